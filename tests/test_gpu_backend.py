"""GPU parity of the fused layer step (cvsa_decode_step via CVSABackend).

Checks the drop-in backend against the reference's own outputs (golden) and
against the oracle backend over multi-step lazy schedules; the selection each
scoring step leaves cached is compared bit-exactly, accept decisions exactly
(away from tau), outputs within the bf16 / fp32 bars. At the full config-2
size, size-independent properties stand in for a full oracle comparison of
every variant: tau above 1 makes every head recover, so the output must equal
dense attention; tau = 0 accepts every head, so it must equal the draft.
"""

import numpy as np
import pytest
import torch

from conftest import sel_sets
from cvsa import synthetic
from cvsa.backend import CVSABackend
from cvsa.runtime.dense import DenseAttentionBackend
from cvsa.kernels import sparse_decode as SD
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _close(a, b, dtype):
    a = a.float().cpu()
    b = torch.as_tensor(b).float().cpu()
    if dtype == torch.float32:
        assert (a - b).abs().max() <= 1e-4, float((a - b).abs().max())
    else:
        assert ((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all(), float((a - b).abs().max())


def test_scoring_step_matches_reference_backend(cuda, golden):
    wl = synthetic.config1()
    d = wl.to(cuda)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=64, block_size=16, num_layers=1,
                     budget_pct=wl.budget_pct, coverage_threshold=wl.tau)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    _close(out, golden["config1_backend_output"], torch.float32)
    idx, n = be.cached_selection(0)
    ref = [[list(r[:int(k)]) for r, k in zip(rows, ns)]
           for rows, ns in zip(golden["config1_backend_sel"], golden["config1_backend_n"])]
    assert sel_sets(idx.cpu(), n.cpu()) == ref
    assert np.array_equal(be._last_accept_mask[0].cpu().numpy().astype(np.uint8),
                          golden["config1_backend_accept"])


def test_lazy_schedule_matches_reference_backend(cuda, golden):
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    d = wl.to(cuda)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16, num_layers=1,
                     budget_pct=wl.budget_pct, coverage_threshold=wl.tau, lazy=True,
                     check_interval=2)
    for step in range(5):
        q = torch.from_numpy(golden[f"small_lazy_q{step}"]).to(torch.bfloat16).to(cuda)
        out = be(q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        be.step_done(0, 1)
        _close(out, golden[f"small_lazy_out{step}"], torch.bfloat16)
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(st[key] - float(golden["small_lazy_stat_" + key])) < 1e-9, key


@pytest.mark.parametrize("lazy", [True, False])
def test_multistep_schedule_vs_oracle_backend(cuda, lazy):
    wl = synthetic.small(seed=21, B=3, Hq=16, Hkv=4, D=128, ctx=(3000, 1200, 4100))
    d = wl.to(cuda)
    kw = dict(num_layers=2, budget_pct=0.08, coverage_threshold=0.9, dense_layers=[1],
              sink_pages=1, local_pages=2)
    if lazy:
        kw.update(lazy=True, check_interval=3)
    else:
        kw.update(reuse_interval=3)
    be = CVSABackend(4, 16, 128, 16, **kw)
    ob = R.OracleBackend(4, 16, 128, 16, **kw)
    g = torch.Generator().manual_seed(4)
    base_q = wl.q.float()
    for step in range(7):
        # drift the query so that some gates flip between steps
        q = (base_q + 0.6 * torch.randn(base_q.shape, generator=g)).to(wl.q.dtype)
        for layer in range(2):
            out = be(q.to(cuda), d.k_cache, d.v_cache, d.block_tables, d.context_lens, layer)
            ref = ob(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, layer)
            _close(out, ref, wl.q.dtype)
            be.step_done(layer, 2)
            ob.step_done(layer, 2)
        gi, gn = be.cached_selection(0)
        oi, on = ob._cached[0]
        assert sel_sets(gi.cpu(), gn.cpu()) == sel_sets(oi, on), step
    gs, os_ = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct",
                "total_pages_attended", "total_pages_max"):
        assert abs(gs[key] - os_[key]) < 1e-9, (key, gs[key], os_[key])


def test_dense_layer_vs_oracle(cuda):
    wl = synthetic.small(seed=8, B=2, Hq=32, Hkv=8, D=128, ctx=(5000, 333))
    d = wl.to(cuda)
    out = DenseAttentionBackend(8, 32, 128, 16)(d.q, d.k_cache, d.v_cache, d.block_tables,
                                                 d.context_lens, 0)
    ref = R.dense_decode(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 8, 4, 16)
    _close(out, ref, torch.bfloat16)


@pytest.fixture(scope="module")
def config2_cpu():
    return synthetic.config2()


def test_config2_scoring_step_vs_oracle(cuda, config2_cpu):
    """Full config 2 (B=32, 8K): selection bit-exact, decisions exact, output in tolerance."""
    wl = config2_cpu
    d = wl.to(cuda)
    be = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                     coverage_threshold=wl.tau, sink_pages=1, local_pages=2,
                     keep_page_scores=True)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    torch.set_num_threads(8)
    r = R.scoring_step(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 8, 4, 16,
                       wl.budget_pct, wl.tau, 1, 2)
    gs = be._layers[0].scores.cpu()
    # scores agree to fp32 rounding
    fin = torch.isfinite(r["page_scores"])
    assert (gs[fin] - r["page_scores"][fin]).abs().max() < 2e-5
    # selection: bit-exact unless a near-tie (gap below the score tolerance)
    gap = R.topk_gap(r["page_scores"], wl.context_lens, 16, int(r["budget"]), 1, 2)
    gi, gn = be.cached_selection(0)
    G_sets, O_sets = sel_sets(gi.cpu(), gn.cpu()), sel_sets(r["page_indices"], r["n_per_head"])
    mism = [(b, h) for b in range(32) for h in range(8) if G_sets[b][h] != O_sets[b][h]]
    assert all(gap[b, h] < 4e-5 for b, h in mism), mism
    assert len(mism) == 0, f"{len(mism)} near-tie selection differences"
    # accept decisions: exact away from tau
    acc = be._last_accept_mask[0].cpu()
    margin = R.coverage_margin(r["coverage"], wl.tau)
    assert torch.equal(acc[margin > 1e-5], r["accept"][margin > 1e-5])
    n_rej = int((~r["accept"]).sum())
    assert 20 <= n_rej <= 100, n_rej          # the calibrated mix: some heads recover
    _close(out, r["output"], torch.bfloat16)


def test_config2_properties_full_size(cuda, config2_cpu):
    """tau > 1: every head recovers -> dense attention; tau = 0: every head keeps the draft."""
    d = config2_cpu.to(cuda)
    dense = DenseAttentionBackend(8, 32, 128, 16)(d.q, d.k_cache, d.v_cache, d.block_tables,
                                                  d.context_lens, 0)
    be = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=0.05, coverage_threshold=1.01,
                     sink_pages=1, local_pages=2)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    assert not be._last_accept_mask[0].any()
    _close(out, dense, torch.bfloat16)
    be0 = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=0.05, coverage_threshold=0.0,
                      sink_pages=1, local_pages=2)
    out0 = be0(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    idx, n = be0.cached_selection(0)
    draft = SD.sparse_decode(d.q, d.k_cache, d.v_cache, d.block_tables, idx, n, d.context_lens,
                             8, 4, 16)
    assert torch.equal(out0, draft)
    st = be0.get_stats()
    assert st["per_head_accept_rate"] == 100.0
    # effective budget = selected pages / all pages
    assert abs(st["effective_budget_pct"] - 28 / 512 * 100) < 1e-9


@pytest.fixture(scope="module")
def config3_cpu():
    return synthetic.config3()


def test_config3_scoring_step_vs_oracle(cuda, config3_cpu):
    """Full config 3 (one 128K sequence, 8192 pages): heads spread over every CTA of
    the stream and rejected heads over dozens of them; selection bit-exact,
    decisions exact, output in tolerance."""
    wl = config3_cpu
    d = wl.to(cuda)
    be = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                     coverage_threshold=wl.tau, sink_pages=1, local_pages=2,
                     keep_page_scores=True)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    torch.set_num_threads(8)
    r = R.scoring_step(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 8, 4, 16,
                       wl.budget_pct, wl.tau, 1, 2)
    gs = be._layers[0].scores.cpu()
    fin = torch.isfinite(r["page_scores"])
    assert (gs[fin] - r["page_scores"][fin]).abs().max() < 2e-5 * max(1.0, float(
        r["page_scores"][fin].abs().max()))
    gap = R.topk_gap(r["page_scores"], wl.context_lens, 16, int(r["budget"]), 1, 2)
    gi, gn = be.cached_selection(0)
    G_sets, O_sets = sel_sets(gi.cpu(), gn.cpu()), sel_sets(r["page_indices"], r["n_per_head"])
    mism = [h for h in range(8) if G_sets[0][h] != O_sets[0][h]]
    assert all(gap[0, h] < 4e-5 for h in mism), mism
    assert len(mism) == 0, f"{len(mism)} near-tie selection differences"
    acc = be._last_accept_mask[0].cpu()
    margin = R.coverage_margin(r["coverage"], wl.tau)
    assert torch.equal(acc[margin > 1e-5], r["accept"][margin > 1e-5])
    assert 1 <= int((~r["accept"]).sum()) <= 7      # the calibrated mix: some heads recover
    _close(out, r["output"], torch.bfloat16)
    # reuse step on the cached selection = the draft over that selection
    be._step = 1
    out_r = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    draft = SD.sparse_decode(d.q, d.k_cache, d.v_cache, d.block_tables, gi, gn, d.context_lens,
                             8, 4, 16)
    assert torch.equal(out_r, draft)


def test_config3_every_head_recovers_equals_dense(cuda, config3_cpu):
    """tau > 1 at 128K: all 8 heads take all 8192 pages, each split over many CTAs."""
    d = config3_cpu.to(cuda)
    dense = DenseAttentionBackend(8, 32, 128, 16)(d.q, d.k_cache, d.v_cache, d.block_tables,
                                                  d.context_lens, 0)
    be = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=0.05, coverage_threshold=1.01,
                     sink_pages=1, local_pages=2)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    assert not be._last_accept_mask[0].any()
    _close(out, dense, torch.bfloat16)
    ref = R.dense_decode(config3_cpu.q, config3_cpu.k_cache, config3_cpu.v_cache,
                         config3_cpu.block_tables, config3_cpu.context_lens, 8, 4, 16)
    _close(out, ref, torch.bfloat16)


def test_step_is_graph_capturable_and_deterministic(cuda):
    wl = synthetic.small(seed=9, B=4, Hq=32, Hkv=8, D=128, ctx=(4096, 2000, 8192, 100))
    d = wl.to(cuda)
    be = CVSABackend(8, 32, 128, 16, num_layers=1, budget_pct=0.05, coverage_threshold=0.9,
                     lazy=True, check_interval=2, sink_pages=1, local_pages=2)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        first = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0).clone()
        be._step = 2            # a lazy check step (warm-up on the capture stream)
        be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        s.synchronize()
        be._step = 2
        with torch.cuda.graph(g, stream=s):
            out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    # same q, same cache: the replayed lazy step reproduces the first step exactly
    assert torch.equal(out, first)


def test_approx_recovery_lazy_matches_reference(cuda):
    """approx_recovery_pct=0.2 over a lazy schedule against the reference's own
    CVSABackend outputs (tests/golden/make_golden_ar.py; every head rejects at
    tau=0.95, so each check step decodes the expanded selections)."""
    import os
    from conftest import GOLDEN
    g = dict(np.load(os.path.join(os.path.dirname(GOLDEN), "reference_outputs_ar.npz")))
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    d = wl.to(cuda)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16, num_layers=1,
                     budget_pct=wl.budget_pct, coverage_threshold=0.95, lazy=True,
                     check_interval=2, approx_recovery_pct=0.2)
    for step in range(4):
        q = torch.from_numpy(g[f"small_ar20_q{step}"]).to(torch.bfloat16).to(cuda)
        out = be(q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        be.step_done(0, 1)
        _close(out, g[f"small_ar20_out{step}"], torch.bfloat16)
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate"):
        assert abs(st[key] - float(g["small_ar20_stat_" + key])) < 1e-9, key


def test_approx_recovery_vs_oracle(cuda):
    """Approximate recovery with forced pages, Llama-8B head geometry, lazy
    schedule with drifting queries: outputs, cached selections and decisions
    against the oracle backend."""
    wl = synthetic.small(seed=12, B=2, Hq=32, Hkv=8, D=128, ctx=(6000, 2500), heavy_alpha=3.0)
    d = wl.to(cuda)
    kw = dict(num_layers=1, budget_pct=0.05, coverage_threshold=0.9, lazy=True, check_interval=2,
              sink_pages=1, local_pages=2, approx_recovery_pct=0.2)
    be = CVSABackend(8, 32, 128, 16, **kw)
    ob = R.OracleBackend(8, 32, 128, 16, **kw)
    g = torch.Generator().manual_seed(6)
    rejected = 0
    for step in range(6):
        q = (wl.q.float() + 0.8 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
        out = be(q.to(cuda), d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        ref = ob(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        _close(out, ref, wl.q.dtype)
        if "accept" in ob.last and ob.last.get("expanded") is not None:
            rejected += int((~ob.last["accept"]).sum())
        gi, gn = be.cached_selection(0)
        oi, on = ob._cached[0]
        assert sel_sets(gi.cpu(), gn.cpu()) == sel_sets(oi, on), step
        be.step_done(0, 1)
        ob.step_done(0, 1)
    assert rejected > 0, "no head took the approximate branch"
    gs, os_ = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate"):
        assert abs(gs[key] - os_[key]) < 1e-9, (key, gs[key], os_[key])


def test_coverage_only_steps_match_reference(cuda):
    """coverage_interval=2 < check_interval=4: coverage-only steps gate the
    cached selection on the last scoring step's page scores (backend.py:
    467-520); outputs and statistics against the reference's own CVSABackend
    (tests/golden/make_golden_cv.py)."""
    import os
    from conftest import GOLDEN
    g = dict(np.load(os.path.join(os.path.dirname(GOLDEN), "reference_outputs_cv.npz")))
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    d = wl.to(cuda)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16, num_layers=1,
                     budget_pct=wl.budget_pct, coverage_threshold=0.16, lazy=True,
                     check_interval=4, coverage_interval=2)
    for step in range(9):
        q = torch.from_numpy(g[f"small_cv_q{step}"]).to(torch.bfloat16).to(cuda)
        out = be(q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        be.step_done(0, 1)
        _close(out, g[f"small_cv_out{step}"], torch.bfloat16)
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(st[key] - float(g["small_cv_stat_" + key])) < 1e-9, key


def test_coverage_only_steps_vs_oracle(cuda):
    """Coverage-only steps with forced pages and Llama-8B head geometry,
    against the oracle backend: outputs, cached selections, statistics."""
    wl = synthetic.small(seed=14, B=2, Hq=32, Hkv=8, D=128, ctx=(5000, 3100), heavy_alpha=5.0)
    d = wl.to(cuda)
    kw = dict(num_layers=1, budget_pct=0.05, coverage_threshold=0.5, lazy=True, check_interval=4,
              coverage_interval=2, sink_pages=1, local_pages=2)
    be = CVSABackend(8, 32, 128, 16, **kw)
    ob = R.OracleBackend(8, 32, 128, 16, **kw)
    g = torch.Generator().manual_seed(8)
    for step in range(10):
        q = (wl.q.float() + 0.5 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
        out = be(q.to(cuda), d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        ref = ob(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        _close(out, ref, wl.q.dtype)
        gi, gn = be.cached_selection(0)
        oi, on = ob._cached[0]
        assert sel_sets(gi.cpu(), gn.cpu()) == sel_sets(oi, on), step
        be.step_done(0, 1)
        ob.step_done(0, 1)
    gs, os_ = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(gs[key] - os_[key]) < 1e-9, (key, gs[key], os_[key])
