"""Parity against the oracle at the benchmark's own shapes for configs 4 and 5.

* Config 4, one head shard at full size: B=8, one KV head with its 8 query
  heads (G=8), 32K context (2048 pages), budget 102 + 3 forced pages -- the
  work one rank does when the 8 KV heads are sharded over 8 GPUs. Scoring
  step: scores to fp32 rounding, selection bit-exact (a difference only
  allowed at a score near-tie, and none may occur), accept decisions exact
  away from tau, output within the bf16 bar; then a reuse step.
* Config 5, ragged at 16 sequences of up to 16K tokens in a pool with a
  shuffled free list, growing by one token per sequence each step through
  cvsa_paged_append, over a lazy schedule: outputs, cached selections and
  statistics against the oracle run on copies of the cache.
"""

import pytest
import torch

from conftest import sel_sets
from cvsa import synthetic
from cvsa.backend import CVSABackend
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _close(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    assert ((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all(), float((a - b).abs().max())


def test_config4_full_shard_vs_oracle(cuda):
    torch.set_num_threads(8)
    wl = synthetic.config4(kv_heads=slice(3, 4))            # rank 3 of 8
    d = wl.to(cuda)
    kw = dict(num_layers=1, budget_pct=wl.budget_pct, coverage_threshold=wl.tau,
              sink_pages=1, local_pages=2)
    be = CVSABackend(1, 8, 128, 16, keep_page_scores=True, reuse_interval=2, **kw)
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    r = R.scoring_step(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 1, 8, 16,
                       wl.budget_pct, wl.tau, 1, 2)
    gs = be._layers[0].scores.cpu()
    fin = torch.isfinite(r["page_scores"])
    assert torch.equal(torch.isfinite(gs), fin)
    assert (gs[fin] - r["page_scores"][fin]).abs().max() < 2e-5
    gap = R.topk_gap(r["page_scores"], wl.context_lens, 16, int(r["budget"]), 1, 2)
    gi, gn = be.cached_selection(0)
    G_sets, O_sets = sel_sets(gi.cpu(), gn.cpu()), sel_sets(r["page_indices"], r["n_per_head"])
    mism = [b for b in range(8) if G_sets[b][0] != O_sets[b][0]]
    assert all(gap[b, 0] < 4e-5 for b in mism), mism
    assert not mism, f"{len(mism)} near-tie selection differences"
    acc = be._last_accept_mask[0].cpu()
    margin = R.coverage_margin(r["coverage"], wl.tau)
    assert torch.equal(acc[margin > 1e-5], r["accept"][margin > 1e-5])
    _close(out, r["output"])
    be.step_done(0, 1)
    # reuse step on the cached selection
    out2 = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    ref2 = R.sparse_decode(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, r["page_indices"],
                           r["n_per_head"], wl.context_lens, 1, 8, 16)
    _close(out2, ref2)


def test_config5_sixteen_sequences_vs_oracle(cuda):
    torch.set_num_threads(8)
    n = 16
    wl = synthetic.config5(device=cuda, seed=5, n_seqs=n, min_len=1024, max_len=16384, grow=24)
    mgr, cache = wl.mgr, wl.cache
    kw = dict(num_layers=1, budget_pct=wl.budget_pct, coverage_threshold=wl.tau, lazy=True,
              check_interval=4, sink_pages=1, local_pages=2)
    be = CVSABackend(8, 32, 128, 16, **kw)
    ob = R.OracleBackend(8, 32, 128, 16, **kw)
    g = torch.Generator(device="cpu").manual_seed(21)
    lens0 = mgr.context_lens.cpu().clone()
    for step in range(6):
        k_new = (0.1 * torch.randn((n, 8, 128), generator=g)).to(torch.bfloat16)
        v_new = torch.randn((n, 8, 128), generator=g).to(torch.bfloat16)
        mgr.append_batch(k_new.to(cuda), v_new.to(cuda))
        q = torch.randn((n, 32, 128), generator=g).to(torch.bfloat16)
        out = be(q.to(cuda), cache.k_cache, cache.v_cache, mgr.block_tables, mgr.context_lens, 0)
        kc, vc = cache.k_cache.cpu(), cache.v_cache.cpu()
        bt, cl = mgr.block_tables.cpu(), mgr.context_lens.cpu()
        ref = ob(q, kc, vc, bt, cl, 0)
        _close(out, ref)
        assert torch.equal(cl, lens0 + step + 1)
        gi, gn = be.cached_selection(0)
        oi, on = ob._cached[0]
        assert sel_sets(gi.cpu(), gn.cpu()) == sel_sets(oi, on), step
        be.step_done(0, 1)
        ob.step_done(0, 1)
    cache.check()
    gs, os_ = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate",
                "total_pages_attended", "total_pages_max"):
        assert abs(gs[key] - os_[key]) < 1e-9, (key, gs[key], os_[key])
