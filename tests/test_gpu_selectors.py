"""GPU parity of the reference's alternative selectors (cvsa/selectors.py,
csrc/quest.cu) against the reference's own outputs and the oracle.

The fixture tests/golden/reference_outputs_sel.npz holds the reference
CVSABackend's per-step outputs, cached selections, gate decisions and
statistics for each selector option (tests/golden/make_golden_sel.py). The
backend here runs the same steps on the GPU; bars: selections equal as sets
with equal counts, gate decisions equal, outputs within the bf16 bar
(2e-2 abs), statistics equal. The Quest kernel is also checked against the
oracle's restatement at a larger ragged size and on the fp32 config-1 pool.
"""

import numpy as np
import pytest
import torch

from conftest import finite_close, sel_sets
from cvsa import synthetic
from cvsa.backend import CVSABackend
from cvsa.kernels.page_scores import quest_page_scores
from oracle import cvsa_ref as R
from test_oracle_selectors import CASES, STAT_KEYS, golden_sets, gsel, step_queries  # noqa: F401

pytestmark = pytest.mark.gpu


def test_quest_kernel_matches_reference(cuda, gsel):
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048)).to(cuda)
    s = quest_page_scores(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, 2)
    finite_close(s.cpu(), gsel["quest_scores"], atol=2e-5, rtol=2e-6)


@pytest.mark.parametrize("case", ["ragged", "config1"])
def test_quest_kernel_matches_oracle(cuda, case):
    if case == "config1":
        wl = synthetic.config1()                       # fp32, D = 64
    else:
        wl = synthetic.small(seed=8, B=3, Hq=32, Hkv=8, D=128, ctx=(37, 4100, 9000))
    ref = R.quest_page_scores(wl.q, wl.k_cache, wl.block_tables, wl.context_lens,
                              wl.num_kv_heads, wl.block_size)
    d = wl.to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    s = quest_page_scores(d.q, d.k_cache, d.block_tables, d.context_lens, wl.num_kv_heads,
                          dev_error=err)
    finite_close(s.cpu(), ref, atol=5e-5, rtol=5e-6)
    assert int(err.item()) == 0


@pytest.mark.parametrize("name,opts,lazy,tau", CASES, ids=[c[0] for c in CASES])
def test_selector_backend_matches_reference(cuda, gsel, name, opts, lazy, tau):
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    d = wl.to(cuda)
    sched = dict(lazy=True, check_interval=2) if lazy else dict(reuse_interval=2)
    be = CVSABackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                     coverage_threshold=tau, **sched, **opts)
    for step, q in enumerate(step_queries(wl)):
        out = be(q.to(cuda), d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        be.step_done(0, 1)
        idx, n = be.cached_selection(0)
        assert np.array_equal(n.cpu().numpy(), gsel[f"sel_{name}_n{step}"]), step
        assert sel_sets(idx.cpu(), n.cpu()) == golden_sets(gsel, name, step), step
        acc = be._last_accept_mask.get(0)
        ref_acc = gsel[f"sel_{name}_acc{step}"]
        if acc is not None and ref_acc[0, 0] != 255:
            assert np.array_equal(acc.cpu().numpy().astype(np.uint8), ref_acc), step
        ref = torch.from_numpy(gsel[f"sel_{name}_out{step}"])
        assert (out.float().cpu() - ref).abs().max() < 2e-2, step
    st = be.get_stats()
    for key in STAT_KEYS:
        assert abs(st[key] - float(gsel[f"sel_{name}_stat_{key}"])) < 1e-9, key


def test_random_reject_gates_all_heads_together(cuda):
    """random_reject_prob = 0.5: every gate accepts or rejects every head at
    once (one draw per gate, backend.py:437-438), and both happen."""
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    d = wl.to(cuda)
    torch.cuda.manual_seed(5)
    be = CVSABackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                     coverage_threshold=0.0, lazy=True, check_interval=1,
                     random_reject_prob=0.5)
    seen = set()
    for q in step_queries(wl, 12):
        be(q.to(cuda), d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        be.step_done(0, 1)
        acc = be._last_accept_mask[0]
        assert bool(acc.all()) or not bool(acc.any())
        seen.add(bool(acc.all()))
    assert seen == {True, False}
    st = be.get_stats()
    assert st["total_coverage_checks"] == 12
