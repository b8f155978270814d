"""The oracle's alternative selectors against the reference itself.

tests/golden/reference_outputs_sel.npz was produced by
tests/golden/make_golden_sel.py, which ran the reference's CVSABackend with
each selector option (selector='quest', light_normalizer, top_p,
static_budget_table, adaptive_selection, random_reject_prob) under the Triton
interpreter on the bf16 ragged case. These tests pin the oracle's
restatements (quest_page_scores, topp_select, static_select,
adaptive_select, OracleBackend with the options) to the reference: the Quest
scores within fp32 summation-order error, then per step the cached selection
(as sets), the page counts, the gate decisions, the output (bf16 bar
2e-2) and the final statistics.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, finite_close, sel_sets
from cvsa import synthetic
from oracle import cvsa_ref as R

SEL = os.path.join(os.path.dirname(GOLDEN), "reference_outputs_sel.npz")
STAT_KEYS = ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
             "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct")
TAU = 0.8
# (name, OracleBackend options, lazy, coverage threshold)
CASES = [
    ("selq", dict(selector="quest"), True, TAU),
    ("ln", dict(selector="quest", light_normalizer=True), True, TAU),
    ("tp", dict(top_p=0.9), True, TAU),
    ("staticpol", dict(static_budget_table={0: [0.05, 0.25]}), True, TAU),
    ("adasel", dict(adaptive_selection=True), True, TAU),
    ("tp_ar", dict(top_p=0.6, approx_recovery_pct=0.2), True, TAU),
    ("tp_fixed", dict(top_p=0.9), False, TAU),
    ("rr0", dict(random_reject_prob=0.0), True, TAU),
    ("rr1", dict(random_reject_prob=1.0), True, TAU),
    ("selq_mix", dict(selector="quest"), True, 0.3),
    ("ln_mix", dict(selector="quest", light_normalizer=True), True, 0.3),
    ("staticpol_mix", dict(static_budget_table={0: [0.05, 0.25]}), True, 0.3),
    ("adasel_mix", dict(adaptive_selection=True), True, 0.3),
]


@pytest.fixture(scope="module")
def gsel():
    return dict(np.load(SEL))


def workload():
    return synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))


def step_queries(wl, steps=5):
    """The queries make_golden_sel.py drew: base + 0.7 N(0, 1) per step (seed 31)."""
    g = torch.Generator().manual_seed(31)
    base = torch.randn(wl.q.shape, generator=g)
    return [(base + 0.7 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
            for _ in range(steps)]


def golden_sets(g, name, step):
    return sel_sets(g[f"sel_{name}_idx{step}"], g[f"sel_{name}_n{step}"])


def test_quest_scores_match_reference(gsel):
    wl = workload()
    s = R.quest_page_scores(wl.q, wl.k_cache, wl.block_tables, wl.context_lens,
                            wl.num_kv_heads, wl.block_size)
    finite_close(s, gsel["quest_scores"], atol=2e-5, rtol=2e-6)


@pytest.mark.parametrize("name,opts,lazy,tau", CASES, ids=[c[0] for c in CASES])
def test_oracle_selector_runs_match_reference(gsel, name, opts, lazy, tau):
    if f"sel_{name}_out0" not in gsel:
        pytest.fail(f"fixture has no case {name}")
    wl = workload()
    sched = dict(lazy=True, check_interval=2) if lazy else dict(reuse_interval=2)
    be = R.OracleBackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=tau, **sched, **opts)
    for step, q in enumerate(step_queries(wl)):
        out = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        be.step_done(0, 1)
        idx, n = be._cached[0]
        assert np.array_equal(n.numpy(), gsel[f"sel_{name}_n{step}"]), step
        assert sel_sets(idx, n) == golden_sets(gsel, name, step), step
        ref = torch.from_numpy(gsel[f"sel_{name}_out{step}"])
        assert (out.float() - ref).abs().max() < 2e-2, step
    st = be.get_stats()
    for key in STAT_KEYS:
        assert abs(st[key] - float(gsel[f"sel_{name}_stat_{key}"])) < 1e-9, key


def test_topp_prefix_reaches_mass():
    """Known answer: probabilities 0.5, 0.3, 0.15, 0.05 (in scrambled page
    order); top_p 0.9 needs the three largest (0.95 >= 0.9 while 0.8 < 0.9)."""
    p = torch.tensor([0.05, 0.3, 0.5, 0.15])
    s = p.log().view(1, 1, 4)
    idx, n, mb = R.topp_select(s, torch.tensor([4]), 0.9)
    assert int(n[0, 0]) == 3 and mb == 3
    assert sorted(idx[0, 0, :3].tolist()) == [1, 2, 3]


def test_adaptive_shares_known_answer():
    """Two heads, base budget 2 (4 slots): head 0 holds the three best pages,
    so its raw share is 3, head 1's is 1; blended half-way to uniform:
    round(1.5 + 1) = 2 (half to even) and round(0.5 + 1) = 2."""
    s = torch.tensor([[[9.0, 8.0, 7.0, 0.0], [6.0, 1.0, 0.5, 0.2]]])
    idx, n, mb = R.adaptive_select(s, 2, torch.tensor([4]), 0.5)
    assert n.tolist() == [[2, 2]]
    s2 = torch.tensor([[[9.0, 8.0, 7.0, 6.5], [6.0, 1.0, 0.5, 0.2]]])
    idx, n, mb = R.adaptive_select(s2, 2, torch.tensor([4]), 0.0)
    assert n.tolist() == [[4, 1]] and mb == 4
