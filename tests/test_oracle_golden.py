"""The CPU oracle against outputs of the reference implementation itself.

tests/golden/reference_outputs.npz was produced by tests/golden/make_golden.py,
which ran the reference's Triton kernels and CVSABackend under the Triton
interpreter on the same seeded inputs. These tests pin the oracle (the checker
of every GPU parity test) to the reference.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, finite_close, input_checksum, sel_sets
from cvsa import synthetic
from oracle import cvsa_ref as R


def _case(name):
    if name == "config1":
        return synthetic.config1()
    return synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))


@pytest.mark.parametrize("case", ["config1", "small"])
def test_inputs_regenerate_bit_identically(golden, case):
    wl = _case(case)
    assert input_checksum(wl) == str(golden[f"{case}_checksum"])


@pytest.mark.parametrize("case", ["config1", "small"])
def test_oracle_scores_match_reference(golden, case):
    wl = _case(case)
    s = R.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, wl.num_kv_heads,
                      wl.num_q_per_kv, wl.block_size)
    # the reference sums in fp32 in its own order; the oracle rounds the exact sum
    finite_close(s, golden[f"{case}_scores"], atol=2e-5, rtol=2e-6)


@pytest.mark.parametrize("case", ["config1", "small"])
def test_oracle_selection_and_gate_match_reference(golden, case):
    wl = _case(case)
    ref_scores = torch.from_numpy(golden[f"{case}_scores"])
    W = wl.block_tables.shape[1]
    budget = R.budget_for(W, wl.budget_pct)
    idx, n = R.select_pages(ref_scores, wl.context_lens, wl.block_size, budget,
                            wl.sink_pages, wl.local_pages)
    assert sel_sets(idx, n) == sel_sets(golden[f"{case}_sel_idx"], golden[f"{case}_sel_n"])
    acc, cov = R.check_coverage(ref_scores, idx, n, wl.tau)
    assert np.array_equal(acc.numpy().astype(np.uint8), golden[f"{case}_accept"])
    assert np.abs(cov.numpy() - golden[f"{case}_coverage"]).max() < 1e-5


@pytest.mark.parametrize("case", ["config1", "small"])
def test_oracle_decode_complement_merge_match_reference(golden, case):
    wl = _case(case)
    idx = torch.from_numpy(golden[f"{case}_sel_idx"])
    n = torch.from_numpy(golden[f"{case}_sel_n"])
    o, m, l = R.sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, idx, n,
                                     wl.context_lens, wl.num_kv_heads, wl.num_q_per_kv,
                                     wl.block_size)
    finite_close(m, golden[f"{case}_m_draft"], atol=1e-5, rtol=1e-6)
    finite_close(l, golden[f"{case}_l_draft"], atol=1e-4, rtol=1e-5)
    finite_close(o, golden[f"{case}_o_draft"], atol=1e-4, rtol=1e-5)
    acc = torch.from_numpy(golden[f"{case}_accept"]).bool()
    comp, nc = R.compute_complement_pages(idx, n, wl.context_lens, wl.block_size, acc)
    assert np.array_equal(nc.numpy(), golden[f"{case}_n_comp"])
    oc, mc, lc = R.sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, comp, nc,
                                        wl.context_lens, wl.num_kv_heads, wl.num_q_per_kv,
                                        wl.block_size)
    out = R.selective_lse_merge(o, m, l, oc, mc, lc, acc, wl.num_q_per_kv, wl.q.dtype)
    ref = torch.from_numpy(golden[f"{case}_output"])
    if wl.q.dtype == torch.float32:
        assert (out - ref).abs().max() < 1e-4
    else:
        # both sides round to bf16 once: at most one bf16 ulp apart
        assert (out.float() - ref).abs().max() < 2e-2


def test_oracle_backend_scoring_step_matches_reference(golden):
    wl = synthetic.config1()
    be = R.OracleBackend(2, 8, 64, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=wl.tau)
    out = be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
    idx, n = be._cached[0]
    assert sel_sets(idx, n) == [[list(r[:int(k)]) for r, k in zip(rows, ns)]
                                for rows, ns in zip(golden["config1_backend_sel"],
                                                    golden["config1_backend_n"])]
    assert np.array_equal(be.last["accept"].numpy().astype(np.uint8),
                          golden["config1_backend_accept"])
    assert (out - torch.from_numpy(golden["config1_backend_output"])).abs().max() < 1e-4


def test_oracle_lazy_schedule_matches_reference(golden):
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be = R.OracleBackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=wl.tau, lazy=True, check_interval=2)
    for step in range(5):
        q = torch.from_numpy(golden[f"small_lazy_q{step}"]).to(torch.bfloat16)
        out = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        be.step_done(0, 1)
        ref = torch.from_numpy(golden[f"small_lazy_out{step}"])
        assert (out.float() - ref).abs().max() < 2e-2, step
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(st[key] - float(golden["small_lazy_stat_" + key])) < 1e-9, key


@pytest.fixture(scope="module")
def golden_ar():
    return dict(np.load(os.path.join(os.path.dirname(GOLDEN), "reference_outputs_ar.npz")))


def test_oracle_approx_recovery_matches_reference(golden_ar):
    """approx_recovery_pct=0.2 (backend.py:780-817) against the reference's
    own CVSABackend (tests/golden/make_golden_ar.py): output, expanded
    selection, accept mask and the recorded work."""
    wl = synthetic.config1()
    be = R.OracleBackend(2, 8, 64, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=wl.tau, approx_recovery_pct=0.2)
    out = be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
    e_idx, e_n = be.last["expanded"]
    assert np.array_equal(e_n.numpy(), golden_ar["config1_ar20_exp_n"])
    assert sel_sets(e_idx, e_n) == [[list(r[:int(k)]) for r, k in zip(rows, ns)]
                                    for rows, ns in zip(golden_ar["config1_ar20_exp_sel"],
                                                        golden_ar["config1_ar20_exp_n"])]
    assert np.array_equal(be.last["accept"].numpy().astype(np.uint8),
                          golden_ar["config1_ar20_accept"])
    assert not bool(be.last["accept"].all())          # the approximate branch ran
    assert (out - torch.from_numpy(golden_ar["config1_ar20_output"])).abs().max() < 1e-4
    st = be.get_stats()
    assert abs(st["effective_budget_pct"]
               - float(golden_ar["config1_ar20_stat_effective_budget_pct"])) < 1e-9


def test_oracle_approx_recovery_lazy_matches_reference(golden_ar):
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be = R.OracleBackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=0.95, lazy=True, check_interval=2,
                         approx_recovery_pct=0.2)
    for step in range(4):
        q = torch.from_numpy(golden_ar[f"small_ar20_q{step}"]).to(torch.bfloat16)
        out = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        be.step_done(0, 1)
        ref = torch.from_numpy(golden_ar[f"small_ar20_out{step}"])
        assert (out.float() - ref).abs().max() < 2e-2, step
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate",
                "effective_budget_pct"):
        assert abs(st[key] - float(golden_ar["small_ar20_stat_" + key])) < 1e-9, key


def test_oracle_coverage_only_steps_match_reference():
    """coverage_interval=2 < check_interval=4 (backend.py:467-520) against the
    reference's own CVSABackend (tests/golden/make_golden_cv.py)."""
    g = dict(np.load(os.path.join(os.path.dirname(GOLDEN), "reference_outputs_cv.npz")))
    wl = synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be = R.OracleBackend(2, 8, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                         coverage_threshold=0.16, lazy=True, check_interval=4,
                         coverage_interval=2)
    for step in range(9):
        q = torch.from_numpy(g[f"small_cv_q{step}"]).to(torch.bfloat16)
        out = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        be.step_done(0, 1)
        assert (out.float() - torch.from_numpy(g[f"small_cv_out{step}"])).abs().max() < 2e-2, step
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(st[key] - float(g["small_cv_stat_" + key])) < 1e-9, key
