"""Known-answer tests of the reference, restated against the oracle (CPU).

Fixtures follow the reference's own tests: tests/test_complement.py:10-100
(exact complement sets), tests/test_lse_merge.py:29-108 (merge equals dense,
seed 42) and tests/test_effective_budget.py:34-95 (work accounting).
"""

import torch

from oracle import cvsa_ref as R


def test_complement_basic():
    # 10 pages; head 0 selects {0,2,4}, head 1 selects {1,3} (3rd slot is padding)
    idx = torch.tensor([[[0, 2, 4], [1, 3, 0]]], dtype=torch.int32)
    n = torch.tensor([[3, 2]], dtype=torch.int32)
    comp, nc = R.compute_complement_pages(idx, n, torch.tensor([160]), 16)
    assert nc.tolist() == [[7, 8]]
    assert set(comp[0, 0, :7].tolist()) == {1, 3, 5, 6, 7, 8, 9}
    assert set(comp[0, 1, :8].tolist()) == {0, 2, 4, 5, 6, 7, 8, 9}


def test_complement_accept_mask():
    idx = torch.tensor([[[0, 1], [1, 2], [2, 3], [3, 4]]], dtype=torch.int32)
    n = torch.full((1, 4), 2, dtype=torch.int32)
    acc = torch.tensor([[True, False, True, False]])
    _, nc = R.compute_complement_pages(idx, n, torch.tensor([80]), 16, acc)
    assert nc.tolist() == [[0, 3, 0, 3]]


def test_complement_full_budget_and_batch():
    _, nc = R.compute_complement_pages(torch.tensor([[[0, 1, 2]]], dtype=torch.int32),
                                       torch.tensor([[3]], dtype=torch.int32),
                                       torch.tensor([48]), 16)
    assert nc.tolist() == [[0]]
    idx = torch.tensor([[[0, 1]], [[0, 1]]], dtype=torch.int32)
    _, nc = R.compute_complement_pages(idx, torch.tensor([[2], [2]], dtype=torch.int32),
                                       torch.tensor([80, 48]), 16)
    assert nc.tolist() == [[3], [1]]


def _unnorm(q, k, v):
    D = q.shape[-1]
    s = torch.einsum("bhd,bhnd->bhn", q, k) / D ** 0.5
    m = s.max(-1).values
    e = (s - m.unsqueeze(-1)).exp()
    return torch.einsum("bhn,bhnd->bhd", e, v), m, e.sum(-1)


def _dense(q, k, v):
    D = q.shape[-1]
    w = torch.softmax(torch.einsum("bhd,bhnd->bhn", q, k) / D ** 0.5, -1)
    return torch.einsum("bhn,bhnd->bhd", w, v)


def test_merge_equals_dense():
    torch.manual_seed(42)
    q = torch.randn(1, 4, 64)
    k = torch.randn(1, 4, 20, 64)
    v = torch.randn(1, 4, 20, 64)
    od, md, ld = _unnorm(q, k[:, :, :5], v[:, :, :5])
    oc, mc, lc = _unnorm(q, k[:, :, 5:], v[:, :, 5:])
    out = R.selective_lse_merge(od, md, ld, oc, mc, lc, torch.zeros(1, 2, dtype=torch.bool), 2,
                                torch.float32)
    assert (out - _dense(q, k, v)).abs().max() < 1e-4


def test_accepted_heads_use_draft_and_all_accepted():
    torch.manual_seed(42)
    kk = torch.randn(1, 2, 20, 64).repeat_interleave(2, 1)
    vv = torch.randn(1, 2, 20, 64).repeat_interleave(2, 1)
    q = torch.randn(1, 4, 64)
    od, md, ld = _unnorm(q, kk[:, :, :5], vv[:, :, :5])
    oc, mc, lc = _unnorm(q, kk[:, :, 5:], vv[:, :, 5:])
    out = R.selective_lse_merge(od, md, ld, oc, mc, lc, torch.tensor([[True, False]]), 2,
                                torch.float32)
    assert (out[:, :2] - od[:, :2] / ld[:, :2].unsqueeze(-1)).abs().max() < 1e-6
    assert (out[:, 2:] - _dense(q, kk, vv)[:, 2:]).abs().max() < 1e-4
    # all accepted, empty complement (m = -inf, l = 0)
    out = R.selective_lse_merge(od, md, ld, torch.zeros_like(od), torch.full_like(md, -1e30),
                                torch.zeros_like(ld), torch.ones(1, 2, dtype=torch.bool), 2,
                                torch.float32)
    assert (out - od / ld.unsqueeze(-1)).abs().max() < 1e-6


def test_effective_budget_accounting():
    be = R.OracleBackend(4, 32, 128, 16, budget_pct=0.05)
    be._record(torch.tensor([64, 128], dtype=torch.int32), 10)
    assert be.attn_work == 10 and be.attn_work_max == (4 + 8) * 4
    be._record(torch.tensor([64, 128], dtype=torch.int32), 5)
    assert be.attn_work == 15 and be.attn_work_max == 96
    st = be.get_stats()
    assert abs(st["effective_budget_pct"] - 15 / 96 * 100) < 1e-9
    be.reset()
    assert "effective_budget_pct" not in be.get_stats()


def test_stable_topk_ties_go_to_lower_index():
    s = torch.tensor([[[1.0, 3.0, 3.0, 3.0, 0.0, 3.0]]])
    idx, n = R.select_pages(s, torch.tensor([96]), 16, budget=2)
    assert idx[0, 0, :int(n[0, 0])].tolist() == [1, 2]
    # forced pages are on top of the budget
    idx, n = R.select_pages(s, torch.tensor([96]), 16, budget=2, sink_pages=1, local_pages=2)
    assert idx[0, 0, :int(n[0, 0])].tolist() == [0, 1, 2, 4, 5]


def test_empty_and_short_sequences():
    s = torch.randn(3, 1, 8)
    cl = torch.tensor([0, 20, 128])       # 0, 2 and 8 valid pages
    s[0, 0, :] = float("-inf")
    s[1, 0, 2:] = float("-inf")
    idx, n = R.select_pages(s, cl, 16, budget=4, sink_pages=1, local_pages=2)
    assert n.tolist() == [[0], [2], [7]]
    assert idx[1, 0, :2].tolist() == [0, 1]
