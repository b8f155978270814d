"""Device-side failure paths, each in a form that cannot fault the GPU.

* Range checks: the kernels are told the pool holds fewer blocks than it
  really does (a view of its first rows), and some block-table entries point
  into the rows beyond the view -- memory that is allocated, so a missed
  check would read valid memory instead of faulting. The kernels must skip
  those pages, set CVSA_DEV_ERR_BLOCK_RANGE, and give the result over the
  remaining pages. Out-of-range page indices in a cached selection
  (CVSA_DEV_ERR_PAGE_RANGE) are checked the same way.
* Bounded waits: cvsa_set_wait_limit(1) makes the attention kernel's waits
  on its producer warp give up at once; the step must return, record
  CVSA_DEV_ERR_TIMEOUT, and a step after the limit is restored (on a reset
  workspace) must be correct again.
"""

import pytest
import torch

from cvsa import _lib, synthetic
from cvsa.backend import CVSABackend
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


def _wl():
    return synthetic.small(seed=5, B=2, Hq=8, Hkv=2, D=128, ctx=(700, 1500))


def _dense_be():
    return CVSABackend(2, 8, 128, 16, num_layers=1, dense_layers=[0])


def test_block_range_skips_pages_and_sets_error(cuda):
    wl = _wl()
    NB = wl.k_cache.shape[0]
    nb = NB - 6                                    # the kernels' view of the pool
    bt = wl.block_tables.clone()
    # three pages of sequence 1 (not the last one) move into rows past the view
    bad = [3, 10, 40]
    for i, p in enumerate(bad):
        bt[1, p] = nb + i
    d = wl.to(cuda)
    kv_k, kv_v = d.k_cache[:nb], d.v_cache[:nb]    # views: rows >= nb still allocated
    be = _dense_be()
    out = be(d.q, kv_k, kv_v, bt.to(cuda), d.context_lens, 0)
    torch.cuda.synchronize()
    assert be.device_errors() & _lib.DEV_ERR_BLOCK_RANGE
    # expected: dense attention over every valid page except the skipped ones
    nv = R.n_valid_pages(wl.context_lens, 16)
    W = bt.shape[1]
    idx = torch.zeros(2, 2, W, dtype=torch.int32)
    n = torch.zeros(2, 2, dtype=torch.int32)
    for b in range(2):
        # every page whose block lies outside the view is skipped (the planted
        # ones, and any the permuted table already placed there)
        keep = [p for p in range(int(nv[b])) if int(bt[b, p]) < nb]
        if b == 1:
            assert not any(p in keep for p in bad)
        idx[b, :, :len(keep)] = torch.tensor(keep, dtype=torch.int32)
        n[b, :] = len(keep)
    ref = R.sparse_decode(wl.q, wl.k_cache, wl.v_cache, bt, idx, n, wl.context_lens, 2, 4, 16)
    assert (out.float().cpu() - ref.float()).abs().max() < BF16_ATOL


def test_block_range_in_scoring_step(cuda):
    """Scoring, selection and attention of a scoring step with out-of-view
    blocks: the error bit is set and the step completes with finite output."""
    wl = _wl()
    NB = wl.k_cache.shape[0]
    nb = NB - 4
    bt = wl.block_tables.clone()
    bt[0, 5] = nb + 1
    d = wl.to(cuda)
    be = CVSABackend(2, 8, 128, 16, num_layers=1, budget_pct=0.1, coverage_threshold=0.9)
    out = be(d.q, d.k_cache[:nb], d.v_cache[:nb], bt.to(cuda), d.context_lens, 0)
    torch.cuda.synchronize()
    assert be.device_errors() & _lib.DEV_ERR_BLOCK_RANGE
    assert torch.isfinite(out.float()).all()


def test_page_range_in_cached_selection(cuda):
    """A reuse step whose cached selection holds a page index past the table
    width: CVSA_DEV_ERR_PAGE_RANGE, the page is skipped, the others attended."""
    wl = _wl()
    d = wl.to(cuda)
    be = CVSABackend(2, 8, 128, 16, num_layers=1, budget_pct=0.1, coverage_threshold=0.0,
                     reuse_interval=4)
    be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)   # scoring step
    be.step_done(0, 1)
    idx, n = be.cached_selection(0)
    W = wl.block_tables.shape[1]
    good = idx.clone()
    idx[0, 1, 0] = W + 7                              # out of the table
    out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)   # reuse
    torch.cuda.synchronize()
    assert be.device_errors() & _lib.DEV_ERR_PAGE_RANGE
    # expected: head (0, 1) without its first cached page, the rest unchanged
    sel = good.cpu().clone()
    nn = n.cpu().clone()
    row = sel[0, 1, 1:int(nn[0, 1])].clone()
    sel[0, 1, :row.numel()] = row
    nn[0, 1] -= 1
    ref = R.sparse_decode(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, sel, nn,
                          wl.context_lens, 2, 4, 16)
    assert (out.float().cpu() - ref.float()).abs().max() < BF16_ATOL


def test_bounded_wait_times_out_and_recovers(cuda):
    wl = _wl()
    d = wl.to(cuda)
    lib = _lib.load()
    be = _dense_be()
    ref = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    try:
        assert lib.cvsa_set_wait_limit(1) == 0
        out = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        torch.cuda.synchronize()                    # the step returned
    finally:
        lib.cvsa_set_wait_limit(0)
    assert be.device_errors() & _lib.DEV_ERR_TIMEOUT
    # a fresh workspace (the timed-out launch may leave its tickets set) and
    # the default limit: the step is correct again
    for ws in be._ws.values():
        ws[2].zero_()
    be._dev_error.zero_()
    out2 = be(d.q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    assert torch.equal(out2, ref)
