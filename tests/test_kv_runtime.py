"""Paged KV runtime: the oracle pinned to the reference, and the CUDA runtime
(cvsa.runtime.kv_cache over cvsa_paged_append / cvsa_paged_gather) against
both.

tests/golden/reference_outputs_kv.npz holds the reference's own
PagedKVCache / SequenceKVManager run (tests/golden/make_golden_kv.py) over a
seeded schedule of prefills and single-token appends: block tables, context
lengths, pages allocated, the allocator position, and digests of the pools.
The bar is bit-exact (index work and copies).
"""

import hashlib
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import cvsa_ref as R

import importlib.util

_spec = importlib.util.spec_from_file_location(
    "make_golden_kv", os.path.join(os.path.dirname(GOLDEN), "make_golden_kv.py"))
G = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(G)


@pytest.fixture(scope="module")
def gkv():
    return dict(np.load(os.path.join(os.path.dirname(GOLDEN), "reference_outputs_kv.npz")))


def digest(t) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().view(-1).view(torch.uint8)
                          .numpy().tobytes()).hexdigest()


def run_oracle():
    ref = R.PagedKVRef(G.NUM_BLOCKS, G.BS, G.H, G.D, torch.bfloat16, G.B, G.MAX_CTX)
    pre, app = G.schedule()
    for b, k, v in pre:
        ref.prefill(b, k, v)
    snap = (ref.block_tables.clone(), ref.context_lens.clone(), list(ref.pages), ref.next_free)
    for b, k, v in app:
        ref.append(b, k, v)
    return ref, snap


def test_oracle_runtime_matches_reference(gkv):
    ref, (t0, l0, p0, f0) = run_oracle()
    assert np.array_equal(t0.numpy(), gkv["pre_tables"])
    assert np.array_equal(l0.numpy(), gkv["pre_lens"])
    assert p0 == gkv["pre_pages"].tolist() and f0 == int(gkv["pre_next_free"])
    assert np.array_equal(ref.block_tables.numpy(), gkv["tables"])
    assert np.array_equal(ref.context_lens.numpy(), gkv["lens"])
    assert ref.pages == gkv["pages"].tolist() and ref.next_free == int(gkv["next_free"])
    assert digest(ref.k) == str(gkv["k_sha"]) and digest(ref.v) == str(gkv["v_sha"])


@pytest.mark.gpu
def test_gpu_prefill_append_gather_match_reference(cuda, gkv):
    """prefill_kv, append_token_kv (one launch per call, the reference's call
    pattern) and gather_pages against the reference's own run."""
    from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
    cache = PagedKVCache(G.NUM_BLOCKS, G.BS, G.H, G.D, dtype=torch.bfloat16, device="cuda")
    mgr = SequenceKVManager(cache, G.B, G.MAX_CTX)
    pre, app = G.schedule()
    for b, k, v in pre:
        mgr.prefill_kv(b, k.to(cuda), v.to(cuda))
    assert np.array_equal(mgr.block_tables.cpu().numpy(), gkv["pre_tables"])
    assert np.array_equal(mgr.context_lens.cpu().numpy(), gkv["pre_lens"])
    assert mgr._pages_allocated == gkv["pre_pages"].tolist()
    assert cache._next_free == int(gkv["pre_next_free"])
    for b, k, v in app:
        mgr.append_token_kv(b, k.to(cuda), v.to(cuda))
    cache.check()
    assert np.array_equal(mgr.block_tables.cpu().numpy(), gkv["tables"])
    assert np.array_equal(mgr.context_lens.cpu().numpy(), gkv["lens"])
    assert mgr._pages_allocated == gkv["pages"].tolist()
    assert cache._next_free == int(gkv["next_free"])
    assert digest(cache.k_cache) == str(gkv["k_sha"])
    assert digest(cache.v_cache) == str(gkv["v_sha"])
    # gather: every sequence's pages, dense, against the oracle pool
    ref, _ = run_oracle()
    for b in range(G.B):
        n = int(mgr.pages_allocated[b])
        blocks = mgr.block_tables[b, :n]
        kg, vg = cache.gather_pages(blocks)
        rk, rv = ref.gather(blocks.cpu())
        assert torch.equal(kg.cpu(), rk) and torch.equal(vg.cpu(), rv)
    kg, vg = cache.gather_pages(mgr.block_tables[0, :2], with_v=False)
    assert vg is None and torch.equal(kg.cpu(), ref.gather([0, 1])[0])
    assert int(cache.dev_error.item()) == 0


@pytest.mark.gpu
def test_gpu_pool_exhaustion_sets_error_and_raises(cuda):
    """A free list shorter than the appends need: the append kernel records
    CVSA_DEV_ERR_POOL (no write, the context does not grow) and
    PagedKVCache.check() raises AssertionError as the reference's allocator
    asserts (kv_cache.py:55-56). The pool itself is larger than the free
    list, so a missed check would still write allocated memory."""
    from cvsa import _lib
    from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
    cache = PagedKVCache(8, 16, 2, 64, dtype=torch.bfloat16, device="cuda")
    # only 3 blocks on the free list of an 8-block pool
    cache.free_list = cache.free_list[:3].clone()
    cache._total_blocks = 3
    mgr = SequenceKVManager(cache, 2, 128)
    k = torch.randn(2, 2, 64, device=cuda, dtype=torch.bfloat16)
    mgr.append_batch(k, k)                       # 2 blocks
    for _ in range(15):
        mgr.append_batch(k, k)                   # pages fill, no new block
    mgr.append_batch(k, k)                       # both need a page: 1 block left
    torch.cuda.synchronize()
    assert int(cache.dev_error.item()) & _lib.DEV_ERR_POOL
    assert sorted(mgr.context_lens.tolist()) == [16, 17]
    with pytest.raises(AssertionError):
        cache.check()


@pytest.mark.gpu
def test_gpu_table_full_sets_error(cuda):
    """Appending past the block table width records CVSA_DEV_ERR_TABLE_FULL."""
    from cvsa import _lib
    from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
    cache = PagedKVCache(8, 16, 1, 64, dtype=torch.bfloat16, device="cuda")
    mgr = SequenceKVManager(cache, 1, 16)        # one page per sequence
    k = torch.randn(1, 1, 64, device=cuda, dtype=torch.bfloat16)
    for _ in range(17):
        mgr.append_batch(k, k)
    torch.cuda.synchronize()
    assert int(cache.dev_error.item()) & _lib.DEV_ERR_TABLE_FULL
    assert int(mgr.context_lens[0]) == 16
    with pytest.raises(ValueError):
        cache.check()
