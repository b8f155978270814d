"""Paged KV cache (drop-in for cvsa/runtime/kv_cache.py).

Layout is the reference's [num_blocks, block_size, num_kv_heads, head_dim]
(kv_cache.py:24-50). Allocation generalises the reference's bump allocator
(kv_cache.py:53-62) to a device-resident free list: blocks are handed out in
free-list order by an atomically advanced head, so a shuffled free list gives
a fragmented pool. Decode-time appends run on the GPU for the whole batch in
one launch (cvsa_paged_append) instead of the reference's per-sequence Python
loop with two `.item()` syncs each (kv_cache.py:133-150).
"""

from dataclasses import dataclass
from typing import Optional

import torch

from cvsa import _lib


@dataclass
class CacheConfig:
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    device: torch.device


class PagedKVCache:
    """Paged KV pool with a device free list."""

    def __init__(self, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.bfloat16, device: str = "cuda",
                 free_list: Optional[torch.Tensor] = None):
        self.config = CacheConfig(num_blocks=num_blocks, block_size=block_size,
                                  num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=dtype,
                                  device=torch.device(device))
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.k_cache = torch.zeros(num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype,
                                   device=device)
        self.v_cache = torch.zeros(num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype,
                                   device=device)
        if free_list is None:
            free_list = torch.arange(num_blocks, dtype=torch.int32)
        if free_list.numel() != num_blocks:
            raise ValueError("free_list must list every block once")
        self.free_list = free_list.to(device=device, dtype=torch.int32).contiguous()
        self.free_head = torch.zeros((1,), dtype=torch.int32, device=device)
        self.dev_error = torch.zeros((1,), dtype=torch.int32, device=device)
        self._total_blocks = num_blocks

    @property
    def _next_free(self) -> int:
        return int(self.free_head.item())

    def allocate_blocks(self, n: int) -> torch.Tensor:
        """Pop n blocks from the free list (host-synchronous, like the reference)."""
        head = int(self.free_head.item())
        assert head + n <= self._total_blocks, \
            f"Out of blocks: need {n}, have {self._total_blocks - head}"
        ids = self.free_list[head:head + n].clone()
        self.free_head += n
        return ids

    def write_kv(self, block_id: int, token_offset: int, k: torch.Tensor, v: torch.Tensor):
        """k, v: [num_kv_heads, head_dim] (kv_cache.py:64-71)."""
        self.k_cache[block_id, token_offset] = k
        self.v_cache[block_id, token_offset] = v

    def write_kv_block(self, block_id: int, k_block: torch.Tensor, v_block: torch.Tensor,
                       n_tokens: int):
        """k_block, v_block: [n_tokens, num_kv_heads, head_dim] (kv_cache.py:73-80)."""
        self.k_cache[block_id, :n_tokens] = k_block[:n_tokens]
        self.v_cache[block_id, :n_tokens] = v_block[:n_tokens]

    def gather_pages(self, block_ids: torch.Tensor, with_v: bool = True):
        """Dense [n_pages * block_size, H_kv, D] copies of the given blocks (GPU gather)."""
        n = block_ids.numel()
        rows = block_ids.to(torch.int32).contiguous()
        k_out = torch.empty((n * self.block_size, self.num_kv_heads, self.head_dim),
                            dtype=self.k_cache.dtype, device=self.k_cache.device)
        v_out = torch.empty_like(k_out) if with_v else None
        lib = _lib.load()
        _lib.check(lib.cvsa_paged_gather(_lib.kv_desc(self.k_cache, self.v_cache),
                                         rows.data_ptr(), n, k_out.data_ptr(), _lib.ptr(v_out),
                                         self.dev_error.data_ptr(),
                                         _lib.stream_ptr(self.k_cache.device)),
                   "cvsa_paged_gather")
        return k_out, v_out

    def check(self):
        """Raise for device-side errors recorded so far (synchronises)."""
        err = int(self.dev_error.item())
        if err & _lib.DEV_ERR_POOL:
            raise AssertionError("Out of blocks: the page pool is exhausted")
        if err & _lib.DEV_ERR_TABLE_FULL:
            raise ValueError("a sequence grew past its block table")
        if err:
            raise RuntimeError(f"paged KV device error bits {err:#x}")

    def reset(self):
        """Free all blocks (does not zero memory)."""
        self.free_head.zero_()
        self.dev_error.zero_()


class SequenceKVManager:
    """Block tables and context lengths of a batch (kv_cache.py:87-150)."""

    def __init__(self, cache: PagedKVCache, batch_size: int, max_context_len: int):
        self.cache = cache
        self.batch_size = batch_size
        self.block_size = cache.block_size
        self.max_pages = (max_context_len + cache.block_size - 1) // cache.block_size
        dev = cache.config.device
        self.block_tables = torch.zeros(batch_size, self.max_pages, dtype=torch.int32, device=dev)
        self.context_lens = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.pages_allocated = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self._seq_ids = torch.arange(batch_size, dtype=torch.int32, device=dev)

    @property
    def _pages_allocated(self):
        return self.pages_allocated.tolist()

    def prefill_kv(self, seq_idx: int, k_all: torch.Tensor, v_all: torch.Tensor):
        """Store prefill K/V [seq_len, num_kv_heads, head_dim] for one sequence."""
        seq_len = k_all.shape[0]
        n_pages = (seq_len + self.block_size - 1) // self.block_size
        if n_pages > self.max_pages:
            raise ValueError(f"prefill of {seq_len} tokens exceeds the block table")
        block_ids = self.cache.allocate_blocks(n_pages)
        self.block_tables[seq_idx, :n_pages] = block_ids
        pad = n_pages * self.block_size - seq_len
        kk, vv = k_all, v_all
        if pad:
            z = torch.zeros((pad,) + tuple(k_all.shape[1:]), dtype=k_all.dtype,
                            device=k_all.device)
            kk = torch.cat([k_all, z])
            vv = torch.cat([v_all, z])
        shp = (n_pages, self.block_size) + tuple(k_all.shape[1:])
        idx = block_ids.long()
        self.cache.k_cache.index_copy_(0, idx, kk.view(shp).to(self.cache.k_cache.dtype))
        self.cache.v_cache.index_copy_(0, idx, vv.view(shp).to(self.cache.v_cache.dtype))
        self.context_lens[seq_idx] = seq_len
        self.pages_allocated[seq_idx] = n_pages

    def append_token_kv(self, seq_idx: int, k: torch.Tensor, v: torch.Tensor):
        """Append one decode token's K/V [num_kv_heads, head_dim] to one sequence."""
        self._append(k.unsqueeze(0), v.unsqueeze(0), self._seq_ids[seq_idx:seq_idx + 1])

    def append_batch(self, k: torch.Tensor, v: torch.Tensor,
                     seq_ids: Optional[torch.Tensor] = None):
        """Append one token per sequence: k, v [n, num_kv_heads, head_dim], one launch."""
        ids = self._seq_ids[:k.shape[0]] if seq_ids is None else seq_ids.to(torch.int32)
        self._append(k, v, ids)

    def _append(self, k, v, ids):
        c = self.cache
        _lib.require_cuda(k, v, c.k_cache)
        k = k.to(c.k_cache.dtype).contiguous()
        v = v.to(c.v_cache.dtype).contiguous()
        lib = _lib.load()
        _lib.check(lib.cvsa_paged_append(
            _lib.kv_desc(c.k_cache, c.v_cache), k.data_ptr(), v.data_ptr(), k.shape[0],
            ids.contiguous().data_ptr(), self.block_tables.data_ptr(), self.max_pages,
            self.context_lens.data_ptr(), self.pages_allocated.data_ptr(), c.free_list.data_ptr(),
            c.free_list.numel(), c.free_head.data_ptr(), c.dev_error.data_ptr(),
            _lib.stream_ptr(c.k_cache.device)), "cvsa_paged_append")
