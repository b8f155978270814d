"""Page scoring: max over tokens of (mean-pooled GQA q) . k, times D^-0.5.

Drop-in for cvsa/kernels/page_scores.py:77-119 (`triton_score_pages`); the
kernel is csrc/score.cu behind cvsa_score_pages. `quest_page_scores` is the
Quest sketch ranking of cvsa/backend.py:572-620 (csrc/quest.cu behind
cvsa_quest_scores).
"""

import torch

from cvsa import _lib


def score_pages(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                context_lens: torch.Tensor, num_kv_heads: int, num_q_per_kv: int,
                block_size: int, out: torch.Tensor = None) -> torch.Tensor:
    """Returns page_scores [B, H_kv, max_pages] float32 (-inf past the context)."""
    dev = _lib.require_cuda(q, k_cache, block_tables, context_lens)
    B, Hq, D = q.shape
    if k_cache.shape[2] != num_kv_heads or Hq != num_kv_heads * num_q_per_kv:
        raise ValueError("head counts do not match q / k_cache")
    if k_cache.shape[1] != block_size:
        raise ValueError("block_size does not match k_cache")
    W = block_tables.shape[1]
    if out is None:
        out = torch.empty((B, num_kv_heads, W), dtype=torch.float32, device=dev)
    q = q.contiguous()
    kvd = _lib.kv_desc(k_cache, k_cache)
    qd = _lib.query_desc(q, block_tables, context_lens)
    lib = _lib.load()
    _lib.check(lib.cvsa_score_pages(qd, kvd, out.data_ptr(), _lib.stream_ptr(dev)),
               "cvsa_score_pages")
    return out


def quest_page_scores(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                      context_lens: torch.Tensor, num_kv_heads: int,
                      out: torch.Tensor = None, dev_error: torch.Tensor = None) -> torch.Tensor:
    """Quest ranking scores [B, H_kv, max_pages] float32 (cvsa/backend.py:572-620):
    per page and KV head, sum_d max(q_d kmin_d, q_d kmax_d) * D^-0.5 over the
    channel-wise key range of its valid tokens, q the group-mean query; -inf
    for pages without a valid token."""
    if q.dim() == 4:
        q = q.squeeze(1)
    dev = _lib.require_cuda(q, k_cache, block_tables, context_lens)
    B, Hq, D = q.shape
    if k_cache.shape[2] != num_kv_heads or Hq % num_kv_heads:
        raise ValueError("head counts do not match q / k_cache")
    W = block_tables.shape[1]
    if out is None:
        out = torch.empty((B, num_kv_heads, W), dtype=torch.float32, device=dev)
    q = q.contiguous()
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    cl = context_lens if context_lens.dtype == torch.int32 else context_lens.to(torch.int32)
    kvd = _lib.kv_desc(k_cache, k_cache)
    qd = _lib.query_desc(q, bt.contiguous(), cl.contiguous())
    lib = _lib.load()
    _lib.check(lib.cvsa_quest_scores(qd, kvd, out.data_ptr(), _lib.ptr(dev_error),
                                     _lib.stream_ptr(dev)), "cvsa_quest_scores")
    return out


# Reference name (cvsa/kernels/page_scores.py:77).
triton_score_pages = score_pages
