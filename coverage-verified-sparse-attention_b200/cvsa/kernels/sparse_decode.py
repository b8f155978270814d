"""Sparse paged decode over selected pages (GQA-packed, split-K, TMA + mma).

Drop-in for cvsa/kernels/sparse_decode.py: `triton_sparse_decode` (:286-350),
`triton_sparse_decode_unnorm` (:537-573), `prepare_reuse_state` (:664-678) and
`triton_sparse_decode_reuse` (:681-721), backed by csrc/attend.cu through
cvsa_sparse_decode. The page list of every (b, kv head) is read once for all
its query heads, split across CTAs, and combined in-kernel by LSE.
"""

from typing import Tuple

import torch

from cvsa import _lib


def _decode(q, k_cache, v_cache, block_tables, page_indices, n_per_head, context_lens,
            num_kv_heads, num_q_per_kv, block_size, want_unnorm: bool, want_out: bool,
            out_dtype=None, unnorm_out=None):
    dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                            context_lens)
    B, Hq, D = q.shape
    if k_cache.shape[2] != num_kv_heads or Hq != num_kv_heads * num_q_per_kv:
        raise ValueError("head counts do not match q / k_cache")
    if k_cache.shape[1] != block_size:
        raise ValueError("block_size does not match k_cache")
    pi = page_indices.to(torch.int32).reshape(B, num_kv_heads, -1).contiguous()
    K = pi.shape[2]
    nph = n_per_head.to(torch.int32).reshape(B, num_kv_heads).contiguous()
    q = q.contiguous()
    kvd = _lib.kv_desc(k_cache, v_cache)
    qd = _lib.query_desc(q, block_tables, context_lens)
    lib = _lib.load()
    o = m = l = out = None
    if want_unnorm and unnorm_out is not None:
        o, m, l = unnorm_out
        for t, shape in ((o, (B, Hq, D)), (m, (B, Hq)), (l, (B, Hq))):
            if (t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous()
                    or t.device != dev):
                raise ValueError("unnorm_out must be contiguous float32 (o, m, l) tensors "
                                 "of shapes [B, Hq, D], [B, Hq], [B, Hq]")
    elif want_unnorm:
        o = torch.empty((B, Hq, D), dtype=torch.float32, device=dev)
        m = torch.empty((B, Hq), dtype=torch.float32, device=dev)
        l = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    odt = out_dtype or q.dtype
    if want_out:
        out = torch.empty((B, Hq, D), dtype=odt, device=dev)
    nbytes = lib.cvsa_decode_workspace_size(qd, kvd, max(K, 1))
    ws = _lib.WORKSPACE.get(nbytes, dev, "decode")
    _lib.check(lib.cvsa_sparse_decode(qd, kvd, pi.data_ptr(), max(K, 1), nph.data_ptr(),
                                      _lib.ptr(o), _lib.ptr(m), _lib.ptr(l), _lib.ptr(out),
                                      _lib.dtype_code(odt), ws.data_ptr(), ws.numel(),
                                      _lib.stream_ptr(dev)), "cvsa_sparse_decode")
    return o, m, l, out


def sparse_decode_unnorm(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                         context_lens, num_kv_heads, num_q_per_kv, block_size=64, out=None
                         ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(O_unnorm [B,H_q,D], M [B,H_q], L [B,H_q]) float32 over the first n_per_head pages.

    `out`, if given, is the (o, m, l) tensors to write (views into one
    exchange buffer, for instance)."""
    o, m, l, _ = _decode(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                         context_lens, num_kv_heads, num_q_per_kv, block_size, True, False,
                         unnorm_out=out)
    return o, m, l


def sparse_decode(q, k_cache, v_cache, block_tables, page_indices, n_per_head, context_lens,
                  num_kv_heads, num_q_per_kv, block_size=64) -> torch.Tensor:
    """Normalised output [B, H_q, D] in q's dtype."""
    _, _, _, out = _decode(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                           context_lens, num_kv_heads, num_q_per_kv, block_size, False, True)
    return out


def prepare_reuse_state(page_indices, n_per_head, num_kv_heads, B):
    """(pi_flat [B*H_kv, K] int32, nph_flat [B*H_kv] int32, K) for the reuse path.

    The CUDA kernel needs no power-of-two padding (the reference pads to
    next_pow2 at sparse_decode.py:669-677); the third element keeps the
    reference's tuple shape and is the list width.
    """
    K = page_indices.shape[2]
    pi_flat = page_indices.to(torch.int32).reshape(B * num_kv_heads, K).contiguous()
    nph_flat = n_per_head.to(torch.int32).reshape(B * num_kv_heads).contiguous()
    return pi_flat, nph_flat, K


def sparse_decode_reuse(q, k_cache, v_cache, block_tables, context_lens, pi_flat, nph_flat,
                        padded_max_selected, num_kv_heads, num_q_per_kv, block_size):
    """Normalised decode on a prepared selection (reuse steps)."""
    B = q.shape[0]
    pi = pi_flat.reshape(B, num_kv_heads, -1)
    nph = nph_flat.reshape(B, num_kv_heads)
    return sparse_decode(q, k_cache, v_cache, block_tables, pi, nph, context_lens,
                         num_kv_heads, num_q_per_kv, block_size)


def recover_merge(q, k_cache, v_cache, block_tables, page_indices, n_per_head, context_lens,
                  accept_mask, o_draft, m_draft, l_draft, num_kv_heads, num_q_per_kv,
                  block_size, output_dtype=None) -> torch.Tensor:
    """Fused exact recovery: complement attention for rejected heads + LSE merge.

    Equivalent to cvsa/backend.py:819-842 (triton_compute_complement, a decode
    over the complement, triton_lse_merge) in one kernel that skips selected
    pages through a bitmap instead of materialising the complement list.
    """
    dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                            context_lens, accept_mask, o_draft, m_draft, l_draft)
    B, Hq, D = q.shape
    pi = page_indices.to(torch.int32).reshape(B, num_kv_heads, -1).contiguous()
    K = pi.shape[2]
    nph = n_per_head.to(torch.int32).reshape(B, num_kv_heads).contiguous()
    am = accept_mask.to(torch.uint8).contiguous()
    q = q.contiguous()
    odt = output_dtype or q.dtype
    out = torch.empty((B, Hq, D), dtype=odt, device=dev)
    kvd = _lib.kv_desc(k_cache, v_cache)
    qd = _lib.query_desc(q, block_tables, context_lens)
    lib = _lib.load()
    nbytes = lib.cvsa_decode_workspace_size(qd, kvd, max(K, 1))
    ws = _lib.WORKSPACE.get(nbytes, dev, "decode")
    od, md, ld = (t.float().contiguous() for t in (o_draft, m_draft, l_draft))
    _lib.check(lib.cvsa_recover_merge(qd, kvd, pi.data_ptr(), max(K, 1), nph.data_ptr(),
                                      am.data_ptr(), od.data_ptr(), md.data_ptr(), ld.data_ptr(),
                                      out.data_ptr(), _lib.dtype_code(odt), ws.data_ptr(),
                                      ws.numel(), _lib.stream_ptr(dev)), "cvsa_recover_merge")
    return out


# Reference names.
triton_sparse_decode = sparse_decode
triton_sparse_decode_unnorm = sparse_decode_unnorm
triton_sparse_decode_reuse = sparse_decode_reuse
