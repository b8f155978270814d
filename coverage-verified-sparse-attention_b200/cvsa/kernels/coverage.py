"""Complement indices, coverage gate and LSE merge.

Drop-in for cvsa/kernels/coverage.py: `triton_compute_complement` (:99-150),
`triton_check_coverage` (:218-265) and `triton_lse_merge` (:329-367), backed
by csrc/select.cu and csrc/merge.cu.
"""

from typing import Tuple

import torch

from cvsa import _lib


def _n_valid_max(context_lens: torch.Tensor, block_size: int) -> int:
    # the reference also syncs here (coverage.py:121)
    return int(((int(context_lens.max().item()) + block_size - 1) // block_size))


def compute_complement(page_indices: torch.Tensor, n_per_head: torch.Tensor,
                       context_lens: torch.Tensor, block_size: int,
                       accept_mask: torch.Tensor = None,
                       max_comp: int = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Valid pages not selected, ascending; n = 0 for accepted heads.

    Returns (complement [B, H_kv, max_comp] int32, n_complement [B, H_kv] int32).
    max_comp defaults to the largest n_valid (one host sync, as the reference).
    """
    dev = _lib.require_cuda(page_indices, n_per_head, context_lens, accept_mask)
    B, H, K = page_indices.shape
    if max_comp is None:
        max_comp = max(_n_valid_max(context_lens, block_size), 1)
    pi = page_indices.to(torch.int32).contiguous()
    nph = n_per_head.to(torch.int32).contiguous()
    am = None if accept_mask is None else accept_mask.to(torch.uint8).contiguous()
    comp = torch.zeros((B, H, max_comp), dtype=torch.int32, device=dev)
    n_comp = torch.zeros((B, H), dtype=torch.int32, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_compute_complement(pi.data_ptr(), K, nph.data_ptr(),
                                           context_lens.data_ptr(), B, H, block_size,
                                           _lib.ptr(am), comp.data_ptr(), max_comp,
                                           n_comp.data_ptr(), _lib.stream_ptr(dev)),
               "cvsa_compute_complement")
    return comp, n_comp


def check_coverage(page_scores: torch.Tensor, selected_indices: torch.Tensor,
                   n_per_head: torch.Tensor, tau: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """(accept_mask [B, H_kv] bool, coverage [B, H_kv] float32)."""
    dev = _lib.require_cuda(page_scores, selected_indices, n_per_head)
    B, H, W = page_scores.shape
    K = selected_indices.shape[2]
    ps = page_scores.float().contiguous()
    si = selected_indices.to(torch.int32).contiguous()
    nph = n_per_head.to(torch.int32).contiguous()
    acc = torch.empty((B, H), dtype=torch.uint8, device=dev)
    cov = torch.empty((B, H), dtype=torch.float32, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_check_coverage(ps.data_ptr(), B, H, W, si.data_ptr(), K, nph.data_ptr(),
                                       float(tau), acc.data_ptr(), cov.data_ptr(),
                                       _lib.stream_ptr(dev)), "cvsa_check_coverage")
    return acc.bool(), cov


def lse_merge(o_draft, m_draft, l_draft, o_comp, m_comp, l_comp, accept_mask,
              num_kv_heads: int, num_q_per_kv: int,
              output_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Selective LSE merge -> [B, H_q, D] in output_dtype."""
    dev = _lib.require_cuda(o_draft, m_draft, l_draft, o_comp, m_comp, l_comp, accept_mask)
    B, Hq, D = o_draft.shape
    args = [t.float().contiguous() for t in (o_draft, m_draft, l_draft, o_comp, m_comp, l_comp)]
    am = accept_mask.to(torch.uint8).contiguous()
    out = torch.empty((B, Hq, D), dtype=output_dtype, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_lse_merge(*[a.data_ptr() for a in args], am.data_ptr(), B, num_kv_heads,
                                  num_q_per_kv, D, out.data_ptr(), _lib.dtype_code(output_dtype),
                                  _lib.stream_ptr(dev)), "cvsa_lse_merge")
    return out


def rank_merge(parts: torch.Tensor, batch: int, num_kv_heads: int, num_q_per_kv: int,
               head_dim: int, out: torch.Tensor, need: torch.Tensor = None) -> torch.Tensor:
    """Fixed-order merge over ranks of page-split partials (cvsa_rank_merge).

    parts [world, stride] float32: rank r's row holds o_unnorm [B, Hq, D],
    m [B, Hq] and l [B, Hq] in that order. Writes the normalised output into
    `out` [B, Hq, D] (its dtype); with `need` [B, H_kv] only the query heads
    of KV heads where need is true. Returns `out`."""
    dev = _lib.require_cuda(parts, out)
    if parts.dtype != torch.float32 or parts.dim() != 2 or not parts.is_contiguous():
        raise ValueError("parts must be a contiguous [world, stride] float32 tensor")
    if not out.is_contiguous() or tuple(out.shape) != (batch, num_kv_heads * num_q_per_kv,
                                                       head_dim):
        raise ValueError("out must be a contiguous [B, Hq, D] tensor")
    nd = None
    if need is not None:
        nd = need.to(torch.uint8).contiguous()
        if nd.numel() != batch * num_kv_heads or nd.device != dev:
            raise ValueError("need must be [B, H_kv] on the device of parts")
    lib = _lib.load()
    _lib.check(lib.cvsa_rank_merge(parts.data_ptr(), parts.shape[0], parts.shape[1], batch,
                                   num_kv_heads, num_q_per_kv, head_dim, _lib.ptr(nd),
                                   out.data_ptr(), _lib.dtype_code(out.dtype),
                                   _lib.stream_ptr(dev)), "cvsa_rank_merge")
    return out


def page_lse(page_scores: torch.Tensor, page_indices: torch.Tensor, n_per_head: torch.Tensor):
    """(lse_all, lse_sel) [B, H_kv] float32 of page scores [B, H_kv, W]: the
    log-sum-exp over every page and over the first n_per_head selected pages
    (cvsa_page_lse; -inf when empty)."""
    dev = _lib.require_cuda(page_scores, page_indices, n_per_head)
    B, H, W = page_scores.shape
    ps = page_scores.float().contiguous()
    pi = page_indices.to(torch.int32).reshape(B, H, -1).contiguous()
    nph = n_per_head.to(torch.int32).reshape(B, H).contiguous()
    if W == 0:
        # no page: both log-sum-exps are over an empty set (no launch)
        lse_all = torch.full((B, H), float("-inf"), dtype=torch.float32, device=dev)
        return lse_all, lse_all.clone()
    if pi.shape[2] == 0:
        # no selection slot: every row's selection is empty
        pi = torch.zeros((B, H, 1), dtype=torch.int32, device=dev)
        nph = torch.zeros((B, H), dtype=torch.int32, device=dev)
    lse_all = torch.empty((B, H), dtype=torch.float32, device=dev)
    lse_sel = torch.empty((B, H), dtype=torch.float32, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_page_lse(ps.data_ptr(), B * H, W, pi.data_ptr(), pi.shape[2],
                                 nph.data_ptr(), lse_all.data_ptr(), lse_sel.data_ptr(),
                                 _lib.stream_ptr(dev)), "cvsa_page_lse")
    return lse_all, lse_sel


def rank_accept(parts: torch.Tensor, off_all: int, off_sel: int, rows: int,
                tau: float) -> torch.Tensor:
    """accept [rows] bool of the coverage gate over ranks (cvsa_rank_accept):
    parts [world, stride] float32 holds each rank's lse_all at off_all and
    lse_sel at off_sel."""
    dev = _lib.require_cuda(parts)
    if parts.dtype != torch.float32 or parts.dim() != 2 or not parts.is_contiguous():
        raise ValueError("parts must be a contiguous [world, stride] float32 tensor")
    acc = torch.empty(rows, dtype=torch.uint8, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_rank_accept(parts.data_ptr(), parts.shape[0], parts.shape[1], off_all,
                                    off_sel, rows, float(tau), acc.data_ptr(),
                                    _lib.stream_ptr(dev)), "cvsa_rank_accept")
    return acc.bool()


# Reference names.
triton_compute_complement = compute_complement
triton_check_coverage = check_coverage
triton_lse_merge = lse_merge
