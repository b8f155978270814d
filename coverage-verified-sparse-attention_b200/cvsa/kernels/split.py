"""Kernels of the page-split step (csrc/split.cu, cvsa_split_*): a sequence's
pages spread over ranks, the selection and the coverage gates taken over the
ranks with two all-gathers per scoring or lazy-check step.

split_propose writes a rank's exchange row (its log-sum-exps and its best
`budget` candidates), split_gate turns the all-gathered rows into the same
global selection and gates on every rank (this rank's share of the selection
comes back), split_attend decodes the chosen selection -- or every valid page
of the rank for a rejected head -- into the partials that the second
all-gather carries to cvsa_rank_merge.
"""

from typing import Optional, Tuple

import torch

from cvsa import _lib


def row_floats(batch: int, num_kv_heads: int, max_sel: int) -> int:
    """Floats of one rank's exchange row: three log-sum-exps and max_sel
    candidate scores per (b, kv head)."""
    rows = batch * num_kv_heads
    return 3 * rows + rows * max_sel


def _desc(world, rank, batch, num_kv_heads, max_pages, block_size, budget, max_sel, sink, local,
          tau) -> _lib.SplitDesc:
    return _lib.SplitDesc(int(world), int(rank), int(batch), int(num_kv_heads), int(max_pages),
                          int(block_size), int(budget), int(max_sel), int(sink), int(local),
                          float(tau))


def split_propose(scores: torch.Tensor, context_lens: torch.Tensor, block_size: int,
                  cached: Optional[Tuple[torch.Tensor, torch.Tensor]], sink: int, local: int,
                  budget: int, max_sel: int, out: torch.Tensor) -> torch.Tensor:
    """Fill `out` (a float32 exchange row of row_floats(B, H, max_sel)) from
    this rank's page scores [B, H, W]; returns the candidates' local pages
    [B, H, max_sel] int32 (-1 unused)."""
    dev = _lib.require_cuda(scores, context_lens, out)
    B, H, W = scores.shape
    if out.dtype != torch.float32 or not out.is_contiguous() or \
            out.numel() < row_floats(B, H, max_sel):
        raise ValueError("out must be a contiguous float32 exchange row")
    sc = scores.float().contiguous()
    cl = context_lens.to(torch.int32).contiguous()
    ci = cn = None
    if cached is not None:
        ci = cached[0].to(torch.int32).reshape(B, H, max_sel).contiguous()
        cn = cached[1].to(torch.int32).reshape(B, H).contiguous()
    prop = torch.empty((B, H, max_sel), dtype=torch.int32, device=dev)
    sd = _desc(1, 0, B, H, W, block_size, budget, max_sel, sink, local, 1.0)
    lib = _lib.load()
    _lib.check(lib.cvsa_split_propose(sd, sc.data_ptr(), cl.data_ptr(), _lib.ptr(ci), _lib.ptr(cn),
                                      out.data_ptr(), prop.data_ptr(), _lib.stream_ptr(dev)),
               "cvsa_split_propose")
    return prop


def split_gate(parts: torch.Tensor, prop: torch.Tensor, context_lens: torch.Tensor,
               block_size: int, max_pages: int, rank: int, budget: int, max_sel: int, sink: int,
               local: int, tau: float, has_cache: bool, stats_mode: int, state: torch.Tensor,
               counters: Optional[torch.Tensor] = None, dev_error: Optional[torch.Tensor] = None):
    """(sel [B, H, max_sel] int32, n [B, H] int32, accept [B, H] uint8,
    bitmap [B, H, ceil(max_pages / 32)] int32) of this rank from the gathered
    exchange rows parts [world, stride]. state [4] int32 (zeroed once) keeps
    the decision word in state[3]; counters [6] int64 are accumulated."""
    dev = _lib.require_cuda(parts, prop, context_lens, state)
    if parts.dtype != torch.float32 or parts.dim() != 2 or not parts.is_contiguous():
        raise ValueError("parts must be a contiguous [world, stride] float32 tensor")
    if state.dtype != torch.int32 or state.numel() < 4 or not state.is_contiguous():
        raise ValueError("state must be 4 contiguous int32")
    B, H, _ = prop.shape
    world = parts.shape[0]
    cl = context_lens.to(torch.int32).contiguous()
    sel = torch.empty((B, H, max_sel), dtype=torch.int32, device=dev)
    n = torch.empty((B, H), dtype=torch.int32, device=dev)
    acc = torch.empty((B, H), dtype=torch.uint8, device=dev)
    bitmap = torch.empty((B, H, (max_pages + 31) // 32), dtype=torch.int32, device=dev)
    sd = _desc(world, rank, B, H, max_pages, block_size, budget, max_sel, sink, local, tau)
    lib = _lib.load()
    _lib.check(lib.cvsa_split_gate(sd, parts.data_ptr(), parts.shape[1], prop.data_ptr(),
                                   cl.data_ptr(), int(bool(has_cache)), int(stats_mode),
                                   sel.data_ptr(), n.data_ptr(), acc.data_ptr(), bitmap.data_ptr(),
                                   state.data_ptr(), _lib.ptr(counters), _lib.ptr(dev_error),
                                   _lib.stream_ptr(dev)), "cvsa_split_gate")
    return sel, n, acc, bitmap


def split_attend(q, k_cache, v_cache, block_tables, context_lens, num_kv_heads, num_q_per_kv,
                 block_size, cached, sel, n, decision, accept, bitmap, out):
    """Partials (o, m, l) into `out` (float32 views of [B, Hq, D], [B, Hq],
    [B, Hq]): the cached selection where decision[0] bit0 is set (decision
    may be None), else the new one, every valid page for a head whose new
    gate rejected; the new selection is copied into `cached` (idx, n) when
    decoded (cached may be None)."""
    dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, context_lens, sel, n, accept,
                            bitmap)
    B, Hq, D = q.shape
    if k_cache.shape[2] != num_kv_heads or Hq != num_kv_heads * num_q_per_kv:
        raise ValueError("head counts do not match q / k_cache")
    o, m, l = out
    for t, shape in ((o, (B, Hq, D)), (m, (B, Hq)), (l, (B, Hq))):
        if t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError("out must be contiguous float32 (o, m, l)")
    max_sel = sel.shape[-1]
    ci = cn = None
    if cached is not None:
        ci, cn = cached
        if ci.dtype != torch.int32 or not ci.is_contiguous() or cn.dtype != torch.int32 or \
                not cn.is_contiguous() or ci.shape[-1] != max_sel:
            raise ValueError("cached must be contiguous int32 (idx [B, H, max_sel], n [B, H])")
    q = q.contiguous()
    kvd = _lib.kv_desc(k_cache, v_cache)
    qd = _lib.query_desc(q, block_tables, context_lens)
    lib = _lib.load()
    nbytes = lib.cvsa_decode_workspace_size(qd, kvd, max_sel)
    ws = _lib.WORKSPACE.get(nbytes, dev, "decode")
    _lib.check(lib.cvsa_split_attend(qd, kvd, _lib.ptr(ci), _lib.ptr(cn), sel.data_ptr(),
                                     n.data_ptr(), max_sel, _lib.ptr(decision),
                                     accept.data_ptr(), bitmap.data_ptr(), o.data_ptr(),
                                     m.data_ptr(), l.data_ptr(), None, ws.data_ptr(), ws.numel(),
                                     _lib.stream_ptr(dev)), "cvsa_split_attend")
    return out
