"""CPU oracle for the CVSA decode step -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline arm of `bench.py`
may import this module, and only as the checker / the timed CPU baseline. The
product path (the `cvsa` package over `libcvsa_b200.so`) never calls it.

This is a pure-PyTorch (CPU) restatement of the reference's algorithm for the
hot path, following DJ-Melvin/coverage-verified-sparse-attention op by op:

  scoring     cvsa/kernels/page_scores.py:90-119 (q_rep mean-pool in q dtype)
              and :41-74 (max over valid tokens of q_rep.k, times D^-0.5)
  selection   cvsa/backend.py:690 (budget) and :737-747 (top-k, n_per_head)
  decode      cvsa/kernels/sparse_decode.py:424-500 (online softmax, o/m/l)
              and :15-132 (normalised variant, clamp l >= 1e-6)
  coverage    cvsa/kernels/coverage.py:160-215 (lse_sel - lse_all, +1e-30)
  complement  cvsa/complement.py:11-69
  merge       cvsa/lse_merge.py:11-54 and cvsa/kernels/coverage.py:274-326
  schedule    cvsa/backend.py:313-366, 392-465, 683-864, 866-881

Precision: `precise=True` (the default, used by the parity tests) computes the
q.k dot products in float64 and rounds each to float32 once, so the oracle's
page scores are the correctly rounded values of the reference's fp32 formula;
`precise=False` keeps the reference's own fp32 arithmetic and is what the
CPU-baseline arm of bench.py times.

Two documented extensions over the reference (both off by default, so the
default behaviour is the reference's):
  * forced pages: the first `sink_pages` and last `local_pages` valid pages of
    every sequence are always selected, and the top-k budget counts only the
    remaining pages;
  * a stable tie rule: top-k orders pages by (score descending, page index
    ascending), where the reference's `torch.topk(sorted=False)` leaves ties
    unspecified. Selections are reported in ascending page order.
One further definition: a sequence with context length 0 has no valid pages
(the reference's formula counts one empty page and its decode returns NaN).

Parity of this oracle is pinned against the reference itself: the fixtures in
tests/golden/ were produced by running the reference's own Triton kernels and
`CVSABackend` under TRITON_INTERPRET=1 (tests/golden/make_golden.py).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch

NEG_INF = float("-inf")


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def n_valid_pages(context_lens: torch.Tensor, block_size: int) -> torch.Tensor:
    """Valid pages per sequence, ceil(ctx / block_size).

    cvsa/backend.py:687 computes ((ctx - 1) / bs).long() + 1, which equals
    ceil(ctx / bs) for ctx >= 1; here ctx = 0 gives 0 pages.
    """
    cl = context_lens.to(torch.int64)
    return (cl + block_size - 1) // block_size


def budget_for(table_width: int, budget_pct: float) -> int:
    """cvsa/backend.py:690 -- budget uses the block-table WIDTH, not n_valid."""
    return max(3, int(table_width * budget_pct))


def q_representative(q: torch.Tensor, num_kv_heads: int) -> torch.Tensor:
    """Mean-pooled GQA query per KV head, rounded to q's dtype.

    cvsa/kernels/page_scores.py:94-95: q.view(B, Hkv, G, D).mean(2) in q's
    dtype. On CUDA torch reduces in fp32 and multiplies by float(1/G) before
    the cast back; that is restated here (sum in order g = 0..G-1).
    """
    B, Hq, D = q.shape
    G = Hq // num_kv_heads
    qf = q.float().view(B, num_kv_heads, G, D)
    acc = qf[:, :, 0].clone()
    for g in range(1, G):
        acc = acc + qf[:, :, g]
    rep = acc * torch.tensor(1.0 / G, dtype=torch.float32)
    return rep.to(q.dtype)


def _gather_pages(cache: torch.Tensor, block_tables: torch.Tensor, b: int,
                  n_pages: int) -> torch.Tensor:
    """[n_pages, bs, Hkv, D] view of sequence b's first n_pages pages."""
    blocks = block_tables[b, :n_pages].long()
    return cache.index_select(0, blocks)


def _dot_f32(a: torch.Tensor, b: torch.Tensor, precise: bool) -> torch.Tensor:
    """fp32 dot products along the last dim (einsum '...d,...d')."""
    if precise:
        return (a.double() * b.double()).sum(-1).float()
    return (a.float() * b.float()).sum(-1)


# --------------------------------------------------------------------------
# a7: page scoring
# --------------------------------------------------------------------------

def score_pages(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                context_lens: torch.Tensor, num_kv_heads: int, num_q_per_kv: int,
                block_size: int, precise: bool = True) -> torch.Tensor:
    """score[b,h,p] = max over valid tokens t of (q_rep[b,h] . K[blk(b,p),t,h]) * D^-0.5.

    cvsa/kernels/page_scores.py:41-74. Pages at or beyond the context and
    padding tokens of the last page score -inf. Returns [B, Hkv, W] float32.
    """
    B, Hq, D = q.shape
    W = block_tables.shape[1]
    scale = torch.tensor(D ** -0.5, dtype=torch.float32)
    q_rep = q_representative(q, num_kv_heads).float()          # [B, Hkv, D]
    nv = n_valid_pages(context_lens, block_size)
    out = torch.full((B, num_kv_heads, W), NEG_INF, dtype=torch.float32)
    for b in range(B):
        n = int(nv[b])
        if n == 0:
            continue
        kp = _gather_pages(k_cache, block_tables, b, n)        # [n, bs, Hkv, D]
        dots = _dot_f32(kp, q_rep[b].view(1, 1, num_kv_heads, D), precise)  # [n, bs, Hkv]
        tok = torch.arange(n).view(n, 1) * block_size + torch.arange(block_size).view(1, -1)
        valid = (tok < int(context_lens[b])).unsqueeze(-1)
        dots = torch.where(valid, dots, torch.tensor(NEG_INF))
        # (dot * scale) then max == max(dot) * scale: fp32 rounding is monotone.
        page_max = (dots * scale).amax(dim=1)                  # [n, Hkv]
        out[b, :, :n] = page_max.t()
    return out


# --------------------------------------------------------------------------
# a8: top-k selection (+ forced pages, stable tie rule)
# --------------------------------------------------------------------------

def select_pages(page_scores: torch.Tensor, context_lens: torch.Tensor, block_size: int,
                 budget: int, sink_pages: int = 0, local_pages: int = 0
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per (b, h): forced pages, plus the top `budget` other valid pages.

    Follows cvsa/backend.py:737-747 (top `budget` by score, n_per_head =
    min(budget, n_valid)) with the stable order (score desc, index asc) and the
    forced-page extension. Returns (page_indices [B,Hkv,max_sel] int32 in
    ascending page order, padded with 0, n_per_head [B,Hkv] int32), where
    max_sel = budget + sink_pages + local_pages.
    """
    B, H, W = page_scores.shape
    max_sel = budget + sink_pages + local_pages
    idx_out = torch.zeros((B, H, max_sel), dtype=torch.int32)
    n_out = torch.zeros((B, H), dtype=torch.int32)
    nv = n_valid_pages(context_lens, block_size)
    for b in range(B):
        n = int(nv[b])
        forced = set(range(min(sink_pages, n))) | set(range(max(0, n - local_pages), n))
        cand = [p for p in range(n) if p not in forced]
        for h in range(H):
            s = page_scores[b, h].tolist()
            # stable: score descending, then page index ascending
            ranked = sorted(cand, key=lambda p: (-s[p], p))
            chosen = sorted(forced | set(ranked[:budget]))
            n_out[b, h] = len(chosen)
            if chosen:
                idx_out[b, h, :len(chosen)] = torch.tensor(chosen, dtype=torch.int32)
    return idx_out, n_out


def topk_indices_stable(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k along the last dim ordered by (score desc, index asc); ascending output."""
    *lead, W = scores.shape
    flat = scores.reshape(-1, W)
    out = torch.zeros((flat.shape[0], k), dtype=torch.int32)
    for r in range(flat.shape[0]):
        s = flat[r].tolist()
        ranked = sorted(range(W), key=lambda p: (-s[p], p))[:k]
        out[r] = torch.tensor(sorted(ranked), dtype=torch.int32)
    return out.reshape(*lead, k)


# --------------------------------------------------------------------------
# a11: coverage gate
# --------------------------------------------------------------------------

def check_coverage(page_scores: torch.Tensor, selected: torch.Tensor,
                   n_per_head: torch.Tensor, tau: float, precise: bool = True
                   ) -> Tuple[torch.Tensor, torch.Tensor]:
    """cov = exp(lse(scores[sel[:n]]) - lse(scores[all])), accept = cov >= tau.

    cvsa/kernels/coverage.py:179-215: max starts at -1e20, -1e20 fills for
    padding, log(sum + 1e-30); tau is compared in fp32. Returns (accept bool
    [B,H], coverage float32 [B,H]).
    """
    B, H, W = page_scores.shape
    dt = torch.float64 if precise else torch.float32
    s = page_scores.to(dt)
    m_all = torch.clamp(s.amax(-1), min=-1e20)
    sum_all = torch.exp(s - m_all.unsqueeze(-1)).sum(-1)
    lse_all = m_all + torch.log(sum_all + 1e-30)
    K = selected.shape[-1]
    rng = torch.arange(K).view(1, 1, K)
    mask = rng < n_per_head.unsqueeze(-1).long()
    safe = torch.where(mask, selected.long(), torch.zeros_like(selected.long()))
    sel = torch.gather(s, 2, safe)
    sel = torch.where(mask, sel, torch.tensor(-1e20, dtype=dt))
    m_sel = sel.amax(-1)
    sum_sel = torch.where(mask, torch.exp(sel - m_sel.unsqueeze(-1)), torch.zeros((), dtype=dt)).sum(-1)
    lse_sel = m_sel + torch.log(sum_sel + 1e-30)
    cov = torch.exp(lse_sel - lse_all).float()
    accept = cov >= torch.tensor(tau, dtype=torch.float32)
    return accept, cov


# --------------------------------------------------------------------------
# a9 / a10: sparse paged decode
# --------------------------------------------------------------------------

def sparse_decode_unnorm(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         block_tables: torch.Tensor, page_indices: torch.Tensor,
                         n_per_head: torch.Tensor, context_lens: torch.Tensor,
                         num_kv_heads: int, num_q_per_kv: int, block_size: int,
                         precise: bool = True
                         ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(o_unnorm [B,Hq,D], m [B,Hq], l [B,Hq]) over the first n_per_head pages.

    cvsa/kernels/sparse_decode.py:454-500: s = (q . k) * D^-0.5 in fp32, tokens
    t < min(bs, ctx - page_start) only; m = max s, l = sum exp(s - m),
    o = sum exp(s - m) v. The result does not depend on page order. A head with
    no valid token returns (0, -inf, 0) (the reference returns NaN there).
    """
    B, Hq, D = q.shape
    G = num_q_per_kv
    scale = torch.tensor(D ** -0.5, dtype=torch.float32)
    acc = torch.float64 if precise else torch.float32
    o = torch.zeros((B, Hq, D), dtype=torch.float32)
    m = torch.full((B, Hq), NEG_INF, dtype=torch.float32)
    l = torch.zeros((B, Hq), dtype=torch.float32)
    for b in range(B):
        ctx = int(context_lens[b])
        for h in range(num_kv_heads):
            n = int(n_per_head[b, h])
            if n <= 0:
                continue
            pages = page_indices[b, h, :n].long()
            blocks = block_tables[b, pages].long()
            kp = k_cache.index_select(0, blocks)[:, :, h]         # [n, bs, D]
            vp = v_cache.index_select(0, blocks)[:, :, h]
            tok = pages.view(-1, 1) * block_size + torch.arange(block_size).view(1, -1)
            valid = (tok < ctx).reshape(-1)
            kt = kp.reshape(-1, D)[valid]
            vt = vp.reshape(-1, D)[valid]
            if kt.shape[0] == 0:
                continue
            qg = q[b, h * G:(h + 1) * G]                           # [G, D]
            dots = _dot_f32(qg.unsqueeze(1), kt.unsqueeze(0), precise)   # [G, T]
            s = dots * scale                                        # fp32, as the reference
            mg = s.amax(-1)                                         # [G]
            p = torch.exp((s.to(acc) - mg.to(acc).unsqueeze(-1)))
            lg = p.sum(-1)
            og = p @ vt.to(acc)
            o[b, h * G:(h + 1) * G] = og.float()
            m[b, h * G:(h + 1) * G] = mg
            l[b, h * G:(h + 1) * G] = lg.float()
    return o, m, l


def sparse_decode(q, k_cache, v_cache, block_tables, page_indices, n_per_head,
                  context_lens, num_kv_heads, num_q_per_kv, block_size,
                  precise: bool = True) -> torch.Tensor:
    """Normalised decode in q's dtype: o / max(l, 1e-6) (sparse_decode.py:126-132)."""
    o, m, l = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, page_indices,
                                   n_per_head, context_lens, num_kv_heads,
                                   num_q_per_kv, block_size, precise)
    return (o / l.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)


def dense_decode(q, k_cache, v_cache, block_tables, context_lens, num_kv_heads,
                 num_q_per_kv, block_size, precise: bool = True) -> torch.Tensor:
    """Attention over every valid page (cvsa/runtime/dense.py:40-68 semantics)."""
    B = q.shape[0]
    W = block_tables.shape[1]
    nv = n_valid_pages(context_lens, block_size)
    idx = torch.arange(W, dtype=torch.int32).view(1, 1, W).expand(B, num_kv_heads, W).contiguous()
    nph = nv.view(B, 1).expand(B, num_kv_heads).to(torch.int32).contiguous()
    return sparse_decode(q, k_cache, v_cache, block_tables, idx, nph, context_lens,
                         num_kv_heads, num_q_per_kv, block_size, precise)


# --------------------------------------------------------------------------
# a12 / a13: complement
# --------------------------------------------------------------------------

def compute_complement_pages(page_indices: torch.Tensor, n_per_head: torch.Tensor,
                             context_lens: torch.Tensor, block_size: int,
                             accept_mask: Optional[torch.Tensor] = None
                             ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Valid pages not selected, ascending; n = 0 for accepted heads.

    cvsa/complement.py:27-69 (mask, then compaction). The reference packs the
    list with a descending float sort, so its order is unspecified; compare as
    sets. Returns (indices [B,H,max_comp] int32, n [B,H] int32), with a
    [B,H,1] zero tensor when no head has a complement (complement.py:60-63).
    """
    B, H, K = page_indices.shape
    nv = n_valid_pages(context_lens, block_size)
    P = max(int(nv.max()) if B else 0, 1)
    # The reference scatters a bool mask (complement.py:42-43); a padding entry
    # that repeats a selected index can then overwrite True with False. The
    # intended set semantics (an OR over the first n_per_head entries) is used.
    sel = torch.zeros((B, H, P), dtype=torch.bool)
    for b in range(B):
        for h in range(H):
            for i in range(int(n_per_head[b, h])):
                p = int(page_indices[b, h, i])
                if 0 <= p < P:
                    sel[b, h, p] = True
    valid = torch.arange(P).view(1, 1, P) < nv.view(B, 1, 1)
    comp = valid & ~sel
    n_comp = comp.sum(-1).to(torch.int32)
    if accept_mask is not None:
        n_comp = torch.where(accept_mask, torch.zeros_like(n_comp), n_comp)
    max_c = int(n_comp.max()) if n_comp.numel() else 0
    if max_c == 0:
        return torch.zeros((B, H, 1), dtype=torch.int32), n_comp
    out = torch.zeros((B, H, max_c), dtype=torch.int32)
    for b in range(B):
        for h in range(H):
            c = int(n_comp[b, h])
            if c:
                out[b, h, :c] = torch.nonzero(comp[b, h]).view(-1)[:c].to(torch.int32)
    return out, n_comp


# --------------------------------------------------------------------------
# a14 / a15: selective LSE merge
# --------------------------------------------------------------------------

def selective_lse_merge(o_draft, m_draft, l_draft, o_comp, m_comp, l_comp,
                        accept_mask, num_q_per_kv, output_dtype=torch.bfloat16):
    """cvsa/lse_merge.py:11-54 restated (accept -> o_d / max(l_d, 1e-6); reject ->
    LSE merge of draft and complement, divided by max(l, 1e-6))."""
    accept_q = accept_mask.repeat_interleave(num_q_per_kv, dim=1)
    o_acc = o_draft / l_draft.clamp(min=1e-6).unsqueeze(-1)
    m_all = torch.maximum(m_draft, m_comp)
    # exp(-inf - (-inf)) would be NaN; a side with m = -inf has no mass.
    sd = torch.where(torch.isinf(m_draft) & (m_draft < 0), torch.zeros_like(m_draft),
                     (m_draft - m_all).exp())
    sc = torch.where(torch.isinf(m_comp) & (m_comp < 0), torch.zeros_like(m_comp),
                     (m_comp - m_all).exp())
    l_m = l_draft * sd + l_comp * sc
    o_m = o_draft * sd.unsqueeze(-1) + o_comp * sc.unsqueeze(-1)
    o_rej = o_m / l_m.clamp(min=1e-6).unsqueeze(-1)
    out = torch.where(accept_q.unsqueeze(-1), o_acc, o_rej)
    return out.to(output_dtype)


# --------------------------------------------------------------------------
# a3: one full scoring step; a4: reuse step
# --------------------------------------------------------------------------

def approx_budget(table_width: int, budget: int, approx_recovery_pct: float) -> int:
    """Pages of the expanded selection (backend.py:782-783)."""
    return min(max(budget + 1, int(table_width * approx_recovery_pct)), table_width)


def scoring_step(q, k_cache, v_cache, block_tables, context_lens, num_kv_heads,
                 num_q_per_kv, block_size, budget_pct, tau, sink_pages=0, local_pages=0,
                 page_scores=None, precise=True, approx_recovery_pct=None
                 ) -> Dict[str, torch.Tensor]:
    """cvsa/backend.py:683-864: exact recovery (complement + LSE merge), or
    with approx_recovery_pct the approximate one of backend.py:780-817 (when
    some head rejects, every head's expanded top-k is attended and rejected
    heads output it; the expansion follows the same forced-page rule as the
    draft selection). `n_recovery` is the recovery work the reference records
    (complement pages of rejected heads, or every head's expanded pages)."""
    W = block_tables.shape[1]
    budget = budget_for(W, budget_pct)
    if page_scores is None:
        page_scores = score_pages(q, k_cache, block_tables, context_lens, num_kv_heads,
                                  num_q_per_kv, block_size, precise)
    idx, nph = select_pages(page_scores, context_lens, block_size, budget,
                            sink_pages, local_pages)
    o_d, m_d, l_d = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, idx, nph,
                                         context_lens, num_kv_heads, num_q_per_kv,
                                         block_size, precise)
    accept, cov = check_coverage(page_scores, idx, nph, tau, precise)
    exp = None
    if bool(accept.all()):
        out = (o_d / l_d.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
        n_comp = torch.zeros_like(nph)
        n_rec = n_comp
    elif approx_recovery_pct is not None:
        eb = approx_budget(W, budget, approx_recovery_pct)
        e_idx, e_n = select_pages(page_scores, context_lens, block_size, eb, sink_pages,
                                  local_pages)
        o_e, m_e, l_e = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, e_idx, e_n,
                                             context_lens, num_kv_heads, num_q_per_kv,
                                             block_size, precise)
        acc_q = accept.repeat_interleave(num_q_per_kv, dim=1).unsqueeze(-1)
        out = torch.where(acc_q, o_d / l_d.clamp(min=1e-6).unsqueeze(-1),
                          o_e / l_e.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
        n_comp = torch.zeros_like(nph)
        n_rec = e_n
        exp = (e_idx, e_n)
    else:
        comp, n_comp = compute_complement_pages(idx, nph, context_lens, block_size, accept)
        o_c, m_c, l_c = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, comp, n_comp,
                                             context_lens, num_kv_heads, num_q_per_kv,
                                             block_size, precise)
        out = selective_lse_merge(o_d, m_d, l_d, o_c, m_c, l_c, accept, num_q_per_kv, q.dtype)
        n_rec = n_comp
    return dict(output=out, page_scores=page_scores, page_indices=idx, n_per_head=nph,
                accept=accept, coverage=cov, o_draft=o_d, m_draft=m_d, l_draft=l_d,
                n_complement=n_comp, n_recovery=n_rec, expanded=exp,
                budget=torch.tensor(budget))


# --------------------------------------------------------------------------
# alternative selectors (cvsa/backend.py:522-681)
# --------------------------------------------------------------------------

def quest_page_scores(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                      context_lens: torch.Tensor, num_kv_heads: int,
                      block_size: int) -> torch.Tensor:
    """Quest ranking scores [B, H_kv, W] f32 (cvsa/backend.py:572-620).

    For each page and KV head: the channel-wise minimum and maximum of the
    keys of its valid tokens (in the pool's dtype), then
    sum_d max(q_d * kmin_d, q_d * kmax_d) in fp32 with q the group mean in
    q's dtype (as page scoring pools it), times D^-0.5. Pages without a valid
    token score -inf.
    """
    B, W = block_tables.shape
    D = q.shape[-1]
    qr = q_representative(q, num_kv_heads).float()                # [B, H, D]
    out = torch.full((B, num_kv_heads, W), NEG_INF, dtype=torch.float32)
    for b in range(B):
        ctx = int(context_lens[b])
        n = min((ctx + block_size - 1) // block_size, W)
        if n == 0:
            continue
        kp = k_cache[block_tables[b, :n].long()]                  # [n, bs, H, D]
        tok = torch.arange(n).view(n, 1) * block_size + torch.arange(block_size).view(1, -1)
        valid = (tok < ctx).view(n, block_size, 1, 1)
        kmin = torch.where(valid, kp, torch.full_like(kp, math.inf)).amin(dim=1).float()
        kmax = torch.where(valid, kp, torch.full_like(kp, -math.inf)).amax(dim=1).float()
        qb = qr[b].view(1, num_kv_heads, D)
        bound = torch.maximum(qb * kmin, qb * kmax).sum(-1) * (D ** -0.5)   # [n, H]
        out[b, :, :n] = bound.t()
    return out


def _stable_desc_order(x: torch.Tensor) -> torch.Tensor:
    """Indices ordering the last dim by (value descending, index ascending)."""
    return torch.sort(x, dim=-1, descending=True, stable=True).indices


def topp_select(sel_scores: torch.Tensor, n_valid: torch.Tensor, top_p: float):
    """cvsa/backend.py:652-681: per head the shortest score-ordered prefix whose
    softmax mass (over every page of the row) reaches top_p, at least 3 pages,
    at most the valid ones. Returns (page_indices [B, H, max_budget] in score
    order, n_per_head, max_budget)."""
    B, H, P = sel_scores.shape
    probs = torch.softmax(sel_scores.float(), dim=-1)
    order = _stable_desc_order(probs)
    mass = torch.gather(probs, -1, order).cumsum(-1)
    need = ((mass < top_p).sum(-1) + 1).clamp(min=3, max=P)
    n = torch.minimum(need, n_valid.view(B, 1).expand(B, H).to(need.dtype)).to(torch.int32)
    mb = int(n.max())
    return order[:, :, :mb].to(torch.int32), n, mb


def static_select(sel_scores: torch.Tensor, fracs, n_valid: torch.Tensor):
    """cvsa/backend.py:622-650: per-head budgets round(frac * W), clamped to
    [3, W], at most the valid pages; the top pages of each head in score
    order. Returns (page_indices, n_per_head, max_budget)."""
    B, H, P = sel_scores.shape
    f = torch.as_tensor(fracs, dtype=torch.float32)
    per = torch.clamp((f * P).round().long(), min=3, max=P)
    n = torch.minimum(per.view(1, H).expand(B, H), n_valid.view(B, 1).expand(B, H))
    mb = int(per.max())
    order = _stable_desc_order(sel_scores)[:, :, :min(mb, P)]
    return order.to(torch.int32), n.to(torch.int32), mb


def adaptive_select(page_scores: torch.Tensor, base_budget: int, n_valid: torch.Tensor,
                    floor_ratio: float):
    """cvsa/backend.py:522-570: the heads of a sequence compete for
    H * base_budget page slots by score (each head's share = how many of the
    H * base_budget best scores of the sequence are its), blended toward the
    uniform budget by floor_ratio, rounded half to even, at least 1 and at most
    the valid pages. Returns (page_indices in score order, n_per_head,
    max_budget)."""
    B, H, P = page_scores.shape
    total = H * base_budget
    flat = page_scores.reshape(B, H * P)
    order = _stable_desc_order(flat)[:, :min(total, H * P)]
    owner = order // P
    wins = torch.zeros(B, H, dtype=torch.float32)
    wins.scatter_add_(-1, owner, torch.ones_like(owner, dtype=torch.float32))
    final = torch.round(wins * (1 - floor_ratio) + base_budget * floor_ratio).to(torch.int32)
    final = torch.minimum(final.clamp(min=1), n_valid.view(B, 1).expand(B, H).to(torch.int32))
    mb = int(final.max())
    idx = _stable_desc_order(page_scores)[:, :, :min(mb, P)]
    return idx.to(torch.int32), final, mb


def uniform_select_unsorted_ref(sel_scores: torch.Tensor, n_valid: torch.Tensor, budget: int):
    """The reference's uniform path (cvsa/backend.py:737-747) with the stable
    tie rule: the top `budget` pages, n_per_head = min(budget, valid pages)."""
    B, H, P = sel_scores.shape
    idx = _stable_desc_order(sel_scores)[:, :, :min(budget, P)]
    n = torch.minimum(torch.full((B, H), budget, dtype=torch.int64),
                      n_valid.view(B, 1).expand(B, H)).to(torch.int32)
    return idx.to(torch.int32), n, budget


def alt_scoring_step(q, k_cache, v_cache, block_tables, context_lens, num_kv_heads,
                     num_q_per_kv, block_size, budget_pct, tau, *, selector="exact",
                     light_normalizer=False, top_p=None, static_fracs=None,
                     adaptive=False, adaptive_floor_ratio=0.5, approx_recovery_pct=None,
                     reject_override=None, page_scores=None, precise=True):
    """cvsa/backend.py:683-864 with the reference's selector options.

    `page_scores` drive the coverage gate (the Quest sketch when
    light_normalizer, else exact); `sel_scores` drive the ranking (the sketch
    when selector == 'quest'). reject_override: None, or True / False to force
    every head to reject / accept (the random-reject counterfactual with its
    draw already taken).
    """
    W = block_tables.shape[1]
    nv = n_valid_pages(context_lens, block_size)
    budget = budget_for(W, budget_pct)
    quest = None
    if page_scores is None:
        if light_normalizer:
            quest = quest_page_scores(q, k_cache, block_tables, context_lens, num_kv_heads,
                                      block_size)
            page_scores = quest
        else:
            page_scores = score_pages(q, k_cache, block_tables, context_lens, num_kv_heads,
                                      num_q_per_kv, block_size, precise)
    sel_scores = page_scores
    if selector == "quest" and not light_normalizer:
        quest = quest_page_scores(q, k_cache, block_tables, context_lens, num_kv_heads,
                                  block_size)
        sel_scores = quest
    if top_p is not None:
        idx, nph, budget = topp_select(sel_scores, nv, top_p)
    elif static_fracs is not None:
        idx, nph, budget = static_select(sel_scores, static_fracs, nv)
    elif adaptive:
        idx, nph, budget = adaptive_select(sel_scores, budget, nv, adaptive_floor_ratio)
    else:
        idx, nph, budget = uniform_select_unsorted_ref(sel_scores, nv, budget)
    o_d, m_d, l_d = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, idx, nph,
                                         context_lens, num_kv_heads, num_q_per_kv,
                                         block_size, precise)
    accept, cov = check_coverage(page_scores, idx, nph, tau, precise)
    if reject_override is not None:
        accept = torch.full_like(accept, not reject_override)
    exp = None
    if bool(accept.all()):
        out = (o_d / l_d.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
        n_rec = torch.zeros_like(nph)
    elif approx_recovery_pct is not None:
        eb = min(max(budget + 1, int(W * approx_recovery_pct)), W)
        e_idx = _stable_desc_order(sel_scores)[:, :, :eb].to(torch.int32)
        e_n = torch.minimum(torch.full_like(nph, eb), nv.view(-1, 1).expand_as(nph).to(nph.dtype))
        o_e, m_e, l_e = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, e_idx, e_n,
                                             context_lens, num_kv_heads, num_q_per_kv,
                                             block_size, precise)
        acc_q = accept.repeat_interleave(num_q_per_kv, dim=1).unsqueeze(-1)
        out = torch.where(acc_q, o_d / l_d.clamp(min=1e-6).unsqueeze(-1),
                          o_e / l_e.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
        n_rec = e_n
        exp = (e_idx, e_n)
    else:
        comp, n_comp = compute_complement_pages(idx, nph, context_lens, block_size, accept)
        o_c, m_c, l_c = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, comp, n_comp,
                                             context_lens, num_kv_heads, num_q_per_kv,
                                             block_size, precise)
        out = selective_lse_merge(o_d, m_d, l_d, o_c, m_c, l_c, accept, num_q_per_kv, q.dtype)
        n_rec = n_comp
    return dict(output=out, page_scores=page_scores, sel_scores=sel_scores, page_indices=idx,
                n_per_head=nph, accept=accept, coverage=cov, n_recovery=n_rec, expanded=exp,
                budget=budget)


class OracleBackend:
    """Scheduling of cvsa/backend.py:313-366 / 392-465 / 866-881 on the oracle ops.

    Lazy mode (lazy=True, check_interval=M): on steps with step % M == 0 the
    pages are rescored and the cached selection is gated; if every (b, h)
    accepts, the cached selection is reused, otherwise a full scoring step
    runs. Other steps reuse the cached selection without a gate. Fixed-interval
    mode rescores every reuse_interval steps. Dense layers attend all pages.
    """

    def __init__(self, num_kv_heads, num_q_heads, head_dim, block_size, num_layers=32,
                 budget_pct=0.10, reuse_interval=16, coverage_threshold=0.90,
                 dense_layers=None, lazy=False, check_interval=None,
                 sink_pages=0, local_pages=0, precise=True, approx_recovery_pct=None,
                 coverage_interval=None, selector="exact", light_normalizer=False,
                 top_p=None, static_budget_table=None, adaptive_selection=False,
                 adaptive_floor_ratio=0.5, random_reject_prob=None, reject_draw=None):
        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.G = num_q_heads // num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.num_layers = num_layers
        self.budget_pct = budget_pct
        self.reuse_interval = reuse_interval
        self.tau = coverage_threshold
        self.dense_layers = set(dense_layers or [])
        self.lazy = lazy
        self.check_interval = check_interval or 1
        self.sink_pages = sink_pages
        self.local_pages = local_pages
        self.precise = precise
        self.approx_recovery_pct = approx_recovery_pct
        self.coverage_interval = coverage_interval or self.check_interval
        # selector options of backend.py:66-76; reject_draw() gives the
        # uniform [0, 1) draws of the random-reject counterfactual
        self.selector = selector
        self.light_normalizer = light_normalizer
        self.top_p = top_p
        self.static_budget_table = static_budget_table
        self.adaptive_selection = adaptive_selection
        self.adaptive_floor_ratio = adaptive_floor_ratio
        self.random_reject_prob = random_reject_prob
        self.reject_draw = reject_draw or (lambda: float(torch.rand(1)))
        self.alt = (selector != "exact" or light_normalizer or top_p is not None
                    or static_budget_table is not None or adaptive_selection
                    or random_reject_prob is not None)
        self.reset()

    def reset(self):
        self._step = 0
        self._cached: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._cached_scores: Dict[int, torch.Tensor] = {}   # backend.py:713
        self.attn_work = 0
        self.attn_work_max = 0
        self.accept_counts = 0
        self.reject_counts = 0
        self.total_scoring_steps = 0
        self.total_coverage_checks = 0
        self.per_head_accept_sum = 0
        self.per_head_total = 0
        self.dense_layer_steps = 0
        self.last: Dict[str, torch.Tensor] = {}

    def step_done(self, layer_idx, num_layers):
        if layer_idx == num_layers - 1:
            self._step += 1

    def _record(self, context_lens, pages):
        nv = n_valid_pages(context_lens, self.block_size)
        self.attn_work += int(pages)
        self.attn_work_max += int(nv.sum()) * self.num_kv_heads

    def _reuse(self, q, k, v, bt, cl, layer_idx):
        idx, nph = self._cached[layer_idx]
        self._record(cl, nph.sum())
        return sparse_decode(q, k, v, bt, idx, nph, cl, self.num_kv_heads, self.G,
                             self.block_size, self.precise)

    def _override(self):
        """backend.py:437-438 / 764-766: one draw per gate, True = reject all."""
        if self.random_reject_prob is None:
            return None
        return self.reject_draw() < self.random_reject_prob

    def _gate_scores(self, q, k, bt, cl):
        if self.light_normalizer:
            return quest_page_scores(q, k, bt, cl, self.num_kv_heads, self.block_size)
        return score_pages(q, k, bt, cl, self.num_kv_heads, self.G, self.block_size,
                           self.precise)

    def _scoring(self, q, k, v, bt, cl, layer_idx, page_scores=None):
        if self.alt:
            fr = None
            if self.static_budget_table is not None:
                fr = self.static_budget_table[layer_idx]
            r = alt_scoring_step(q, k, v, bt, cl, self.num_kv_heads, self.G, self.block_size,
                                 self.budget_pct, self.tau, selector=self.selector,
                                 light_normalizer=self.light_normalizer, top_p=self.top_p,
                                 static_fracs=fr, adaptive=self.adaptive_selection,
                                 adaptive_floor_ratio=self.adaptive_floor_ratio,
                                 approx_recovery_pct=self.approx_recovery_pct,
                                 reject_override=self._override(), page_scores=page_scores,
                                 precise=self.precise)
        else:
            r = scoring_step(q, k, v, bt, cl, self.num_kv_heads, self.G, self.block_size,
                             self.budget_pct, self.tau, self.sink_pages, self.local_pages,
                             page_scores, self.precise, self.approx_recovery_pct)
        self._cached[layer_idx] = (r["page_indices"], r["n_per_head"])
        self._cached_scores[layer_idx] = r["page_scores"]
        self._record(cl, r["n_per_head"].sum() + r["n_recovery"].sum())
        self.total_scoring_steps += 1
        if not self.lazy:
            self.per_head_accept_sum += int(r["accept"].sum())
            self.per_head_total += r["accept"].numel()
            if bool(r["accept"].all()):
                self.accept_counts += 1
            else:
                self.reject_counts += 1
        self.last = r
        return r["output"]

    def __call__(self, q, k, v, bt, cl, layer_idx):
        if layer_idx in self.dense_layers:
            self.dense_layer_steps += 1
            nv = n_valid_pages(cl, self.block_size)
            self._record(cl, nv.sum() * self.num_kv_heads)
            return dense_decode(q, k, v, bt, cl, self.num_kv_heads, self.G,
                                self.block_size, self.precise)
        if self.lazy:
            # backend.py:335-358: scoring every check_interval steps, the
            # coverage-only gate every coverage_interval steps in between
            if self._step % self.check_interval == 0 or layer_idx not in self._cached:
                return self._lazy(q, k, v, bt, cl, layer_idx)
            if self._step % self.coverage_interval == 0 and layer_idx in self._cached_scores:
                return self._coverage_only(q, k, v, bt, cl, layer_idx)
            return self._reuse(q, k, v, bt, cl, layer_idx)
        if self._step % self.reuse_interval == 0 or layer_idx not in self._cached:
            return self._scoring(q, k, v, bt, cl, layer_idx)
        return self._reuse(q, k, v, bt, cl, layer_idx)

    def _coverage_only(self, q, k, v, bt, cl, layer_idx):
        """backend.py:467-520: gate the cached selection on the page scores of
        the last scoring step (no fresh scores); reuse it if every head
        accepts, else a scoring step on fresh scores."""
        idx, nph = self._cached[layer_idx]
        accept, cov = check_coverage(self._cached_scores[layer_idx], idx, nph, self.tau,
                                     self.precise)
        ov = self._override()
        if ov is not None:
            accept = torch.full_like(accept, not ov)
        self.per_head_accept_sum += int(accept.sum())
        self.per_head_total += accept.numel()
        self.total_coverage_checks += 1
        self.last = dict(cached_accept=accept, cached_coverage=cov)
        if bool(accept.all()):
            self.accept_counts += 1
            return self._reuse(q, k, v, bt, cl, layer_idx)
        self.reject_counts += 1
        return self._scoring(q, k, v, bt, cl, layer_idx)

    def _lazy(self, q, k, v, bt, cl, layer_idx):
        scores = self._gate_scores(q, k, bt, cl)
        self.total_coverage_checks += 1
        if layer_idx in self._cached:
            idx, nph = self._cached[layer_idx]
            accept, cov = check_coverage(scores, idx, nph, self.tau, self.precise)
            ov = self._override()
            if ov is not None:
                accept = torch.full_like(accept, not ov)
            self.per_head_accept_sum += int(accept.sum())
            self.per_head_total += accept.numel()
            self.last = dict(cached_accept=accept, cached_coverage=cov, page_scores=scores)
            if bool(accept.all()):
                self.accept_counts += 1
                return self._reuse(q, k, v, bt, cl, layer_idx)
        self.reject_counts += 1
        out = self._scoring(q, k, v, bt, cl, layer_idx, page_scores=scores)
        return out

    def get_stats(self) -> dict:
        total_checks = max(self.total_coverage_checks, self.total_scoring_steps, 1)
        st = {
            "total_scoring_steps": self.total_scoring_steps,
            "total_coverage_checks": self.total_coverage_checks,
            "all_accepted_pct": self.accept_counts / total_checks * 100,
            "some_rejected_pct": self.reject_counts / total_checks * 100,
            "per_head_accept_rate": self.per_head_accept_sum / max(self.per_head_total, 1) * 100,
            "total_decode_steps": self._step,
        }
        if self.attn_work_max > 0:
            st["effective_budget_pct"] = self.attn_work / self.attn_work_max * 100
            st["total_pages_attended"] = self.attn_work
            st["total_pages_max"] = self.attn_work_max
        return st


def coverage_margin(cov: torch.Tensor, tau: float) -> torch.Tensor:
    """|cov - tau|, used to attribute an accept mismatch to a near-tie."""
    return (cov.double() - float(torch.tensor(tau, dtype=torch.float32))).abs()


def topk_gap(page_scores: torch.Tensor, context_lens: torch.Tensor, block_size: int,
             budget: int, sink_pages: int = 0, local_pages: int = 0) -> torch.Tensor:
    """Score gap between the last selected and first unselected candidate per (b, h).

    A selection mismatch between two implementations whose scores agree to
    within eps can only occur where this gap is <= 2 * eps.
    """
    B, H, W = page_scores.shape
    nv = n_valid_pages(context_lens, block_size)
    gap = torch.full((B, H), math.inf, dtype=torch.float64)
    for b in range(B):
        n = int(nv[b])
        forced = set(range(min(sink_pages, n))) | set(range(max(0, n - local_pages), n))
        cand = [p for p in range(n) if p not in forced]
        if len(cand) <= budget:
            continue
        for h in range(H):
            vals = sorted((float(page_scores[b, h, p]) for p in cand), reverse=True)
            gap[b, h] = vals[budget - 1] - vals[budget]
    return gap


# --------------------------------------------------------------------------
# paged KV runtime (cvsa/runtime/kv_cache.py:24-150)
# --------------------------------------------------------------------------

class PagedKVRef:
    """CPU restatement of PagedKVCache + SequenceKVManager
    (cvsa/runtime/kv_cache.py:24-150): a pool [num_blocks, block_size, H, D]
    with a bump allocator (blocks handed out in order, kv_cache.py:53-62),
    per-sequence block tables and context lengths; prefill writes whole
    pages (:110-128), a decode append takes a new block when its token starts
    a page past the ones allocated (:130-150)."""

    def __init__(self, num_blocks, block_size, num_kv_heads, head_dim, dtype, batch_size,
                 max_context_len):
        self.bs = block_size
        self.k = torch.zeros(num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.next_free = 0
        self.total = num_blocks
        self.max_pages = (max_context_len + block_size - 1) // block_size
        self.block_tables = torch.zeros(batch_size, self.max_pages, dtype=torch.int32)
        self.context_lens = torch.zeros(batch_size, dtype=torch.int32)
        self.pages = [0] * batch_size

    def allocate(self, n):
        assert self.next_free + n <= self.total, "Out of blocks"
        ids = list(range(self.next_free, self.next_free + n))
        self.next_free += n
        return ids

    def prefill(self, b, k_all, v_all):
        n_tok = k_all.shape[0]
        n_pages = (n_tok + self.bs - 1) // self.bs
        ids = self.allocate(n_pages)
        for p, blk in enumerate(ids):
            self.block_tables[b, p] = blk
            t0, t1 = p * self.bs, min((p + 1) * self.bs, n_tok)
            self.k[blk, :t1 - t0] = k_all[t0:t1]
            self.v[blk, :t1 - t0] = v_all[t0:t1]
        self.context_lens[b] = n_tok
        self.pages[b] = n_pages

    def append(self, b, k, v):
        pos = int(self.context_lens[b])
        page, off = pos // self.bs, pos % self.bs
        if off == 0 and page >= self.pages[b]:
            self.block_tables[b, page] = self.allocate(1)[0]
            self.pages[b] += 1
        blk = int(self.block_tables[b, page])
        self.k[blk, off] = k
        self.v[blk, off] = v
        self.context_lens[b] += 1

    def gather(self, blocks):
        """Dense [n * block_size, H, D] copies of the given blocks' K and V."""
        idx = torch.as_tensor(blocks, dtype=torch.long)
        return (self.k[idx].reshape(-1, *self.k.shape[2:]),
                self.v[idx].reshape(-1, *self.v.shape[2:]))


# --------------------------------------------------------------------------
# page split over ranks (the scoring / lazy-check step of
# cvsa/backend.py:683-864 and :392-465 with every sequence's pages spread over
# ranks): restatement of the three per-rank ops of a split step
# --------------------------------------------------------------------------

def _lse_rows(x: torch.Tensor) -> torch.Tensor:
    """log-sum-exp over the last dim (-inf when empty or all -inf)."""
    if x.shape[-1] == 0:
        return torch.full(x.shape[:-1], NEG_INF, dtype=torch.float32)
    return torch.logsumexp(x.float(), -1)


def split_propose(scores: torch.Tensor, context_lens: torch.Tensor, block_size: int,
                  cached, sink: int, local: int, budget: int, max_sel: int,
                  out: torch.Tensor) -> torch.Tensor:
    """A rank's exchange row: [lse_all | lse_cached | lse_forced | candidate
    scores] over its B * H rows (the candidates: the best `budget` of its
    pages outside its forced ones, finite scores only, ranked (score desc,
    page asc), written in page order and -inf padded to max_sel). Returns the
    candidates' local pages [B, H, max_sel] (-1 unused)."""
    B, H, W = scores.shape
    rows = B * H
    nv = n_valid_pages(context_lens, block_size).clamp(max=W)
    lse_all = _lse_rows(scores).reshape(rows)
    lse_c = torch.full((B, H), NEG_INF)
    lse_f = torch.full((B, H), NEG_INF)
    cand_s = torch.full((B, H, max_sel), NEG_INF)
    prop = torch.full((B, H, max_sel), -1, dtype=torch.int32)
    for b in range(B):
        n = int(nv[b])
        f_hi = min(sink, n)
        t_lo = max(n - local, f_hi)
        forced = list(range(f_hi)) + list(range(t_lo, n))
        for h in range(H):
            s = scores[b, h]
            if forced:
                lse_f[b, h] = _lse_rows(s[torch.tensor(forced)])
            if cached is not None:
                ci, cn = cached
                ents = [int(p) for p in ci[b, h, :int(cn[b, h])] if 0 <= int(p) < W]
                if ents:
                    lse_c[b, h] = _lse_rows(s[torch.tensor(ents)])
            sl = s.tolist()
            cand = [p for p in range(f_hi, t_lo) if math.isfinite(sl[p])]
            best = sorted(sorted(cand, key=lambda p: (-sl[p], p))[:budget])
            for j, p in enumerate(best):
                cand_s[b, h, j] = sl[p]
                prop[b, h, j] = p
    out[:rows] = lse_all
    out[rows:2 * rows] = lse_c.reshape(rows)
    out[2 * rows:3 * rows] = lse_f.reshape(rows)
    out[3 * rows:3 * rows + rows * max_sel] = cand_s.reshape(-1)
    return prop


def split_gate(parts: torch.Tensor, prop: torch.Tensor, context_lens: torch.Tensor,
               block_size: int, max_pages: int, rank: int, budget: int, max_sel: int,
               sink: int, local: int, tau: float, has_cache: bool, stats_mode: int,
               state: torch.Tensor, counters: torch.Tensor):
    """The same decisions on every rank from the gathered rows parts [N, stride]:
    lse_all over ranks, the lazy gate of the cached selection (batch decision
    in state[3]), the global top-`budget` of the candidates (position order is
    page order), its gate against lse_all with every rank's forced pages added,
    and this rank's share of it (sink, chosen, local; ascending). Counts the
    step in `counters` (scoring, accept, reject, heads accepted, checks, heads
    total) the way cvsa/backend.py:420-465 (lazy) and :775-862 do. Returns
    (sel, n, accept uint8, bitmap)."""
    N = parts.shape[0]
    B, H, _ = prop.shape
    rows = B * H
    lse_all = torch.logsumexp(parts[:, :rows].float(), 0)
    lse_c = torch.logsumexp(parts[:, rows:2 * rows].float(), 0)
    forced = parts[:, 2 * rows:3 * rows].float()                       # [N, rows]
    cand = parts[:, 3 * rows:3 * rows + rows * max_sel].reshape(N, rows, max_sel)
    cand = cand.permute(1, 0, 2).reshape(rows, N * max_sel)
    acc0 = torch.exp(lse_c - lse_all) >= tau
    nv = n_valid_pages(context_lens, block_size).clamp(max=max_pages)
    sel = torch.zeros((B, H, max_sel), dtype=torch.int32)
    n = torch.zeros((B, H), dtype=torch.int32)
    acc = torch.zeros((B, H), dtype=torch.uint8)
    words = (max_pages + 31) // 32
    bitmap = torch.zeros((B, H, words), dtype=torch.int64)
    for i in range(rows):
        b, h = divmod(i, H)
        c = cand[i].tolist()
        fin = [j for j in range(len(c)) if math.isfinite(c[j])]
        chosen = sorted(fin, key=lambda j: (-c[j], j))[:budget]
        terms = torch.tensor([c[j] for j in chosen] + forced[:, i].tolist())
        lse_sel = _lse_rows(terms)
        acc[b, h] = int(bool(torch.exp(lse_sel - lse_all[i]) >= tau))
        mine = sorted(j - rank * max_sel for j in chosen
                      if rank * max_sel <= j < (rank + 1) * max_sel)
        nvb = int(nv[b])
        f_hi = min(sink, nvb)
        t_lo = max(nvb - local, f_hi)
        pages = list(range(f_hi)) + [int(prop[b, h, j]) for j in mine] + list(range(t_lo, nvb))
        n[b, h] = len(pages)
        if pages:
            sel[b, h, :len(pages)] = torch.tensor(pages, dtype=torch.int32)
        for p in pages:
            bitmap[b, h, p // 32] |= 1 << (p % 32)
    reuse = bool(has_cache) and bool(acc0.all())
    state[3] = 1 if reuse else 0
    check, lazy = bool(stats_mode & 1), bool(stats_mode & 2)
    SC, AC, RJ, HA, CK, HT = range(6)
    if check:
        counters[CK] += 1
    if check and not has_cache:
        counters[RJ] += 1
    if check and has_cache:
        counters[HT] += rows
        counters[HA] += int(acc0.sum())
        counters[AC if reuse else RJ] += 1
        if not reuse:
            counters[SC] += 1
    else:
        counters[SC] += 1
    if not lazy:
        counters[HA] += int(acc.sum())
        counters[HT] += rows
    bitmap = torch.where(bitmap >= 2 ** 31, bitmap - 2 ** 32, bitmap).to(torch.int32)
    return sel, n, acc, bitmap


def split_attend(q, k_cache, v_cache, block_tables, context_lens, num_kv_heads, num_q_per_kv,
                 block_size, cached, sel, n, decision, accept, bitmap, out):
    """Partials of a split step: the cached selection where decision[0] bit0
    is set, else the new one; a head whose new gate rejected attends every
    valid page of the rank (draft and complement of backend.py:818-844).
    Copies the new selection into `cached` when it is the one decoded."""
    B = q.shape[0]
    H = num_kv_heads
    W = block_tables.shape[1]
    reuse = decision is not None and (int(decision[0]) & 1) == 1
    if reuse:
        idx, cnt = cached[0].clone(), cached[1].clone()
    else:
        nv = n_valid_pages(context_lens, block_size).clamp(max=W)
        every = torch.arange(W, dtype=torch.int32).view(1, 1, W).expand(B, H, W)
        width = max(W, sel.shape[-1])
        idx = torch.zeros((B, H, width), dtype=torch.int32)
        cnt = torch.zeros((B, H), dtype=torch.int32)
        for b in range(B):
            for h in range(H):
                if int(accept[b, h]):
                    k = int(n[b, h])
                    idx[b, h, :k] = sel[b, h, :k]
                    cnt[b, h] = k
                else:
                    idx[b, h, :W] = every[b, h]
                    cnt[b, h] = int(nv[b])
        if cached is not None:
            cached[0].copy_(sel)
            cached[1].copy_(n)
    o, m, l = sparse_decode_unnorm(q, k_cache, v_cache, block_tables, idx, cnt, context_lens,
                                   num_kv_heads, num_q_per_kv, block_size)
    for dst, src in zip(out, (o, m, l)):
        dst.copy_(src)
    return out
