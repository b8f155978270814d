"""The reference's alternative page selectors on the B200 kernels.

cvsa/backend.py:522-681 offers, besides the uniform top-k of the exact page
scores: the Quest sketch ranking (selector='quest', optionally also as the
gate's normaliser, light_normalizer), per-head top-p budgets (top_p), offline
per-head budgets (static_budget_table), cross-head budget competition
(adaptive_selection) and a random-reject counterfactual (random_reject_prob).
`AltStep` runs a layer step with those options the way the reference's
_lazy_step / _scoring_step / _reuse_step / _coverage_only_step do, each stage
on the GPU: page scores (csrc/score.cu) or the Quest sketch (csrc/quest.cu),
the uniform top-k (csrc/select.cu) or the selector functions below, the draft
decode (csrc/attend*.cu), the coverage gate (csrc/select.cu), and exact
recovery fused with the LSE merge (cvsa_recover_merge) or the approximate one
(a second top-k and decode). Decisions are read on the host where the
reference reads them (`accept_mask.all()`, the random draw), so these steps
are not graph-capturable, as the reference's are not.

Selections of the per-head-budget selectors are in score order (the first
n_per_head entries of a row are the head's pages); ties in score go to the
lower page index.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from cvsa import _lib
from cvsa.kernels.coverage import check_coverage, compute_complement
from cvsa.kernels.page_scores import quest_page_scores, score_pages
from cvsa.kernels.select import budget_for, select_pages
from cvsa.kernels.sparse_decode import recover_merge, sparse_decode, sparse_decode_unnorm


def _desc_order(x: torch.Tensor) -> torch.Tensor:
    """Indices ordering the last dim by value descending, index ascending."""
    return torch.sort(x, dim=-1, descending=True, stable=True).indices


def topp_select(sel_scores: torch.Tensor, n_valid: torch.Tensor, top_p: float):
    """backend.py:652-681: the shortest score-ordered prefix of each head whose
    softmax mass (temperature 1: the scores carry D^-0.5) reaches top_p, at
    least 3 pages and at most the valid ones. Returns (page_indices
    [B, H, max_budget] int32 in score order, n_per_head int32, max_budget)."""
    B, H, P = sel_scores.shape
    probs = torch.softmax(sel_scores.float(), dim=-1)
    order = _desc_order(probs)
    below = torch.gather(probs, -1, order).cumsum(-1) < top_p
    need = (below.sum(-1) + 1).clamp(min=3, max=P)
    n = torch.minimum(need, n_valid.view(B, 1).to(need.dtype)).to(torch.int32)
    mb = int(n.max())                     # host read, as backend.py:677
    return order[:, :, :mb].to(torch.int32).contiguous(), n, mb


def static_select(sel_scores: torch.Tensor, fracs: torch.Tensor, n_valid: torch.Tensor):
    """backend.py:622-650: head h keeps round(fracs[h] * W) pages (half to
    even), clamped to [3, W] and to the valid pages; its best pages in score
    order. Returns (page_indices, n_per_head, max_budget)."""
    B, H, P = sel_scores.shape
    per = torch.clamp((fracs.to(sel_scores.device, torch.float32) * P).round().long(),
                      min=3, max=P)
    n = torch.minimum(per.view(1, H), n_valid.view(B, 1).to(per.dtype)).to(torch.int32)
    mb = int(per.max())
    idx = _desc_order(sel_scores)[:, :, :min(mb, P)]
    return idx.to(torch.int32).contiguous(), n, mb


def adaptive_select(page_scores: torch.Tensor, base_budget: int, n_valid: torch.Tensor,
                    floor_ratio: float):
    """backend.py:522-570: the KV heads of a sequence compete for
    H * base_budget slots -- a head's raw share is how many of the sequence's
    H * base_budget best page scores are its own -- blended toward the uniform
    budget (round(raw (1 - f) + base f), half to even), at least 1, at most
    the valid pages. Returns (page_indices in score order, n_per_head,
    max_budget)."""
    B, H, P = page_scores.shape
    slots = min(H * base_budget, H * P)
    best = _desc_order(page_scores.reshape(B, H * P))[:, :slots]
    share = torch.zeros(B, H, dtype=torch.float32, device=page_scores.device)
    share.scatter_add_(-1, best // P, torch.ones_like(best, dtype=torch.float32))
    n = torch.round(share * (1 - floor_ratio) + base_budget * floor_ratio).to(torch.int32)
    n = torch.minimum(n.clamp(min=1), n_valid.view(B, 1).to(torch.int32))
    mb = int(n.max())
    idx = _desc_order(page_scores)[:, :, :min(mb, P)]
    return idx.to(torch.int32).contiguous(), n, mb


class AltStep:
    """Layer steps of CVSABackend with the reference's selector options.

    Holds its own per-layer cached selections and page scores; updates the
    backend's device counters (the same statistics as the fused path)."""

    def __init__(self, be):
        self.be = be
        self.cached: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        self.scores: Dict[int, torch.Tensor] = {}
        fr = be.static_budget_table
        self.fracs = None if fr is None else {int(k): torch.as_tensor(v, dtype=torch.float32)
                                              for k, v in fr.items()}

    def reset(self):
        self.cached = {}
        self.scores = {}

    # ---- helpers ----------------------------------------------------------
    def _ctr(self, i, v):
        self.be._counters[i] += v

    def _record(self, cl, pages):
        """backend.py:368-390: pages attended, and what dense attention would
        attend (every valid page of every KV head)."""
        nv = (cl.to(torch.int64) + self.be.block_size - 1) // self.be.block_size
        self._ctr(_lib.CTR_PAGES_ATTENDED, pages)
        self._ctr(_lib.CTR_PAGES_MAX, nv.sum() * self.be.num_kv_heads)

    def _override(self, accept: torch.Tensor) -> torch.Tensor:
        """backend.py:437-438 / 490-491 / 764-766: one uniform draw per gate on
        the accept mask's device; below random_reject_prob every head rejects,
        else every head accepts."""
        p = self.be.random_reject_prob
        if p is None:
            return accept
        reject = torch.rand(1, device=accept.device).item() < p
        return torch.zeros_like(accept) if reject else torch.ones_like(accept)

    def _gate_scores(self, q, k, bt, cl):
        be = self.be
        if be.light_normalizer:
            return quest_page_scores(q, k, bt, cl, be.num_kv_heads)
        return score_pages(q, k, bt, cl, be.num_kv_heads, be.num_q_per_kv, be.block_size)

    def _decode(self, q, k, v, bt, cl, idx, n):
        be = self.be
        return sparse_decode(q, k, v, bt, idx, n, cl, be.num_kv_heads, be.num_q_per_kv,
                             be.block_size)

    # ---- steps -------------------------------------------------------------
    def __call__(self, q, k, v, bt, cl, layer_idx):
        be = self.be
        has_cache = layer_idx in self.cached
        if be.lazy:
            step = be._step
            if step % be.check_interval == 0 or not has_cache:
                return self.lazy(q, k, v, bt, cl, layer_idx)
            if step % be.coverage_interval == 0 and layer_idx in self.scores:
                return self.coverage_only(q, k, v, bt, cl, layer_idx)
            return self.reuse(q, k, v, bt, cl, layer_idx)
        if be._step % be.reuse_interval == 0 or not has_cache:
            return self.scoring(q, k, v, bt, cl, layer_idx)
        return self.reuse(q, k, v, bt, cl, layer_idx)

    def reuse(self, q, k, v, bt, cl, layer_idx):
        """backend.py:866-881."""
        idx, n = self.cached[layer_idx]
        self._record(cl, n.sum())
        return self._decode(q, k, v, bt, cl, idx, n)

    def _gate_cached(self, scores, layer_idx):
        """Gate the cached selection on `scores`; returns (accept, all)."""
        be = self.be
        idx, n = self.cached[layer_idx]
        acc, _cov = check_coverage(scores, idx, n, be.tau)
        acc = self._override(acc)
        self._ctr(_lib.CTR_HEAD_ACCEPT, acc.sum())
        self._ctr(_lib.CTR_HEAD_TOTAL, acc.numel())
        return acc, bool(acc.all())

    def lazy(self, q, k, v, bt, cl, layer_idx):
        """backend.py:392-465."""
        scores = self._gate_scores(q, k, bt, cl)
        self._ctr(_lib.CTR_COVERAGE_CHECKS, 1)
        if layer_idx in self.cached:
            acc, all_ok = self._gate_cached(scores, layer_idx)
            if all_ok:
                self._ctr(_lib.CTR_ACCEPT_STEPS, 1)
                self.be._last_accept_mask[layer_idx] = acc
                return self.reuse(q, k, v, bt, cl, layer_idx)
        self._ctr(_lib.CTR_REJECT_STEPS, 1)
        return self.scoring(q, k, v, bt, cl, layer_idx, page_scores=scores)

    def coverage_only(self, q, k, v, bt, cl, layer_idx):
        """backend.py:467-520: the gate on the page scores cached at the last
        scoring step; reuse if every head accepts, else a scoring step on
        fresh scores."""
        acc, all_ok = self._gate_cached(self.scores[layer_idx], layer_idx)
        self._ctr(_lib.CTR_COVERAGE_CHECKS, 1)
        if all_ok:
            self._ctr(_lib.CTR_ACCEPT_STEPS, 1)
            self.be._last_accept_mask[layer_idx] = acc
            return self.reuse(q, k, v, bt, cl, layer_idx)
        self._ctr(_lib.CTR_REJECT_STEPS, 1)
        return self.scoring(q, k, v, bt, cl, layer_idx)

    def scoring(self, q, k, v, bt, cl, layer_idx, page_scores: Optional[torch.Tensor] = None):
        """backend.py:683-864 with the selector options."""
        be = self.be
        H, G, bs = be.num_kv_heads, be.num_q_per_kv, be.block_size
        B = q.shape[0]
        W = bt.shape[1]
        nv = ((cl.to(torch.int64) + bs - 1) // bs).clamp(max=W)
        budget = budget_for(W, be.budget_pct)
        if page_scores is None:
            page_scores = self._gate_scores(q, k, bt, cl)
        self.scores[layer_idx] = page_scores
        sel_scores = page_scores
        if be.selector == "quest" and not be.light_normalizer:
            sel_scores = quest_page_scores(q, k, bt, cl, H)
        if be.top_p is not None:
            idx, n, budget = topp_select(sel_scores, nv, be.top_p)
        elif self.fracs is not None:
            idx, n, budget = static_select(sel_scores, self.fracs[layer_idx], nv)
        elif be.adaptive_selection:
            idx, n, budget = adaptive_select(sel_scores, budget, nv, be.adaptive_floor_ratio)
        else:
            idx, n = select_pages(sel_scores, cl, bs, budget)
        o_d, m_d, l_d = sparse_decode_unnorm(q, k, v, bt, idx, n, cl, H, G, bs)
        acc, _cov = check_coverage(page_scores, idx, n, be.tau)
        acc = self._override(acc)
        be._last_accept_mask[layer_idx] = acc
        all_ok = bool(acc.all())
        rec_pages = None
        if all_ok:
            out = (o_d / l_d.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
            if not be.lazy:
                self._ctr(_lib.CTR_ACCEPT_STEPS, 1)
        elif be.approx_recovery_pct is not None:
            # backend.py:780-817: every head's expanded top-k of the selector's
            # scores; rejected heads output it
            eb = min(max(budget + 1, int(W * be.approx_recovery_pct)), W)
            e_idx, e_n = select_pages(sel_scores, cl, bs, eb)
            o_e = sparse_decode(q, k, v, bt, e_idx, e_n, cl, H, G, bs)
            o_dn = (o_d / l_d.clamp(min=1e-6).unsqueeze(-1)).to(q.dtype)
            acc_q = acc.repeat_interleave(G, dim=1).unsqueeze(-1)
            out = torch.where(acc_q, o_dn, o_e)
            rec_pages = e_n.sum()
            be._last_expanded_selection[layer_idx] = (e_idx, e_n)
            if not be.lazy:
                self._ctr(_lib.CTR_REJECT_STEPS, 1)
        else:
            # backend.py:818-844: complement attention merged by LSE (fused)
            out = recover_merge(q, k, v, bt, idx, n, cl, acc, o_d, m_d, l_d, H, G, bs,
                                output_dtype=q.dtype)
            comp, n_comp = compute_complement(idx, n, cl, bs, acc)
            rec_pages = n_comp.sum()
            be._last_expanded_selection[layer_idx] = (comp, n_comp)
            if not be.lazy:
                self._ctr(_lib.CTR_REJECT_STEPS, 1)
        self._record(cl, n.sum() if rec_pages is None else n.sum() + rec_pages)
        self.cached[layer_idx] = (idx, n)
        self._ctr(_lib.CTR_SCORING_STEPS, 1)
        if not be.lazy:
            self._ctr(_lib.CTR_HEAD_ACCEPT, acc.sum())
            self._ctr(_lib.CTR_HEAD_TOTAL, acc.numel())
        return out
