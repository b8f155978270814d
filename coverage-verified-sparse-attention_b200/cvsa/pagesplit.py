"""Page-split CVSA step: each rank holds a contiguous range of every
sequence's pages (one long sequence spread over GPUs, config 3 across ranks).

The reference has no multi-GPU path; this follows its single-GPU semantics
(cvsa/backend.py:683-864 scoring step, :392-465 lazy step, :866-881 reuse)
with the selection, the attention partials and the coverage sums combined
over the ranks:

  1. every rank scores its pages and proposes its best `budget` non-forced
     pages (score, global page index); an all-gather of the proposals lets
     every rank take the same global top-`budget` (score descending, page
     ascending; proposals are concatenated in rank order, so table position
     order is page order). Forced pages: the sink pages live on rank 0, the
     local pages on the last rank;
  2. every rank attends its share of the selection (unnormalised partial
     (o, m, l)) and sums its pages' log-sum-exp terms (all valid pages, and
     the selected ones); an all-gather of both lets every rank merge them in
     fixed rank order: the draft output, coverage exp(lse_sel - lse_all) and
     the accept mask (coverage.py:160-215) are identical on every rank;
  3. if a head rejects, exact recovery: every rank attends all its valid
     pages of the rejected heads (draft and complement partition them, so
     this is the merged result of backend.py:818-844) and a third all-gather
     merges them.
Reuse steps need only exchange 2 (partials). A lazy check step gathers the
cached selection's coverage sums first; every rank then takes the same
decision from the same merged sums.

No step reads a device value on the host: the lazy decision and the accept
mask stay on the device and gate the work instead of branching around it. A
lazy check step always runs the scoring step's launches and exchanges, and
where the cached selection passed, its pages are the ones attended and kept;
exact recovery always runs, attending no pages for heads that need none. The
launches and exchanges of a step depend only on its host-known kind (first,
check, reuse), so a layer's steps can be captured in CUDA graphs, NCCL
all-gathers included, and every rank issues the same collectives.

A step is a generator that yields each 1-D float32 tensor to all-gather and
receives the [world, n] result; `run_step` drives it with torch.distributed,
and tests can drive the ranks of one process in lockstep.
"""

from typing import Callable, Dict, List, Optional, Tuple

import torch

from cvsa.kernels.select import budget_for

NEG_INF = float("-inf")


def page_range(n_pages: torch.Tensor, rank: int, world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """[lo, hi) of each sequence's pages held by `rank`: contiguous, sizes differ by <= 1."""
    n = n_pages.to(torch.int64)
    return n * rank // world, n * (rank + 1) // world


def shard_sequence(k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                   context_lens: torch.Tensor, rank: int, world: int, block_size: int):
    """This rank's part of a paged batch: a pool holding only its pages, its
    block tables (local page p = global page lo + p) and local context lengths
    (tokens inside its range; the last rank keeps the partial last page)."""
    ctx = context_lens.to(torch.int64).cpu()
    nv = (ctx + block_size - 1) // block_size
    lo, hi = page_range(nv, rank, world)
    B = block_tables.shape[0]
    W = int((hi - lo).max()) if B else 0
    bt_cpu = block_tables.cpu()
    blocks = []
    table = torch.zeros((B, max(W, 1)), dtype=torch.int32)
    for b in range(B):
        ids = bt_cpu[b, int(lo[b]):int(hi[b])].long()
        table[b, :ids.numel()] = torch.arange(len(blocks), len(blocks) + ids.numel(),
                                              dtype=torch.int32)
        blocks.extend(ids.tolist())
    idx = torch.tensor(blocks, dtype=torch.long, device=k_cache.device)
    k_local = k_cache.index_select(0, idx).contiguous()
    v_local = v_cache.index_select(0, idx).contiguous()
    cl_local = (torch.minimum(hi * block_size, ctx) - lo * block_size).clamp(min=0)
    return (k_local, v_local, table.to(k_cache.device),
            cl_local.to(torch.int32).to(k_cache.device))


class DeviceOps:
    """The kernels of a page-split step: this package's CUDA ops.

    score_pages, select_pages; decode_unnorm(..., out=(o, m, l)) writes its
    partial into the given views of the exchange buffer; rank_merge(parts,
    B, H_kv, G, D, out, need=None) merges the all-gathered partials of the
    ranks in rank order into `out` (cvsa_rank_merge); page_lse(scores, idx,
    n) gives a rank's two coverage log-sum-exps (cvsa_page_lse) and
    rank_accept(parts, off_all, off_sel, rows, tau) the gate over the
    gathered ones (cvsa_rank_accept)."""

    def __init__(self):
        from cvsa.kernels import coverage, page_scores, select, sparse_decode
        self.score_pages = page_scores.score_pages
        self.select_pages = select.select_pages
        self.decode_unnorm = sparse_decode.sparse_decode_unnorm
        self.rank_merge = coverage.rank_merge
        self.page_lse = coverage.page_lse
        self.rank_accept = coverage.rank_accept


def run_step(gen, allgather: Callable[[torch.Tensor], torch.Tensor]):
    """Drive a step generator: each yielded 1-D tensor is all-gathered."""
    try:
        x = next(gen)
        while True:
            x = gen.send(allgather(x))
    except StopIteration as e:
        return e.value


def dist_allgather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    import torch.distributed as dist

    def ag(x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(group)
        x = x.contiguous()
        if x.is_cuda:
            out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x, group=group)
            return out
        outs = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(outs, x, group=group)
        return torch.stack(outs)
    return ag


def _pack(*ts: torch.Tensor) -> torch.Tensor:
    return torch.cat([t.reshape(-1).to(torch.float32) for t in ts])


def _unpack(flat: torch.Tensor, *shapes) -> List[torch.Tensor]:
    out, off = [], 0
    for s in shapes:
        n = 1
        for d in s:
            n *= d
        out.append(flat[..., off:off + n].reshape(flat.shape[:-1] + tuple(s)))
        off += n
    return out


def _compact(mask: torch.Tensor, values: torch.Tensor, width: int, fill):
    """Entries of `values` where `mask`, in order, left-aligned in `width` slots."""
    order = torch.argsort((~mask).to(torch.int8), dim=-1, stable=True)
    v = torch.gather(values, -1, order)[..., :width]
    m = torch.gather(mask, -1, order)[..., :width]
    return torch.where(m, v, torch.full_like(v, fill)), m.sum(-1).to(torch.int32)


class PageSplitBackend:
    """CVSA step over the pages a rank holds (see the module docstring).

    Called like CVSABackend with this rank's pool, block tables and local
    context lengths (shard_sequence), plus the global context lengths and the
    global block-table width (the budget is int(W * budget_pct), backend.py:690).
    """

    # device-side counters: the decisions never reach the host during a step,
    # and a step captured in a CUDA graph counts on every replay
    _C_SCORING, _C_ACCEPT, _C_REJECT, _C_HEADS_ACC, _C_CHECKS, _C_HEADS_TOTAL = range(6)

    def __init__(self, num_kv_heads: int, num_q_heads: int, head_dim: int, block_size: int,
                 rank: int, world: int, num_layers: int = 32, budget_pct: float = 0.10,
                 reuse_interval: int = 16, coverage_threshold: float = 0.90, lazy: bool = False,
                 check_interval: Optional[int] = None, sink_pages: int = 0, local_pages: int = 0,
                 process_group=None, ops=None):
        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.G = num_q_heads // num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.rank, self.world = rank, world
        self.num_layers = num_layers
        self.budget_pct = budget_pct
        self.reuse_interval = reuse_interval
        self.tau = coverage_threshold
        self.lazy = lazy
        self.check_interval = check_interval or 1
        self.sink_pages, self.local_pages = sink_pages, local_pages
        self.process_group = process_group
        self.ops = ops or DeviceOps()
        self._cached: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._step = 0
        self._ctr: Optional[torch.Tensor] = None

    @property
    def stats(self) -> Dict[str, int]:
        """scoring_steps, coverage_checks, accept_steps, reject_steps,
        heads_accepted, heads_total (reads the device counters)."""
        c = self._ctr.tolist() if self._ctr is not None else [0] * 6
        return dict(scoring_steps=c[self._C_SCORING], coverage_checks=c[self._C_CHECKS],
                    accept_steps=c[self._C_ACCEPT], reject_steps=c[self._C_REJECT],
                    heads_accepted=c[self._C_HEADS_ACC], heads_total=c[self._C_HEADS_TOTAL])

    def step_done(self, layer_idx: int, num_layers: int):
        if layer_idx == num_layers - 1:
            self._step += 1

    def cached_selection(self, layer_idx: int):
        """(local page indices [B, H_kv, max_sel] ascending, counts) of a layer."""
        return self._cached.get(layer_idx)

    def __call__(self, q, k_cache, v_cache, block_tables, context_lens, layer_idx,
                 global_context_lens, global_table_width):
        gen = self.step(q, k_cache, v_cache, block_tables, context_lens, layer_idx,
                        global_context_lens, global_table_width)
        return run_step(gen, dist_allgather(self.process_group))

    def _counters(self, dev) -> torch.Tensor:
        if self._ctr is None:
            self._ctr = torch.zeros(6, dtype=torch.int64, device=dev)
        return self._ctr

    # ---- the step ---------------------------------------------------------
    def step(self, q, k, v, bt, cl, layer_idx, ctx_g, W_g):
        """Generator: yields tensors to all-gather, returns the output [B, Hq, D]."""
        B, Hq, D = q.shape
        H, G, bs = self.num_kv_heads, self.G, self.block_size
        r, N = self.rank, self.world
        dev = q.device
        budget = budget_for(int(W_g), self.budget_pct)
        sink_r = self.sink_pages if r == 0 else 0
        local_r = self.local_pages if r == N - 1 else 0
        max_sel = budget + self.sink_pages + self.local_pages
        cached = self._cached.get(layer_idx)
        ctr = self._counters(dev)
        if self.lazy:
            check = self._step % self.check_interval == 0 or cached is None
        else:
            check = False
        scoring = (self._step % self.reuse_interval == 0 or cached is None) if not self.lazy \
            else check

        def attend(idx, n):
            return self.ops.decode_unnorm(q, k, v, bt, idx, n, cl, H, G, bs)

        n_part = B * Hq * (D + 2)

        def exchange_partial(idx, n, extra=()):
            """Attend (idx, n) straight into an exchange buffer ([o | m | l]
            then `extra`), all-gather it; returns the [N, stride] rows and the
            gathered extras."""
            buf = torch.empty(n_part + sum(t.numel() for t in extra), dtype=torch.float32,
                              device=dev)
            o = buf[:B * Hq * D].view(B, Hq, D)
            m = buf[B * Hq * D:B * Hq * (D + 1)].view(B, Hq)
            l = buf[B * Hq * (D + 1):n_part].view(B, Hq)
            self.ops.decode_unnorm(q, k, v, bt, idx, n, cl, H, G, bs, out=(o, m, l))
            off = n_part
            for t in extra:
                buf[off:off + t.numel()].copy_(t.reshape(-1))
                off += t.numel()
            got = yield buf
            return got, _unpack(got[:, n_part:], *[tuple(t.shape) for t in extra])

        out = torch.empty((B, Hq, D), dtype=q.dtype, device=dev)
        if not scoring and not check:                           # reuse step
            got, _ = yield from exchange_partial(*cached)
            return self.ops.rank_merge(got, B, H, G, D, out)

        # the rank's page range of every sequence (only scoring and check
        # steps need it)
        nv_g = (ctx_g.to(device=dev, dtype=torch.int64) + bs - 1) // bs
        lo, hi = page_range(nv_g, r, N)
        nv_r = hi - lo                                          # [B]
        capturing = dev.type == "cuda" and torch.cuda.is_current_stream_capturing()
        if B and not capturing and int((nv_g // N).min()) < self.sink_pages + self.local_pages:
            raise ValueError("every rank needs at least sink_pages + local_pages pages "
                             "of every sequence")
        scores = self.ops.score_pages(q, k, bt, cl, H, G, bs)          # [B, H, W_r] f32
        BH = B * H
        reuse = None            # device bool: the cached selection passed the lazy gate
        if check:
            # lazy accounting of backend.py:420-465: every check counts; a layer
            # without a cached selection counts as a reject
            ctr[self._C_CHECKS] += 1
        if check and cached is None:
            ctr[self._C_REJECT] += 1
        if check and cached is not None:
            # each rank's log-sum-exps over its pages (all, cached selection);
            # the gate takes them over the ranks
            got = yield _pack(*self.ops.page_lse(scores, *cached))
            acc0 = self.ops.rank_accept(got, 0, BH, BH, self.tau).view(B, H)
            ctr[self._C_HEADS_TOTAL] += acc0.numel()
            reuse = acc0.all()
            ctr[self._C_HEADS_ACC] += acc0.sum()
            ctr[self._C_ACCEPT] += reuse
            ctr[self._C_REJECT] += ~reuse
            ctr[self._C_SCORING] += ~reuse
        else:
            ctr[self._C_SCORING] += 1

        # ---- scoring step (gated by `reuse` on a lazy check step) ----
        # proposals: this rank's selection at the common width max_sel, page
        # order, forced and unused slots at -inf (never chosen over a page)
        idx_l, n_l = self.ops.select_pages(scores, cl, bs, budget, sink_r, local_r,
                                           max_sel=max_sel)
        pos = torch.arange(max_sel, device=dev).view(1, 1, max_sel)
        il = idx_l.long()
        forced = (il < sink_r) | (il >= (nv_r.view(B, 1, 1) - local_r))
        cand = (pos < n_l.unsqueeze(-1)) & ~forced
        cs = torch.gather(scores, -1, il.clamp(min=0)).masked_fill(~cand, NEG_INF)
        got = yield cs.reshape(-1)                              # [N, B * H * max_sel]
        # rank order then slot order: table position order is global page order
        tab_s = got.view(N, B, H, max_sel).permute(1, 2, 0, 3).reshape(B, H, N * max_sel)
        tab_s = tab_s.contiguous()
        tab_len = torch.full((B,), N * max_sel * bs, dtype=torch.int32, device=dev)
        tpos, tn = self.ops.select_pages(tab_s, tab_len, bs, budget, 0, 0)
        tp = tpos.long().clamp(min=0)
        chosen = (torch.arange(tp.shape[-1], device=dev).view(1, 1, -1) < tn.unsqueeze(-1)) \
            & torch.isfinite(torch.gather(tab_s, -1, tp))
        # my pages of the global selection (a position of my block maps to the
        # page in that slot of my proposals), with my forced pages, ascending
        mine = chosen & (tp // max_sel == r)
        loc = torch.gather(il, -1, tp % max_sel)
        sink_idx = torch.arange(sink_r, device=dev).view(1, 1, -1).expand(B, H, sink_r)
        tail = (nv_r.view(B, 1, 1) - local_r + torch.arange(local_r, device=dev).view(1, 1, -1)
                ).expand(B, H, local_r)
        all_idx = torch.cat([sink_idx, loc, tail], -1)
        all_mask = torch.cat([sink_idx >= 0, mine, tail >= 0], -1)
        idx_new, n_new = _compact(all_mask, all_idx, max_sel, 0)
        idx_new = idx_new.to(torch.int32)
        if reuse is not None:
            idx_new = torch.where(reuse, cached[0], idx_new)
            n_new = torch.where(reuse, cached[1], n_new)
        idx_new, n_new = idx_new.contiguous(), n_new.contiguous()
        got, _ = yield from exchange_partial(idx_new, n_new,
                                             self.ops.page_lse(scores, idx_new, n_new))
        self.ops.rank_merge(got, B, H, G, D, out)
        if cached is not None and cached[0].shape == idx_new.shape:
            # in place: a captured reuse step keeps reading the same buffers
            cached[0].copy_(idx_new)
            cached[1].copy_(n_new)
        else:
            self._cached[layer_idx] = (idx_new, n_new)
        acc = self.ops.rank_accept(got, n_part, n_part + BH, BH, self.tau).view(B, H)
        if not self.lazy:
            ctr[self._C_HEADS_ACC] += acc.sum()
            ctr[self._C_HEADS_TOTAL] += acc.numel()
        # exact recovery: rejected heads attend every valid page of the range
        # and their merged result replaces the draft; heads that need none
        # (accepted, or the cached selection passed the lazy gate) attend no
        # pages and keep the draft
        need = ~acc if reuse is None else ~acc & ~reuse
        Wr = scores.shape[-1]
        every = torch.arange(Wr, device=dev, dtype=torch.int32).view(1, 1, Wr).expand(B, H, Wr)
        n_rec = torch.where(need, nv_r.view(B, 1).to(torch.int32).expand(B, H),
                            torch.zeros_like(n_new))
        got, _ = yield from exchange_partial(every.contiguous(), n_rec.contiguous())
        return self.ops.rank_merge(got, B, H, G, D, out, need=need)
