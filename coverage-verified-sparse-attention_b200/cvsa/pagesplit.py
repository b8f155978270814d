"""Page-split CVSA step: each rank holds a contiguous range of every
sequence's pages (one long sequence spread over GPUs, config 3 across ranks).

The reference has no multi-GPU path; this follows its single-GPU semantics
(cvsa/backend.py:683-864 scoring step, :392-465 lazy step, :866-881 reuse)
with the selection, the coverage sums and the attention partials combined
over the ranks in two exchanges:

  1. every rank scores its pages and writes one exchange row
     (cvsa_split_propose): its log-sum-exps over all its pages, over its part
     of the cached selection (the lazy gate) and over its forced pages (the
     sink pages live on rank 0, the local pages on the last rank), and its
     best `budget` non-forced candidates' scores in page order. All-gather A.
  2. from the gathered rows every rank takes the same decisions
     (cvsa_split_gate): the lazy gate of the cached selection and the batch
     decision; the global top-`budget` of the candidates (score descending,
     page ascending; rows concatenate in rank order, so position order is
     page order) and its coverage gate; it keeps its own share of the new
     selection (sink, its chosen pages, local) in ascending page order.
  3. every rank attends its share (cvsa_split_attend): the cached selection
     when every head accepted it, else the new one; a head whose new gate
     rejected attends every valid page of the rank, which over the ranks is
     the exact recovery of backend.py:818-844 (draft and complement
     together). All-gather B of the partials (o, m, l); every rank merges
     them in rank order (cvsa_rank_merge).
A reuse step attends the cached selection and needs only exchange B.

No step reads a device value on the host: the lazy decision and the accept
masks stay on the device and gate the work instead of branching around it,
and the counters are device tensors. The launches and exchanges of a step
depend only on its host-known kind (first, check, reuse), so a layer's steps
can be captured in CUDA graphs, NCCL all-gathers included, and every rank
issues the same collectives.

A step is a generator that yields each 1-D float32 tensor to all-gather and
receives the [world, n] result; `run_step` drives it with torch.distributed,
and tests can drive the ranks of one process in lockstep. With an `exchange`
(cvsa.peer.PeerExchange) the step yields nothing: exchange A is an all-gather
kernel over NVLink peer memory and exchange B one kernel that pushes the
partials and merges them.
"""

from typing import Callable, Dict, Optional, Tuple

import torch

from cvsa.kernels.select import budget_for

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

    score_pages; split_propose / split_gate / split_attend (cvsa_split_*,
    see the module docstring); decode_unnorm(..., out=(o, m, l)) for reuse
    steps writes its partial into the given views of the exchange buffer;
    rank_merge(parts, B, H_kv, G, D, out) merges the all-gathered partials of
    the ranks in rank order into `out` (cvsa_rank_merge)."""

    def __init__(self):
        from cvsa.kernels import coverage, page_scores, sparse_decode, split
        self.score_pages = page_scores.score_pages
        self.split_propose = split.split_propose
        self.split_gate = split.split_gate
        self.split_attend = split.split_attend
        self.decode_unnorm = sparse_decode.sparse_decode_unnorm
        self.rank_merge = coverage.rank_merge


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


class PageSplitBackend:
    """CVSA step over the pages a rank holds (see the module docstring).

    Called like CVSABackend with this rank's pool, block tables and local
    context lengths (shard_sequence), plus the global context lengths and the
    global block-table width (the budget is int(W * budget_pct), backend.py:690).
    """

    # device-side counters (CVSA_SPLIT_CTR_* order), accumulated by
    # cvsa_split_gate: the decisions never reach the host during a step, and
    # a step captured in a CUDA graph counts on every replay
    _C_SCORING, _C_ACCEPT, _C_REJECT, _C_HEADS_ACC, _C_CHECKS, _C_HEADS_TOTAL = range(6)

    def __init__(self, num_kv_heads: int, num_q_heads: int, head_dim: int, block_size: int,
                 rank: int, world: int, num_layers: int = 32, budget_pct: float = 0.10,
                 reuse_interval: int = 16, coverage_threshold: float = 0.90, lazy: bool = False,
                 check_interval: Optional[int] = None, sink_pages: int = 0, local_pages: int = 0,
                 process_group=None, ops=None, exchange=None):
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
        # a cvsa.peer.PeerExchange: the two exchanges and the merge run as
        # NVLink peer-memory kernels instead of yielding to an all-gather
        self.exchange = exchange
        self._cached: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._step = 0
        self._ctr: Optional[torch.Tensor] = None
        self._gate_state: Optional[torch.Tensor] = None

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

    @staticmethod
    def exchange_row_cap(batch: int, num_kv_heads: int, num_q_heads: int, head_dim: int,
                         max_sel: int) -> int:
        """Floats a PeerExchange for this backend must carry per rank: the
        larger of the proposal row and the partial row."""
        rows = batch * num_kv_heads
        return max(3 * rows + rows * max_sel, batch * num_q_heads * (head_dim + 2))

    def _counters(self, dev) -> torch.Tensor:
        if self._ctr is None:
            self._ctr = torch.zeros(6, dtype=torch.int64, device=dev)
        return self._ctr

    def _state(self, dev) -> torch.Tensor:
        """int32 [4] of cvsa_split_gate: CTA tickets and accept counts (left
        zeroed), the decision word (state[3], bit0: the cached selection is
        decoded)."""
        if self._gate_state is None:
            self._gate_state = torch.zeros(4, dtype=torch.int32, device=dev)
        return self._gate_state

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
        if cached is not None and tuple(cached[0].shape) != (B, H, max_sel):
            cached = None                   # another batch: no selection to reuse
        ctr = self._counters(dev)
        if self.lazy:
            check = self._step % self.check_interval == 0 or cached is None
        else:
            check = False
        scoring = (self._step % self.reuse_interval == 0 or cached is None) if not self.lazy \
            else check

        n_part = B * Hq * (D + 2)
        buf = torch.empty(n_part, dtype=torch.float32, device=dev)   # exchange B
        o = buf[:B * Hq * D].view(B, Hq, D)
        m = buf[B * Hq * D:B * Hq * (D + 1)].view(B, Hq)
        l = buf[B * Hq * (D + 1):].view(B, Hq)
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=dev)
        if not scoring and not check:                           # reuse step
            self.ops.decode_unnorm(q, k, v, bt, cached[0], cached[1], cl, H, G, bs,
                                   out=(o, m, l))
            if self.exchange is not None:
                return self.exchange.merge(buf, B, H, G, D, out)
            got = yield buf
            return self.ops.rank_merge(got, B, H, G, D, out)

        capturing = dev.type == "cuda" and torch.cuda.is_current_stream_capturing()
        if B and not capturing:
            nv_g = (ctx_g.to(torch.int64) + bs - 1) // bs
            if int((nv_g // N).min()) < self.sink_pages + self.local_pages:
                raise ValueError("every rank needs at least sink_pages + local_pages pages "
                                 "of every sequence")
        scores = self.ops.score_pages(q, k, bt, cl, H, G, bs)          # [B, H, W_r] f32
        W_r = scores.shape[-1]
        has_cache = check and cached is not None
        stats_mode = (1 if check else 0) | (2 if self.lazy else 0)
        row = torch.empty(3 * B * H + B * H * max_sel, dtype=torch.float32, device=dev)
        prop = self.ops.split_propose(scores, cl, bs, cached if has_cache else None, sink_r,
                                      local_r, budget, max_sel, row)
        if self.exchange is not None:
            got = self.exchange.allgather(row)                  # exchange A
        else:
            got = yield row                                     # exchange A
        state = self._state(dev)
        sel, n, acc, bitmap = self.ops.split_gate(got, prop, cl, bs, W_r, r, budget, max_sel,
                                                  sink_r, local_r, self.tau, has_cache,
                                                  stats_mode, state, ctr)
        if cached is None:
            cached = (torch.zeros((B, H, max_sel), dtype=torch.int32, device=dev),
                      torch.zeros((B, H), dtype=torch.int32, device=dev))
            self._cached[layer_idx] = cached
        # decodes (and, when chosen, commits in place) the new selection;
        # a captured reuse step keeps reading the same cache buffers
        self.ops.split_attend(q, k, v, bt, cl, H, G, bs, cached, sel, n,
                              state[3:4] if has_cache else None, acc, bitmap, out=(o, m, l))
        if self.exchange is not None:
            return self.exchange.merge(buf, B, H, G, D, out)   # exchange B and merge
        got = yield buf                                         # exchange B
        return self.ops.rank_merge(got, B, H, G, D, out)
