"""CVSA attention backend on the B200 kernels (drop-in for cvsa/backend.py).

`CVSABackend` keeps the reference's constructor, call signature and
statistics (cvsa/backend.py:45-311) so the reference's decode loops use it
unchanged. What differs is where the work happens: each layer call is ONE
C-ABI call (cvsa_decode_step) that enqueues the whole step on the current
stream -- page scoring, top-k selection, coverage gate, sparse decode, exact
recovery and LSE merge -- with the lazy schedule's batch-global decision
(backend.py:446, `accept_mask.all()`) taken on the device. There is no host
synchronisation on the hot path, so a layer step can be captured in a CUDA
graph; statistics live in device counters read once by get_stats().

Scheduling follows the reference:
  * dense layer          -> attention over every valid page (backend.py:327-333)
  * lazy, step % M == 0  -> _lazy_step: fresh scores, gate the cached
                            selection, reuse it if every (b, h) accepts, else a
                            full scoring step (backend.py:392-465)
  * lazy, other steps    -> _reuse_step (backend.py:866-881)
  * fixed interval R     -> scoring step every R steps, reuse between
                            (backend.py:361-366)
A layer without a cached selection takes a scoring step (the reference's
_reuse_step re-enters __call__ with step - 1 for that case).

Extensions (off by default): `sink_pages` / `local_pages` always-kept pages,
the stable (score desc, page index asc) top-k order, and `process_group`:
the KV heads are sharded over the ranks of a torch.distributed group (one
process per GPU; this rank holds `num_kv_heads` of them with their
`num_q_heads` query heads), and the lazy step's batch-global decision is
all-reduced (MIN of one int32) over the group between the selection and the
attention kernels, so every rank reuses or re-selects together exactly as
one GPU holding all heads would. The reference's options that select
pages differently (selector='quest' and light_normalizer, top_p,
static_budget_table, adaptive_selection) and the random-reject
counterfactual (random_reject_prob) run as host-orchestrated steps over the
same kernels plus the Quest sketch kernel (cvsa/selectors.py), reading the
decisions on the host where the reference does. A coverage_interval below
check_interval runs the reference's coverage-only steps (backend.py:467-520):
the cached selection is gated on the page scores kept from the last scoring
step, and the host reads the decision, as the reference does. Approximate recovery (approx_recovery_pct, backend.py:780-817)
decodes each rejected head's expanded selection in the same attention
kernel; the pages-attended statistic counts the pages read (the reference
also decodes, and counts, the expanded selection of accepted heads).
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Tuple

import torch

from cvsa import _lib
from cvsa.kernels.select import budget_for


class _LayerState:
    __slots__ = ("key", "cached_idx", "cached_n", "has_cache", "accept", "accept_bool",
                 "coverage", "flags", "scores", "ckey", "kvd", "qd", "cfg", "io", "ws_bytes",
                 "scored", "has_scored")

    def __init__(self, key, B, Hkv, max_sel, W, device, keep_scores):
        self.key = key
        self.ckey = None
        self.cached_idx = torch.zeros((B, Hkv, max_sel), dtype=torch.int32, device=device)
        self.cached_n = torch.zeros((B, Hkv), dtype=torch.int32, device=device)
        self.has_cache = False
        self.accept = torch.ones((B, Hkv), dtype=torch.uint8, device=device)
        self.accept_bool = self.accept.view(torch.bool)
        self.coverage = torch.ones((B, Hkv), dtype=torch.float32, device=device)
        self.flags = torch.zeros((1,), dtype=torch.int32, device=device)
        self.scores = (torch.empty((B, Hkv, W), dtype=torch.float32, device=device)
                       if keep_scores else None)
        # page scores of the last scoring step (coverage-only steps gate on them)
        self.scored = None
        self.has_scored = False


_MODE_COVERAGE_ONLY = -100   # host-side marker: gate on cached scores, then reuse or rescore


class StepHandle:
    """A layer step in flight: `out` (final once `decision` is None) and, for
    the selection half of a phased lazy step, the int32 device word holding
    this rank's decision (bit0: every head of this rank accepted)."""
    __slots__ = ("out", "decision", "args")

    def __init__(self, out, decision, args):
        self.out = out
        self.decision = decision
        self.args = args


class CVSABackend:
    """CVSA backend: draft with sparse attention, verify with coverage, recover."""

    def __init__(
        self,
        num_kv_heads: int,
        num_q_heads: int,
        head_dim: int,
        block_size: int,
        num_layers: int = 32,
        budget_pct: float = 0.10,
        reuse_interval: int = 16,
        coverage_threshold: float = 0.90,
        dense_layers: Optional[List[int]] = None,
        lazy: bool = False,
        check_interval: Optional[int] = None,
        coverage_interval: Optional[int] = None,
        approx_recovery_pct: Optional[float] = None,
        adaptive_selection: bool = False,
        adaptive_floor_ratio: float = 0.5,
        random_reject_prob: Optional[float] = None,
        static_budget_table: Optional[Dict[int, List[float]]] = None,
        selector: str = "exact",
        top_p: Optional[float] = None,
        light_normalizer: bool = False,
        sink_pages: int = 0,
        local_pages: int = 0,
        keep_page_scores: bool = False,
        process_group=None,
        peer_exchange=None,
    ):
        # argument checks of the reference (backend.py:150-178)
        if selector not in ("exact", "quest"):
            raise ValueError(f"Unknown selector: {selector!r}")
        if light_normalizer and selector != "quest":
            raise ValueError(
                "light_normalizer=True requires selector='quest' "
                "(the sketch supplies both selection and normalizer)")
        if top_p is not None and not (0.0 < top_p < 1.0):
            raise ValueError(f"top_p must be in (0, 1), got {top_p}")
        if num_q_heads % num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if sink_pages < 0 or local_pages < 0:
            raise ValueError("sink_pages/local_pages must be >= 0")
        if approx_recovery_pct is not None and not (0.0 < approx_recovery_pct <= 1.0):
            raise ValueError(f"approx_recovery_pct must be in (0, 1], got {approx_recovery_pct}")
        alt = (selector != "exact" or light_normalizer or top_p is not None
               or static_budget_table is not None or adaptive_selection
               or random_reject_prob is not None)
        if alt and (sink_pages or local_pages):
            raise ValueError("sink_pages/local_pages apply to the uniform top-k only, "
                             "not with the reference's selector options")
        if alt and process_group is not None:
            raise ValueError("the selector options run on one GPU (no process_group)")

        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_q_per_kv = num_q_heads // num_kv_heads
        self.budget_pct = budget_pct
        self.reuse_interval = reuse_interval
        self.tau = coverage_threshold
        self._dense_layers = set(dense_layers or [])
        self.approx_recovery_pct = approx_recovery_pct
        self.lazy = lazy
        self.check_interval = check_interval or 1
        self.coverage_interval = coverage_interval or self.check_interval
        self.adaptive_selection = adaptive_selection
        self.adaptive_floor_ratio = adaptive_floor_ratio
        self.random_reject_prob = random_reject_prob
        self.static_budget_table = static_budget_table
        self.selector = selector
        self.top_p = top_p
        self.light_normalizer = light_normalizer
        self.sink_pages = sink_pages
        self.local_pages = local_pages
        self.keep_page_scores = keep_page_scores
        self.process_group = process_group
        # a cvsa.peer.PeerExchange over the same ranks: the decision word is
        # reduced by an NVLink peer-memory kernel instead of dist.all_reduce
        self.peer_exchange = peer_exchange
        self._decision_views: Dict[int, torch.Tensor] = {}  # workspace ptr -> int32 view

        self._layers: Dict[int, _LayerState] = {}
        self._ws: Dict[tuple, tuple] = {}  # (stream, private) -> (ptr, bytes, tensor)
        self._counters: Optional[torch.Tensor] = None   # int64[8] device
        self._dev_error: Optional[torch.Tensor] = None
        self._step = 0
        self._dense_layer_steps = 0
        self._last_accept_mask: Dict[int, Optional[torch.Tensor]] = {}
        self._last_expanded_selection: Dict[int, Optional[Tuple[torch.Tensor, torch.Tensor]]] = {}
        self._track_timing = False
        self._timing_events = None   # caller-owned cudaEvent_t array (bench.py)
        self._pending_events: list = []
        # the reference's buckets (backend.py:217-220) plus 'dense'; the
        # complement and the LSE merge run inside the attention kernel, so
        # their buckets stay at zero and the time counts under 'ar_recovery'
        self._kernel_times_ms = {"scoring": 0.0, "coverage": 0.0, "sparse_draft": 0.0,
                                 "ar_recovery": 0.0, "lse_merge": 0.0, "complement": 0.0,
                                 "dense": 0.0}
        self._kernel_counts = {k: 0 for k in self._kernel_times_ms}
        # the reference's selector options run as host-orchestrated steps over
        # the same kernels (cvsa/selectors.py); None: the fused C-ABI step
        self._alt = None
        if alt:
            from cvsa.selectors import AltStep
            self._alt = AltStep(self)

    # ---- bookkeeping (backend.py:225-311) -------------------------------
    def enable_timing(self, track: bool = True):
        """Per-kernel CUDA-event timing (backend.py:225-250). Buckets: 'scoring'
        (page scoring), 'coverage' (top-k selection + coverage gate),
        'sparse_draft' (attention of reuse steps), 'ar_recovery' (attention of
        scoring steps: draft + complement recovery + merge, one kernel),
        'lse_merge' and 'complement' (the reference's keys; always zero, as
        that work is fused into 'ar_recovery') and 'dense'. Recording events
        between kernels disables launch overlap."""
        self._track_timing = track

    def _flush_timing(self):
        if not self._pending_events:
            return
        torch.cuda.synchronize()
        for mode, ev in self._pending_events:
            pairs = []
            if mode in (_lib.MODE_SCORE, _lib.MODE_LAZY):
                pairs = [("scoring", _lib.EV_SCORE_BEGIN), ("coverage", _lib.EV_SELECT_BEGIN),
                         ("ar_recovery", _lib.EV_ATTEND_BEGIN)]
            elif mode == _lib.MODE_REUSE:
                pairs = [("sparse_draft", _lib.EV_ATTEND_BEGIN)]
            else:
                pairs = [("dense", _lib.EV_ATTEND_BEGIN)]
            for name, i in pairs:
                self._kernel_times_ms[name] += ev[i].elapsed_time(ev[i + 1])
                self._kernel_counts[name] += 1
        self._pending_events.clear()

    def reset(self):
        self._step = 0
        for st in self._layers.values():
            st.has_cache = False
        if self._alt is not None:
            self._alt.reset()
        self._last_accept_mask = {}
        self._last_expanded_selection = {}
        if self._counters is not None:
            self._counters.zero_()
        if self._dev_error is not None:
            self._dev_error.zero_()
        self._dense_layer_steps = 0
        for k in self._kernel_times_ms:
            self._kernel_times_ms[k] = 0.0
            self._kernel_counts[k] = 0
        self._pending_events.clear()

    @property
    def is_scoring_step(self):
        return self._step % self.reuse_interval == 0

    def step_done(self, layer_idx: int, num_layers: int):
        if layer_idx == num_layers - 1:
            self._step += 1

    def _counter_values(self) -> List[int]:
        if self._counters is None:
            return [0] * _lib.NUM_COUNTERS
        return [int(x) for x in self._counters.tolist()]

    def get_stats(self) -> dict:
        c = self._counter_values()
        scoring = c[_lib.CTR_SCORING_STEPS]
        checks = c[_lib.CTR_COVERAGE_CHECKS]
        total_checks = max(checks, scoring, 1)
        stats = {
            "total_scoring_steps": scoring,
            "total_coverage_checks": checks,
            "all_accepted_pct": c[_lib.CTR_ACCEPT_STEPS] / total_checks * 100,
            "some_rejected_pct": c[_lib.CTR_REJECT_STEPS] / total_checks * 100,
            "per_head_accept_rate": c[_lib.CTR_HEAD_ACCEPT] / max(c[_lib.CTR_HEAD_TOTAL], 1) * 100,
            "total_decode_steps": self._step,
            "lazy": self.lazy,
            "check_interval": self.check_interval if self.lazy else None,
            "rescore_rate": scoring / max(checks, 1) * 100 if self.lazy else 100.0,
            "dense_layer_steps": self._dense_layer_steps,
        }
        if c[_lib.CTR_PAGES_MAX] > 0:
            stats["effective_budget_pct"] = c[_lib.CTR_PAGES_ATTENDED] / c[_lib.CTR_PAGES_MAX] * 100
            stats["total_pages_attended"] = c[_lib.CTR_PAGES_ATTENDED]
            stats["total_pages_max"] = c[_lib.CTR_PAGES_MAX]
        if self._track_timing:
            self._flush_timing()
            n_decode = max(self._step, 1)
            stats["kernel_times_ms_total"] = dict(self._kernel_times_ms)
            stats["kernel_counts"] = dict(self._kernel_counts)
            stats["kernel_ms_per_decode_step"] = {
                k: v / n_decode for k, v in self._kernel_times_ms.items()}
        return stats

    def device_errors(self) -> int:
        """CVSA_DEV_ERR_* bits raised by the kernels so far (synchronises)."""
        return 0 if self._dev_error is None else int(self._dev_error.item())

    # ---- the step --------------------------------------------------------
    def _ensure(self, device: torch.device):
        if self._counters is None or self._counters.device != device:
            self._counters = torch.zeros((_lib.NUM_COUNTERS,), dtype=torch.int64, device=device)
            self._dev_error = torch.zeros((1,), dtype=torch.int32, device=device)

    def _layer_state(self, layer_idx, B, W, max_sel, device) -> _LayerState:
        key = (B, W, max_sel, device)
        st = self._layers.get(layer_idx)
        if st is None or st.key != key:
            cv = self._coverage_only_enabled()
            st = _LayerState(key, B, self.num_kv_heads, max_sel, W, device,
                             self.keep_page_scores or cv)
            if cv:
                st.scored = torch.empty_like(st.scores)
            self._layers[layer_idx] = st
        return st

    def _coverage_only_enabled(self) -> bool:
        return self.lazy and self.coverage_interval != self.check_interval

    def _mode_for(self, layer_idx: int, st: _LayerState) -> int:
        if layer_idx in self._dense_layers:
            return _lib.MODE_DENSE
        if self.lazy:
            if self._step % self.check_interval == 0 or not st.has_cache:
                return _lib.MODE_LAZY
            if (self._step % self.coverage_interval == 0 and st.has_scored
                    and self._coverage_only_enabled()):
                return _MODE_COVERAGE_ONLY
            return _lib.MODE_REUSE
        if self._step % self.reuse_interval == 0 or not st.has_cache:
            return _lib.MODE_SCORE
        return _lib.MODE_REUSE

    def __call__(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_tables: torch.Tensor, context_lens: torch.Tensor,
                 layer_idx: int) -> torch.Tensor:
        h = self.begin_step(q, k_cache, v_cache, block_tables, context_lens, layer_idx,
                            phased=self.process_group is not None)
        if h.decision is not None:
            exchange_decision(h.decision, self.process_group, self.peer_exchange)
            self.finish_step(h)
        return h.out

    def begin_step(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   block_tables: torch.Tensor, context_lens: torch.Tensor, layer_idx: int,
                   phased: bool = False) -> "StepHandle":
        """Enqueue a layer step. With `phased` a lazy check step stops after
        the selection: the handle's `decision` is the device word to combine
        over the ranks holding the other KV heads (MIN), and finish_step runs
        the attention. Other steps (and phased=False) run whole; their handle
        has decision None and `out` is final."""
        self._last_accept_mask.pop(layer_idx, None)
        self._last_expanded_selection.pop(layer_idx, None)
        if q.dim() == 4:
            q = q.squeeze(1)
        dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, context_lens)
        self._ensure(dev)
        if self._alt is not None and layer_idx not in self._dense_layers:
            bt_a = block_tables if block_tables.dtype == torch.int32 else \
                block_tables.to(torch.int32)
            cl_a = context_lens if context_lens.dtype == torch.int32 else \
                context_lens.to(torch.int32)
            out = self._alt(q.contiguous(), k_cache, v_cache, bt_a.contiguous(),
                            cl_a.contiguous(), layer_idx)
            return StepHandle(out, None, None)
        B, Hq, D = q.shape
        W = block_tables.shape[1]
        budget = budget_for(W, self.budget_pct)
        max_sel = budget + self.sink_pages + self.local_pages
        st = self._layer_state(layer_idx, B, W, max_sel, dev)
        mode = self._mode_for(layer_idx, st)
        if mode == _MODE_COVERAGE_ONLY:
            mode = self._coverage_only(st, layer_idx)
        if mode == _lib.MODE_DENSE:
            self._dense_layer_steps += 1

        q = q.contiguous()
        bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
        cl = context_lens if context_lens.dtype == torch.int32 else context_lens.to(torch.int32)
        bt = bt.contiguous()
        cl = cl.contiguous()
        out = torch.empty_like(q)
        lib = _lib.load()
        stream = _lib.stream_ptr(dev)
        # descriptors are rebuilt (and validated) only when the caller's
        # tensors change; decode loops pass the same cache and tables each step
        ckey = (k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape, k_cache.stride(),
                k_cache.dtype, bt.data_ptr(), cl.data_ptr(), q.shape, q.dtype, stream)
        if st.ckey != ckey:
            st.kvd = _lib.kv_desc(k_cache, v_cache)
            st.qd = _lib.query_desc(q, bt, cl)
            if self.approx_recovery_pct is None:
                recovery, exp_budget = _lib.RECOVERY_EXACT, 0
            else:
                # backend.py:782-783
                recovery = _lib.RECOVERY_APPROX
                exp_budget = min(max(budget + 1, int(W * self.approx_recovery_pct)), W)
            st.cfg = _lib.StepConfig(mode, budget, self.sink_pages, self.local_pages,
                                     float(self.tau), recovery, 0, 1 if self.lazy else 0,
                                     exp_budget)
            st.io = _lib.StepIO(st.cached_idx.data_ptr(), st.cached_n.data_ptr(), max_sel, 0,
                                out.data_ptr(), _lib.ptr(st.scores), st.accept.data_ptr(),
                                st.coverage.data_ptr(), self._counters.data_ptr(),
                                st.flags.data_ptr(), self._dev_error.data_ptr())
            st.ws_bytes = lib.cvsa_step_workspace_size(st.qd, st.kvd, st.cfg, max_sel)
            st.ckey = ckey
        kvd, qd, cfg, io = st.kvd, st.qd, st.cfg, st.io
        qd.q = q.data_ptr()
        io.out = out.data_ptr()
        io.timing_events = None
        cfg.mode = mode
        cfg.has_cache = 1 if st.has_cache else 0
        ws = self._workspace(st.ws_bytes, dev, stream, private=phased)
        events = None
        if self._timing_events is not None:
            io.timing_events = ctypes.cast(self._timing_events, ctypes.c_void_p)
        elif self._track_timing:
            events = [torch.cuda.Event(enable_timing=True) for _ in range(_lib.NUM_EVENTS)]
            for e in events:
                e.record()      # torch creates the cudaEvent_t at its first record
            arr = (ctypes.c_void_p * _lib.NUM_EVENTS)(*[e.cuda_event for e in events])
            io.timing_events = ctypes.cast(arr, ctypes.c_void_p)
        # the handle holds every tensor the descriptors point at (q and the
        # tables may be fresh contiguous copies): the attention half of a
        # phased step runs after this call returns, and a tensor freed here
        # could be handed to work enqueued before it
        handle = StepHandle(out, None, (qd, kvd, cfg, io, ws, stream, out.data_ptr(),
                                        (q, bt, cl, k_cache, v_cache)))
        if phased and mode == _lib.MODE_LAZY:
            # heads sharded over ranks: the lazy decision is exchanged between
            # the selection and the attention halves of the step
            io.phase = _lib.PHASE_SELECT
            rc = lib.cvsa_decode_step(qd, kvd, cfg, io, ws[0], ws[1], stream)
            io.phase = _lib.PHASE_ALL
            if rc:
                _lib.check(rc, "cvsa_decode_step (select)")
            handle.decision = self._decision_view(ws)
        else:
            rc = lib.cvsa_decode_step(qd, kvd, cfg, io, ws[0], ws[1], stream)
            if rc:
                _lib.check(rc, "cvsa_decode_step")
        if events is not None:
            self._pending_events.append((mode, events))
        if mode in (_lib.MODE_SCORE, _lib.MODE_LAZY):
            st.has_cache = True
            self._last_accept_mask[layer_idx] = st.accept_bool
            if st.scored is not None:
                # keep this step's scores if it rescored (step_flags bit1), as
                # the reference caches page_scores in _scoring_step only
                # (backend.py:713); decided on the device
                rescored = (st.flags & 2).bool()
                torch.where(rescored, st.scores, st.scored, out=st.scored)
                st.has_scored = True
        return handle

    def _coverage_only(self, st: _LayerState, layer_idx: int) -> int:
        """backend.py:467-520: gate the cached selection on the page scores of
        the last scoring step, without scoring. Returns the step to run:
        REUSE if every head accepts, else SCORE (fresh scores). The decision is
        read on the host, as the reference does (`accept_mask.all()`)."""
        from cvsa.kernels.coverage import check_coverage
        acc, _cov = check_coverage(st.scored, st.cached_idx, st.cached_n, self.tau)
        c = self._counters
        c[_lib.CTR_HEAD_ACCEPT] += acc.sum()
        c[_lib.CTR_HEAD_TOTAL] += acc.numel()
        c[_lib.CTR_COVERAGE_CHECKS] += 1
        if bool(acc.all()):
            c[_lib.CTR_ACCEPT_STEPS] += 1
            self._last_accept_mask[layer_idx] = acc
            return _lib.MODE_REUSE
        c[_lib.CTR_REJECT_STEPS] += 1
        return _lib.MODE_SCORE

    def finish_step(self, h: "StepHandle") -> torch.Tensor:
        """Run the attention half of a phased step (after its decision word
        holds the combined decision); returns the step's output."""
        if h.decision is None:
            return h.out
        qd, kvd, cfg, io, ws, stream, out_ptr, _alive = h.args
        io.phase = _lib.PHASE_ATTEND
        io.out = out_ptr
        rc = _lib.load().cvsa_decode_step(qd, kvd, cfg, io, ws[0], ws[1], stream)
        io.phase = _lib.PHASE_ALL
        if rc:
            _lib.check(rc, "cvsa_decode_step (attend)")
        h.decision = None
        h.args = None
        return h.out

    def _decision_view(self, ws) -> torch.Tensor:
        """int32 view of the workspace's lazy-decision word (cvsa_step_decision_word)."""
        view = self._decision_views.get(ws[0])
        if view is None:
            word = ctypes.c_void_p()
            _lib.check(_lib.load().cvsa_step_decision_word(ws[0], ctypes.byref(word)),
                       "cvsa_step_decision_word")
            off = word.value - ws[0]
            view = ws[2][off:off + 4].view(torch.int32)
            self._decision_views[ws[0]] = view
        return view

    def _workspace(self, nbytes: int, dev: torch.device, stream: int, private: bool = False):
        """(pointer, bytes, tensor) of a zeroed 256-aligned workspace for this
        stream. Whole steps run one after another in stream order, so backends
        share one; a phased step keeps its selection in the workspace until its
        attention half, so it takes one of its own."""
        key = (stream, private)
        ws = self._ws.get(key)
        if ws is None or ws[1] < nbytes:
            tag = f"step-{stream}" + (f"-{id(self)}" if private else "")
            buf = _lib.WORKSPACE.get(nbytes, dev, tag)
            ws = (buf.data_ptr(), buf.numel(), buf)
            self._ws[key] = ws
        return ws

    # ---- tracing helpers -------------------------------------------------
    def cached_selection(self, layer_idx: int) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        """(page_indices [B,H_kv,max_sel], n_per_head) cached for a layer: ascending
        page order, or score order for the per-head-budget selectors."""
        if self._alt is not None and layer_idx in self._alt.cached:
            return self._alt.cached[layer_idx]
        st = self._layers.get(layer_idx)
        if st is None or not st.has_cache:
            return None
        return st.cached_idx, st.cached_n

    def last_step_flags(self, layer_idx: int) -> Optional[torch.Tensor]:
        """Device word: bit0 every head accepted, bit1 the selection was rescored."""
        st = self._layers.get(layer_idx)
        return None if st is None else st.flags


def exchange_decision(decision: torch.Tensor, group, peer=None) -> torch.Tensor:
    """All-reduce the lazy decision word over `group` (MIN: bit0 stays set only
    if every rank's heads all accepted their cached selection), in place, in
    stream order. backend.py:446 takes `accept_mask.all()` over every head of
    the batch; with the heads sharded over ranks that is this reduction. With
    `peer` (a cvsa.peer.PeerExchange over the same ranks) it is one NVLink
    peer-memory kernel (cvsa_peer_min_i32)."""
    if peer is not None:
        return peer.min_i32(decision)
    import torch.distributed as dist
    dist.all_reduce(decision, op=dist.ReduceOp.MIN, group=group)
    return decision


def shard_heads(num_kv_heads: int, num_q_heads: int, rank: int, world: int) -> Tuple[slice, slice]:
    """KV heads and query heads rank `rank` of `world` holds: contiguous equal
    blocks, query heads following their KV heads (GQA groups stay whole)."""
    if num_kv_heads % world or num_q_heads % num_kv_heads:
        raise ValueError(f"{num_kv_heads} KV heads do not shard over {world} ranks")
    per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    return slice(rank * per, (rank + 1) * per), slice(rank * per * g, (rank + 1) * per * g)
