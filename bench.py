"""bench.py -- CVSA decode step on B200 (one JSON line from rank 0).

Workload (N=1): BASELINE config 2 -- Llama-3.1-8B attention geometry, B=32
sequences of 8192 tokens (512 pages of 16), Hq=32, Hkv=8, D=128, bf16 paged
KV with a permuted page table, budget 5 % (25 pages) + 3 forced pages,
tau=0.9, lazy schedule M=4 (page scoring + coverage gate every 4 steps,
selection reuse between), over 32 layers with 32 independent KV pools
(1.07 GB of K+V each, so every layer's inputs exceed the 126 MB L2).
Synthetic seeded data (no checkpoints, no datasets).

A step is one decode step through all 32 layers (`CVSABackend.__call__` per
layer, i.e. one cvsa_decode_step C-ABI call per layer). The metric is the
achieved HBM bandwidth on the KV bytes the CVSA algorithm reads (whole job,
GB/s): scoring steps read every valid page's K, every step reads the selected
pages' K+V, and recovery reads the complement pages' K+V of rejected heads;
the per-layer step time (us/layer) is reported beside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cvsa|reference]

--impl reference times the reference's algorithm on the host cores: the
pure-PyTorch restatement in oracle/cvsa_ref.py (the reference itself is
Triton + PyTorch and cannot run without its GPU kernels), on a bounded sample
of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "coverage-verified-sparse-attention_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

M_INTERVAL = 4
LAYERS = 32
KP_BYTES = 16 * 128 * 2        # one K (or V) page of one KV head, bf16
METRIC = "CVSA decode-step achieved HBM GB/s on algorithmic KV bytes (config 2, 8K ctx)"
WORKLOAD = ("config2: Llama-3.1-8B attention, B=32, Hq=32, Hkv=8, D=128, bf16, ctx=8192 "
            "(512 pages x 16), budget 5% (25) + sink 1 + local 2, tau=0.9, lazy M=4, "
            "32 layers with independent pools")


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU, sampled
    through NVML every 2 ms from a thread while the timed region runs, plus
    one sample when it starts and one when it ends (the config-2 region is
    about 15 ms, shorter than nvidia-smi's sampling period). The GPU is found
    by UUID, so CUDA_VISIBLE_DEVICES cannot point it at another device;
    without NVML, nvidia-smi is polled instead."""

    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.nv = None
        self.handle = None
        self.samples = []        # (sm_mhz, reason bits)
        self.smax = None
        self.proc = None
        self.lines = []
        self.t = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            try:
                uuid = str(torch.cuda.get_device_properties(index).uuid)
                uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nv = None

    def _sample(self):
        nv, h = self.nv, self.handle
        try:
            fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), int(fn(h))))
        except Exception:
            pass

    def _poll(self):
        while not self._stop.wait(0.002):
            self._sample()

    def start(self):
        if self.nv is not None:
            self._sample()
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nv is not None:
            self._stop.set()
            self.t.join(timeout=5)
            self._sample()
            sm = [c for c, _ in self.samples]
            bits = 0
            for _, r in self.samples:
                bits |= r
            reasons = sorted(nm for bit, nm in self.REASONS.items() if bits & bit)
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                    "reasons": reasons, "samples": len(sm), "source": "NVML, 2 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return ws, rank, local


def _barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _scoring_pages(context_lens, hkv):
    nv = (context_lens.to(torch.int64) + 15) // 16
    return int(nv.sum()) * hkv


# ----------------------------------------------------------------------------
# reference (CPU) arm
# ----------------------------------------------------------------------------

class CpuSample:
    """The oracle restatement of the reference path, timed on the host cores.

    Sample: one layer of config 2 (all 32 sequences, 8K context) under the
    lazy M=4 schedule, in the reference's fp32 arithmetic, with every host
    thread. A CPU "step" is one M=4 cycle (lazy check step + 3 reuse steps).
    """

    def __init__(self, threads: int = None):
        from cvsa import synthetic
        from oracle import cvsa_ref as R

        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.wl = synthetic.config2(device="cpu", seed=123)
        wl = self.wl
        self.be = R.OracleBackend(8, 32, 128, 16, num_layers=1, budget_pct=wl.budget_pct,
                                  coverage_threshold=wl.tau, lazy=True,
                                  check_interval=M_INTERVAL, sink_pages=1, local_pages=2,
                                  precise=False)

    def cycle(self):
        """Run one M=4 cycle; returns (seconds, algorithmic KV bytes)."""
        wl, be = self.wl, self.be
        w0, lazy0 = be.attn_work, be.total_coverage_checks
        t0 = time.perf_counter()
        for _ in range(M_INTERVAL):
            be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
            be.step_done(0, 1)
        dt = time.perf_counter() - t0
        pages = be.attn_work - w0
        lazy = be.total_coverage_checks - lazy0
        nbytes = pages * 2 * KP_BYTES + lazy * _scoring_pages(wl.context_lens, 8) * KP_BYTES
        return dt, nbytes


CPU_SAMPLE_DESC = ("one layer of config 2 (all 32 sequences, 8K ctx) under the lazy M=4 schedule, "
                   "one M=4 cycle (lazy check + 3 reuse steps) per step, fp32 torch restatement "
                   "of the reference on CPU")


def run_reference(args, ws, rank):
    if rank != 0:
        return
    cs = CpuSample()
    threads = cs.threads
    for _ in range(args.warmup):
        cs.cycle()
    tot_t, tot_b = 0.0, 0
    for _ in range(args.steps):
        dt, nb = cs.cycle()
        tot_t += dt
        tot_b += nb
    value = tot_b / tot_t / 1e9
    sample = CPU_SAMPLE_DESC
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": sample},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# CUDA arm
# ----------------------------------------------------------------------------

def build_layers(dev, layers):
    from cvsa import synthetic
    wls = []
    for l in range(layers):
        wls.append(synthetic.config2(device=dev, seed=1000 + l, gen_device=str(dev)))
    torch.cuda.synchronize()
    return wls


C3_LAYERS = 16


def measure_config3(dev, steps, warmup, ws):
    """Config 3 (single 128K sequence, Llama-8B geometry, 5 % budget): the same
    graph-captured lazy M=4 schedule over C3_LAYERS independent layers (537 MB of
    K+V each). Returns the achieved GB/s on algorithmic KV bytes and us/layer."""
    from cvsa import _lib, synthetic
    from cvsa.backend import CVSABackend

    wls = [synthetic.config3(device=dev, seed=3000 + l, gen_device=str(dev))
           for l in range(C3_LAYERS)]
    torch.cuda.synchronize()
    B, Hq, D = wls[0].q.shape
    hkv = wls[0].num_kv_heads
    scoring = sum(_scoring_pages(wl.context_lens, hkv) * KP_BYTES for wl in wls)
    be = CVSABackend(hkv, Hq, D, 16, num_layers=C3_LAYERS, budget_pct=0.05,
                     coverage_threshold=0.9, lazy=True, check_interval=M_INTERVAL,
                     sink_pages=1, local_pages=2)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = {}
    with torch.cuda.stream(side):
        for _ in range(warmup):
            for l, wl in enumerate(wls):
                be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
                be.step_done(l, C3_LAYERS)
        side.synchronize()
        for kind, step_idx in (("lazy", 0), ("reuse", 1)):
            g = torch.cuda.CUDAGraph()
            be._step = step_idx
            with torch.cuda.graph(g, stream=side):
                for l, wl in enumerate(wls):
                    be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
            graphs[kind] = g
    torch.cuda.current_stream(dev).wait_stream(side)
    for s in range(M_INTERVAL):
        graphs["lazy" if s % M_INTERVAL == 0 else "reuse"].replay()
    torch.cuda.synchronize()
    lazy_steps = sum(1 for s in range(steps) if s % M_INTERVAL == 0)
    _barrier(ws)
    torch.cuda.synchronize()
    c0 = be._counter_values()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        graphs["lazy" if s % M_INTERVAL == 0 else "reuse"].replay()
    e1.record()
    torch.cuda.synchronize()
    _barrier(ws)
    ms = _max_over_ranks(e0.elapsed_time(e1), ws)
    c1 = be._counter_values()
    pages = c1[_lib.CTR_PAGES_ATTENDED] - c0[_lib.CTR_PAGES_ATTENDED]
    nbytes = _sum_over_ranks(float(pages * 2 * KP_BYTES + lazy_steps * scoring), ws)
    stats = be.get_stats()
    del graphs
    return {"workload": "config3: B=1, Hq=32, Hkv=8, D=128, bf16, ctx=131072 (8192 pages), "
                        f"budget 5% (409) + sink 1 + local 2, tau=0.9, lazy M=4, {C3_LAYERS} "
                        "layers with independent pools (537 MB K+V each)",
            "value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "us_per_layer": ms * 1e3 / (steps * C3_LAYERS), "steps": steps,
            "per_head_accept_rate": stats.get("per_head_accept_rate")}


C4_LAYERS = 80
C4_POOLS = 16


def measure_config4(dev, steps, warmup, ws, rank):
    """Config 4 (Llama-70B attention: B=8, Hq=64, Hkv=8, D=128, ctx 32768, 80
    layers), KV heads sharded over the ranks: rank r holds KV heads
    [8r/N, 8(r+1)/N) and their query heads, and the lazy check step reduces
    the batch-global decision (one int32, MIN, an NVLink peer-memory kernel)
    between its selection and attention halves. Layer l reads pool l % C4_POOLS (each pool 1.07 GB / N of
    K+V, so consecutive uses of a pool are 15 pools apart, far beyond L2). The
    lazy-check and reuse steps are captured as CUDA graphs (the all-reduce
    inside) and timed separately; times are the max over ranks."""
    from cvsa import _lib, synthetic
    from cvsa.backend import CVSABackend, shard_heads

    kv_s, q_s = shard_heads(8, 64, rank, ws)
    pools = [synthetic.config4(device=dev, kv_heads=kv_s, seed=4000 + i)
             for i in range(C4_POOLS)]
    torch.cuda.synchronize()
    B, Hq, D = pools[0].q.shape
    hkv = pools[0].num_kv_heads
    pg = None
    if ws > 1:
        import torch.distributed as dist
        pg = dist.group.WORLD
    px = None
    if ws > 1:
        from cvsa.peer import PeerExchange
        px = PeerExchange(4, group=pg, device=dev)
    be = CVSABackend(hkv, Hq, D, 16, num_layers=C4_LAYERS, budget_pct=0.05,
                     coverage_threshold=0.9, lazy=True, check_interval=M_INTERVAL,
                     sink_pages=1, local_pages=2, process_group=pg, peer_exchange=px)

    def step():
        for l in range(C4_LAYERS):
            wl = pools[l % C4_POOLS]
            be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
            be.step_done(l, C4_LAYERS)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs, launch = {}, ("CUDA graph per step kind (the decision's NVLink peer-memory MIN "
                          "kernel inside the lazy-check graph)")
    with torch.cuda.stream(side):
        for _ in range(max(warmup, M_INTERVAL)):
            step()
        side.synchronize()
        ok = 1
        try:
            for kind, step_idx in (("lazy", 0), ("reuse", 1)):
                g = torch.cuda.CUDAGraph()
                be._step = step_idx
                with torch.cuda.graph(g, stream=side):
                    for l in range(C4_LAYERS):
                        wl = pools[l % C4_POOLS]
                        be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
                graphs[kind] = g
        except Exception:  # noqa: BLE001 - capture unsupported here: time eager steps
            ok = 0
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = int(t.item())
    if not ok:
        graphs = {}
        launch = "eager (graph capture of the collective failed)"

    def run(kind, n):
        be._step = 0 if kind == "lazy" else 1
        if graphs:
            graphs[kind].replay()
            for _ in range(n - 1):
                graphs[kind].replay()
        else:
            for _ in range(n):
                be._step = 0 if kind == "lazy" else 1
                for l in range(C4_LAYERS):
                    wl = pools[l % C4_POOLS]
                    be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)

    res = {}
    n = max(steps // 2, 2)
    for kind in ("lazy", "reuse"):
        run(kind, 1)
        torch.cuda.synchronize()
        _barrier(ws)
        c0 = be._counter_values()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        run(kind, n)
        e1.record()
        torch.cuda.synchronize()
        _barrier(ws)
        ms = _max_over_ranks(e0.elapsed_time(e1), ws)
        c1 = be._counter_values()
        pages = c1[_lib.CTR_PAGES_ATTENDED] - c0[_lib.CTR_PAGES_ATTENDED]
        scoring = (n * C4_LAYERS * _scoring_pages(pools[0].context_lens, hkv) * KP_BYTES
                   if kind == "lazy" else 0)
        per_rank_bytes = float(pages * 2 * KP_BYTES + scoring)
        res[kind] = (ms * 1e3 / (n * C4_LAYERS), _sum_over_ranks(per_rank_bytes, ws) / (ms * 1e-3) / 1e9)
    stats = be.get_stats()
    del graphs
    if px is not None:
        torch.cuda.synchronize()
        if int(px.dev_error.item()):
            launch += "; peer exchange reported a timeout"
        px.close()
    us_layer = (res["lazy"][0] + (M_INTERVAL - 1) * res["reuse"][0]) / M_INTERVAL
    step_s = us_layer * C4_LAYERS * 1e-6
    gbs = (res["lazy"][1] * res["lazy"][0] + (M_INTERVAL - 1) * res["reuse"][1] * res["reuse"][0]) / (
        M_INTERVAL * us_layer)
    return {"workload": "config4: Llama-70B attention, B=8, Hq=64, Hkv=8, D=128, bf16, ctx=32768 "
                        "(2048 pages), budget 5% (102) + sink 1 + local 2, tau=0.9, lazy M=4, "
                        f"{C4_LAYERS} layers over {C4_POOLS} rotating pools",
            "parallelism": f"KV heads sharded over {ws} GPU(s): {hkv} KV + {Hq} query heads each",
            "launch": launch,
            "us_per_layer_lazy_check": res["lazy"][0], "us_per_layer_reuse": res["reuse"][0],
            "us_per_layer": us_layer, "tokens_per_s": B / step_s,
            "value": gbs, "unit": "GB/s (all GPUs, algorithmic KV bytes)",
            "frac_of_peak": gbs / (_peaks()[0] * ws),
            "per_head_accept_rate_rank0": stats.get("per_head_accept_rate")}


C3S_LAYERS = 4


def measure_config3_split(dev, steps, ws, rank, peer=False):
    """Config 3 (one 128K sequence) with its pages split over the ranks
    (cvsa.pagesplit): every rank scores, proposes and attends its contiguous
    page range; the proposal rows (candidates and coverage sums) and the
    attention partials are all-gathered (NCCL, two per lazy-check step, one
    per reuse step) and merged in rank order. Lazy M=4 over C3S_LAYERS layers; the lazy-check
    step and the reuse step (all layers each) are captured as CUDA graphs with
    the all-gathers inside and timed separately; times are the max over
    ranks."""
    from cvsa import synthetic
    from cvsa.pagesplit import PageSplitBackend, dist_allgather, run_step, shard_sequence

    pools = []
    for l in range(C3S_LAYERS):
        wl = synthetic.config3(device=dev, seed=3000 + l, gen_device=str(dev))
        k, v, bt, cl = shard_sequence(wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens,
                                      rank, ws, 16)
        pools.append((wl.q, k, v, bt, cl, wl.context_lens, wl.block_tables.shape[1]))
        del wl
    torch.cuda.synchronize()
    pg = None
    if ws > 1:
        import torch.distributed as dist
        pg = dist.group.WORLD
    px = None
    if peer and ws > 1:
        from cvsa.kernels.select import budget_for
        from cvsa.peer import PeerExchange
        W = pools[0][6]
        max_sel = budget_for(int(W), 0.05) + 3
        px = PeerExchange(PageSplitBackend.exchange_row_cap(1, 8, 32, 128, max_sel), group=pg,
                          device=dev)
    pb = PageSplitBackend(8, 32, 128, 16, rank, ws, num_layers=C3S_LAYERS, budget_pct=0.05,
                          coverage_threshold=0.9, lazy=True, check_interval=M_INTERVAL,
                          sink_pages=1, local_pages=2, process_group=pg, exchange=px)
    if ws > 1:
        ag = dist_allgather(pg)
    else:
        def ag(x):
            return x.unsqueeze(0)

    def one_step():
        for l, (q, k, v, bt, cl, ctx, W) in enumerate(pools):
            run_step(pb.step(q, k, v, bt, cl, l, ctx, W), ag)
            pb.step_done(l, C3S_LAYERS)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = {}
    with torch.cuda.stream(side):
        for _ in range(M_INTERVAL + 1):
            one_step()
        side.synchronize()
        # the eager warm-up steps' counts (a replayed graph advances only the
        # device-side counters)
        stats = pb.stats
        ok = 1
        try:
            for kind, step_idx in (("check", 0), ("reuse", 1)):
                g = torch.cuda.CUDAGraph()
                pb._step = step_idx
                with torch.cuda.graph(g, stream=side):
                    for l, (q, k, v, bt, cl, ctx, W) in enumerate(pools):
                        run_step(pb.step(q, k, v, bt, cl, l, ctx, W), ag)
                graphs[kind] = g
        except Exception:  # noqa: BLE001 - capture unsupported here: time eager steps
            ok = 0
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    if ws > 1:
        t = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = int(t.item())
    if not ok:
        graphs = {}

    def run(kind, n):
        for _ in range(n):
            if graphs:
                graphs[kind].replay()
            else:
                pb._step = 0 if kind == "check" else 1
                one_step()

    res = {}
    n = max(steps // 2, 2)
    for kind in ("check", "reuse"):
        run(kind, 1)
        torch.cuda.synchronize()
        _barrier(ws)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        run(kind, n)
        e1.record()
        torch.cuda.synchronize()
        _barrier(ws)
        res[kind] = _max_over_ranks(e0.elapsed_time(e1), ws) * 1e3 / (n * C3S_LAYERS)
    del graphs
    us_layer = (res["check"] + (M_INTERVAL - 1) * res["reuse"]) / M_INTERVAL
    breakdown = _split_breakdown(pb, pools, ag, ws)
    errors = 0
    if px is not None:
        torch.cuda.synchronize()
        errors = int(px.dev_error.item())
        px.close()
    xname = "NVLink peer-memory kernels (all-gather; push + merge)" if px is not None else \
        "NCCL all-gathers"
    return {"workload": "config3: B=1, Hq=32, Hkv=8, D=128, bf16, ctx=131072 (8192 pages), "
                        f"pages split contiguously over {ws} GPU(s), lazy M=4, {C3S_LAYERS} layers",
            "us_per_layer_lazy_check": res["check"], "us_per_layer_reuse": res["reuse"],
            "us_per_layer": us_layer, "steps_per_kind": n,
            "exchange": xname, "exchange_errors": errors,
            "launch": (f"CUDA graph per step kind ({xname} inside)" if ok else
                       "eager (graph capture failed)"),
            "breakdown_us_per_layer": breakdown,
            "stats_rank0_warmup": stats}


def _split_breakdown(pb, pools, ag, ws):
    """Per-op device time of one eager lazy-check step and one eager reuse
    step of the page split (CUDA events around every kernel call and every
    all-gather on the current stream; max over ranks, per layer). The events
    separate the launches (no overlap), so the sum exceeds the graph-replayed
    step."""
    import types
    from cvsa.pagesplit import run_step

    names = ("score_pages", "split_propose", "split_gate", "split_attend", "decode_unnorm",
             "rank_merge")
    records = []

    def wrap(label, fn):
        def call(*a, **k):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*a, **k)
            e1.record()
            records.append((label, e0, e1))
            return r
        return call

    ops = pb.ops
    pb.ops = types.SimpleNamespace(**{nm: wrap(nm, getattr(ops, nm)) for nm in names})
    tag = wrap("all_gather", ag)
    px = pb.exchange
    if px is not None:
        pb.exchange = types.SimpleNamespace(allgather=wrap("all_gather", px.allgather),
                                            merge=wrap("exchange_merge", px.merge))
    out = {}
    try:
        for kind, step_idx in (("check", 0), ("reuse", 1)):
            records.clear()
            pb._step = step_idx
            # hold the stream (a fixed spin of about 25 ms) while the host
            # enqueues the step, so no event pair spans host launch gaps, and
            # let the ranks meet on the device after it, so no exchange
            # absorbs the ranks' start skew
            torch.cuda._sleep(50_000_000)
            if ws > 1:
                import torch.distributed as dist
                dist.all_reduce(torch.zeros(1, device="cuda"))
            for l, (q, k, v, bt, cl, ctx, W) in enumerate(pools):
                run_step(pb.step(q, k, v, bt, cl, l, ctx, W), tag)
            torch.cuda.synchronize()
            tot = {}
            for label, e0, e1 in records:
                tot[label] = tot.get(label, 0.0) + e0.elapsed_time(e1)
            out[kind] = {label: _max_over_ranks(tot.get(label, 0.0), ws) * 1e3 / len(pools)
                         for label in ("score_pages", "split_propose", "all_gather", "split_gate",
                                       "split_attend", "decode_unnorm", "rank_merge",
                                       "exchange_merge")}
    finally:
        pb.ops = ops
        pb.exchange = px
    return out


C5_STEPS = 256


def measure_config5(dev, warmup, ws, rank):
    """Config 5: 64 ragged sequences (1K-64K tokens) in a pool with a shuffled
    free list; every step appends one token per sequence (cvsa_paged_append,
    new pages taken on the device) and runs one lazy-M=4 layer step. Nearly
    every head fails tau, so scoring steps recover almost every page. The
    append, the lazy-check step and the reuse step are captured as CUDA graphs;
    C5_STEPS steps are timed (max over ranks; each rank its own batch), and
    the appends alone separately."""
    from cvsa import _lib, synthetic
    from cvsa.backend import CVSABackend

    grow = C5_STEPS + 3 * M_INTERVAL + 16
    wl = synthetic.config5(device=dev, seed=5000 + rank, grow=grow)
    mgr, cache = wl.mgr, wl.cache
    B, Hq, D = wl.q.shape
    hkv = cache.num_kv_heads
    be = CVSABackend(hkv, Hq, D, 16, num_layers=1, budget_pct=wl.budget_pct,
                     coverage_threshold=wl.tau, lazy=True, check_interval=M_INTERVAL,
                     sink_pages=wl.sink_pages, local_pages=wl.local_pages)

    def decode():
        be(wl.q, cache.k_cache, cache.v_cache, mgr.block_tables, mgr.context_lens, 0)

    def append():
        mgr.append_batch(wl.k_new, wl.v_new)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = {}
    with torch.cuda.stream(side):
        for _ in range(M_INTERVAL):              # one eager cycle (the first step scores)
            append()
            decode()
            be.step_done(0, 1)
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            append()
        graphs["append"] = g
        for kind, step_idx in (("lazy", 0), ("reuse", 1)):
            g = torch.cuda.CUDAGraph()
            be._step = step_idx
            with torch.cuda.graph(g, stream=side):
                decode()
            graphs[kind] = g
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    lens0 = mgr.context_lens.to(torch.int64).cpu()   # before the timed steps

    def run(n, with_decode=True):
        for s in range(n):
            graphs["append"].replay()
            if with_decode:
                graphs["lazy" if s % M_INTERVAL == 0 else "reuse"].replay()

    _barrier(ws)
    torch.cuda.synchronize()
    c0 = be._counter_values()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    run(C5_STEPS)
    e1.record()
    torch.cuda.synchronize()
    _barrier(ws)
    ms = _max_over_ranks(e0.elapsed_time(e1), ws)
    c1 = be._counter_values()
    pages = c1[_lib.CTR_PAGES_ATTENDED] - c0[_lib.CTR_PAGES_ATTENDED]
    scoring = sum(int(((lens0 + s + 1 + 15) // 16).sum()) * hkv * KP_BYTES
                  for s in range(C5_STEPS) if s % M_INTERVAL == 0)
    nbytes = _sum_over_ranks(float(pages * 2 * KP_BYTES + scoring), ws)
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    n_app = 16
    a0.record()
    run(n_app, with_decode=False)
    a1.record()
    torch.cuda.synchronize()
    app_us = _max_over_ranks(a0.elapsed_time(a1), ws) * 1e3 / n_app
    cache.check()
    stats = be.get_stats()
    del graphs
    return {"workload": f"config5: {B} ragged sequences, lengths U[1024, 65536] (+1 token per "
                        "step), Hq=32, Hkv=8, D=128, bf16, shuffled free list, budget 5% of the "
                        f"table width + sink 1 + local 2, tau=0.9, lazy M=4, {C5_STEPS} steps of "
                        "append + one layer",
            "value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s (algorithmic KV bytes)",
            "us_per_step": ms * 1e3 / C5_STEPS, "append_us": app_us,
            "frac_of_peak": nbytes / (ms * 1e-3) / 1e9 / (_peaks()[0] * ws),
            "per_head_accept_rate": stats.get("per_head_accept_rate"),
            "launch": "CUDA graphs: append, lazy-check step, reuse step"}


# DRAM bytes (read + write) per algorithmic byte of each launch kind, from the
# ncu captures of the config-2 bench workload (profiles/stream_attend_config2.md,
# profiles/score_stream_config2.md): a launch's traffic is this ratio times the
# algorithmic bytes of the same launch kind in this run (traffic grows with the
# pages a launch reads; the captured launches' own rejection mix differs from a
# given run's).
NCU_TRAFFIC_RATIO = {"attend_check": (233.66e6 + 3.54e6) / 233.2e6,
                     "attend_reuse": (59.17e6 + 0.76e6) / 58.7e6,
                     "score": (537.30e6 + 3.75e6) / 536.87e6}


def roofline_table(kern, att_pages, layers, score_bytes, peak, peak_kind):
    """Achieved HBM bandwidth of each hot kernel over the timed cycle, the
    one with the largest share of kernel time first.

    Per launch: algorithmic bytes (scoring: every valid page's K; attention:
    the K+V of the pages it attends, from the device counters of one replay of
    each graph) / the launch's CUDA-event duration, averaged over the layers
    of the M=4 cycle (one lazy-check step, M-1 reuse steps)."""
    mean = statistics.mean
    out = []
    n_check, n_reuse = 1, M_INTERVAL - 1
    if kern["attend_scoring"] and kern["attend_reuse"]:
        b_check = att_pages["lazy"] * 2 * KP_BYTES / layers
        b_reuse = att_pages["reuse"] * 2 * KP_BYTES / layers
        t_check, t_reuse = mean(kern["attend_scoring"]), mean(kern["attend_reuse"])
        launches = n_check + n_reuse
        avg_bytes = (n_check * b_check + n_reuse * b_reuse) / launches
        avg_ms = (n_check * t_check + n_reuse * t_reuse) / launches
        traffic = (n_check * NCU_TRAFFIC_RATIO["attend_check"] * b_check
                   + n_reuse * NCU_TRAFFIC_RATIO["attend_reuse"] * b_reuse) / launches
        out.append(dict(kernel="stream_attend_kernel", launch="cycle mean (1 check + "
                        f"{n_reuse} reuse launches)", time_ms_per_cycle=avg_ms * launches,
                        algorithmic_bytes_per_launch=avg_bytes, avg_launch_ms=avg_ms,
                        traffic=traffic))
        for name, b, t, tr in (("check", b_check, t_check,
                                NCU_TRAFFIC_RATIO["attend_check"] * b_check),
                               ("reuse", b_reuse, t_reuse,
                                NCU_TRAFFIC_RATIO["attend_reuse"] * b_reuse)):
            out.append(dict(kernel="stream_attend_kernel", launch=name,
                            time_ms_per_cycle=t * (n_check if name == "check" else n_reuse),
                            algorithmic_bytes_per_launch=b, avg_launch_ms=t, traffic=tr))
    if kern["score"]:
        t = mean(kern["score"])
        out.append(dict(kernel="score_stream_kernel", launch="check", time_ms_per_cycle=t,
                        algorithmic_bytes_per_launch=score_bytes, avg_launch_ms=t,
                        traffic=NCU_TRAFFIC_RATIO["score"] * score_bytes))
    if kern["select"]:
        t = mean(kern["select"])
        # the kernel the selection dispatch picks for config 2's 512-page tables
        out.append(dict(kernel="select_gate_big_kernel<4, 128>", launch="check",
                        time_ms_per_cycle=t,
                        algorithmic_bytes_per_launch=0, avg_launch_ms=t, traffic=None,
                        note="reads 0.5 MB of page scores from L2; latency-bound"))
    for r in out:
        ach = r["algorithmic_bytes_per_launch"] / (r["avg_launch_ms"] * 1e-3) / 1e9
        r.update(bound="hbm", achieved=ach, peak=peak, unit="GB/s", frac=ach / peak,
                 peak_kind=peak_kind)
    # the headline entry: the cycle-mean of the kernel with the largest time share
    heads = [r for r in out if r["launch"] not in ("check", "reuse")
             or r["kernel"] != "stream_attend_kernel"]
    heads.sort(key=lambda r: -r["time_ms_per_cycle"])
    rest = [r for r in out if r not in heads[:1]]
    return heads[:1] + rest


def run_cvsa(args, ws, rank, local):
    import ctypes

    from cvsa import _lib
    from cvsa.backend import CVSABackend

    dev = torch.device("cuda", local)
    layers = args.layers
    wls = build_layers(dev, layers)
    B, Hq, D = wls[0].q.shape
    hkv = wls[0].num_kv_heads
    scoring_bytes_per_layer = [_scoring_pages(wl.context_lens, hkv) * KP_BYTES for wl in wls]

    def make_backend():
        return CVSABackend(hkv, Hq, D, 16, num_layers=layers, budget_pct=0.05,
                           coverage_threshold=0.9, lazy=True, check_interval=M_INTERVAL,
                           sink_pages=1, local_pages=2)

    def eager_step(be, qs=None, outs=None):
        for l, wl in enumerate(wls):
            q = wl.q if qs is None else qs[l]
            o = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
            if outs is not None:
                outs[l] = o
            be.step_done(l, layers)

    def alg_bytes(be, c0, lazy_steps):
        c1 = be._counter_values()
        pages = c1[_lib.CTR_PAGES_ATTENDED] - c0[_lib.CTR_PAGES_ATTENDED]
        return pages * 2 * KP_BYTES + lazy_steps * sum(scoring_bytes_per_layer)

    def timed(be, k, fn, lazy_steps):
        _barrier(ws)
        torch.cuda.synchronize()
        c0 = be._counter_values()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(k):
            fn(s)
        e1.record()
        torch.cuda.synchronize()
        _barrier(ws)
        return e0.elapsed_time(e1), alg_bytes(be, c0, lazy_steps)

    warm = args.warmup + ((-args.warmup) % M_INTERVAL)   # timed region starts a cycle
    lazy_steps = sum(1 for s in range(args.steps) if s % M_INTERVAL == 0)

    # ---- device-resident timing (value): the step captured in CUDA graphs ----
    # One graph for a lazy check step and one for a reuse step, each holding the
    # 32 layer calls (3 kernels per layer on check steps, 1 on reuse steps).
    be = make_backend()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = {}
    with torch.cuda.stream(side):
        for _ in range(warm):
            eager_step(be)
        side.synchronize()
        for kind, step_idx in (("lazy", 0), ("reuse", 1)):
            g = torch.cuda.CUDAGraph()
            be._step = step_idx
            with torch.cuda.graph(g, stream=side):
                for l, wl in enumerate(wls):
                    be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
            graphs[kind] = g
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    for s in range(M_INTERVAL):                      # warm the graphs
        graphs["lazy" if s % M_INTERVAL == 0 else "reuse"].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ms, nbytes = timed(be, args.steps,
                       lambda s: graphs["lazy" if s % M_INTERVAL == 0 else "reuse"].replay(),
                       lazy_steps)
    clk = clocks.stop()
    ms_max = _max_over_ranks(ms, ws)
    bytes_all = _sum_over_ranks(float(nbytes), ws)
    value = bytes_all / (ms_max * 1e-3) / 1e9
    us_per_layer = ms_max * 1e3 / (args.steps * layers)
    launches = (lazy_steps * 3 + (args.steps - lazy_steps) * 1) * layers
    stats = be.get_stats()

    # ---- per-kernel times: the same graphs captured with CUDA events ----
    # around each launch (events between kernels disable launch overlap)
    ev_graphs = {}
    ev_sets = {"lazy": [], "reuse": []}
    with torch.cuda.stream(side):
        for kind, step_idx in (("lazy", 0), ("reuse", 1)):
            g = torch.cuda.CUDAGraph()
            be._step = step_idx
            sets = []
            for _ in wls:
                evs = [torch.cuda.Event(enable_timing=True) for _ in range(_lib.NUM_EVENTS)]
                for e in evs:
                    e.record()       # torch creates the cudaEvent_t at its first record
                sets.append((evs, (ctypes.c_void_p * _lib.NUM_EVENTS)(
                    *[e.cuda_event for e in evs])))
            side.synchronize()
            with torch.cuda.graph(g, stream=side):
                for l, wl in enumerate(wls):
                    be._timing_events = sets[l][1]
                    be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
                be._timing_events = None
            ev_graphs[kind] = g
            ev_sets[kind] = sets
    torch.cuda.current_stream(dev).wait_stream(side)
    kern = {"score": [], "select": [], "attend_scoring": [], "attend_reuse": []}
    att_pages = {"lazy": 0, "reuse": 0}      # pages attended by one replay of each graph
    for rep in range(2):
        for kind in ("lazy", "reuse"):
            c_a = be._counter_values()[_lib.CTR_PAGES_ATTENDED]
            ev_graphs[kind].replay()
            torch.cuda.synchronize()
            if rep == 0:
                continue
            att_pages[kind] = be._counter_values()[_lib.CTR_PAGES_ATTENDED] - c_a
            for evs, _ in ev_sets[kind]:
                att = evs[_lib.EV_ATTEND_BEGIN].elapsed_time(evs[_lib.EV_ATTEND_END])
                if kind == "lazy":
                    kern["score"].append(evs[_lib.EV_SCORE_BEGIN].elapsed_time(
                        evs[_lib.EV_SCORE_END]))
                    kern["select"].append(evs[_lib.EV_SELECT_BEGIN].elapsed_time(
                        evs[_lib.EV_SELECT_END]))
                    kern["attend_scoring"].append(att)
                else:
                    kern["attend_reuse"].append(att)
    del ev_graphs
    score_ms = statistics.mean(kern["score"]) if kern["score"] else None
    score_bytes = scoring_bytes_per_layer[0]
    peak, peak_kind = _peaks()
    rooflines = roofline_table(kern, att_pages, layers, score_bytes, peak, peak_kind)
    reuse_ms = statistics.mean(kern["attend_reuse"]) if kern["attend_reuse"] else None
    sel_pages = B * hkv * 28
    reuse_bytes = sel_pages * 2 * KP_BYTES

    # ---- eager device-resident timing (one C-ABI call per layer, no graph) ----
    be2 = make_backend()
    for _ in range(warm):
        eager_step(be2)
    ms_eager, _ = timed(be2, args.steps, lambda s: eager_step(be2), lazy_steps)
    ms_eager = _max_over_ranks(ms_eager, ws)

    # ---- end-to-end through the public API with host buffers ----
    be3 = make_backend()
    q_host = [wl.q.cpu().pin_memory() for wl in wls]
    out_host = [torch.empty_like(h).pin_memory() for h in q_host]
    q_dev = [torch.empty_like(wl.q) for wl in wls]

    # Every step uploads each layer's q from pinned memory and reads each
    # layer's output back, all inside the timed region. The uploads run on a
    # copy stream (layer l's step waits only for its own q) and each output
    # is read back on a second copy stream as soon as its layer is done, so
    # the copies overlap the other layers' kernels; the step ends when the
    # last read-back has landed.
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    q_ready = [torch.cuda.Event() for _ in wls]
    o_ready = [torch.cuda.Event() for _ in wls]

    def e2e_step(_s=0):
        up.wait_stream(comp)              # the previous step's layers are done with q_dev
        with torch.cuda.stream(up):
            for l in range(layers):
                q_dev[l].copy_(q_host[l], non_blocking=True)
                q_ready[l].record(up)
        for l, wl in enumerate(wls):
            comp.wait_event(q_ready[l])
            o = be3(q_dev[l], wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, l)
            o_ready[l].record(comp)
            down.wait_event(o_ready[l])
            with torch.cuda.stream(down):
                out_host[l].copy_(o, non_blocking=True)
                o.record_stream(down)
            be3.step_done(l, layers)
        comp.wait_stream(down)

    for _ in range(warm):
        e2e_step()
    torch.cuda.synchronize()
    ms_e, nbytes_e = timed(be3, args.steps, e2e_step, lazy_steps)
    ms_e = _max_over_ranks(ms_e, ws)
    e2e_val = _sum_over_ranks(float(nbytes_e), ws) / (ms_e * 1e-3) / 1e9
    h2d = sum(h.numel() * h.element_size() for h in q_host)
    del graphs

    # ---- config 3 (128K single sequence): the metric's second context ----
    c3 = None
    if not args.no_c3:
        c3 = measure_config3(dev, args.steps, warm, ws)
        c3["frac_of_peak"] = c3["value"] / (_peaks()[0] * ws)
    c4 = None
    if not args.no_c4:
        c4 = measure_config4(dev, args.steps, warm, ws, rank)
    c5 = None
    if not args.no_c5:
        c5 = measure_config5(dev, warm, ws, rank)
    c3s = None
    if not args.no_c3:
        c3s = measure_config3_split(dev, args.steps, ws, rank, peer=ws > 1)
        if ws > 1:
            nccl = measure_config3_split(dev, args.steps, ws, rank, peer=False)
            c3s["nccl_all_gathers"] = {k: nccl[k] for k in (
                "us_per_layer_lazy_check", "us_per_layer_reuse", "us_per_layer")}

    # ---- CPU baseline (rank 0, N=1 only) ----
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cs = CpuSample()
        cs.cycle()                       # warm-up cycle (first step has no cache)
        tot_t, tot_b, cycles = 0.0, 0, 0
        while tot_t < 10.0:
            dt, nb = cs.cycle()
            tot_t += dt
            tot_b += nb
            cycles += 1
        cpu = {"value": tot_b / tot_t / 1e9, "unit": "GB/s", "cores": cs.threads,
               "kind": "port", "sample": CPU_SAMPLE_DESC + f"; {cycles} cycles, {tot_t:.1f} s",
               "ms_per_layer_step": tot_t * 1e3 / (M_INTERVAL * cycles)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": warm, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) + planted heavy pages; no checkpoints)",
            "config": {"workload": WORKLOAD, "batch_per_gpu": B, "ctx": 8192, "layers": layers,
                       "schedule": f"lazy M={M_INTERVAL}",
                       "launch": "CUDA graph per step kind (lazy check / reuse), 32 layers each",
                       "l2": "inputs larger than L2 (1.07 GB K+V per layer, 32 pools)",
                       "parallelism": f"{ws} independent replicas (weak scaling)"},
            "us_per_layer": us_per_layer,
            "eager_us_per_layer": ms_eager * 1e3 / (args.steps * layers),
            "tokens_per_s": B * ws * args.steps / (ms_max * 1e-3),
            # the kernel with the largest share of the step's kernel time
            "roofline": rooflines[0],
            "rooflines": rooflines,
            "kernels": {
                "score_ms": score_ms,
                "select_ms": statistics.mean(kern["select"]) if kern["select"] else None,
                "attend_scoring_ms": (statistics.mean(kern["attend_scoring"])
                                      if kern["attend_scoring"] else None),
                "attend_reuse_ms": reuse_ms,
                "attend_reuse_gbs": reuse_bytes / (reuse_ms * 1e-3) / 1e9 if reuse_ms else None,
            },
            "cvsa_stats": {k: stats[k] for k in ("per_head_accept_rate", "effective_budget_pct",
                                                 "total_scoring_steps", "total_coverage_checks")
                           if k in stats},
            "e2e": {"value": e2e_val, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": h2d, "ms_per_step": ms_e / args.steps,
                    "path": "CVSABackend.__call__ per layer (eager); every layer's q uploaded "
                            "from pinned memory and its output read back each step, on copy "
                            "streams overlapping the other layers' kernels"},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if c3 is not None:
            line["config3_128k"] = c3
        if c4 is not None:
            line["config4_70b_head_sharded"] = c4
        if c5 is not None:
            line["config5_ragged_append"] = c5
        if c3s is not None:
            line["config3_page_split"] = c3s
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


KERNEL_CASES = ("select_warp", "select_big", "quest", "score_general", "attend_general",
                "page_lse", "rank_merge", "append", "gather", "config3_step", "split_propose",
                "split_gate")


def run_kernel_case(name: str, reps: int = 3):
    """One kernel on a small fixed workload, `reps` launches (the ncu capture
    targets of profiles/: `ncu -k regex:<kernel> -c 1 python bench.py
    --kernel-case <name>`). Inputs are sized above L2 where the kernel reads
    the KV pool."""
    from cvsa import synthetic
    from cvsa.kernels import coverage as C
    from cvsa.kernels import page_scores as PS
    from cvsa.kernels import select as SEL
    from cvsa.kernels import sparse_decode as SD
    dev = torch.device("cuda", 0)
    if name in ("select_warp", "quest"):
        wl = synthetic.config2(device=dev, seed=1000, gen_device=str(dev))
    elif name in ("select_big", "config3_step"):
        wl = synthetic.config3(device=dev, seed=3000, gen_device=str(dev))
    elif name in ("score_general", "attend_general"):
        # fp32 pool: the general-layout kernels (score_pages_kernel, attend_kernel)
        wl = synthetic.small(device="cpu", seed=2, B=16, Hq=32, Hkv=8, D=128,
                             ctx=(8192,) * 16, dtype=torch.float32).to(dev)
    elif name in ("split_propose", "split_gate"):
        wl = None
    else:
        wl = synthetic.small(device="cpu", seed=2, B=8, Hq=32, Hkv=8, D=128,
                             ctx=(8192,) * 8).to(dev)
    if name == "config3_step":
        # one config-3 layer through the backend: a scoring step (score,
        # selection over 8192 pages, attention with recovery) then reuse steps
        from cvsa.backend import CVSABackend
        be = CVSABackend(wl.num_kv_heads, wl.q.shape[1], 128, 16, num_layers=1,
                         budget_pct=0.05, coverage_threshold=0.9, lazy=True, check_interval=4,
                         sink_pages=1, local_pages=2)
        for _ in range(reps + 1):
            be(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
            be.step_done(0, 1)
        torch.cuda.synchronize()
        print(json.dumps({"kernel_case": name, "reps": reps}), flush=True)
        return
    if name in ("split_propose", "split_gate"):
        # the page split's proposal over config 3 on one of 8 ranks (8 rows of
        # 1024 pages) and its gate over the 8 ranks' gathered rows
        from cvsa.kernels import split as SK
        gen = torch.Generator().manual_seed(7)
        H8, W8, budget8, max_sel8 = 8, 1024, 409, 412
        lens8 = torch.full((1,), W8 * 16, dtype=torch.int32, device=dev)
        rows8 = []
        for r in range(8):
            sc8 = torch.randn((1, H8, W8), generator=gen).to(dev)
            row8 = torch.empty(SK.row_floats(1, H8, max_sel8), device=dev)
            prop8 = SK.split_propose(sc8, lens8, 16, None, 1 if r == 0 else 0,
                                     2 if r == 7 else 0, budget8, max_sel8, row8)
            rows8.append(row8)
        parts8 = torch.stack(rows8)
        state8 = torch.zeros(4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        for _ in range(reps):
            if name == "split_propose":
                SK.split_propose(sc8, lens8, 16, None, 0, 2, budget8, max_sel8, row8)
            else:
                SK.split_gate(parts8, prop8, lens8, 16, W8, 7, budget8, max_sel8, 0, 2, 0.9,
                              False, 0, state8)
        torch.cuda.synchronize()
        print(json.dumps({"kernel_case": name, "reps": reps}), flush=True)
        return
    H, G = wl.num_kv_heads, wl.num_q_per_kv
    W = wl.block_tables.shape[1]
    scores = PS.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, H, G, 16)
    budget = SEL.budget_for(W, 0.05)
    idx, n = SEL.select_pages(scores, wl.context_lens, 16, budget, 1, 2)
    torch.cuda.synchronize()
    for _ in range(reps):
        if name in ("select_warp", "select_big"):
            SEL.select_pages(scores, wl.context_lens, 16, budget, 1, 2)
        elif name == "quest":
            PS.quest_page_scores(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, H)
        elif name == "score_general":
            PS.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, H, G, 16)
        elif name == "attend_general":
            SD.sparse_decode(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, idx, n,
                             wl.context_lens, H, G, 16)
        elif name == "page_lse":
            C.page_lse(scores, idx, n)
        elif name == "rank_merge":
            B, Hq, D = wl.q.shape
            parts = torch.randn((8, B * Hq * (D + 2)), device=dev)
            C.rank_merge(parts, B, H, G, D, torch.empty_like(wl.q))
        elif name == "append":
            from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
            cache = PagedKVCache(64 * 64, 16, 8, 128, device="cuda")
            mgr = SequenceKVManager(cache, 64, 4096)
            kn = torch.randn((64, 8, 128), device=dev, dtype=torch.bfloat16)
            for _t in range(16):
                mgr.append_batch(kn, kn)
        elif name == "gather":
            from cvsa.runtime.kv_cache import PagedKVCache
            cache = PagedKVCache(4096, 16, 8, 128, device="cuda")
            cache.gather_pages(torch.randperm(4096, device=dev)[:2048])
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": name, "reps": reps}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="cvsa", choices=["cvsa", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-c3", action="store_true", help="skip the config-3 (128K) measurement")
    ap.add_argument("--no-c4", action="store_true",
                    help="skip the config-4 (70B, KV heads sharded over the GPUs) measurement")
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the config-5 (ragged batch with appends) measurement")
    ap.add_argument("--kernel-case", choices=KERNEL_CASES, default=None,
                    help="run one kernel on a small fixed case (profiling target), no bench line")
    args = ap.parse_args()
    if args.kernel_case:
        run_kernel_case(args.kernel_case)
        return
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, ws, rank)
        return
    ws, rank, local = _dist()
    try:
        run_cvsa(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
