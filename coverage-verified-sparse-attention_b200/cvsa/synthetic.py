"""Seeded synthetic decode workloads with the shapes of the CVSA benchmark configs.

No model checkpoints or datasets are used: queries, keys and values are drawn
from N(0, 1) and a few "heavy" pages per (sequence, KV head) get keys aligned
with that head's query, so page coverage varies across heads the way it does
on real attention. Each generator returns a `Workload` whose tensors live on
`device`; generation runs on `gen_device` (CPU for bit-identical inputs across
machines, CUDA for fast generation of large pools).

  config 1  B=1,  Hq=8,  Hkv=2, D=64,  fp32, ctx 4096 (256 pages), top-k 32 + 3 forced
  config 2  B=32, Hq=32, Hkv=8, D=128, bf16, ctx 8192 (512 pages), 5 % + 3 forced
  config 3  B=1,  Hq=32, Hkv=8, D=128, bf16, ctx 131072 (8192 pages), drifting keys
The heavy-key strength alpha of each config was calibrated so that a mix of
heads pass and fail tau = 0.9 (recorded in `Workload.meta`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import torch


@dataclass
class Workload:
    name: str
    q: torch.Tensor             # [B, Hq, D]
    k_cache: torch.Tensor       # [NB, bs, Hkv, D]
    v_cache: torch.Tensor
    block_tables: torch.Tensor  # [B, W] int32
    context_lens: torch.Tensor  # [B] int32
    num_kv_heads: int
    block_size: int
    budget_pct: float
    tau: float
    sink_pages: int
    local_pages: int
    check_interval: int
    meta: Dict = field(default_factory=dict)

    @property
    def num_q_per_kv(self) -> int:
        return self.q.shape[1] // self.num_kv_heads

    def to(self, device) -> "Workload":
        d = dict(self.__dict__)
        for k in ("q", "k_cache", "v_cache", "block_tables", "context_lens"):
            d[k] = d[k].to(device)
        return Workload(**d)

    def kv_bytes(self) -> int:
        return self.k_cache.numel() * self.k_cache.element_size()


# Calibrated heavy-key strengths (alpha), see the generators' docstrings.
ALPHA_C1 = (5.5, 2.5)       # head 0 passes tau=0.9, head 1 fails
ALPHA_C2 = 6.5              # about a fifth of (b, h) fail tau=0.9
ALPHA_C3 = 6.0              # 6 of 8 heads pass tau=0.9 at seed 0
ALPHA_C4 = 11.0             # 14 of 64 (b, h) fail tau=0.9 at seed 0


def _unit_group_query(q: torch.Tensor, num_kv_heads: int) -> torch.Tensor:
    """Unit-norm mean query of each KV group, [B, Hkv, D] fp32."""
    B, Hq, D = q.shape
    m = q.float().view(B, num_kv_heads, Hq // num_kv_heads, D).mean(2)
    return m / m.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def _randn(shape, gen, device, dtype=torch.float32):
    return torch.randn(shape, generator=gen, device=device, dtype=dtype)


def config1(device="cpu", seed: int = 0, alpha=ALPHA_C1) -> Workload:
    """B=1, Hq=8, Hkv=2, D=64, fp32, ctx 4096; 4 heavy pages per KV head.

    Draw order: q, K, V ~ N(0, 1); then per KV head 4 heavy page positions
    (uniform among the non-forced pages 1..253) whose 16 keys become
    alpha_h * 3 * q_hat_h + 0.5 * N(0, 1). alpha = (5.5, 2.5) makes head 0
    pass and head 1 fail tau = 0.9 (the literal recipe, alpha = 1, passes no
    head). Budget: top-32 of 256 pages plus forced pages {0, 254, 255}.
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    B, Hq, Hkv, D, bs, ctx = 1, 8, 2, 64, 16, 4096
    W = ctx // bs
    q = _randn((B, Hq, D), g, "cpu")
    k = _randn((W, bs, Hkv, D), g, "cpu")
    v = _randn((W, bs, Hkv, D), g, "cpu")
    qh = _unit_group_query(q, Hkv)
    heavy = {}
    for h in range(Hkv):
        cand = torch.arange(1, W - 2)
        pos = cand[torch.randperm(cand.numel(), generator=g)[:4]]
        heavy[h] = sorted(pos.tolist())
        for p in pos.tolist():
            k[p, :, h, :] = alpha[h] * 3.0 * qh[0, h] + 0.5 * _randn((bs, D), g, "cpu")
    bt = torch.arange(W, dtype=torch.int32).view(1, W)
    cl = torch.tensor([ctx], dtype=torch.int32)
    wl = Workload("config1", q, k, v, bt, cl, Hkv, bs, budget_pct=32 / 256, tau=0.90,
                  sink_pages=1, local_pages=2, check_interval=4,
                  meta=dict(alpha=list(alpha), heavy_pages=heavy, seed=seed))
    return wl.to(device)


def config2(device="cpu", seed: int = 0, alpha: float = ALPHA_C2, batch: int = 32,
            ctx: int = 8192, gen_device: Optional[str] = None,
            dtype: torch.dtype = torch.bfloat16) -> Workload:
    """Llama-3.1-8B geometry: B=32, Hq=32, Hkv=8, D=128, bf16, ctx 8192.

    Pool of B*512 pages with a randomly permuted page table. q, K, V ~ N(0, 1).
    Per (b, h): U{2..8} heavy pages at random non-forced positions, strength
    s ~ logU[1, 4], keys s * alpha * q_hat + 0.5 * N(0, 1). alpha = 6.5 leaves
    51 of the 256 (b, h) heads (20 %) below tau = 0.9 at seed 0 (alpha = 5:
    56 % fail, alpha = 8: 6 %). Budget int(512 * 0.05) = 25 plus forced pages
    {0, 510, 511}.
    """
    gd = gen_device or (device if str(device).startswith("cuda") else "cpu")
    g = torch.Generator(device=gd).manual_seed(seed)
    gc = torch.Generator(device="cpu").manual_seed(seed + 1)
    B, Hq, Hkv, D, bs = batch, 32, 8, 128, 16
    W = ctx // bs
    NB = B * W
    q = _randn((B, Hq, D), g, gd).to(dtype)
    k = torch.empty((NB, bs, Hkv, D), dtype=dtype, device=gd)
    v = torch.empty((NB, bs, Hkv, D), dtype=dtype, device=gd)
    chunk = 4096
    for s0 in range(0, NB, chunk):
        n = min(chunk, NB - s0)
        k[s0:s0 + n] = _randn((n, bs, Hkv, D), g, gd).to(dtype)
    for s0 in range(0, NB, chunk):
        n = min(chunk, NB - s0)
        v[s0:s0 + n] = _randn((n, bs, Hkv, D), g, gd).to(dtype)
    perm = torch.randperm(NB, generator=gc).to(torch.int32)
    bt = perm.view(B, W).contiguous()
    qh = _unit_group_query(q, Hkv)                          # on gd
    n_heavy = torch.randint(2, 9, (B, Hkv), generator=gc)
    heavy = {}
    for b in range(B):
        for h in range(Hkv):
            nh = int(n_heavy[b, h])
            cand = torch.arange(1, W - 2)
            pos = cand[torch.randperm(cand.numel(), generator=gc)[:nh]]
            strength = torch.exp(torch.empty(nh).uniform_(0.0, math.log(4.0), generator=gc))
            heavy[(b, h)] = (pos.tolist(), strength.tolist())
            blocks = bt[b, pos].long().to(gd)
            noise = _randn((nh, bs, D), g, gd)
            keys = (strength.to(gd).view(nh, 1, 1) * alpha * qh[b, h].view(1, 1, D)
                    + 0.5 * noise)
            k[blocks, :, h, :] = keys.to(dtype)
    cl = torch.full((B,), ctx, dtype=torch.int32)
    wl = Workload("config2", q, k, v, bt, cl, Hkv, bs, budget_pct=0.05, tau=0.90,
                  sink_pages=1, local_pages=2, check_interval=4,
                  meta=dict(alpha=alpha, seed=seed, n_heavy=n_heavy.tolist()))
    return wl.to(device)


def config4(device="cpu", kv_heads: slice = slice(0, 8), seed: int = 0,
            alpha: float = ALPHA_C4, batch: int = 8, ctx: int = 32768,
            dtype: torch.dtype = torch.bfloat16) -> Workload:
    """Llama-70B attention geometry, one shard of its KV heads: B=8, Hq=64,
    Hkv=8, D=128, bf16, ctx 32768 (2048 pages). `kv_heads` selects the KV
    heads this rank holds (with their query heads); every head's keys, values
    and planted pages come from generators seeded by the head index, so a
    shard equals the same slice of the unsharded workload whatever the rank
    count. Pool of B*2048 pages with a randomly permuted page table (shared by
    all heads). Per (b, h): U{2..8} heavy pages, strength s ~ logU[1, 4], keys
    s * alpha * q_hat + 0.5 * N(0, 1); q_hat is the unit mean query of the
    head's group. Budget int(2048 * 0.05) = 102 plus forced pages {0, 2046,
    2047}; tau = 0.9. alpha = 11 leaves 14 of the 64 (b, h) heads (22 %)
    below tau at seed 0 (measured with the GPU backend; alpha = 9: 39 %,
    alpha = 14: 11 %).
    """
    gd = device if str(device).startswith("cuda") else "cpu"
    B, Hq, Hkv, D, bs = batch, 64, 8, 128, 16
    G = Hq // Hkv
    W = ctx // bs
    NB = B * W
    heads = list(range(kv_heads.start, kv_heads.stop))
    gq = torch.Generator(device=gd).manual_seed(seed)
    q_full = _randn((B, Hq, D), gq, gd).to(dtype)
    q = q_full[:, heads[0] * G:(heads[-1] + 1) * G].contiguous()
    qh = _unit_group_query(q_full, Hkv)
    gt = torch.Generator(device="cpu").manual_seed(seed + 1)
    bt = torch.randperm(NB, generator=gt).to(torch.int32).view(B, W).contiguous()
    k = torch.empty((NB, bs, len(heads), D), dtype=dtype, device=gd)
    v = torch.empty((NB, bs, len(heads), D), dtype=dtype, device=gd)
    n_heavy = {}
    for j, h in enumerate(heads):
        gh = torch.Generator(device=gd).manual_seed(seed * 1000 + 17 + h)
        gp = torch.Generator(device="cpu").manual_seed(seed * 1000 + 500 + h)
        k[:, :, j, :] = _randn((NB, bs, D), gh, gd).to(dtype)
        v[:, :, j, :] = _randn((NB, bs, D), gh, gd).to(dtype)
        nh_b = torch.randint(2, 9, (B,), generator=gp)
        for b in range(B):
            nh = int(nh_b[b])
            n_heavy[(b, h)] = nh
            cand = torch.arange(1, W - 2)
            pos = cand[torch.randperm(cand.numel(), generator=gp)[:nh]]
            strength = torch.exp(torch.empty(nh).uniform_(0.0, math.log(4.0), generator=gp))
            blocks = bt[b, pos].long().to(gd)
            keys = (strength.to(gd).view(nh, 1, 1) * alpha * qh[b, h].view(1, 1, D)
                    + 0.5 * _randn((nh, bs, D), gh, gd))
            k[blocks, :, j, :] = keys.to(dtype)
    cl = torch.full((B,), ctx, dtype=torch.int32)
    wl = Workload("config4", q, k, v, bt, cl, len(heads), bs, budget_pct=0.05, tau=0.90,
                  sink_pages=1, local_pages=2, check_interval=4,
                  meta=dict(alpha=alpha, seed=seed, kv_heads=(heads[0], heads[-1] + 1)))
    return wl.to(device)


def config3(device="cpu", seed: int = 0, alpha: float = ALPHA_C3, ctx: int = 131072,
            gen_device: Optional[str] = None, dtype: torch.dtype = torch.bfloat16,
            rho: float = 0.999) -> Workload:
    """Single 128K sequence, Llama-8B geometry, keys with a drifting mean.

    Keys: mu_t = rho * mu_{t-1} + sqrt(1 - rho^2) * eta_t (eta ~ N(0, I_D) per
    KV head), k_t = mu_t + N(0, 1); V ~ N(0, 1); 16 heavy pages per head with
    keys s * alpha * q_hat + 0.5 * N(0, 1), s ~ logU[1, 4]. The AR(1) recursion
    is evaluated in closed form over chunks (float64). Budget
    int(8192 * 0.05) = 409 plus forced pages.
    """
    gd = gen_device or (device if str(device).startswith("cuda") else "cpu")
    g = torch.Generator(device=gd).manual_seed(seed)
    gc = torch.Generator(device="cpu").manual_seed(seed + 1)
    B, Hq, Hkv, D, bs = 1, 32, 8, 128, 16
    W = ctx // bs
    T = ctx
    q = _randn((B, Hq, D), g, gd).to(dtype)
    # AR(1) mean per (head, dim) along tokens, chunked closed form
    c = math.sqrt(1.0 - rho * rho)
    mu = torch.empty((T, Hkv, D), dtype=torch.float32, device=gd)
    prev = torch.zeros((Hkv, D), dtype=torch.float64, device=gd)
    L = 2048
    pw = rho ** torch.arange(L, dtype=torch.float64, device=gd)       # rho^j
    for t0 in range(0, T, L):
        n = min(L, T - t0)
        eta = _randn((n, Hkv, D), g, gd).double()
        # mu_{t0+j} = rho^{j+1} prev + c * sum_{i<=j} rho^{j-i} eta_i
        scaled = eta / pw[:n].view(n, 1, 1)
        acc = torch.cumsum(scaled, 0) * pw[:n].view(n, 1, 1)
        blk = rho * pw[:n].view(n, 1, 1) * prev.view(1, Hkv, D) + c * acc
        mu[t0:t0 + n] = blk.float()
        prev = blk[-1]
    k = (mu + _randn((T, Hkv, D), g, gd)).to(dtype).view(W, bs, Hkv, D)
    del mu
    v = _randn((W, bs, Hkv, D), g, gd).to(dtype)
    perm = torch.randperm(W, generator=gc).to(torch.int32)
    kp = torch.empty_like(k)
    vp = torch.empty_like(v)
    kp[perm.long().to(gd)] = k
    vp[perm.long().to(gd)] = v
    k, v = kp, vp
    bt = perm.view(1, W).contiguous()
    qh = _unit_group_query(q, Hkv)
    heavy = {}
    for h in range(Hkv):
        cand = torch.arange(1, W - 2)
        pos = cand[torch.randperm(cand.numel(), generator=gc)[:16]]
        strength = torch.exp(torch.empty(16).uniform_(0.0, math.log(4.0), generator=gc))
        heavy[h] = (pos.tolist(), strength.tolist())
        blocks = bt[0, pos].long().to(gd)
        keys = (strength.to(gd).view(16, 1, 1) * alpha * qh[0, h].view(1, 1, D)
                + 0.5 * _randn((16, bs, D), g, gd))
        k[blocks, :, h, :] = keys.to(dtype)
    cl = torch.tensor([ctx], dtype=torch.int32)
    wl = Workload("config3", q, k, v, bt, cl, Hkv, bs, budget_pct=0.05, tau=0.90,
                  sink_pages=1, local_pages=2, check_interval=4,
                  meta=dict(alpha=alpha, seed=seed, rho=rho))
    return wl.to(device)


def small(device="cpu", seed: int = 0, B: int = 2, Hq: int = 8, Hkv: int = 2, D: int = 128,
          ctx=(1000, 2048), W: Optional[int] = None, dtype=torch.bfloat16,
          heavy_alpha: float = 4.0, shuffle: bool = True, budget_pct: float = 0.1,
          sink_pages: int = 1, local_pages: int = 2, tau: float = 0.9) -> Workload:
    """Reduced-size workload for parity tests: ragged contexts, planted pages."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    bs = 16
    ctx = list(ctx) if isinstance(ctx, (list, tuple)) else [ctx] * B
    assert len(ctx) == B
    nvs = [(c + bs - 1) // bs for c in ctx]
    W = W or max(max(nvs), 1)
    NB = max(sum(nvs), 1) + 8
    q = _randn((B, Hq, D), g, "cpu").to(dtype)
    k = _randn((NB, bs, Hkv, D), g, "cpu")
    v = _randn((NB, bs, Hkv, D), g, "cpu").to(dtype)
    perm = torch.randperm(NB, generator=g) if shuffle else torch.arange(NB)
    bt = torch.zeros((B, W), dtype=torch.int32)
    off = 0
    for b in range(B):
        bt[b, :nvs[b]] = perm[off:off + nvs[b]].to(torch.int32)
        off += nvs[b]
    qh = _unit_group_query(q, Hkv)
    for b in range(B):
        for h in range(Hkv):
            if nvs[b] < 4:
                continue
            nh = int(torch.randint(1, 5, (1,), generator=g))
            pos = torch.randperm(nvs[b], generator=g)[:nh]
            for p in pos.tolist():
                s = float(torch.empty(1).uniform_(0.5, 2.0, generator=g))
                k[int(bt[b, p]), :, h, :] = (s * heavy_alpha * qh[b, h]
                                             + 0.5 * _randn((bs, D), g, "cpu"))
    cl = torch.tensor(ctx, dtype=torch.int32)
    wl = Workload("small", q, k.to(dtype), v, bt, cl, Hkv, bs, budget_pct=budget_pct, tau=tau,
                  sink_pages=sink_pages, local_pages=local_pages, check_interval=4,
                  meta=dict(seed=seed))
    return wl.to(device)


@dataclass
class RaggedWorkload:
    """A batch in a paged pool that grows by one token per sequence per step."""
    name: str
    cache: object               # cvsa.runtime.kv_cache.PagedKVCache
    mgr: object                 # cvsa.runtime.kv_cache.SequenceKVManager
    q: torch.Tensor             # [B, Hq, D] query of every step
    k_new: torch.Tensor         # [B, Hkv, D] appended token of every step
    v_new: torch.Tensor
    budget_pct: float
    tau: float
    sink_pages: int
    local_pages: int
    check_interval: int
    meta: Dict = field(default_factory=dict)


def config5(device="cuda", seed: int = 0, n_seqs: int = 64, min_len: int = 1024,
            max_len: int = 65536, grow: int = 256, Hq: int = 32, Hkv: int = 8, D: int = 128,
            dtype: torch.dtype = torch.bfloat16) -> RaggedWorkload:
    """Ragged batch: n_seqs sequences with lengths ~ U[min_len, max_len], room
    to grow by `grow` tokens each, in a pool whose free list is shuffled (pages
    are handed out in random order, so every table is fragmented). K = 0.1 *
    N(0, 1), V ~ N(0, 1), no planted pages: attention is diffuse and nearly
    every head fails tau = 0.9, so scoring steps recover almost every page.
    The block-table width is the longest possible sequence, so the budget
    int(W * 0.05) is the same for every sequence (the reference's budget
    comes from the table width, backend.py:690).
    """
    from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
    bs = 16
    gc = torch.Generator(device="cpu").manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (n_seqs,), generator=gc)
    pages = ((lens + grow + bs - 1) // bs).tolist()
    nb = int(sum(pages)) + n_seqs
    free = torch.randperm(nb, generator=gc).to(torch.int32)
    cache = PagedKVCache(nb, bs, Hkv, D, dtype=dtype, device=device, free_list=free)
    mgr = SequenceKVManager(cache, n_seqs, max_len + grow)
    g = torch.Generator(device=device).manual_seed(seed + 1)
    for b in range(n_seqs):
        n = int(lens[b])
        k = 0.1 * torch.randn((n, Hkv, D), generator=g, device=device)
        v = torch.randn((n, Hkv, D), generator=g, device=device)
        mgr.prefill_kv(b, k.to(dtype), v.to(dtype))
    q = torch.randn((n_seqs, Hq, D), generator=g, device=device).to(dtype)
    k_new = (0.1 * torch.randn((n_seqs, Hkv, D), generator=g, device=device)).to(dtype)
    v_new = torch.randn((n_seqs, Hkv, D), generator=g, device=device).to(dtype)
    return RaggedWorkload("config5", cache, mgr, q, k_new, v_new, budget_pct=0.05, tau=0.9,
                          sink_pages=1, local_pages=2, check_interval=4,
                          meta=dict(seed=seed, lens=lens.tolist(), grow=grow))
