"""Head-sharded steps on one GPU: 2 or 8 shards, each a backend holding an
equal block of the KV heads (and their query heads; 8 shards leave one KV
head per shard, as on 8 GPUs), run the phased lazy step through begin_step /
finish_step with their decision words combined by MIN between the halves --
what the ranks do with an all-reduce -- and must reproduce one backend
holding every head: identical cached selections, outputs within the bf16
bar, the same reuse / rescore choices. The check step is built so the first
half of the heads accept their cached selection while the rest reject, so
the combined decision differs from some shards' own.
"""

import pytest
import torch

from cvsa import synthetic
from cvsa.backend import CVSABackend, shard_heads
from cvsa.kernels.select import budget_for
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _close(a, b):
    a, b = a.float(), b.float()
    assert ((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all(), float((a - b).abs().max())


@pytest.mark.parametrize("world", [2, 8])
def test_shards_match_one_backend(cuda, world):
    Hkv, Hq, D = 8, 32, 128
    wl = synthetic.small(seed=11, B=2, Hq=Hq, Hkv=Hkv, D=D, ctx=(4096, 2500), heavy_alpha=5.0)
    d = wl.to(cuda)
    g = torch.Generator(device="cpu").manual_seed(5)
    q_fresh = torch.randn(wl.q.shape, generator=g).to(wl.q.dtype)
    q_check = wl.q.clone()
    q_check[:, Hq // 2:] = q_fresh[:, Hq // 2:] * 3
    # tau between the shards' worst coverages of their cached selections at
    # the check step (oracle): shard 0's heads all accept, some of shard 1's
    # reject, so the combined decision overrides shard 0's own
    budget = budget_for(wl.block_tables.shape[1], 0.05)
    s0 = R.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, Hkv, Hq // Hkv, 16)
    idx0, n0 = R.select_pages(s0, wl.context_lens, 16, budget, 1, 2)
    s2 = R.score_pages(q_check, wl.k_cache, wl.block_tables, wl.context_lens, Hkv, Hq // Hkv, 16)
    _, cov2 = R.check_coverage(s2, idx0, n0, 0.5)
    min_a, min_b = float(cov2[:, :Hkv // 2].min()), float(cov2[:, Hkv // 2:].min())
    assert min_a > min_b + 0.05, (min_a, min_b)
    tau = (min_a + min_b) / 2
    kw = dict(head_dim=D, block_size=16, num_layers=1, budget_pct=0.05, coverage_threshold=tau,
              lazy=True, check_interval=2, sink_pages=1, local_pages=2)
    full = CVSABackend(Hkv, Hq, **kw)
    shards = []
    for r in range(world):
        kv_s, q_s = shard_heads(Hkv, Hq, r, world)
        be = CVSABackend(Hkv // world, Hq // world, **kw)
        shards.append((be, kv_s, q_s, d.k_cache[:, :, kv_s].contiguous(),
                       d.v_cache[:, :, kv_s].contiguous()))

    saw_split_decision = False
    for step in range(5):
        # check step 2: shard 1's query heads move away from their cached
        # pages; shard 0's stay
        q = (q_check if step == 2 else wl.q).to(cuda)
        out_full = full(q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        handles = [be.begin_step(q[:, q_s].contiguous(), kc, vc, d.block_tables, d.context_lens,
                                 0, phased=True)
                   for be, kv_s, q_s, kc, vc in shards]
        if handles[0].decision is not None:
            local = [int(h.decision.item()) for h in handles]
            saw_split_decision |= len(set(local)) > 1
            combined = handles[0].decision.clone()
            for h in handles[1:]:
                combined = torch.minimum(combined, h.decision)
            for h in handles:
                h.decision.copy_(combined)
            for (be, *_), h in zip(shards, handles):
                be.finish_step(h)
        out_sh = torch.cat([h.out for h in handles], dim=1)
        torch.cuda.synchronize()
        _close(out_sh, out_full)
        idx_f, n_f = full.cached_selection(0)
        for (be, kv_s, *_rest) in shards:
            idx_s, n_s = be.cached_selection(0)
            assert torch.equal(n_s, n_f[:, kv_s]), step
            for b in range(n_f.shape[0]):
                for h in range(n_s.shape[1]):
                    k = int(n_s[b, h])
                    assert torch.equal(idx_s[b, h, :k], idx_f[b, kv_s.start + h, :k]), (step, b, h)
        full.step_done(0, 1)
        for be, *_ in shards:
            be.step_done(0, 1)
    assert saw_split_decision, "the check step did not split the shards' decisions"
