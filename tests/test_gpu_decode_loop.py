"""The reference's batched decode loop driven against the package.

eval/latency_benchmark.py:361-460 (benchmark_decode_batched) builds one
PagedKVCache + SequenceKVManager per layer, prefills every sequence with the
same K/V, and then each decode step, per layer: appends the new token's K/V
sequence by sequence with manager.append_token_kv(b, ...) (:447-450), calls
backend(q, cache.k_cache, cache.v_cache, manager.block_tables,
manager.context_lens, layer_idx) (:452-454) and finally
backend.step_done(layer_idx, num_layers). No checkpoint is available, so the
model's projections are replaced by seeded synthetic q / k / v of the same
shapes; the call pattern and the data flow through the caches are the
reference's. The same schedule runs on the oracle (PagedKVRef +
OracleBackend, CPU); per step and layer the outputs must agree within the
bf16 bar, the context lengths and block tables exactly, and the final
statistics exactly.
"""

import pytest
import torch

from cvsa.backend import CVSABackend
from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu

B, HQ, HKV, D, BS = 3, 8, 2, 128, 16
LAYERS, PREFILL, STEPS = 2, 300, 24


def test_reference_decode_loop_call_pattern(cuda):
    g = torch.Generator().manual_seed(123)
    max_ctx = PREFILL + STEPS + 16
    n_pages = (PREFILL + BS - 1) // BS
    num_blocks = (n_pages + 16 + 64) * B
    kw = dict(num_layers=LAYERS, budget_pct=0.1, coverage_threshold=0.9, lazy=True,
              check_interval=4, dense_layers=[0])
    be = CVSABackend(HKV, HQ, D, BS, **kw)
    ob = R.OracleBackend(HKV, HQ, D, BS, **kw)
    caches, mgrs, refs = [], [], []
    for _ in range(LAYERS):
        cache = PagedKVCache(num_blocks, BS, HKV, D, dtype=torch.bfloat16, device="cuda")
        mgr = SequenceKVManager(cache, B, max_ctx)
        ref = R.PagedKVRef(num_blocks, BS, HKV, D, torch.bfloat16, B, max_ctx)
        k = torch.randn((PREFILL, HKV, D), generator=g).to(torch.bfloat16)
        v = torch.randn((PREFILL, HKV, D), generator=g).to(torch.bfloat16)
        for b in range(B):                           # every sequence the same prompt
            mgr.prefill_kv(b, k.to(cuda), v.to(cuda))
            ref.prefill(b, k, v)
        caches.append(cache)
        mgrs.append(mgr)
        refs.append(ref)
    be.reset()
    for step in range(STEPS):
        for layer in range(LAYERS):
            cache, mgr, ref = caches[layer], mgrs[layer], refs[layer]
            q = torch.randn((B, HQ, D), generator=g).to(torch.bfloat16)
            k = torch.randn((B, HKV, D), generator=g).to(torch.bfloat16)
            v = torch.randn((B, HKV, D), generator=g).to(torch.bfloat16)
            kd, vd = k.to(cuda), v.to(cuda)
            for b in range(B):
                mgr.append_token_kv(b, kd[b], vd[b])
                ref.append(b, k[b], v[b])
            out = be(q.to(cuda), cache.k_cache, cache.v_cache, mgr.block_tables,
                     mgr.context_lens, layer)
            want = ob(q, ref.k, ref.v, ref.block_tables, ref.context_lens, layer)
            assert (out.float().cpu() - want.float()).abs().max() < 2e-2, (step, layer)
            be.step_done(layer, LAYERS)
            ob.step_done(layer, LAYERS)
        for layer in range(LAYERS):
            assert torch.equal(mgrs[layer].context_lens.cpu(), refs[layer].context_lens)
            assert torch.equal(mgrs[layer].block_tables.cpu(), refs[layer].block_tables)
    for c in caches:
        c.check()
    st, so = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        assert abs(st[key] - so[key]) < 1e-9, key
    assert st["total_decode_steps"] == STEPS
