"""A ragged batch that grows while it decodes (SURVEY config 5, reduced).

Sequences of very different lengths live in a pool whose free list is
shuffled; every step appends one token per sequence on the device
(cvsa_paged_append: new pages come off the free list when a page fills) and
runs one lazy-schedule layer step. The same steps run through the oracle
backend on copies of the cache: outputs within the bf16 bar, cached
selections identical, statistics equal; the appended tokens land where the
block tables say, and pages are never handed out twice.
"""

import pytest
import torch

from conftest import sel_sets
from cvsa import synthetic
from cvsa.backend import CVSABackend
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _close(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    assert ((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all(), float((a - b).abs().max())


def test_ragged_growing_batch_vs_oracle(cuda):
    wl = synthetic.config5(device=cuda, seed=3, n_seqs=4, min_len=20, max_len=2200, grow=40,
                           Hq=8, Hkv=2, D=128)
    mgr, cache = wl.mgr, wl.cache
    kw = dict(num_layers=1, budget_pct=0.1, coverage_threshold=0.9, lazy=True, check_interval=2,
              sink_pages=1, local_pages=2)
    be = CVSABackend(2, 8, 128, 16, **kw)
    ob = R.OracleBackend(2, 8, 128, 16, **kw)
    g = torch.Generator(device="cpu").manual_seed(9)
    lens0 = mgr.context_lens.cpu().clone()
    for step in range(24):
        k_new = (0.1 * torch.randn((4, 2, 128), generator=g)).to(torch.bfloat16)
        v_new = torch.randn((4, 2, 128), generator=g).to(torch.bfloat16)
        mgr.append_batch(k_new.to(cuda), v_new.to(cuda))
        q = torch.randn((4, 8, 128), generator=g).to(torch.bfloat16)
        out = be(q.to(cuda), cache.k_cache, cache.v_cache, mgr.block_tables, mgr.context_lens, 0)
        kc, vc = cache.k_cache.cpu(), cache.v_cache.cpu()
        bt, cl = mgr.block_tables.cpu(), mgr.context_lens.cpu()
        ref = ob(q, kc, vc, bt, cl, 0)
        _close(out, ref)
        # the appended token sits at position len - 1 of its sequence
        assert torch.equal(cl, lens0 + step + 1)
        for b in range(4):
            pos = int(cl[b]) - 1
            blk = int(bt[b, pos // 16])
            assert torch.equal(kc[blk, pos % 16], k_new[b])
            assert torch.equal(vc[blk, pos % 16], v_new[b])
        gi, gn = be.cached_selection(0)
        oi, on = ob._cached[0]
        assert sel_sets(gi.cpu(), gn.cpu()) == sel_sets(oi, on), step
        be.step_done(0, 1)
        ob.step_done(0, 1)
    cache.check()
    # every page in use appears in exactly one table slot
    used = [int(bt[b, p]) for b in range(4) for p in range((int(cl[b]) + 15) // 16)]
    assert len(used) == len(set(used))
    gs, os_ = be.get_stats(), ob.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate",
                "total_pages_attended", "total_pages_max"):
        assert abs(gs[key] - os_[key]) < 1e-9, (key, gs[key], os_[key])
