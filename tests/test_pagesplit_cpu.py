"""Page-split step on CPU ranks (gloo, world size 2 and 3) with the oracle's ops.

Each rank holds a contiguous range of every sequence's pages
(pagesplit.shard_sequence) and runs PageSplitBackend with the oracle's
scoring, split proposal / gate / attention and merge in place of the CUDA
kernels, exchanging the proposal rows and the partials over a real gloo
group. Every rank's output must
equal the oracle backend's over the whole context (the single-GPU
semantics), its cached selection must be the oracle's selection restricted
to its pages, and every rank must take the same reuse / rescore decisions.
The device path (the same generator with the CUDA kernels) is checked in
tests/test_gpu_pagesplit.py.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cvsa import synthetic
from cvsa.pagesplit import PageSplitBackend, dist_allgather, page_range, run_step, shard_sequence
from oracle import cvsa_ref as R


class OracleOps:
    """The oracle's restatement of the kernels a page-split step runs."""
    score_pages = staticmethod(R.score_pages)
    split_propose = staticmethod(R.split_propose)
    split_gate = staticmethod(R.split_gate)
    split_attend = staticmethod(R.split_attend)

    @staticmethod
    def decode_unnorm(q, k, v, bt, idx, n, cl, H, G, bs, out=None):
        o, m, l = R.sparse_decode_unnorm(q, k, v, bt, idx, n, cl, H, G, bs)
        if out is None:
            return o, m, l
        for dst, src in zip(out, (o, m, l)):
            dst.copy_(src)
        return out

    @staticmethod
    def rank_merge(parts, B, H, G, D, out, need=None):
        """The LSE merge of cvsa/lse_merge.py:11-54 taken over the ranks
        (dim 0), in rank order, normalised by max(l, 1e-6)."""
        Hq = H * G
        o = parts[:, :B * Hq * D].reshape(-1, B, Hq, D)
        m = parts[:, B * Hq * D:B * Hq * (D + 1)].reshape(-1, B, Hq)
        l = parts[:, B * Hq * (D + 1):B * Hq * (D + 2)].reshape(-1, B, Hq)
        M = m.amax(0)
        w = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m),
                        torch.exp(m - torch.where(torch.isinf(M), torch.zeros_like(M), M)))
        res = (o * w.unsqueeze(-1)).sum(0) / (l * w).sum(0).clamp(min=1e-6).unsqueeze(-1)
        if need is None:
            out.copy_(res)
        else:
            nq = need.repeat_interleave(G, dim=1).unsqueeze(-1)
            out.copy_(torch.where(nq, res.to(out.dtype), out))
        return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        wl = synthetic.small(seed=21, B=2, Hq=8, Hkv=2, D=64, ctx=(3000, 1700),
                             dtype=torch.float32, heavy_alpha=4.0, budget_pct=0.1)
        kw = dict(num_layers=1, budget_pct=0.1, coverage_threshold=0.9, lazy=True,
                  check_interval=2, sink_pages=1, local_pages=2)
        ob = R.OracleBackend(2, 8, 64, 16, **kw)
        pb = PageSplitBackend(2, 8, 64, 16, rank, world, ops=OracleOps(), **kw)
        k, v, bt, cl = shard_sequence(wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens,
                                      rank, world, 16)
        nv = (wl.context_lens.long() + 15) // 16
        lo, hi = page_range(nv, rank, world)
        g = torch.Generator().manual_seed(3)
        ag = dist_allgather()
        for step in range(5):
            q = wl.q + 0.7 * torch.randn(wl.q.shape, generator=g)
            ref = ob(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
            out = run_step(pb.step(q, k, v, bt, cl, 0, wl.context_lens,
                                   wl.block_tables.shape[1]), ag)
            assert (out - ref).abs().max() <= 1e-4, (step, float((out - ref).abs().max()))
            oi, on = ob._cached[0]
            li, ln = pb.cached_selection(0)
            for b in range(2):
                for h in range(2):
                    full = [p for p in oi[b, h, :int(on[b, h])].tolist()
                            if int(lo[b]) <= p < int(hi[b])]
                    mine = [p + int(lo[b]) for p in li[b, h, :int(ln[b, h])].tolist()]
                    assert mine == full, (step, b, h, mine, full)
            ob.step_done(0, 1)
            pb.step_done(0, 1)
        os_ = ob.get_stats()
        results[rank] = (pb.stats["scoring_steps"], os_["total_scoring_steps"],
                         pb.stats["coverage_checks"], os_["total_coverage_checks"],
                         pb.stats["accept_steps"], ob.accept_counts,
                         pb.stats["reject_steps"], ob.reject_counts)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_page_split_matches_oracle(world):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    assert len(results) == world
    for r in range(world):
        got = results[r]
        assert got[0::2] == got[1::2], got
