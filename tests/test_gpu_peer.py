"""NVLink peer-memory exchanges (cvsa.peer.PeerExchange, csrc/peer.cu).

On one GPU: a one-rank group exercises the push, flag and bounded wait of
every kernel against plain results (the row gathered is the row pushed, the
minimum is the input, the merge equals cvsa_rank_merge of the one row), and
consecutive calls alternate the two buffer slots. On two or more GPUs (one
process per GPU, NCCL group): all-gather, minimum and merge against NCCL and
cvsa_rank_merge on the same rows, over several calls of different sizes, and
the page split run with the peer exchange against the same split with NCCL
all-gathers.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _merge_rows(world, B, H, G, D, gen):
    """world partial rows [o | m | l] with some -inf (empty) rows."""
    rows = B * H * G
    parts = torch.randn((world, rows * (D + 2)), generator=gen)
    m = parts[:, rows * D:rows * (D + 1)]
    l = parts[:, rows * (D + 1):]
    l.copy_(l.abs() + 0.5)
    m[0, 3] = float("-inf")
    return parts


def test_peer_one_rank(cuda):
    from cvsa.kernels.coverage import rank_merge
    from cvsa.peer import PeerExchange
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, H, G, D = 2, 4, 4, 64
        px = PeerExchange(max(4100, B * H * G * (D + 2)), device=cuda)
        gen = torch.Generator().manual_seed(5)
        for n in (1, 37, 1024, 4100):
            x = torch.randn(n, generator=gen).to(cuda)
            got = px.allgather(x)
            assert got.shape == (1, n) and torch.equal(got[0], x)
        w = torch.randint(-5, 5, (3,), generator=gen, dtype=torch.int32).to(cuda)
        ref = w.clone()
        assert torch.equal(px.min_i32(w), ref)
        for _ in range(3):
            parts = _merge_rows(1, B, H, G, D, gen).to(cuda)
            out = torch.empty((B, H * G, D), dtype=torch.float32, device=cuda)
            ref = torch.empty_like(out)
            px.merge(parts[0].contiguous(), B, H, G, D, out)
            rank_merge(parts, B, H, G, D, ref)
            assert torch.allclose(out, ref, rtol=1e-6, atol=1e-6)
        torch.cuda.synchronize()
        assert int(px.dev_error.item()) == 0
        px.close()
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        from cvsa import synthetic
        from cvsa.kernels.coverage import rank_merge
        from cvsa.pagesplit import PageSplitBackend, dist_allgather, run_step, shard_sequence
        from cvsa.peer import PeerExchange
        B, H, G, D = 2, 8, 4, 128
        wl = synthetic.small(seed=41, B=B, Hq=H * G, Hkv=H, D=D, ctx=(9000, 4100),
                             heavy_alpha=4.0, budget_pct=0.05).to(dev)
        max_sel = 64
        px = PeerExchange(PageSplitBackend.exchange_row_cap(B, H, H * G, D, max_sel),
                          device=dev)
        gen = torch.Generator().manual_seed(100 + rank)
        ok = True
        for n in (5, 1024, 3000, B * H * G * (D + 2)):
            x = torch.randn(n, generator=gen).to(dev)
            ref = torch.empty((world, n), device=dev)
            dist.all_gather_into_tensor(ref, x)
            ok &= bool(torch.equal(px.allgather(x), ref))
        w = torch.randint(-9, 9, (4,), generator=gen, dtype=torch.int32).to(dev)
        ref = w.clone()
        dist.all_reduce(ref, op=dist.ReduceOp.MIN)
        ok &= bool(torch.equal(px.min_i32(w), ref))
        part = _merge_rows(1, B, H, G, D, gen)[0].to(dev)
        parts = torch.empty((world, part.numel()), device=dev)
        dist.all_gather_into_tensor(parts, part)
        out = torch.empty((B, H * G, D), dtype=torch.float32, device=dev)
        ref = torch.empty_like(out)
        px.merge(part, B, H, G, D, out)
        rank_merge(parts, B, H, G, D, ref)
        ok &= bool(torch.allclose(out, ref, rtol=1e-6, atol=1e-6))
        # the page split over the peer exchange against the same split over NCCL
        k, v, bt, cl = shard_sequence(wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens,
                                      rank, world, 16)
        kw = dict(num_layers=1, budget_pct=0.05, coverage_threshold=0.9, lazy=True,
                  check_interval=2, sink_pages=1, local_pages=2)
        pn = PageSplitBackend(H, H * G, D, 16, rank, world, **kw)
        pp = PageSplitBackend(H, H * G, D, 16, rank, world, exchange=px, **kw)
        ag = dist_allgather()
        qg = torch.Generator().manual_seed(7)
        for step in range(5):
            q = (wl.q.float().cpu() + 0.6 * torch.randn(wl.q.shape, generator=qg)).to(
                wl.q.dtype).to(dev)
            a = run_step(pn.step(q, k, v, bt, cl, 0, wl.context_lens, wl.block_tables.shape[1]),
                         ag)
            b = run_step(pp.step(q, k, v, bt, cl, 0, wl.context_lens, wl.block_tables.shape[1]),
                         ag)
            ok &= bool(torch.allclose(a.float(), b.float(), rtol=1e-2, atol=1e-2))
            ci, cn = pn.cached_selection(0)
            di, dn = pp.cached_selection(0)
            ok &= bool(torch.equal(cn, dn))
            for bb in range(B):
                for hh in range(H):
                    nn = int(cn[bb, hh])
                    ok &= bool(torch.equal(ci[bb, hh, :nn], di[bb, hh, :nn]))
            pn.step_done(0, 1)
            pp.step_done(0, 1)
        ok &= pn.stats == pp.stats
        torch.cuda.synchronize()
        ok &= int(px.dev_error.item()) == 0
        px.close()
        results[rank] = ok
    finally:
        dist.destroy_process_group()


def test_peer_two_gpus():
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs (the one-GPU test covers the kernels on one rank)")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    assert len(results) == world and all(results.values()), dict(results)


def test_peer_wait_runs_out(cuda):
    """A rank that never arrives: a two-rank exchange on one GPU whose second
    rank's buffer is a plain local buffer nobody writes into this rank's. With
    the wait limit cut to a few polls, every call returns and records
    CVSA_DEV_ERR_TIMEOUT (no hang); the words that did land are still right;
    with the limit restored a one-rank exchange on the same buffer runs clean."""
    import ctypes
    from cvsa import _lib
    lib = _lib.load()
    n = 300
    nbytes = lib.cvsa_peer_buffer_bytes(2, n)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        h = ctypes.create_string_buffer(64)
        _lib.check(lib.cvsa_peer_alloc(nbytes, ctypes.byref(p), h), "cvsa_peer_alloc")
        bufs.append(p.value)
    try:
        bases = torch.tensor(bufs, dtype=torch.int64, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        desc = _lib.PeerDesc(bases.data_ptr(), 2, 0, n, err.data_ptr())
        x = torch.randn(n, device=cuda)
        out = torch.full((2, n), 7.0, device=cuda)
        lib.cvsa_set_wait_limit(64)
        try:
            _lib.check(lib.cvsa_peer_allgather(ctypes.byref(desc), x.data_ptr(), n,
                                               out.data_ptr(), _lib.stream_ptr(cuda)),
                       "cvsa_peer_allgather")
            torch.cuda.synchronize()
        finally:
            lib.cvsa_set_wait_limit(0)
        assert int(err.item()) & _lib.DEV_ERR_TIMEOUT
        assert torch.equal(out[0], x)            # this rank's own row landed
        # a clean one-rank exchange on the same buffer afterwards
        err.zero_()
        lib.cvsa_peer_free(ctypes.c_void_p(bufs.pop()))
        one = _lib.PeerDesc(bases.data_ptr(), 1, 0, n, err.data_ptr())
        out1 = torch.empty((1, n), device=cuda)
        _lib.check(lib.cvsa_peer_allgather(ctypes.byref(one), x.data_ptr(), n, out1.data_ptr(),
                                           _lib.stream_ptr(cuda)), "cvsa_peer_allgather")
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and torch.equal(out1[0], x)
    finally:
        for p in bufs:
            lib.cvsa_peer_free(ctypes.c_void_p(p))
