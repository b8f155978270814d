"""Page-split step on the GPU kernels: ranks emulated in one process.

The ranks of a page split (each holding a contiguous range of every
sequence's pages) run PageSplitBackend with the CUDA kernels; their step
generators are driven in lockstep, each exchange served by stacking the
ranks' tensors -- what all_gather returns. Every rank's output must match
the oracle (OracleBackend over the whole context, CPU) and CVSABackend within
the bf16 bar, and the ranks' cached selections, mapped back to global pages,
must together be the oracle's cached selection, across a lazy schedule with
rescoring and reuse steps.
"""

import pytest
import torch

from cvsa import synthetic
from cvsa.backend import CVSABackend
from cvsa.pagesplit import PageSplitBackend, page_range, shard_sequence
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _lockstep(gens):
    xs = [next(g) for g in gens]
    while True:
        stacked = torch.stack(xs)
        outs, done = [], 0
        for g in gens:
            try:
                outs.append(g.send(stacked))
            except StopIteration as e:
                outs.append(e.value)
                done += 1
        if done:
            assert done == len(gens), "ranks left the exchange at different points"
            return outs
        xs = outs


def _check_close(out, ref, step):
    a, b = out.float(), ref.float()
    assert ((a - b).abs() <= 2e-2 + 1e-2 * b.abs()).all(), (step, float((a - b).abs().max()))


@pytest.mark.parametrize("world", [2, 4])
def test_page_split_matches_one_gpu(cuda, world):
    wl = synthetic.small(seed=31, B=2, Hq=32, Hkv=8, D=128, ctx=(9000, 4100), heavy_alpha=4.0,
                         budget_pct=0.05)
    d = wl.to(cuda)
    kw = dict(num_layers=1, budget_pct=0.05, coverage_threshold=0.9, lazy=True,
              check_interval=2, sink_pages=1, local_pages=2)
    full = CVSABackend(8, 32, 128, 16, **kw)
    ob = R.OracleBackend(8, 32, 128, 16, **kw)
    ranks = []
    nv = (wl.context_lens.long() + 15) // 16
    for r in range(world):
        k, v, bt, cl = shard_sequence(d.k_cache, d.v_cache, d.block_tables, d.context_lens,
                                      r, world, 16)
        ranks.append((PageSplitBackend(8, 32, 128, 16, r, world, **kw), k, v, bt, cl,
                      page_range(nv, r, world)))
    g = torch.Generator(device="cpu").manual_seed(4)
    for step in range(6):
        q = (wl.q.float() + 0.6 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype).to(cuda)
        ref = full(q, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        oref = ob(q.cpu(), wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        _check_close(ref.cpu(), oref, step)
        outs = _lockstep([pb.step(q, k, v, bt, cl, 0, d.context_lens, d.block_tables.shape[1])
                          for pb, k, v, bt, cl, _ in ranks])
        for out in outs:
            _check_close(out, ref, step)
            _check_close(out.cpu(), oref, step)
        fi, fn = ob._cached[0]
        for b in range(2):
            for h in range(8):
                union = []
                for pb, *_rest, (lo, hi) in ranks:
                    li, ln = pb.cached_selection(0)
                    union += [p + int(lo[b]) for p in li[b, h, :int(ln[b, h])].tolist()]
                assert union == fi[b, h, :int(fn[b, h])].tolist(), (step, b, h)
        full.step_done(0, 1)
        ob.step_done(0, 1)
        for pb, *_ in ranks:
            pb.step_done(0, 1)


def test_page_split_steps_replay_as_graphs(cuda):
    """The check and reuse steps of two lockstep ranks, captured once each as
    CUDA graphs (no device value is read on the host inside a step), replayed
    over a lazy schedule with fresh queries copied into the captured input:
    every replay must match CVSABackend's step, and the in-place cached
    selections its cached selection."""
    world = 2
    wl = synthetic.small(seed=32, B=2, Hq=32, Hkv=8, D=128, ctx=(8000, 5000), heavy_alpha=4.0,
                         budget_pct=0.05)
    d = wl.to(cuda)
    kw = dict(num_layers=1, budget_pct=0.05, coverage_threshold=0.9, lazy=True,
              check_interval=2, sink_pages=1, local_pages=2)
    full = CVSABackend(8, 32, 128, 16, **kw)
    nv = (wl.context_lens.long() + 15) // 16
    ranks = []
    for r in range(world):
        k, v, bt, cl = shard_sequence(d.k_cache, d.v_cache, d.block_tables, d.context_lens,
                                      r, world, 16)
        ranks.append((PageSplitBackend(8, 32, 128, 16, r, world, **kw), k, v, bt, cl,
                      page_range(nv, r, world)))
    qbuf = d.q.clone()
    W = d.block_tables.shape[1]

    def lockstep():
        return _lockstep([pb.step(qbuf, k, v, bt, cl, 0, d.context_lens, W)
                          for pb, k, v, bt, cl, _ in ranks])

    g = torch.Generator(device="cpu").manual_seed(9)
    queries = [(wl.q.float() + 0.6 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
               for _ in range(8)]
    # step 0 eager: no cached selection yet
    qbuf.copy_(queries[0].to(cuda))
    outs0 = lockstep()
    ref = full(qbuf, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
    for out in outs0:
        _check_close(out, ref, 0)
    full.step_done(0, 1)
    graphs, static = {}, {}
    for kind, step_idx in (("check", 0), ("reuse", 1)):
        for pb, *_ in ranks:
            pb._step = step_idx
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            static[kind] = lockstep()
        graphs[kind] = gr
    for step in range(1, 8):
        kind = "check" if step % 2 == 0 else "reuse"
        qbuf.copy_(queries[step].to(cuda))
        graphs[kind].replay()
        ref = full(qbuf, d.k_cache, d.v_cache, d.block_tables, d.context_lens, 0)
        torch.cuda.synchronize()
        for out in static[kind]:
            _check_close(out, ref, step)
        fi, fn = full.cached_selection(0)
        for b in range(2):
            for h in range(8):
                union = []
                for pb, *_rest, (lo, hi) in ranks:
                    li, ln = pb.cached_selection(0)
                    union += [p + int(lo[b]) for p in li[b, h, :int(ln[b, h])].tolist()]
                assert union == fi[b, h, :int(fn[b, h])].tolist(), (step, b, h)
        full.step_done(0, 1)


def _rank_scores(gen, B, H, W, lens, ties):
    """Page scores of one rank: -inf past each sequence's valid pages, some
    exact ties (ties=True), one non-finite valid page."""
    s = torch.randn((B, H, W), generator=gen)
    if ties:
        s = (s * 4).round() / 4           # many equal values
    nv = (lens.long() + 15) // 16
    for b in range(B):
        s[b, :, int(nv[b]):] = float("-inf")
        if int(nv[b]) > 3:
            s[b, 0, 2] = float("-inf")      # a valid page with a -inf score
    return s


@pytest.mark.parametrize("world,ties", [(3, True), (2, False), (4, True)])
def test_split_kernels_match_oracle(cuda, world, ties):
    """cvsa_split_propose / cvsa_split_gate against their oracle restatement
    on the same inputs: exchange rows (log-sum-exps within 1e-5, candidates and
    their pages exactly), then from the same gathered rows every rank's
    selection, bitmap, gate, decision word and counters exactly (gates away
    from the threshold). Ragged ranks, one with fewer candidates than the
    budget, forced sink / local pages, ties and a -inf page."""
    from cvsa.kernels import split as SK
    gen = torch.Generator().manual_seed(100 + world)
    B, H, budget, sink, local = 3, 4, 7, 1, 2
    max_sel = budget + sink + local
    lens_all = torch.tensor([[700, 100, 2000], [650, 40, 1900], [600, 90, 1800],
                             [640, 60, 1700]], dtype=torch.int32)[:world]
    W = int(((lens_all.long() + 15) // 16).max())
    rows_dev, props, inputs = [], [], []
    for r in range(world):
        lens = lens_all[r]
        s = _rank_scores(gen, B, H, W, lens, ties)
        sink_r = sink if r == 0 else 0
        local_r = local if r == world - 1 else 0
        ci = torch.randint(0, W, (B, H, max_sel), generator=gen, dtype=torch.int32)
        cn = torch.randint(0, max_sel + 1, (B, H), generator=gen, dtype=torch.int32)
        n_row = SK.row_floats(B, H, max_sel)
        row_d = torch.empty(n_row, dtype=torch.float32, device=cuda)
        prop_d = SK.split_propose(s.to(cuda), lens.to(cuda), 16, (ci.to(cuda), cn.to(cuda)),
                                  sink_r, local_r, budget, max_sel, row_d)
        row_o = torch.empty(n_row, dtype=torch.float32)
        prop_o = R.split_propose(s, lens, 16, (ci, cn), sink_r, local_r, budget, max_sel, row_o)
        rd = row_d.cpu()
        rows = B * H
        assert torch.allclose(rd[:3 * rows], row_o[:3 * rows], atol=1e-5, rtol=1e-5,
                              equal_nan=False), r
        assert torch.equal(rd[3 * rows:], row_o[3 * rows:]), r
        assert torch.equal(prop_d.cpu(), prop_o), r
        rows_dev.append(rd)
        props.append((prop_d, prop_o))
        inputs.append((lens, sink_r, local_r))
    parts = torch.stack(rows_dev)
    tau = 0.6
    for r in range(world):
        lens, sink_r, local_r = inputs[r]
        state_d = torch.zeros(4, dtype=torch.int32, device=cuda)
        ctr_d = torch.zeros(6, dtype=torch.int64, device=cuda)
        state_o = torch.zeros(4, dtype=torch.int32)
        ctr_o = torch.zeros(6, dtype=torch.int64)
        for has_cache, mode in ((True, 3), (False, 3), (False, 0)):
            got_d = SK.split_gate(parts.to(cuda), props[r][0], lens.to(cuda), 16, W, r, budget,
                                  max_sel, sink_r, local_r, tau, has_cache, mode, state_d, ctr_d)
            got_o = R.split_gate(parts, props[r][1], lens, 16, W, r, budget, max_sel, sink_r,
                                 local_r, tau, has_cache, mode, state_o, ctr_o)
            sel_d, n_d, acc_d, bm_d = (t.cpu() for t in got_d)
            sel_o, n_o, acc_o, bm_o = got_o
            assert torch.equal(n_d, n_o), (r, has_cache)
            for b in range(B):
                for h in range(H):
                    k = int(n_o[b, h])
                    assert sel_d[b, h, :k].tolist() == sel_o[b, h, :k].tolist(), (r, b, h)
            assert torch.equal(bm_d, bm_o), r
            assert torch.equal(acc_d, acc_o), r
            assert int(state_d[3]) == int(state_o[3]), r
            assert torch.equal(state_d[:3].cpu(), torch.zeros(3, dtype=torch.int32)), r
        assert torch.equal(ctr_d.cpu(), ctr_o), r
