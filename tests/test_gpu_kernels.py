"""GPU parity of each kernel entry point against the oracle and the reference.

Bars (from the north star): selection and accept decisions bit-exact (ties to
the lower page index); outputs within 1e-4 in fp32 and 2e-2 abs / 1e-2 rel in
bf16; coverage within 1e-3 (tested far tighter, 2e-5).
"""

import numpy as np
import pytest
import torch

from conftest import finite_close, sel_sets
from cvsa import synthetic
from cvsa.kernels import coverage as C
from cvsa.kernels import page_scores as P
from cvsa.kernels import select as S
from cvsa.kernels import sparse_decode as SD
from cvsa.complement import compute_complement_pages
from cvsa.lse_merge import selective_lse_merge
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_RTOL = 2e-2, 1e-2
F32_ATOL = 1e-4


def _golden_case(name):
    if name == "config1":
        return synthetic.config1()
    return synthetic.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))


def _out_close(a, b, dtype):
    a = a.float().cpu()
    b = torch.as_tensor(b).float().cpu()
    if dtype == torch.float32:
        assert (a - b).abs().max() <= F32_ATOL, float((a - b).abs().max())
    else:
        assert ((a - b).abs() <= BF16_ATOL + BF16_RTOL * b.abs()).all(), \
            float((a - b).abs().max())


def _dev(wl, cuda):
    return wl.to(cuda)


# ---------------------------------------------------------------- golden ---
@pytest.mark.parametrize("case", ["config1", "small"])
def test_kernels_match_reference_outputs(cuda, golden, case):
    wl = _golden_case(case)
    d = _dev(wl, cuda)
    H, G, bs = wl.num_kv_heads, wl.num_q_per_kv, wl.block_size
    s = P.triton_score_pages(d.q, d.k_cache, d.block_tables, d.context_lens, H, G, bs)
    finite_close(s.cpu(), golden[f"{case}_scores"], atol=2e-5, rtol=2e-6)
    idx = torch.from_numpy(golden[f"{case}_sel_idx"]).to(cuda)
    n = torch.from_numpy(golden[f"{case}_sel_n"]).to(cuda)
    o, m, l = SD.triton_sparse_decode_unnorm(d.q, d.k_cache, d.v_cache, d.block_tables, idx, n,
                                             d.context_lens, H, G, bs)
    finite_close(m.cpu(), golden[f"{case}_m_draft"], atol=1e-5, rtol=1e-6)
    if wl.q.dtype == torch.float32:
        finite_close(l.cpu(), golden[f"{case}_l_draft"], atol=1e-4, rtol=1e-5)
        finite_close(o.cpu(), golden[f"{case}_o_draft"], atol=1e-4, rtol=1e-5)
    gs = torch.from_numpy(golden[f"{case}_scores"]).to(cuda)
    acc, cov = C.triton_check_coverage(gs, idx, n, wl.tau)
    assert np.array_equal(acc.cpu().numpy().astype(np.uint8), golden[f"{case}_accept"])
    assert np.abs(cov.cpu().numpy() - golden[f"{case}_coverage"]).max() < 2e-5
    comp, nc = C.triton_compute_complement(idx, n, d.context_lens, bs, acc)
    assert np.array_equal(nc.cpu().numpy(), golden[f"{case}_n_comp"])
    # fused recovery (complement attention skipping selected pages + merge)
    out = SD.recover_merge(d.q, d.k_cache, d.v_cache, d.block_tables, idx, n, d.context_lens, acc,
                           o, m, l, H, G, bs)
    _out_close(out, golden[f"{case}_output"], wl.q.dtype)
    # unfused path of the reference: complement decode + merge kernel
    oc, mc, lc = SD.triton_sparse_decode_unnorm(d.q, d.k_cache, d.v_cache, d.block_tables, comp,
                                                nc, d.context_lens, H, G, bs)
    out2 = C.triton_lse_merge(o, m, l, oc, mc, lc, acc, H, G, wl.q.dtype)
    _out_close(out2, golden[f"{case}_output"], wl.q.dtype)


# ----------------------------------------------------------- selection ---
def _select_cases():
    g = torch.Generator().manual_seed(5)
    cases = []
    # random scores, ragged contexts, forced pages
    s = torch.randn(3, 4, 300, generator=g)
    cl = torch.tensor([4800, 17, 1], dtype=torch.int32)
    cases.append((s, cl, 25, 1, 2))
    # heavy ties: small integer scores, so the tie rule decides most picks
    s = torch.randint(0, 4, (2, 3, 512), generator=g).float()
    cl = torch.tensor([8192, 5000], dtype=torch.int32)
    cases.append((s, cl, 25, 0, 0))
    cases.append((s, cl, 40, 1, 2))
    # budget larger than the candidates; empty sequence
    s = torch.randn(2, 2, 64, generator=g)
    cl = torch.tensor([0, 100], dtype=torch.int32)
    cases.append((s, cl, 10, 1, 2))
    # long table (128K context), all candidates tied
    s = torch.zeros(1, 2, 8192)
    cl = torch.tensor([131072], dtype=torch.int32)
    cases.append((s, cl, 409, 1, 2))
    # -0.0 / +0.0 and denormals
    s = torch.tensor([[[0.0, -0.0, 1e-40, -1e-40, 0.0, 3.0, -0.0, 1e-40]]])
    cases.append((s, torch.tensor([128], dtype=torch.int32), 3, 0, 0))
    # long tables (one CTA of 1024 threads per head): random, ragged
    s = torch.randn(2, 3, 2000, generator=g)
    cl = torch.tensor([32000, 20000], dtype=torch.int32)
    cases.append((s, cl, 100, 1, 2))
    s = torch.randn(1, 2, 8192, generator=g) * 3
    cases.append((s, torch.tensor([131072], dtype=torch.int32), 409, 1, 2))
    # 12000 pages with heavy ties
    s = torch.randint(0, 8, (1, 4, 12000), generator=g).float()
    cases.append((s, torch.tensor([190000], dtype=torch.int32), 600, 1, 2))
    # scores on a 0.02 grid: a few equal keys inside the k-th key's value bin
    s = torch.round(torch.randn(2, 3, 4096, generator=g) * 50) / 50
    cases.append((s, torch.tensor([65536, 40000], dtype=torch.int32), 204, 1, 2))
    # 16384 pages (16 per thread)
    s = torch.randn(1, 2, 16384, generator=g)
    cases.append((s, torch.tensor([262144], dtype=torch.int32), 819, 1, 2))
    # non-finite candidate scores: -inf inside the valid range and one +inf
    s = torch.randn(1, 2, 3000, generator=g)
    s[0, 0, 100:400] = float("-inf")
    s[0, 1, 1234] = float("inf")
    cases.append((s, torch.tensor([48000], dtype=torch.int32), 150, 1, 2))
    return cases


@pytest.mark.parametrize("ci", range(12))
def test_select_bit_exact(cuda, ci):
    s, cl, budget, sink, local = _select_cases()[ci]
    nv = R.n_valid_pages(cl, 16)
    W = s.shape[-1]
    s = s.clone()
    for b in range(s.shape[0]):
        s[b, :, int(nv[b]):] = float("-inf")
    ri, rn = R.select_pages(s, cl, 16, budget, sink, local)
    gi, gn = S.select_pages(s.to(cuda), cl.to(cuda), 16, budget, sink, local)
    assert torch.equal(gn.cpu(), rn)
    # identical ascending lists, not only sets
    for b in range(s.shape[0]):
        for h in range(s.shape[1]):
            k = int(rn[b, h])
            assert gi[b, h, :k].cpu().tolist() == ri[b, h, :k].tolist(), (b, h)


def test_coverage_vs_oracle(cuda):
    g = torch.Generator().manual_seed(7)
    s = torch.randn(4, 8, 512, generator=g) * 3
    s[:, :, 400:] = float("-inf")
    cl = torch.full((4,), 400 * 16, dtype=torch.int32)
    idx, n = R.select_pages(s, cl, 16, 25, 1, 2)
    for tau in (0.5, 0.9, 0.99):
        ra, rc = R.check_coverage(s, idx, n, tau)
        ga, gc = C.triton_check_coverage(s.to(cuda), idx.to(cuda), n.to(cuda), tau)
        assert (gc.cpu() - rc).abs().max() < 2e-5
        margin = R.coverage_margin(rc, tau)
        decided = margin > 1e-5
        assert torch.equal(ga.cpu()[decided], ra[decided])


def test_complement_known_answers(cuda):
    idx = torch.tensor([[[0, 2, 4], [1, 3, 0]]], dtype=torch.int32, device=cuda)
    n = torch.tensor([[3, 2]], dtype=torch.int32, device=cuda)
    comp, nc = compute_complement_pages(idx, n, torch.tensor([160], dtype=torch.int32,
                                                              device=cuda), 16)
    assert nc.cpu().tolist() == [[7, 8]]
    assert comp[0, 0, :7].cpu().tolist() == [1, 3, 5, 6, 7, 8, 9]
    assert comp[0, 1, :8].cpu().tolist() == [0, 2, 4, 5, 6, 7, 8, 9]
    acc = torch.tensor([[True, False]], device=cuda)
    _, nc = compute_complement_pages(idx, n, torch.tensor([160], dtype=torch.int32, device=cuda),
                                     16, acc)
    assert nc.cpu().tolist() == [[0, 8]]


# -------------------------------------------------------------- decode ---
DECODE_SHAPES = [
    # B, Hq, Hkv, D, ctx, dtype
    (2, 8, 2, 128, (1000, 2048), torch.bfloat16),
    (3, 32, 8, 128, (4096, 17, 3000), torch.bfloat16),
    (2, 16, 2, 64, (700, 1600), torch.bfloat16),
    (2, 8, 1, 256, (999, 640), torch.bfloat16),
    (2, 8, 2, 128, (1000, 2048), torch.float16),
    (1, 8, 2, 64, (4096,), torch.float32),
    (2, 12, 2, 128, (512, 800), torch.bfloat16),      # G = 6
]


@pytest.mark.parametrize("shape", DECODE_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}x{s[3]}-{s[5]}")
def test_decode_and_recovery_vs_oracle(cuda, shape):
    B, Hq, Hkv, D, ctx, dt = shape
    wl = synthetic.small(seed=11, B=B, Hq=Hq, Hkv=Hkv, D=D, ctx=ctx, dtype=dt)
    d = wl.to(cuda)
    G, bs = wl.num_q_per_kv, wl.block_size
    s = R.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, Hkv, G, bs)
    gs = P.score_pages(d.q, d.k_cache, d.block_tables, d.context_lens, Hkv, G, bs)
    finite_close(gs.cpu(), s, atol=2e-5, rtol=2e-6)
    W = wl.block_tables.shape[1]
    idx, n = R.select_pages(s, wl.context_lens, bs, R.budget_for(W, 0.1), 1, 2)
    o, m, l = R.sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, idx, n,
                                     wl.context_lens, Hkv, G, bs)
    go, gm, gl = SD.sparse_decode_unnorm(d.q, d.k_cache, d.v_cache, d.block_tables,
                                         idx.to(cuda), n.to(cuda), d.context_lens, Hkv, G, bs)
    finite_close(gm.cpu(), m, atol=2e-5, rtol=2e-6)
    ref_norm = o / l.clamp(min=1e-6).unsqueeze(-1)
    _out_close(go.cpu() / gl.cpu().clamp(min=1e-6).unsqueeze(-1), ref_norm, dt)
    gout = SD.sparse_decode(d.q, d.k_cache, d.v_cache, d.block_tables, idx.to(cuda), n.to(cuda),
                            d.context_lens, Hkv, G, bs)
    assert gout.dtype == dt
    _out_close(gout, ref_norm.to(dt), dt)
    # exact recovery for a mixed accept mask
    acc = torch.zeros((B, Hkv), dtype=torch.bool)
    acc[:, 0] = True
    comp, nc = R.compute_complement_pages(idx, n, wl.context_lens, bs, acc)
    oc, mc, lc = R.sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, comp, nc,
                                        wl.context_lens, Hkv, G, bs)
    ref = R.selective_lse_merge(o, m, l, oc, mc, lc, acc, G, dt)
    gout = SD.recover_merge(d.q, d.k_cache, d.v_cache, d.block_tables, idx.to(cuda), n.to(cuda),
                            d.context_lens, acc.to(cuda), go, gm, gl, Hkv, G, bs)
    _out_close(gout, ref, dt)
    # rejected heads equal dense attention over all valid pages
    dense = R.dense_decode(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, Hkv, G,
                           bs)
    rej = ~acc.repeat_interleave(G, 1)
    _out_close(gout.cpu()[rej], dense[rej], dt)


def test_decode_empty_and_padded_selections(cuda):
    wl = synthetic.small(seed=2, B=3, Hq=8, Hkv=2, D=128, ctx=(16, 0, 400))
    d = wl.to(cuda)
    idx = torch.zeros((3, 2, 5), dtype=torch.int32)
    idx[0] = torch.tensor([0, 0, 0, 0, 0])
    idx[2, 0] = torch.tensor([24, 3, 0, 0, 0])      # page 24 lies past the context (25 pages)
    idx[2, 1] = torch.tensor([1, 2, 5, 6, 7])
    n = torch.tensor([[1, 0], [0, 0], [3, 5]], dtype=torch.int32)
    o, m, l = R.sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables, idx, n,
                                     wl.context_lens, 2, 4, 16)
    go, gm, gl = SD.sparse_decode_unnorm(d.q, d.k_cache, d.v_cache, d.block_tables, idx.to(cuda),
                                         n.to(cuda), d.context_lens, 2, 4, 16)
    finite_close(gm.cpu(), m, atol=2e-5, rtol=2e-6)
    assert torch.isfinite(go).all() and torch.isfinite(gl).all()
    assert (gl.cpu()[m == float("-inf")] == 0).all()
    out = SD.sparse_decode(d.q, d.k_cache, d.v_cache, d.block_tables, idx.to(cuda), n.to(cuda),
                           d.context_lens, 2, 4, 16)
    assert torch.isfinite(out.float()).all()
    assert (out.float().cpu()[m == float("-inf")] == 0).all()


def test_lse_merge_vs_reference_formula(cuda):
    g = torch.Generator().manual_seed(1)
    B, Hkv, G, D = 4, 8, 4, 128
    od, oc = torch.randn(B, Hkv * G, D, generator=g), torch.randn(B, Hkv * G, D, generator=g)
    md, mc = torch.randn(B, Hkv * G, generator=g), torch.randn(B, Hkv * G, generator=g)
    ld = torch.rand(B, Hkv * G, generator=g) + 0.1
    lc = torch.rand(B, Hkv * G, generator=g) + 0.1
    for rate in (0.0, 0.5, 1.0):
        acc = torch.rand(B, Hkv, generator=g) < rate
        ref = R.selective_lse_merge(od, md, ld, oc, mc, lc, acc, G, torch.float32)
        out = selective_lse_merge(*(t.to(cuda) for t in (od, md, ld, oc, mc, lc, acc)), G,
                                  torch.float32)
        assert (out.cpu() - ref).abs().max() < 1e-5
        out16 = selective_lse_merge(*(t.to(cuda) for t in (od, md, ld, oc, mc, lc, acc)), G,
                                    torch.bfloat16)
        # one bf16 rounding of the same fp32 value: within the bf16 bar
        assert ((out16.float().cpu() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()


@pytest.mark.parametrize("world", [1, 3, 8])
def test_rank_merge_vs_fp32_formula(cuda, world):
    """cvsa_rank_merge against the fp32 LSE merge over ranks (rank order),
    with empty partials (m = -inf, l = 0, o = 0) on some ranks and rows empty
    on every rank; `need` leaves the other heads' rows untouched."""
    from cvsa.kernels.coverage import rank_merge
    g = torch.Generator().manual_seed(world)
    B, Hkv, G, D = 3, 4, 4, 128
    Hq = Hkv * G
    o = torch.randn(world, B, Hq, D, generator=g)
    m = torch.randn(world, B, Hq, generator=g) * 3
    l = torch.rand(world, B, Hq, generator=g) + 0.1
    empty = torch.rand(world, B, Hq, generator=g) < 0.3
    empty[:, 0, 0] = True                                   # a row empty on every rank
    o[empty.unsqueeze(-1).expand_as(o)] = 0
    m[empty] = float("-inf")
    l[empty] = 0
    parts = torch.cat([o.reshape(world, -1), m.reshape(world, -1), l.reshape(world, -1),
                       torch.randn(world, 7, generator=g)], 1).contiguous()
    M = m.amax(0)
    w = torch.where(empty, torch.zeros_like(m),
                    torch.exp(m - torch.where(torch.isinf(M), torch.zeros_like(M), M)))
    ref = (o * w.unsqueeze(-1)).sum(0) / (l * w).sum(0).clamp(min=1e-6).unsqueeze(-1)
    out = rank_merge(parts.to(cuda), B, Hkv, G, D, torch.empty(B, Hq, D, device=cuda))
    assert (out.cpu() - ref).abs().max() < 1e-5
    assert (out[0, 0] == 0).all()
    out16 = rank_merge(parts.to(cuda), B, Hkv, G, D,
                       torch.empty(B, Hq, D, dtype=torch.bfloat16, device=cuda))
    assert ((out16.float().cpu() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()
    need = torch.rand(B, Hkv, generator=g) < 0.5
    keep = torch.full((B, Hq, D), 7.0)
    got = rank_merge(parts.to(cuda), B, Hkv, G, D, keep.clone().to(cuda), need=need.to(cuda))
    nq = need.repeat_interleave(G, dim=1).unsqueeze(-1)
    want = torch.where(nq, ref, keep)
    assert (got.cpu() - want).abs().max() < 1e-5


def test_page_lse_and_rank_accept_vs_fp32(cuda):
    """cvsa_page_lse against torch.logsumexp (pages past the context at -inf,
    a row with no valid page, a head with an empty selection), then
    cvsa_rank_accept against the fp32 gate over 3 ranks' gathered sums."""
    from cvsa.kernels.coverage import page_lse, rank_accept
    g = torch.Generator().manual_seed(5)
    B, H, W, K = 3, 8, 700, 40
    scores = torch.randn(B, H, W, generator=g) * 4
    scores[:, :, 650:] = float("-inf")
    scores[0, 0] = float("-inf")
    idx = torch.sort(torch.randint(0, 650, (B, H, K), generator=g), -1).values.to(torch.int32)
    n = torch.randint(0, K + 1, (B, H), generator=g).to(torch.int32)
    n[1, 1] = 0
    mask = torch.arange(K).view(1, 1, K) < n.unsqueeze(-1)
    sel = torch.gather(scores, -1, idx.long()).masked_fill(~mask, float("-inf"))
    ref_all, ref_sel = torch.logsumexp(scores, -1), torch.logsumexp(sel, -1)
    la, ls = page_lse(scores.to(cuda), idx.to(cuda), n.to(cuda))
    for got, ref in ((la.cpu(), ref_all), (ls.cpu(), ref_sel)):
        assert torch.equal(torch.isinf(got), torch.isinf(ref))
        fin = torch.isfinite(ref)
        assert ((got[fin] - ref[fin]).abs() <= 1e-5 + 1e-6 * ref[fin].abs()).all()
    world, R = 3, B * H
    sa = torch.randn(world, R, generator=g) + 5
    ss = sa - torch.rand(world, R, generator=g) * 0.4
    ss[1, :4] = float("-inf")                               # a rank with no selected page
    parts = torch.cat([torch.randn(world, 5, generator=g), sa, ss,
                       torch.randn(world, 3, generator=g)], 1).contiguous()
    cov = torch.exp(torch.logsumexp(ss, 0) - torch.logsumexp(sa, 0))
    tau = float(cov.median())
    acc = rank_accept(parts.to(cuda), 5, 5 + R, R, tau).cpu()
    clear = (cov - tau).abs() > 1e-5
    assert torch.equal(acc[clear], (cov >= tau)[clear])
