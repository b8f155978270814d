"""The allocation-free decode entry point, cvsa_sparse_decode_noalloc.

It exists for callers that cannot allocate device memory where they decode
(a server whose memory pool is reserved up front, a host runtime that owns all
allocations) and so cannot pass a workspace: its scratch is an array inside
the library. These tests call it through the C ABI and check that it returns
what the workspace-based cvsa_sparse_decode returns on the same inputs, on two
calls in a row with different shapes (the shared scratch must not carry state
from one call into the next), and that a shape too large for the scratch is
refused with a clear error. This file is collected last on purpose.
"""

import pytest
import torch

from cvsa import _lib
from cvsa import synthetic
from oracle import cvsa_ref as R

pytestmark = pytest.mark.gpu


def _decode_both(wl, cuda):
    d = wl.to(cuda)
    Hkv, G, bs = wl.num_kv_heads, wl.num_q_per_kv, wl.block_size
    s = R.score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, Hkv, G, bs)
    W = wl.block_tables.shape[1]
    idx, n = R.select_pages(s, wl.context_lens, bs, R.budget_for(W, 0.1), 1, 2)
    idx, n = idx.to(cuda), n.to(cuda)
    B, Hq, D = wl.q.shape
    K = idx.shape[2]
    lib = _lib.load()
    kvd = _lib.kv_desc(d.k_cache, d.v_cache)
    qd = _lib.query_desc(d.q, d.block_tables, d.context_lens)
    stream = _lib.stream_ptr(cuda)
    res = {}
    for name in ("workspace", "noalloc"):
        o = torch.empty((B, Hq, D), dtype=torch.float32, device=cuda)
        m = torch.empty((B, Hq), dtype=torch.float32, device=cuda)
        l = torch.empty((B, Hq), dtype=torch.float32, device=cuda)
        out = torch.empty((B, Hq, D), dtype=wl.q.dtype, device=cuda)
        if name == "workspace":
            nbytes = lib.cvsa_decode_workspace_size(qd, kvd, K)
            ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device=cuda)
            ws = ws[(-ws.data_ptr()) % 256:]
            rc = lib.cvsa_sparse_decode(qd, kvd, idx.data_ptr(), K, n.data_ptr(), o.data_ptr(),
                                        m.data_ptr(), l.data_ptr(), out.data_ptr(),
                                        _lib.dtype_code(wl.q.dtype), ws.data_ptr(), ws.numel(),
                                        stream)
        else:
            rc = lib.cvsa_sparse_decode_noalloc(qd, kvd, idx.data_ptr(), K, n.data_ptr(),
                                                o.data_ptr(), m.data_ptr(), l.data_ptr(),
                                                out.data_ptr(), _lib.dtype_code(wl.q.dtype),
                                                stream)
        _lib.check(rc, name)
        torch.cuda.synchronize()
        res[name] = (o.cpu(), m.cpu(), l.cpu(), out.float().cpu())
    return res


def _same(res):
    (o1, m1, l1, y1), (o2, m2, l2, y2) = res["workspace"], res["noalloc"]
    fin = torch.isfinite(m1)
    assert torch.equal(fin, torch.isfinite(m2))
    assert (m1[fin] - m2[fin]).abs().max() <= 2e-5
    assert (l1 - l2).abs().max() <= 1e-4 * (1 + l1.abs().max())
    assert (o1 - o2).abs().max() <= 1e-4 * (1 + o1.abs().max())
    assert ((y1 - y2).abs() <= 2e-2 + 1e-2 * y1.abs()).all()


def test_noalloc_matches_workspace_decode_twice(cuda):
    # first call: several items per head (tickets and partials are used)
    _same(_decode_both(synthetic.small(seed=31, B=3, Hq=32, Hkv=8, D=128,
                                       ctx=(6000, 300, 4100)), cuda))
    # second call, different shapes, on the scratch the first call left behind
    _same(_decode_both(synthetic.small(seed=32, B=2, Hq=16, Hkv=2, D=64, ctx=(2500, 900)),
                       cuda))


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    # fp32 KV takes the general-layout kernel, whose item scratch grows with
    # the selection width (the bf16/f16 stream kernel's scratch does not)
    lib = _lib.load()
    B, Hkv, D = 64, 8, 128
    q = torch.zeros((B, 32, D), dtype=torch.float32, device=cuda)
    k = torch.zeros((8, 16, Hkv, D), dtype=torch.float32, device=cuda)
    bt = torch.zeros((B, 8), dtype=torch.int32, device=cuda)
    cl = torch.full((B,), 128, dtype=torch.int32, device=cuda)
    K = 2048                                  # a selection far wider than the scratch allows
    idx = torch.zeros((B, Hkv, K), dtype=torch.int32, device=cuda)
    n = torch.ones((B, Hkv), dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    rc = lib.cvsa_sparse_decode_noalloc(_lib.query_desc(q, bt, cl), _lib.kv_desc(k, k),
                                        idx.data_ptr(), K, n.data_ptr(), None, None, None,
                                        out.data_ptr(), _lib.DTYPE_F32, _lib.stream_ptr(cuda))
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"no-alloc scratch holds" in lib.cvsa_last_error()
