"""Shared test setup.

Markers: `gpu` tests need a CUDA device (B200) and call the kernels through
the C ABI; everything else runs on CPU. The oracle (oracle/cvsa_ref.py) is the
checker; fixtures in tests/golden/ hold outputs of the reference itself.
"""

import hashlib
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "coverage-verified-sparse-attention_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_outputs.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN, allow_pickle=False))


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for gpu tests; fails (never skips) without one."""
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    return torch.device("cuda:0")


def input_checksum(wl) -> str:
    """sha256 over the raw bytes of a workload's inputs (as make_golden.py)."""
    h = hashlib.sha256()
    for t in (wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens):
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def finite_close(a, b, atol, rtol):
    """Assert equal -inf positions and |a-b| <= atol + rtol|b| elsewhere."""
    a = torch.as_tensor(a).double()
    b = torch.as_tensor(b).double()
    assert a.shape == b.shape, (a.shape, b.shape)
    fa, fb = torch.isfinite(a), torch.isfinite(b)
    assert torch.equal(fa, fb), "non-finite positions differ"
    assert torch.equal(a[~fa], b[~fb]), "non-finite values differ"
    d = (a[fa] - b[fb]).abs()
    lim = atol + rtol * b[fb].abs()
    bad = d > lim
    assert not bad.any(), f"max excess {float((d - lim).max()):.3e}, max diff {float(d.max()):.3e}"


def sel_sets(idx, n):
    idx = torch.as_tensor(idx)
    n = torch.as_tensor(n)
    B, H = n.shape
    return [[sorted(idx[b, h, :int(n[b, h])].tolist()) for h in range(H)] for b in range(B)]
