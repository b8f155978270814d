"""C-ABI library and host-side logic, without a GPU.

The library must load and export every entry point include/cvsa_b200.h
declares; argument validation must reject bad calls before touching CUDA; the
Python mirror of the reference interface must keep its argument checks,
scheduling and error behaviour, and must refuse CPU tensors (no fallback).
"""

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT
from cvsa import _lib
from cvsa.backend import CVSABackend
from cvsa.kernels.select import budget_for

HEADER = os.path.join(ROOT, "include", "cvsa_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cvsa_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding covers the whole header
    assert set(names) == set(_lib.exported_symbols())


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.cvsa_abi_version() == _lib.ABI_VERSION == 2
    assert lib.cvsa_status_string(0) == b"ok"
    assert lib.cvsa_status_string(-5) == b"page pool exhausted"


def test_validation_rejects_before_any_cuda_call():
    lib = _lib.load()
    assert lib.cvsa_score_pages(None, None, None, None) == _lib.ERR_INVALID
    assert b"kv descriptor" in lib.cvsa_last_error()
    kv = _lib.KvDesc(16, 16, _lib.DTYPE_BF16, 10, 16, 8, 128, 0, 16 * 8 * 128, 8 * 128, 128)
    qd = _lib.QueryDesc(16, _lib.DTYPE_BF16, 2, 30, 4, 16, 16)    # 30 q heads, 8 kv heads
    assert lib.cvsa_score_pages(qd, kv, 16, None) == _lib.ERR_INVALID
    assert b"multiple of num_kv_heads" in lib.cvsa_last_error()
    qd.num_q_heads = 32
    kv.head_dim = 96
    kv.stride_head = 96
    assert lib.cvsa_score_pages(qd, kv, 16, None) == _lib.ERR_UNSUPPORTED
    # misaligned rows
    kv.head_dim = 128
    kv.stride_head = 128
    kv.k_cache = 8
    assert lib.cvsa_score_pages(qd, kv, 16, None) == _lib.ERR_INVALID
    # max_sel smaller than budget + forced pages
    assert lib.cvsa_select_pages(16, 2, 8, 4, 16, 16, 3, 1, 2, 16, 5, 16, None) == _lib.ERR_INVALID
    # workspace too small for a decode
    kv.k_cache = 16
    rc = lib.cvsa_sparse_decode(qd, kv, 16, 8, 16, 16, 16, 16, None, 2, 256, 1, None)
    assert rc == _lib.ERR_WORKSPACE
    need = lib.cvsa_decode_workspace_size(qd, kv, 8)
    assert need > 0
    cfg = _lib.StepConfig(_lib.MODE_LAZY, 25, 1, 2, 0.9, _lib.RECOVERY_EXACT, 0, 1)
    assert lib.cvsa_step_workspace_size(qd, kv, cfg, 28) > need
    cfg.mode = 7
    io = _lib.StepIO(16, 16, 28, 0, 16, None, None, None, None, None, None)
    assert lib.cvsa_decode_step(qd, kv, cfg, io, 256, 1 << 30, None) == _lib.ERR_INVALID
    # page-split rank merge: no ranks, rows shorter than [o | m | l], unknown dtype
    bf16 = _lib.DTYPE_BF16
    assert lib.cvsa_rank_merge(16, 0, 2 * 32 * 130, 2, 8, 4, 128, None, 16, bf16, None) \
        == _lib.ERR_INVALID
    assert lib.cvsa_rank_merge(16, 2, 2 * 32 * 130 - 1, 2, 8, 4, 128, None, 16, bf16, None) \
        == _lib.ERR_INVALID
    assert b"row_stride" in lib.cvsa_last_error()
    assert lib.cvsa_rank_merge(16, 2, 2 * 32 * 130, 2, 8, 4, 128, None, 16, 9, None) \
        == _lib.ERR_INVALID
    # page-split coverage sums and gate: empty widths, offsets past the row
    assert lib.cvsa_page_lse(16, 8, 0, 16, 4, 16, 16, 16, None) == _lib.ERR_INVALID
    assert lib.cvsa_rank_accept(16, 2, 100, 0, 90, 16, 0.9, 16, None) == _lib.ERR_INVALID
    assert lib.cvsa_rank_accept(16, 0, 100, 0, 16, 16, 0.9, 16, None) == _lib.ERR_INVALID


def test_status_codes_map_to_reference_exceptions():
    lib = _lib.load()
    lib.cvsa_score_pages(None, None, None, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID)
    with pytest.raises(AssertionError):
        _lib.check(_lib.ERR_POOL)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA)


def test_backend_argument_checks_match_reference():
    with pytest.raises(ValueError):
        CVSABackend(8, 32, 128, 16, selector="bogus")
    with pytest.raises(ValueError):
        CVSABackend(8, 32, 128, 16, light_normalizer=True)
    with pytest.raises(ValueError):
        CVSABackend(8, 32, 128, 16, top_p=1.5)
    with pytest.raises(ValueError):
        CVSABackend(8, 32, 128, 16, approx_recovery_pct=1.5)
    CVSABackend(8, 32, 128, 16, approx_recovery_pct=0.2)     # supported
    # the reference's selector options construct (cvsa/selectors.py runs them)
    for kw in (dict(adaptive_selection=True), dict(top_p=0.9), dict(selector="quest"),
               dict(selector="quest", light_normalizer=True), dict(random_reject_prob=0.2),
               dict(static_budget_table={0: [0.1] * 8})):
        assert CVSABackend(8, 32, 128, 16, **kw)._alt is not None
    assert CVSABackend(8, 32, 128, 16)._alt is None
    # forced pages are an extension of the uniform top-k only
    with pytest.raises(ValueError):
        CVSABackend(8, 32, 128, 16, top_p=0.9, sink_pages=1)


def test_budget_uses_table_width():
    assert budget_for(512, 0.05) == 25
    assert budget_for(8192, 0.05) == 409
    assert budget_for(20, 0.05) == 3
    assert budget_for(256, 32 / 256) == 32


def test_schedule_follows_reference():
    class St:
        has_cache = True

    st = St()
    be = CVSABackend(8, 32, 128, 16, lazy=True, check_interval=4, dense_layers=[0])
    modes = []
    for step in range(8):
        be._step = step
        modes.append((be._mode_for(0, st), be._mode_for(1, st)))
    assert [m[0] for m in modes] == [_lib.MODE_DENSE] * 8
    assert [m[1] for m in modes] == [_lib.MODE_LAZY, _lib.MODE_REUSE, _lib.MODE_REUSE,
                                     _lib.MODE_REUSE] * 2
    st.has_cache = False
    assert be._mode_for(1, st) == _lib.MODE_LAZY
    fixed = CVSABackend(8, 32, 128, 16, reuse_interval=16)
    st.has_cache = True
    fixed._step = 16
    assert fixed._mode_for(1, st) == _lib.MODE_SCORE
    fixed._step = 17
    assert fixed._mode_for(1, st) == _lib.MODE_REUSE
    st.has_cache = False
    assert fixed._mode_for(1, st) == _lib.MODE_SCORE
    be.step_done(30, 32)
    be._step = 0
    be.step_done(31, 32)
    assert be._step == 1


def test_cpu_tensors_are_refused_no_fallback():
    be = CVSABackend(2, 8, 64, 16)
    q = torch.zeros(1, 8, 64)
    k = torch.zeros(4, 16, 2, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        be(q, k, k, torch.zeros(1, 4, dtype=torch.int32), torch.tensor([64], dtype=torch.int32), 0)
