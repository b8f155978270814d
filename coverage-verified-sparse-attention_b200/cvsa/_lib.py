"""ctypes binding of libcvsa_b200.so (include/cvsa_b200.h).

The library is the product: every CVSA op in this package is a call into it on
the current CUDA stream. There is no CPU or Triton fallback -- if the library
cannot be loaded, or a tensor is not on a CUDA device, the call raises.

Status codes map to the exception types the reference raises for the same
conditions: CVSA_ERR_INVALID -> ValueError (cvsa/backend.py:150-178),
CVSA_ERR_POOL -> AssertionError (cvsa/runtime/kv_cache.py:55-56), the rest
-> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcvsa_b200.so")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_POOL = 0, -1, -2, -3, -4, -5
MODE_SCORE, MODE_LAZY, MODE_REUSE, MODE_DENSE = 0, 1, 2, 3
RECOVERY_EXACT, RECOVERY_NONE, RECOVERY_APPROX = 0, 1, 2
(CTR_PAGES_ATTENDED, CTR_PAGES_MAX, CTR_HEAD_ACCEPT, CTR_HEAD_TOTAL, CTR_ACCEPT_STEPS,
 CTR_REJECT_STEPS, CTR_SCORING_STEPS, CTR_COVERAGE_CHECKS) = range(8)
NUM_COUNTERS = 8
EV_SCORE_BEGIN, EV_SCORE_END, EV_SELECT_BEGIN, EV_SELECT_END, EV_ATTEND_BEGIN, EV_ATTEND_END = (
    range(6))
NUM_EVENTS = 6
DEV_ERR_BLOCK_RANGE, DEV_ERR_PAGE_RANGE, DEV_ERR_POOL, DEV_ERR_TABLE_FULL, DEV_ERR_TIMEOUT = (
    1, 2, 4, 8, 16)

_TORCH_TO_DT = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}


class KvDesc(ctypes.Structure):
    _fields_ = [
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("dtype", ctypes.c_int32), ("num_blocks", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("reserved0", ctypes.c_int32),
        ("stride_block", ctypes.c_int64), ("stride_token", ctypes.c_int64),
        ("stride_head", ctypes.c_int64),
    ]


class QueryDesc(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("batch", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32), ("max_pages", ctypes.c_int32),
        ("block_tables", ctypes.c_void_p), ("context_lens", ctypes.c_void_p),
    ]


class StepConfig(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32), ("budget", ctypes.c_int32),
        ("sink_pages", ctypes.c_int32), ("local_pages", ctypes.c_int32),
        ("tau", ctypes.c_float), ("recovery", ctypes.c_int32),
        ("has_cache", ctypes.c_int32), ("lazy_stats", ctypes.c_int32),
        ("approx_budget", ctypes.c_int32),
    ]


class StepIO(ctypes.Structure):
    _fields_ = [
        ("cached_indices", ctypes.c_void_p), ("cached_n", ctypes.c_void_p),
        ("max_sel", ctypes.c_int32), ("phase", ctypes.c_int32),
        ("out", ctypes.c_void_p), ("page_scores", ctypes.c_void_p),
        ("accept", ctypes.c_void_p), ("coverage", ctypes.c_void_p),
        ("counters", ctypes.c_void_p), ("step_flags", ctypes.c_void_p),
        ("dev_error", ctypes.c_void_p), ("timing_events", ctypes.c_void_p),
    ]


class SplitDesc(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("batch", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32), ("max_pages", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("budget", ctypes.c_int32), ("max_sel", ctypes.c_int32),
        ("sink_pages", ctypes.c_int32), ("local_pages", ctypes.c_int32), ("tau", ctypes.c_float),
    ]


class PeerDesc(ctypes.Structure):
    _fields_ = [
        ("bases", ctypes.c_void_p), ("world", ctypes.c_int32), ("rank", ctypes.c_int32),
        ("row_cap", ctypes.c_int64), ("dev_error", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_SIGS = {
    "cvsa_abi_version": ([], ctypes.c_int),
    "cvsa_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "cvsa_last_error": ([], ctypes.c_char_p),
    "cvsa_score_pages": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _P], ctypes.c_int),
    "cvsa_quest_scores": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _P, _P],
                          ctypes.c_int),
    "cvsa_select_pages": ([_P, _I, _I, _I, _P, _I, _I, _I, _I, _P, _I, _P, _P], ctypes.c_int),
    "cvsa_check_coverage": ([_P, _I, _I, _I, _P, _I, _P, ctypes.c_float, _P, _P, _P], ctypes.c_int),
    "cvsa_compute_complement": ([_P, _I, _P, _P, _I, _I, _I, _P, _P, _I, _P, _P], ctypes.c_int),
    "cvsa_decode_workspace_size": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _I],
                                   ctypes.c_size_t),
    "cvsa_sparse_decode": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _I, _P, _P, _P,
                            _P, _P, _I, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "cvsa_lse_merge": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _I, _P], ctypes.c_int),
    "cvsa_page_lse": ([_P, _I, _I, _P, _I, _P, _P, _P, _P], ctypes.c_int),
    "cvsa_rank_accept": ([_P, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I,
                          ctypes.c_float, _P, _P], ctypes.c_int),
    "cvsa_split_row_floats": ([ctypes.POINTER(SplitDesc)], ctypes.c_int64),
    "cvsa_split_propose": ([ctypes.POINTER(SplitDesc), _P, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "cvsa_split_gate": ([ctypes.POINTER(SplitDesc), _P, ctypes.c_int64, _P, _P, _I, _I, _P, _P,
                         _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "cvsa_split_attend": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _P, _P, _P, _I,
                           _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "cvsa_peer_buffer_bytes": ([_I, ctypes.c_int64], ctypes.c_size_t),
    "cvsa_peer_alloc": ([ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _P], ctypes.c_int),
    "cvsa_peer_open": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "cvsa_peer_close": ([_P], ctypes.c_int),
    "cvsa_peer_free": ([_P], ctypes.c_int),
    "cvsa_peer_allgather": ([ctypes.POINTER(PeerDesc), _P, ctypes.c_int64, _P, _P], ctypes.c_int),
    "cvsa_peer_min_i32": ([ctypes.POINTER(PeerDesc), _P, ctypes.c_int64, _P, _P], ctypes.c_int),
    "cvsa_peer_merge": ([ctypes.POINTER(PeerDesc), _P, _I, _I, _I, _I, _P, _P, _I, _P],
                        ctypes.c_int),
    "cvsa_rank_merge": ([_P, _I, ctypes.c_int64, _I, _I, _I, _I, _P, _P, _I, _P], ctypes.c_int),
    "cvsa_recover_merge": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _I, _P, _P, _P,
                            _P, _P, _P, _I, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "cvsa_step_workspace_size": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc),
                                  ctypes.POINTER(StepConfig), _I], ctypes.c_size_t),
    "cvsa_decode_step": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc),
                          ctypes.POINTER(StepConfig), ctypes.POINTER(StepIO), _P, ctypes.c_size_t,
                          _P], ctypes.c_int),
    "cvsa_set_wait_limit": ([ctypes.c_uint32], ctypes.c_int),
    "cvsa_workspace_reset": ([_P, ctypes.c_size_t, _P], ctypes.c_int),
    "cvsa_step_decision_word": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "cvsa_paged_append": ([ctypes.POINTER(KvDesc), _P, _P, _I, _P, _P, _I, _P, _P, _P, _I, _P, _P,
                           _P], ctypes.c_int),
    "cvsa_paged_gather": ([ctypes.POINTER(KvDesc), _P, _I, _P, _P, _P, _P], ctypes.c_int),
    "cvsa_sparse_decode_noalloc": ([ctypes.POINTER(QueryDesc), ctypes.POINTER(KvDesc), _P, _I, _P,
                                    _P, _P, _P, _P, _I, _P], ctypes.c_int),
}
NOALLOC_SCRATCH_BYTES = 8 << 20
ABI_VERSION = 2
# cvsa_decode_step phases (include/cvsa_b200.h CVSA_PHASE_*)
PHASE_ALL, PHASE_SELECT, PHASE_ATTEND = 0, 1, 2

_lib = None
_lock = threading.Lock()


def exported_symbols():
    """Names of every entry point this binding expects the library to export."""
    return sorted(_SIGS)


def load(path: Optional[str] = None) -> ctypes.CDLL:
    """Load libcvsa_b200.so once (raises if it is missing: no fallback)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"libcvsa_b200.so not found at {p}; build it with "
                "`python coverage-verified-sparse-attention_b200/build_lib.py` "
                "(the CVSA ops have no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.cvsa_abi_version() != ABI_VERSION:
            raise RuntimeError("libcvsa_b200.so ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = (load().cvsa_last_error() or b"").decode()
    text = f"{what}: {msg}" if what else msg
    if status == ERR_INVALID:
        raise ValueError(text)
    if status == ERR_POOL:
        raise AssertionError(text)
    raise RuntimeError(f"{text} (status {status})")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}")


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("CVSA ops run on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def kv_desc(k_cache: torch.Tensor, v_cache: torch.Tensor) -> KvDesc:
    """[num_blocks, block_size, num_kv_heads, head_dim] pools (kv_cache.py:38-43)."""
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache/v_cache must both be [num_blocks, block_size, H_kv, D]")
    if k_cache.dtype != v_cache.dtype:
        raise ValueError("k_cache and v_cache dtypes differ")
    if k_cache.stride() != v_cache.stride() or k_cache.stride(3) != 1:
        raise ValueError("k_cache/v_cache must share strides with a contiguous head_dim")
    nb, bs, h, d = k_cache.shape
    return KvDesc(k_cache.data_ptr(), v_cache.data_ptr(), dtype_code(k_cache.dtype), nb, bs, h, d,
                  0, k_cache.stride(0), k_cache.stride(1), k_cache.stride(2))


def query_desc(q: Optional[torch.Tensor], block_tables: torch.Tensor,
               context_lens: torch.Tensor, num_q_heads: Optional[int] = None) -> QueryDesc:
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise ValueError("block_tables and context_lens must be int32")
    if not block_tables.is_contiguous() or not context_lens.is_contiguous():
        raise ValueError("block_tables/context_lens must be contiguous")
    B, W = block_tables.shape
    if q is not None:
        if q.dim() != 3 or not q.is_contiguous():
            raise ValueError("q must be a contiguous [B, H_q, D] tensor")
        return QueryDesc(q.data_ptr(), dtype_code(q.dtype), B, q.shape[1], W,
                         block_tables.data_ptr(), context_lens.data_ptr())
    return QueryDesc(None, DTYPE_BF16, B, num_q_heads or 1, W, block_tables.data_ptr(),
                     context_lens.data_ptr())


class Workspace:
    """Per-device, per-stream cache of zeroed workspace buffers, grown on demand.

    Kernels that use a ticket counter leave it at zero, so a buffer is zeroed
    once, when it is created.
    """

    def __init__(self):
        self._bufs = {}

    def get(self, nbytes: int, device: torch.device, tag: str = "") -> torch.Tensor:
        key = (device, torch.cuda.current_stream(device).cuda_stream, tag)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 256) + 256, dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        off = (-buf.data_ptr()) % 256
        return buf[off:]


WORKSPACE = Workspace()
