"""Exchanges between the ranks of one node over NVLink peer memory
(csrc/peer.cu, cvsa_peer_*): the page split's all-gathers and its merge of the
attention partials, and the head-sharded step's decision all-reduce, each one
kernel launch instead of a library collective.

Every rank allocates one exchange buffer, the buffers' CUDA IPC handles are
passed around once over the process group (all_gather_object), and every
rank maps the others'. A call stores this rank's row into every rank's buffer
over NVLink, each word beside the call's number in one 8-byte store, and
reads the other ranks' words as they land (bounded waits); all ranks must make
the same sequence of calls with the same sizes (as the step's collectives
already do). The calls are graph-capturable.
"""

import ctypes
from typing import Optional

import torch

from cvsa import _lib


class PeerExchange:
    """One rank's end of the exchange (see the module docstring).

    row_cap: the largest row (float32 words) any call will exchange."""

    def __init__(self, row_cap: int, group=None, device: Optional[torch.device] = None):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer exchanges span at most 8 ranks (one node)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.row_cap = (int(row_cap) + 3) // 4 * 4
        lib = _lib.load()
        nbytes = lib.cvsa_peer_buffer_bytes(self.world, self.row_cap)
        if nbytes == 0:
            raise ValueError("bad peer buffer shape")
        # every step that can fail on one rank is followed by an exchange of
        # the outcome, so all ranks fail together instead of waiting forever
        # in the next collective
        handle = ctypes.create_string_buffer(64)
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            st = lib.cvsa_peer_alloc(nbytes, ctypes.byref(ptr), handle)
        self._own = ptr.value if st == _lib.OK else None
        self._opened = []
        got = [None] * self.world
        dist.all_gather_object(got, (st == _lib.OK, handle.raw), group=group)
        if not all(ok for ok, _ in got):
            self._release()
            raise RuntimeError("cvsa_peer_alloc failed on a rank")
        bases, ok = [], True
        with torch.cuda.device(self.device):
            for q, (_, h) in enumerate(got):
                if q == self.rank:
                    bases.append(self._own)
                    continue
                hb = ctypes.create_string_buffer(bytes(h), 64)
                p = ctypes.c_void_p()
                if lib.cvsa_peer_open(hb, ctypes.byref(p)) != _lib.OK:
                    ok = False
                    break
                self._opened.append(p.value)
                bases.append(p.value)
        oks = [None] * self.world
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self._release()
            raise RuntimeError("cvsa_peer_open failed on a rank: " +
                               _lib.load().cvsa_last_error().decode(errors="replace"))
        self.bases = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.dev_error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._desc = _lib.PeerDesc(self.bases.data_ptr(), self.world, self.rank, self.row_cap,
                                   self.dev_error.data_ptr())
        torch.cuda.synchronize(self.device)
        dist.barrier(group)

    def _release(self):
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.cvsa_peer_close(ctypes.c_void_p(p))
            if self._own is not None:
                lib.cvsa_peer_free(ctypes.c_void_p(self._own))
        self._opened, self._own = [], None

    def allgather(self, x: torch.Tensor) -> torch.Tensor:
        """[world, n] float32: every rank's x (1-D float32, n <= row_cap), in rank order."""
        if x.dtype != torch.float32 or x.dim() != 1 or not x.is_contiguous():
            raise ValueError("x must be a contiguous 1-D float32 tensor")
        out = torch.empty((self.world, x.numel()), dtype=torch.float32, device=x.device)
        _lib.check(_lib.load().cvsa_peer_allgather(ctypes.byref(self._desc), x.data_ptr(),
                                                   x.numel(), out.data_ptr(),
                                                   _lib.stream_ptr(x.device)),
                   "cvsa_peer_allgather")
        return out

    def min_i32(self, x: torch.Tensor) -> torch.Tensor:
        """x (int32, contiguous) replaced in place by its minimum over the ranks."""
        if x.dtype != torch.int32 or not x.is_contiguous():
            raise ValueError("x must be contiguous int32")
        _lib.check(_lib.load().cvsa_peer_min_i32(ctypes.byref(self._desc), x.data_ptr(),
                                                 x.numel(), x.data_ptr(),
                                                 _lib.stream_ptr(x.device)), "cvsa_peer_min_i32")
        return x

    def merge(self, part: torch.Tensor, batch: int, num_kv_heads: int, num_q_per_kv: int,
              head_dim: int, out: torch.Tensor, need: Optional[torch.Tensor] = None
              ) -> torch.Tensor:
        """Exchange this rank's partial row [o | m | l] and write the merge of
        every rank's into out [B, Hq, D] (cvsa_rank_merge's arithmetic)."""
        if part.dtype != torch.float32 or not part.is_contiguous():
            raise ValueError("part must be a contiguous float32 row")
        if not out.is_contiguous() or tuple(out.shape) != (batch, num_kv_heads * num_q_per_kv,
                                                           head_dim):
            raise ValueError("out must be a contiguous [B, Hq, D] tensor")
        nd = None if need is None else need.to(torch.uint8).contiguous()
        _lib.check(_lib.load().cvsa_peer_merge(ctypes.byref(self._desc), part.data_ptr(), batch,
                                               num_kv_heads, num_q_per_kv, head_dim,
                                               _lib.ptr(nd), out.data_ptr(),
                                               _lib.dtype_code(out.dtype),
                                               _lib.stream_ptr(part.device)), "cvsa_peer_merge")
        return out

    def close(self):
        """Unmap the peers' buffers and free this rank's (after a barrier, so
        no rank still writes into it). Captured graphs using the exchange must
        be released first."""
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        self._release()
