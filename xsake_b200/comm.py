"""NCCL communicator of the C ABI (``xsake_comm_*``) for the calibration exchange.

The attention path needs no collective: (batch, head) units are independent.  Calibration has one
exchange, a float64 sum all-reduce of per-head entropy sums, which ``calibration.calibrate`` runs
through torch.distributed by default; ``Comm`` provides the same exchange through the library's
own NCCL entry points, for processes that bind the C ABI without torch.distributed (the reference
reduces across devices with jax.lax.pmean, distributed/pmap_trainer.py:54-55).
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _device as dev
from . import _lib


def unique_id() -> bytes:
    """A fresh 128-byte NCCL id; rank 0 creates it and hands it to every rank out of band."""
    lib = _lib.load()
    buf = (C.c_uint8 * 128)()
    _lib.check(lib.xsake_comm_unique_id(buf))
    return bytes(buf)


class Comm:
    """One rank of an NCCL communicator over ``nranks`` processes (one GPU each).

    Every host-side wait of this rank is bounded by ``timeout_s`` (None: unbounded): a rank that
    never joins makes the constructor raise ``XsakeError`` with code ``XSAKE_ETIMEOUT`` after that
    long (the communicator is aborted; the process and its GPU stay usable), and ``wait`` does the
    same for a collective a peer never entered."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device=None, timeout_s: float = 300.0):
        if len(uid) != 128:
            raise ValueError("the NCCL unique id has 128 bytes")
        if device is not None:
            dev.require_cuda()
            torch.cuda.set_device(device)
        self._lib = _lib.load()
        self._uid = (C.c_uint8 * 128).from_buffer_copy(uid)
        self._comm = C.c_void_p()
        self.timeout_ms = 0 if timeout_s is None else max(1, int(timeout_s * 1000))
        _lib.check(self._lib.xsake_comm_init_ex(self._uid, nranks, rank, self.timeout_ms, C.byref(self._comm)))
        self.nranks, self.rank = nranks, rank

    def wait(self, timeout_s: float = None) -> None:
        """Block (bounded) until the current stream has finished the collectives on it."""
        ms = self.timeout_ms if timeout_s is None else max(1, int(timeout_s * 1000))
        _lib.check(self._lib.xsake_comm_wait(self._comm, dev.stream_ptr(), ms))

    def allreduce_sum_f64(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over ranks of a contiguous float64 CUDA tensor (stream-ordered)."""
        if self._comm is None:
            raise RuntimeError("communicator destroyed")
        if t.dtype != torch.float64 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("allreduce_sum_f64 needs a contiguous float64 CUDA tensor")
        _lib.check(self._lib.xsake_comm_allreduce_sum_f64(self._comm, t.data_ptr(), t.numel(), dev.stream_ptr()))
        return t

    def destroy(self) -> None:
        if self._comm is not None:
            _lib.check(self._lib.xsake_comm_destroy(self._comm))
            self._comm = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.destroy()
