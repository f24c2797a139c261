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
    """One rank of an NCCL communicator over ``nranks`` processes (one GPU each)."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device=None):
        if len(uid) != 128:
            raise ValueError("the NCCL unique id has 128 bytes")
        dev.require_cuda()
        if device is not None:
            torch.cuda.set_device(device)
        self._lib = _lib.load()
        self._uid = (C.c_uint8 * 128).from_buffer_copy(uid)
        self._comm = C.c_void_p()
        _lib.check(self._lib.xsake_comm_init(self._uid, nranks, rank, C.byref(self._comm)))
        self.nranks, self.rank = nranks, rank

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
