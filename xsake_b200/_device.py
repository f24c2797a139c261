"""Device-buffer plumbing for the Python operators.

Operators accept either CUDA ``torch.Tensor``s (used in place, results stay on the device)
or host arrays (NumPy, including ``ml_dtypes.bfloat16``), which are copied to the current
CUDA device and whose results are copied back to NumPy.  PyTorch is used here only to own
device memory and to name the current stream; every computation is a libxsake_hads kernel.
"""

from __future__ import annotations

import numpy as np

try:
    import torch
except ImportError as e:  # pragma: no cover - torch is part of the supported environment
    raise ImportError("xsake_b200 needs torch for device buffers") from e

from . import _lib


def require_cuda():
    if not torch.cuda.is_available():
        raise _lib.XsakeError(_lib.XSAKE_ECUDA, "no CUDA device: xsake_b200 operators run only on "
                                                "B200 GPUs (there is no CPU fallback)")
    _lib.load()


def _bf16_np():
    import ml_dtypes
    return np.dtype(ml_dtypes.bfloat16)


def to_device(x, dtype=None):
    """Return (tensor on cuda, was_host).  ``dtype`` is an optional torch dtype to cast to."""
    require_cuda()
    if isinstance(x, torch.Tensor):
        t = x
        was_host = not t.is_cuda
        if was_host:
            t = t.cuda()
    else:
        a = np.asarray(x)
        was_host = True
        if a.dtype == _bf16_np():
            t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
        elif a.dtype == np.bool_:
            t = torch.from_numpy(np.ascontiguousarray(a).astype(np.uint8))
        else:
            t = torch.from_numpy(np.ascontiguousarray(a))
        t = t.cuda()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t, was_host


def host_tensor(a) -> "torch.Tensor":
    """A CPU torch view of a host array (NumPy bfloat16 viewed through int16, bool as uint8)."""
    a = np.asarray(a)
    if a.dtype == _bf16_np():
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    if a.dtype == np.bool_:
        return torch.from_numpy(np.ascontiguousarray(a).astype(np.uint8))
    return torch.from_numpy(np.ascontiguousarray(a))


def to_host(t: "torch.Tensor"):
    t = t.detach()
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(_bf16_np())
    return t.cpu().numpy()


def stream_ptr():
    return torch.cuda.current_stream().cuda_stream


def xsake_dtype(t: "torch.Tensor") -> int:
    if t.dtype == torch.float32:
        return _lib.XSAKE_F32
    if t.dtype == torch.bfloat16:
        return _lib.XSAKE_BF16
    raise TypeError(f"unsupported dtype {t.dtype}; use float32 or bfloat16")


def workspace(nbytes: int, device) -> "torch.Tensor":
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)
