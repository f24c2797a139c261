"""Row softmax with the reference's signatures (kernels/pallas/fused_softmax.py:26-87).

``fused_softmax(x, block_size=256, use_pallas=True)`` and ``fused_softmax_pallas(x,
block_size=256)`` compute softmax over the last axis in one read and one write of the data
(fp32 statistics, output in the input dtype).  ``block_size`` (rows per Pallas program in the
reference) has no meaning for the warp-per-row kernel and is accepted for compatibility.
"""

from __future__ import annotations

import torch

from . import _device as dev
from . import _lib


def softmax_forward(x: torch.Tensor) -> torch.Tensor:
    dev.require_cuda()
    x = x.contiguous()
    y = torch.empty_like(x)
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    _lib.check(_lib.load().xsake_softmax_fwd(dev.xsake_dtype(x), rows, cols, x.data_ptr(),
                                             y.data_ptr(), dev.stream_ptr()))
    return y


def softmax_backward(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    dev.require_cuda()
    y, dy = y.contiguous(), dy.contiguous().to(y.dtype)
    dx = torch.empty_like(y)
    cols = y.shape[-1]
    rows = y.numel() // cols if cols else 0
    _lib.check(_lib.load().xsake_softmax_bwd(dev.xsake_dtype(y), rows, cols, y.data_ptr(),
                                             dy.data_ptr(), dx.data_ptr(), dev.stream_ptr()))
    return dx


class _Softmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = softmax_forward(x)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, dy):
        (y,) = ctx.saved_tensors
        return softmax_backward(y, dy)


def fused_softmax_pallas(x, block_size: int = 256):
    del block_size
    t, was_host = dev.to_device(x)
    if t.requires_grad and torch.is_grad_enabled():
        y = _Softmax.apply(t)
    else:
        y = softmax_forward(t)
    return dev.to_host(y) if was_host else y


def fused_softmax(x, block_size: int = 256, use_pallas: bool = True):
    """Softmax over the last axis on the GPU (``use_pallas`` kept for signature parity)."""
    del use_pallas
    return fused_softmax_pallas(x, block_size)
