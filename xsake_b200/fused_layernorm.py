"""LayerNorm with the reference's signatures (kernels/pallas/fused_layernorm.py:26-119).

``fused_layernorm(x, gamma, beta, eps=1e-5, block_size=64, use_pallas=True)`` and
``fused_layernorm_pallas(x, gamma, beta, block_size=64, eps=1e-5)``: fp32 two-pass statistics
over the last axis, ``y = gamma * (x - mean) / sqrt(var + eps) + beta``, output in x's dtype
(the Pallas path's rule, :51,87).  gamma/beta are used as fp32.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _device as dev
from . import _lib


def layernorm_forward(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                      return_stats: bool = False):
    dev.require_cuda()
    x = x.contiguous()
    d = x.shape[-1]
    rows = x.numel() // d
    g = gamma.to(device=x.device, dtype=torch.float32).contiguous()
    b = beta.to(device=x.device, dtype=torch.float32).contiguous()
    if g.numel() != d or b.numel() != d:
        raise ValueError(f"gamma/beta must have {d} elements")
    y = torch.empty_like(x)
    mean = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device) if return_stats else None
    rstd = torch.empty_like(mean) if return_stats else None
    _lib.check(_lib.load().xsake_layernorm_fwd(
        dev.xsake_dtype(x), rows, d, x.data_ptr(), g.data_ptr(), b.data_ptr(), float(eps), y.data_ptr(),
        mean.data_ptr() if return_stats else None, rstd.data_ptr() if return_stats else None,
        dev.stream_ptr()))
    return (y, mean, rstd) if return_stats else y


def layernorm_backward(x, gamma, mean, rstd, dy):
    dev.require_cuda()
    x = x.contiguous()
    d = x.shape[-1]
    rows = x.numel() // d
    g = gamma.to(device=x.device, dtype=torch.float32).contiguous()
    dy = dy.to(x.dtype).contiguous()
    dx = torch.empty_like(x)
    dg = torch.empty(d, dtype=torch.float32, device=x.device)
    db = torch.empty_like(dg)
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_layernorm_bwd_workspace_size(rows, d, C.byref(n)))
    ws = dev.workspace(n.value, x.device)
    _lib.check(lib.xsake_layernorm_bwd(dev.xsake_dtype(x), rows, d, x.data_ptr(), g.data_ptr(),
                                       mean.contiguous().data_ptr(), rstd.contiguous().data_ptr(),
                                       dy.data_ptr(), dx.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                       ws.data_ptr(), ws.numel(), dev.stream_ptr()))
    return dx, dg, db


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, eps):
        y, mean, rstd = layernorm_forward(x, gamma, beta, eps, return_stats=True)
        ctx.save_for_backward(x, gamma, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, mean, rstd = ctx.saved_tensors
        dx, dg, db = layernorm_backward(x, gamma, mean, rstd, dy)
        return dx, dg.to(gamma.dtype), db.to(gamma.dtype), None


def fused_layernorm_pallas(x, gamma, beta, block_size: int = 64, eps: float = 1e-5):
    del block_size
    t, was_host = dev.to_device(x)
    g, _ = dev.to_device(gamma)
    b, _ = dev.to_device(beta)
    if torch.is_grad_enabled() and (t.requires_grad or g.requires_grad or b.requires_grad):
        y = _LayerNorm.apply(t, g, b, float(eps))
    else:
        y = layernorm_forward(t, g, b, eps)
    return dev.to_host(y) if was_host else y


def fused_layernorm(x, gamma, beta, eps: float = 1e-5, block_size: int = 64, use_pallas: bool = True):
    """LayerNorm over the last axis on the GPU (``use_pallas`` kept for signature parity)."""
    del use_pallas
    return fused_layernorm_pallas(x, gamma, beta, block_size, eps)
