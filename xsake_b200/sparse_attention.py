"""Block-sparse attention with the reference's operator signatures, on libxsake_hads kernels.

Reference: kernels/pallas/sparse_attention.py
  * ``sparse_attention(q, k, v, block_mask, block_size=128, scale=None, causal=False,
    use_pallas=True) -> (out, None)``                                    :257-281
  * ``sparse_attention_pallas(q, k, v, block_mask, block_q=128, block_k=128, sm_scale=None,
    causal=False) -> out``                                                :161-252
  * ``_broadcast_mask``                                                   :286-298
Output semantics are those of ``sparse_attention_reference`` (:45-91): the token-level causal
mask is applied when ``causal`` is true, and a query row whose every score is masked attends
uniformly to all keys.  (The reference's Pallas kernel ignores ``causal``; its CPU path does
not.)

Inputs are ``[batch, heads, seq, d_head]`` float32 or bfloat16 CUDA tensors (any strides with
a unit last stride) or host arrays; ``block_mask`` is a bool mask of shape ``[nq, nk]``,
``[heads, nq, nk]`` or ``[batch, heads, nq, nk]`` with ``nq = nk = seq / block_size``, or a
``CompiledMask``.  Block masks are compiled into a device plan once and cached.
"""

from __future__ import annotations

import ctypes as C
import hashlib
from collections import OrderedDict
from typing import Optional, Tuple

import numpy as np
import torch

from . import _device as dev
from . import _lib


# ----------------------------------------------------------------------------- mask plans
class CompiledMask:
    """A block mask compiled for one (batch, heads, seq, block_size, causal) problem."""

    def __init__(self, plan: torch.Tensor, dims: _lib.MaskDims):
        self.plan = plan
        self.dims = dims
        self._stats = None

    @property
    def batch(self):
        return self.dims.batch

    @property
    def heads(self):
        return self.dims.heads

    @property
    def seq(self):
        return self.dims.seq

    @property
    def block_size(self):
        return self.dims.block_size

    @property
    def causal(self):
        return bool(self.dims.causal)

    def stats(self) -> dict:
        """Active block pairs after the causal cut (n_a), computed 64x64 tiles, fully masked
        q-blocks and forward work items.  Synchronises the current stream."""
        if self._stats is None:
            out = (C.c_int64 * 4)()
            _lib.check(_lib.load().xsake_mask_plan_stats(self.plan.data_ptr(), dev.stream_ptr(), out))
            self._stats = {"active_blocks": out[0], "computed_tiles": out[1],
                           "empty_qblocks": out[2], "work_items": out[3]}
        return self._stats


def _mask_4d(block_mask):
    if isinstance(block_mask, torch.Tensor):
        m = block_mask
    else:
        m = np.asarray(block_mask)
    nd = m.ndim
    if nd == 2:
        m = m[None, None]
    elif nd == 3:
        m = m[None]
    elif nd != 4:
        raise ValueError(f"block_mask must be 2-, 3- or 4-D, got shape {tuple(m.shape)}")
    return m


def _mask_key(m) -> bytes:
    if isinstance(m, torch.Tensor):
        if m.is_cuda:
            return b"cuda" + repr((m.data_ptr(), m._version, tuple(m.shape), m.dtype)).encode()
        m = m.numpy()
    a = np.ascontiguousarray(np.asarray(m).astype(bool, copy=False))
    return hashlib.blake2b(a.tobytes() + repr(a.shape).encode(), digest_size=16).digest()


_CACHE: "OrderedDict[tuple, CompiledMask]" = OrderedDict()
_CACHE_MAX = 32


def compile_block_mask(block_mask, batch: int, heads: int, seq: int, block_size: int,
                       causal: bool, device=None) -> CompiledMask:
    """Compile ``block_mask`` (broadcast like ``_broadcast_mask``) into a device plan."""
    dev.require_cuda()
    if isinstance(block_mask, CompiledMask):
        cm = block_mask
        if (cm.batch, cm.heads, cm.seq, cm.block_size, cm.causal) != (batch, heads, seq, block_size,
                                                                       bool(causal)):
            raise ValueError(f"CompiledMask was built for (batch, heads, seq, block_size, causal) = "
                             f"{(cm.batch, cm.heads, cm.seq, cm.block_size, cm.causal)}, called with "
                             f"{(batch, heads, seq, block_size, bool(causal))}")
        return cm
    if block_size <= 0 or seq % block_size:
        raise ValueError(f"block_size {block_size} must divide seq {seq}")
    nb = seq // block_size
    m = _mask_4d(block_mask)
    Bm, Hm, nq, nk = (int(s) for s in m.shape)
    if nq != nb or nk != nb:
        raise ValueError(f"block_mask has {nq}x{nk} blocks, expected {nb}x{nb} "
                         f"(seq {seq} / block_size {block_size})")
    if Bm not in (1, batch) or Hm not in (1, heads):
        raise ValueError(f"block_mask leading dims {(Bm, Hm)} do not broadcast to {(batch, heads)}")
    device = device or torch.device("cuda", torch.cuda.current_device())
    key = (_mask_key(m), batch, heads, seq, block_size, bool(causal), str(device))
    hit = _CACHE.get(key)
    if hit is not None:
        _CACHE.move_to_end(key)
        return hit
    lib = _lib.load()
    dims = _lib.MaskDims(batch, heads, seq, Bm, Hm, block_size, int(bool(causal)))
    nbytes = C.c_size_t(0)
    _lib.check(lib.xsake_mask_plan_bytes(C.byref(dims), C.byref(nbytes)))
    mt, _ = dev.to_device(m)
    mt = mt.to(device=device, dtype=torch.uint8).contiguous() if mt.dtype != torch.uint8 else \
        mt.to(device).contiguous()
    plan = torch.empty(nbytes.value, dtype=torch.uint8, device=device)
    _lib.check(lib.xsake_mask_compile(C.byref(dims), mt.data_ptr(), plan.data_ptr(), nbytes.value,
                                      dev.stream_ptr()))
    cm = CompiledMask(plan, dims)
    cm._mask_ref = mt  # keep the source alive until the compile kernels have run
    _CACHE[key] = cm
    if len(_CACHE) > _CACHE_MAX:
        _CACHE.popitem(last=False)
    return cm


# ----------------------------------------------------------------------------- descriptors
def _strides(t: torch.Tensor):
    if t.stride(-1) != 1:
        raise ValueError("the last (d_head) dimension must be contiguous")
    return (C.c_int64 * 3)(*t.stride()[:3])


def _desc(q, k, v, o, cm: CompiledMask, scale):
    B, H, S, D = q.shape
    d = _lib.AttnDesc()
    d.dtype = dev.xsake_dtype(q)
    d.batch, d.heads, d.seq, d.head_dim = B, H, S, D
    d.block_size = cm.block_size
    d.causal = int(cm.causal)
    d.mask_batch, d.mask_heads = cm.dims.mask_batch, cm.dims.mask_heads
    d.scale = float(scale) if scale else 0.0
    d.q_stride, d.k_stride, d.v_stride, d.o_stride = _strides(q), _strides(k), _strides(v), _strides(o)
    return d


def _check_qkv(q, k, v):
    if q.dim() != 4:
        raise ValueError(f"q must be [batch, heads, seq, d_head], got {tuple(q.shape)}")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share one dtype")
    dev.xsake_dtype(q)


def _unit_last(t):
    return t if t.stride(-1) == 1 else t.contiguous()


# ----------------------------------------------------------------------------- forward / backward
def attention_forward(q, k, v, block_mask, block_size: int = 128, scale: Optional[float] = None,
                      causal: bool = False):
    """Returns (out, lse) as CUDA tensors; out has q's shape/dtype, lse is fp32 [B, H, S]."""
    dev.require_cuda()
    q, _ = dev.to_device(q)
    k, _ = dev.to_device(k)
    v, _ = dev.to_device(v)
    q, k, v = _unit_last(q), _unit_last(k), _unit_last(v)
    _check_qkv(q, k, v)
    B, H, S, D = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    o = torch.empty_like(q)   # q's layout: a [B, S, H, D] view stays one, with no transpose copy
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device)
    d = _desc(q, k, v, o, cm, scale)
    lib = _lib.load()
    ws_n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_fwd_workspace_size(C.byref(d), C.byref(ws_n)))
    ws = dev.workspace(ws_n.value, q.device)
    _lib.check(lib.xsake_attn_fwd(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(),
                                  v.data_ptr(), o.data_ptr(), lse.data_ptr(), ws.data_ptr(),
                                  ws.numel(), dev.stream_ptr()))
    return o, lse


def attention_backward(q, k, v, o, lse, dout, block_mask, block_size: int = 128,
                       scale: Optional[float] = None, causal: bool = False):
    """Gradients (dq, dk, dv) of ``attention_forward`` for upstream gradient ``dout``."""
    dev.require_cuda()
    q, k, v, o, dout = (_unit_last(dev.to_device(t)[0]) for t in (q, k, v, o, dout))
    lse = dev.to_device(lse, torch.float32)[0].contiguous()
    _check_qkv(q, k, v)
    B, H, S, D = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    # o, dout, dq, dk, dv share one set of strides (the descriptor's o_stride): o's layout, when
    # o is dense (a strided view such as [B, S, H, D] memory seen as [B, H, S, D]), else packed
    if tuple(torch.empty_like(o).stride()) != tuple(o.stride()):
        o = o.contiguous()
    if tuple(dout.stride()) != tuple(o.stride()):
        dout = torch.empty_like(o).copy_(dout)
    dq = torch.empty_like(o)
    dk = torch.empty_like(o)
    dv = torch.empty_like(o)
    d = _desc(q, k, v, dq, cm, scale)
    lib = _lib.load()
    ws_n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_bwd_workspace_size(C.byref(d), C.byref(ws_n)))
    ws = dev.workspace(ws_n.value, q.device)
    _lib.check(lib.xsake_attn_bwd(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(),
                                  v.data_ptr(), o.data_ptr(), lse.data_ptr(), dout.data_ptr(),
                                  dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(),
                                  ws.numel(), dev.stream_ptr()))
    return dq, dk, dv


class SparseAttentionFunction(torch.autograd.Function):
    """Autograd wrapper (the reference has no VJP for its Pallas path)."""

    @staticmethod
    def forward(ctx, q, k, v, cm: CompiledMask, scale):
        o, lse = attention_forward(q, k, v, cm, cm.block_size, scale, cm.causal)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cm, ctx.scale = cm, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        cm = ctx.cm
        dq, dk, dv = attention_backward(q, k, v, o, lse, do, cm, cm.block_size, ctx.scale, cm.causal)
        return dq, dk, dv, None, None


def sparse_attention_autograd(q, k, v, block_mask, block_size: int = 128, scale=None,
                              causal: bool = False):
    B, H, S, _ = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    return SparseAttentionFunction.apply(q, k, v, cm, scale)


# ----------------------------------------------------------------------------- reference API
def _finish(out: torch.Tensor, was_host: bool):
    return dev.to_host(out) if was_host else out


def sparse_attention_pallas(q, k, v, block_mask, block_q: int = 128, block_k: int = 128,
                            sm_scale: Optional[float] = None, causal: bool = False):
    """Drop-in for sparse_attention.py:161-252 (returns the output only)."""
    if block_q != block_k:
        raise ValueError("block_q must equal block_k")
    was_host = not (isinstance(q, torch.Tensor) and q.is_cuda)
    if isinstance(q, torch.Tensor) and q.requires_grad and torch.is_grad_enabled():
        out = sparse_attention_autograd(q, k, v, block_mask, block_q, sm_scale, causal)
    else:
        out, _ = attention_forward(q, k, v, block_mask, block_q, sm_scale, causal)
    return _finish(out, was_host)


def attention_probabilities(q, k, block_mask, block_size: int = 128, scale: Optional[float] = None,
                            causal: bool = False):
    """The attention weights of ``sparse_attention_reference`` (sparse_attention.py:45-91):
    fp32 [B, H, S, S] softmax over all S keys of ``q k^T * scale`` with masked entries at
    finfo(float32).min (a fully masked row is uniform).  Computed on the GPU (fp32 CUDA-core
    scores); NumPy in, NumPy out, CUDA tensor in, CUDA tensor out."""
    was_host = not (isinstance(q, torch.Tensor) and q.is_cuda)
    q, k = (_unit_last(dev.to_device(t)[0]) for t in (q, k))
    if q.dim() != 4 or k.shape != q.shape or k.dtype != q.dtype:
        raise ValueError(f"q and k must be [batch, heads, seq, d_head] of one dtype, got {tuple(q.shape)} "
                         f"{tuple(k.shape)}")
    B, H, S, D = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    p = torch.empty((B, H, S, S), dtype=torch.float32, device=q.device)
    d = _desc(q, k, k, q, cm, scale)
    _lib.check(_lib.load().xsake_attn_probs(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(),
                                            p.data_ptr(), dev.stream_ptr()))
    return dev.to_host(p) if was_host else p


def sparse_attention(q, k, v, block_mask, block_size: int = 128, scale: Optional[float] = None,
                     causal: bool = False, use_pallas: bool = True) -> Tuple[object, Optional[object]]:
    """Drop-in for sparse_attention.py:257-281.  ``use_pallas=True`` returns ``(out, None)`` as
    the reference does on GPU; ``use_pallas=False`` also returns the attention weights, the
    second output of the reference CPU path (``attention_probabilities``).  Both run on the GPU."""
    out = sparse_attention_pallas(q, k, v, block_mask, block_size, block_size, scale, causal)
    if use_pallas:
        return out, None
    return out, attention_probabilities(q, k, block_mask, block_size, scale, causal)


def broadcast_mask(block_mask, batch: int, heads: int, nb: int):
    """``_broadcast_mask`` (sparse_attention.py:286-298) for host masks."""
    m = _mask_4d(block_mask)
    if isinstance(m, torch.Tensor):
        return m.expand(batch, heads, nb, m.shape[-1])
    return np.broadcast_to(m, (batch, heads, nb, m.shape[-1]))
