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
    """A block mask compiled for one (batch, heads, seq, block_size, causal) problem.

    ``units`` (a sorted tuple of unit ids ``b * heads + h``, or None for every unit) are the
    (batch, head) units the attention calls with this plan compute: a rank of a job whose
    batch x heads is sharded over GPUs compiles a plan of its own units, and the kernels then
    read and write only those units' rows."""

    def __init__(self, plan: torch.Tensor, dims: _lib.MaskDims, units=None):
        self.plan = plan
        self.dims = dims
        self.units = units
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
        """Active block pairs after the causal cut (n_a) of the selected units, 64x64 tiles the
        forward computes with the pairing the plan chose, fully masked q-blocks, forward work
        items, and the plan compiler's choices (pairing, split pieces).  Synchronises the
        current stream."""
        if self._stats is None:
            info = _lib.PlanInfo()
            _lib.check(_lib.load().xsake_mask_plan_info(self.plan.data_ptr(), dev.stream_ptr(), C.byref(info)))
            self._stats = {"active_blocks": info.active_blocks, "computed_tiles": info.computed_tiles,
                           "empty_qblocks": info.empty_qblocks, "work_items": info.work_items,
                           "selected_units": info.selected_units,
                           "pairing": _PAIRING_NAMES.get(info.pairing, str(info.pairing)),
                           "split_items": info.split_items, "split_slots": info.split_slots,
                           "split_cap": info.split_cap, "workers": info.workers}
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


# Recently seen host masks by object identity: (bool snapshot, digest).  A hit still compares
# the whole content (a mask may have been written in place), which is cheaper than hashing it.
_SEEN: "OrderedDict[int, tuple]" = OrderedDict()
_SEEN_MAX = 8


def _mask_key(m, ident: int) -> bytes:
    """Content key of a block mask (``ident``: id of the caller's object).  A CUDA mask is copied
    to the host (nq * nk bytes per mask head; this synchronises its stream), so a plan is never
    matched by a tensor's address, which the caching allocator reuses."""
    if isinstance(m, torch.Tensor):
        m = m.detach().cpu().numpy()
    a = np.ascontiguousarray(np.asarray(m).astype(bool, copy=False))
    seen = _SEEN.get(ident)
    if seen is not None and seen[0].shape == a.shape and np.array_equal(seen[0], a):
        _SEEN.move_to_end(ident)
        return seen[1]
    key = hashlib.blake2b(a.tobytes() + repr(a.shape).encode(), digest_size=16).digest()
    _SEEN[ident] = (a.copy(), key)
    if len(_SEEN) > _SEEN_MAX:
        _SEEN.popitem(last=False)
    return key


def _units_tuple(units, batch: int, heads: int):
    if units is None:
        return None
    u = sorted({int(x) for x in np.asarray(units).reshape(-1)})
    if not u:
        raise ValueError("units must name at least one (batch, head) unit")
    if u[0] < 0 or u[-1] >= batch * heads:
        raise ValueError(f"unit ids must lie in [0, batch * heads = {batch * heads})")
    return None if len(u) == batch * heads else tuple(u)


_CACHE: "OrderedDict[tuple, CompiledMask]" = OrderedDict()
_CACHE_MAX = 32


_PAIRINGS = {"auto": 0, "query_chunk": 1, "unit": 2}
_PAIRING_NAMES = {0: "query_chunk", 1: "unit"}


def compile_block_mask(block_mask, batch: int, heads: int, seq: int, block_size: int,
                       causal: bool, device=None, units=None, workers: int = 0,
                       pairing: str = "auto") -> CompiledMask:
    """Compile ``block_mask`` (broadcast like ``_broadcast_mask``) into a device plan.

    ``units`` (unit ids ``b * heads + h``; None = all) restricts the plan to those (batch,
    head) units.  ``workers`` (0 = two per SM of the device) is the concurrency the forward's
    split rule assumes.  ``pairing`` fixes how the tensor-core forward groups rows into work
    items ("query_chunk": chunks 2t, 2t+1 of one unit; "unit": chunk j of two units that share
    the mask); "auto" lets the plan compiler choose from the mask."""
    if pairing not in _PAIRINGS:
        raise ValueError(f"pairing must be one of {sorted(_PAIRINGS)}, got {pairing!r}")
    dev.require_cuda()
    units = _units_tuple(units, batch, heads)
    if isinstance(block_mask, CompiledMask):
        cm = block_mask
        if (cm.batch, cm.heads, cm.seq, cm.block_size, cm.causal) != (batch, heads, seq, block_size,
                                                                       bool(causal)):
            raise ValueError(f"CompiledMask was built for (batch, heads, seq, block_size, causal) = "
                             f"{(cm.batch, cm.heads, cm.seq, cm.block_size, cm.causal)}, called with "
                             f"{(batch, heads, seq, block_size, bool(causal))}")
        if units is not None and cm.units != units:
            raise ValueError("CompiledMask was built for other units")
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
    key = (_mask_key(m, id(block_mask)), batch, heads, seq, block_size, bool(causal), str(device), units,
           int(workers), pairing)
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
    ut = None
    if units is not None:
        ut = torch.tensor(units, dtype=torch.int32).to(device)
    opts = _lib.PlanOptions(ut.data_ptr() if ut is not None else None, len(units) if units else 0,
                            int(workers), _PAIRINGS[pairing])
    _lib.check(lib.xsake_mask_compile_ex(C.byref(dims), C.byref(opts), mt.data_ptr(), plan.data_ptr(),
                                         nbytes.value, dev.stream_ptr()))
    cm = CompiledMask(plan, dims, units)
    cm._mask_ref = (mt, ut)  # keep the sources alive until the compile kernels have run
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


def sparse_attention_shard(q, k, v, block_mask, units, block_size: int = 128, sm_scale: Optional[float] = None,
                           causal: bool = False, out=None, buffers=None):
    """Forward of the (batch, head) units ``units`` (ids ``b * heads + h``) of one job: the share
    of a rank when the job's batch x heads is split over GPUs (the reference runs a job on one
    device, sparse_attention.py:161-252; units are independent, so the split needs no exchange).

    ``q``, ``k``, ``v`` are the job's ``[B, H, S, D]`` tensors.  CUDA tensors are used in place and
    the result is a CUDA tensor whose rows of other units are unspecified.  Host tensors (torch
    CPU tensors, pinned for asynchronous copies, or NumPy arrays) have only the listed units'
    ``[S, D]`` slices copied to the device and the output slices copied back into ``out`` (a host
    tensor of q's shape and dtype, allocated when None; other units' rows are left as they are),
    stream-ordered on the current stream.  ``buffers`` (q, k, v, o device tensors of the job's
    shape) may be passed to reuse device memory across calls."""
    was_host = not (isinstance(q, torch.Tensor) and q.is_cuda)
    if not was_host:
        B, H, S, _ = q.shape
        cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device, units=units)
        return attention_forward(q, k, v, cm, block_size, sm_scale, causal)[0]
    dev.require_cuda()
    ht = [x if isinstance(x, torch.Tensor) else dev.host_tensor(x) for x in (q, k, v)]
    if ht[0].dim() != 4 or any(t.shape != ht[0].shape or t.dtype != ht[0].dtype for t in ht):
        raise ValueError("q, k, v must be [batch, heads, seq, d_head] of one shape and dtype")
    B, H, S, D = ht[0].shape
    device = torch.device("cuda", torch.cuda.current_device())
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, device, units=units)
    sel = cm.units if cm.units is not None else tuple(range(B * H))
    if buffers is None:
        buffers = tuple(torch.empty(ht[0].shape, dtype=ht[0].dtype, device=device) for _ in range(4))
    qd, kd, vd, od = buffers
    # one copy per run of consecutive unit ids (a run is contiguous [S, D] slices of [B*H, S, D])
    runs, start = [], sel[0]
    for a, b in zip(sel, sel[1:] + (None,)):
        if b != a + 1:
            runs.append((start, a + 1))
            start = b
    flat = lambda t: t.contiguous().view(B * H, S, D)   # noqa: E731
    hq, hk, hv = (flat(t) for t in ht)
    fq, fk, fv = (t.view(B * H, S, D) for t in (qd, kd, vd))
    for lo, hi in runs:
        for d_, h_ in ((fq, hq), (fk, hk), (fv, hv)):
            d_[lo:hi].copy_(h_[lo:hi], non_blocking=True)
    o, _ = attention_forward(qd, kd, vd, cm, block_size, sm_scale, causal)
    if out is None:
        out = torch.empty(ht[0].shape, dtype=ht[0].dtype, pin_memory=True)
    fo, ho = o.view(B * H, S, D), out.view(B * H, S, D)
    for lo, hi in runs:
        ho[lo:hi].copy_(fo[lo:hi], non_blocking=True)
    return out


def attention_probabilities(q, k, block_mask, block_size: int = 128, scale: Optional[float] = None,
                            causal: bool = False):
    """The attention weights of ``sparse_attention_reference`` (sparse_attention.py:45-91):
    fp32 [B, H, S, S] softmax over all S keys of ``q k^T * scale`` with masked entries at
    finfo(float32).min (a fully masked row is uniform).  Computed on the GPU with fp32-accurate
    scores (tensor cores at d_head 64, CUDA cores otherwise); NumPy in, NumPy out, CUDA tensor
    in, CUDA tensor out."""
    was_host = not (isinstance(q, torch.Tensor) and q.is_cuda)
    q, k = (_unit_last(dev.to_device(t)[0]) for t in (q, k))
    if q.dim() != 4 or k.shape != q.shape or k.dtype != q.dtype:
        raise ValueError(f"q and k must be [batch, heads, seq, d_head] of one dtype, got {tuple(q.shape)} "
                         f"{tuple(k.shape)}")
    B, H, S, D = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    p = torch.empty((B, H, S, S), dtype=torch.float32, device=q.device)
    d = _desc(q, k, k, q, cm, scale)
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_probs_workspace_size(C.byref(d), C.byref(n)))
    ws = dev.workspace(n.value, q.device)
    _lib.check(lib.xsake_attn_probs_ex(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(), p.data_ptr(),
                                       ws.data_ptr(), ws.numel(), dev.stream_ptr()))
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
