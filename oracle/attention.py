"""Oracle (test infrastructure): NumPy restatement of ``sparse_attention_reference``.

Reference: kernels/pallas/sparse_attention.py
  * ``_broadcast_mask``              :286-298
  * ``sparse_attention_reference``   :45-91  (dense scores, token mask = block mask
    repeated by ``block_size`` (:76-77), AND lower-triangular when causal (:79-81),
    masked scores replaced by ``finfo.min`` (:87), softmax (:88), P.V (:89))
  * the Pallas forward keeps ``lse = m + log(l)`` per row (:156)

The backward is the closed form of JAX autodiff through those ops (the reference
defines no VJP of its own): with P = softmax(masked scores) and O = P V,
  dV = P^T dO,  dP = dO V^T,  dS = P * (dP - rowsum(dO * O)),
  dS = 0 on masked entries (``jnp.where`` passes no gradient to the masked branch),
  dQ = scale * dS K,  dK = scale * dS^T Q.

All arithmetic runs in float64 unless ``compute_dtype`` says otherwise, so the
oracle is more accurate than either the reference or the CUDA path.  Work is done
one (batch, head) slice at a time so that S=4096 fits in host memory.
"""

from __future__ import annotations

import numpy as np

# Fill value of masked scores: jnp.finfo(float32).min (sparse_attention.py:87).
MASK_FILL = float(np.finfo(np.float32).min)


def broadcast_mask(block_mask, batch: int, heads: int, nb: int) -> np.ndarray:
    """Broadcast a 2/3/4-D block mask to [batch, heads, nb, nk] (sparse_attention.py:286-298)."""
    bm = np.asarray(block_mask).astype(bool)
    if bm.ndim == 2:
        bm = bm[None, None]
    elif bm.ndim == 3:
        bm = bm[None]
    elif bm.ndim != 4:
        raise ValueError(f"block_mask must be 2-, 3- or 4-D, got shape {bm.shape}")
    return np.broadcast_to(bm, (batch, heads, nb, bm.shape[-1]))


def token_mask(block_mask_2d: np.ndarray, block_size: int, seq: int, causal: bool) -> np.ndarray:
    """Token-level mask [seq, seq] of one head (sparse_attention.py:76-81)."""
    tm = np.repeat(np.repeat(block_mask_2d, block_size, axis=0), block_size, axis=1)
    tm = tm[:seq, :seq]
    if causal:
        tm = tm & np.tri(seq, seq, dtype=bool)
    return tm


def _slice_forward(q, k, v, tmask, scale, compute_dtype):
    """One (b, h) slice: returns O [S, D], P [S, S], lse [S] (natural log)."""
    q = q.astype(compute_dtype, copy=False)
    k = k.astype(compute_dtype, copy=False)
    v = v.astype(compute_dtype, copy=False)
    s = (q @ k.T) * compute_dtype(scale)
    s = np.where(tmask, s, compute_dtype(MASK_FILL))
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(axis=-1, keepdims=True)
    p = e / l
    o = p @ v
    lse = (m + np.log(l))[:, 0]
    return o, p, lse


def sparse_attention_reference(q, k, v, block_mask, block_size: int = 128, scale=None,
                               causal: bool = False, compute_dtype=np.float64,
                               return_weights: bool = True, return_lse: bool = False):
    """Dense masked attention with the semantics of sparse_attention.py:45-91.

    q, k, v: [B, H, S, D] (any float dtype; upcast to ``compute_dtype``).
    block_mask: [nq, nk], [H, nq, nk] or [B, H, nq, nk] bool.  A 4-D mask with a
    real batch dimension is honoured per batch (the reference's CPU path only
    accepts batch 1 there; its Pallas path broadcasts the same way as here).

    Returns (out [B,H,S,D], attn_weights [B,H,S,S] or None[, lse [B,H,S]]).
    """
    q = np.asarray(q)
    B, H, S, D = q.shape
    scale = scale or float(D ** -0.5)           # same falsy rule as :69
    if S % block_size:
        raise ValueError("block_size must divide seq")
    nb = S // block_size
    bm = broadcast_mask(block_mask, B, H, nb)
    out = np.empty((B, H, S, D), dtype=compute_dtype)
    lse = np.empty((B, H, S), dtype=compute_dtype)
    attn = np.empty((B, H, S, S), dtype=compute_dtype) if return_weights else None
    cache = {}
    for b in range(B):
        for h in range(H):
            key = bm[b, h].tobytes()
            tm = cache.get(key)
            if tm is None:
                tm = cache[key] = token_mask(bm[b, h], block_size, S, causal)
            o, p, l = _slice_forward(q[b, h], np.asarray(k)[b, h], np.asarray(v)[b, h], tm,
                                     scale, compute_dtype)
            out[b, h] = o
            lse[b, h] = l
            if return_weights:
                attn[b, h] = p
    if return_lse:
        return out, attn, lse
    return out, attn


def sparse_attention_backward(q, k, v, do, block_mask, block_size: int = 128, scale=None,
                              causal: bool = False, compute_dtype=np.float64):
    """Closed-form gradients (dq, dk, dv) of ``sparse_attention_reference`` (float64 unless
    ``compute_dtype`` says otherwise; float32 is ~30x faster for large bf16 checks, whose
    2e-2 tolerance is far above float32 rounding)."""
    q = np.asarray(q, dtype=compute_dtype)
    k = np.asarray(k, dtype=compute_dtype)
    v = np.asarray(v, dtype=compute_dtype)
    do = np.asarray(do, dtype=compute_dtype)
    B, H, S, D = q.shape
    scale = scale or float(D ** -0.5)
    nb = S // block_size
    bm = broadcast_mask(block_mask, B, H, nb)
    dq = np.empty_like(q)
    dk = np.empty_like(k)
    dv = np.empty_like(v)
    for b in range(B):
        for h in range(H):
            tm = token_mask(bm[b, h], block_size, S, causal)
            o, p, _ = _slice_forward(q[b, h], k[b, h], v[b, h], tm, scale, compute_dtype)
            g = do[b, h]
            dv[b, h] = p.T @ g
            dp = g @ v[b, h].T
            delta = (g * o).sum(axis=-1, keepdims=True)
            ds = p * (dp - delta)
            ds = np.where(tm, ds, compute_dtype(0.0))
            dq[b, h] = (ds @ k[b, h]) * compute_dtype(scale)
            dk[b, h] = (ds.T @ q[b, h]) * compute_dtype(scale)
    return dq, dk, dv


def active_block_count(block_mask, batch: int, heads: int, nb: int, causal: bool,
                       block_size: int = 64) -> int:
    """n_a: number of active (q-block, kv-block) tiles over B*H after the causal cut.

    This is the unit of the ``4 * D * bs * bs`` FLOP accounting of one forward
    (observability/flops_counter.py:23-36 counts ``4*B*H*S^2*D*(1-sparsity)``).
    """
    bm = broadcast_mask(block_mask, batch, heads, nb).copy()
    if causal:
        bm = bm & np.tri(nb, bm.shape[-1], dtype=bool)
    return int(bm.sum())
