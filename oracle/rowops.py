"""Oracle (test infrastructure): row softmax and LayerNorm, forward and backward.

Reference:
  * ``fused_softmax`` -> ``jax.nn.softmax(x, axis=-1)`` on CPU
    (kernels/pallas/fused_softmax.py:87); the Pallas body is the same
    max / exp / normalise (:33-36).  jax.nn.softmax subtracts the row max and
    divides by the row sum, so a row of all -inf yields NaN.
  * ``fused_layernorm`` (kernels/pallas/fused_layernorm.py:43-51 Pallas body with
    fp32 statistics and output cast to x.dtype; :116-119 CPU formula):
    mean, biased variance of (x - mean), x_hat = (x - mean)/sqrt(var + eps),
    y = gamma * x_hat + beta.
Backwards are the closed forms of autodiff through those formulas.
All arithmetic in float64 unless stated.
"""

from __future__ import annotations

import numpy as np


def softmax(x, compute_dtype=np.float64):
    x = np.asarray(x).astype(compute_dtype)
    with np.errstate(invalid="ignore"):
        m = x.max(axis=-1, keepdims=True)
        e = np.exp(x - m)
        return e / e.sum(axis=-1, keepdims=True)


def softmax_backward(y, dy):
    y = np.asarray(y, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    return y * (dy - (dy * y).sum(axis=-1, keepdims=True))


def layernorm(x, gamma, beta, eps: float = 1e-5, compute_dtype=np.float64, return_stats=False):
    x = np.asarray(x).astype(compute_dtype)
    g = np.asarray(gamma).astype(compute_dtype)
    b = np.asarray(beta).astype(compute_dtype)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + compute_dtype(eps))
    y = g * ((x - mean) * rstd) + b
    if return_stats:
        return y, mean[..., 0], rstd[..., 0]
    return y


def layernorm_backward(x, gamma, dy, eps: float = 1e-5):
    """Returns (dx, dgamma, dbeta) in float64."""
    x = np.asarray(x, dtype=np.float64)
    g = np.asarray(gamma, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    d = x.shape[-1]
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + eps)
    xhat = (x - mean) * rstd
    gdy = dy * g
    dx = rstd * (gdy - gdy.mean(axis=-1, keepdims=True)
                 - xhat * (gdy * xhat).sum(axis=-1, keepdims=True) / d)
    red = tuple(range(x.ndim - 1))
    dgamma = (dy * xhat).sum(axis=red)
    dbeta = dy.sum(axis=red)
    return dx, dgamma, dbeta
