"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

The reference's benchmarks draw q, k, v from one ``jax.random.PRNGKey(0)`` (so
q == k == v there, benchmarks/attention_benchmark.py:36-41).  JAX is not available
and the configurations ask for independent draws, so every tensor here comes from
``numpy.random.default_rng(seed)`` in a fixed order.  No dataset is involved.

Configurations (seed = 1000 + id):
  0  fp32 attention fwd, B=1 H=12 S=1024 D=64, 64x64 blocks, calibrated HADS masks
  1  softmax fp32 [8*12*1024, 1024] ~ N(0, 2^2) with causal -inf; LayerNorm bf16
     [8192, 768] ~ N(0,1), gamma = 1 + 0.1 N(0,1), beta = 0.1 N(0,1), eps 1e-5
  2  calibration: 50 batches of B=8 H=12 S=1024 D=64 fp32 q, k; q of head h * tau_h
  3  bf16 attention fwd+bwd, B=4 H=12 S=4096 D=64, dO ~ N(0,1)
tau_h = linspace(0.25, 4, H)[h] scales q of head h so that head entropies differ.
"""

from __future__ import annotations

import numpy as np

SEED_BASE = 1000


def tau(heads: int) -> np.ndarray:
    return np.linspace(0.25, 4.0, heads).astype(np.float32)


def qkv(batch, heads, seq, d, seed, scale_q_by_tau=True, with_do=False):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
    k = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
    v = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
    if scale_q_by_tau:
        q *= tau(heads)[None, :, None, None]
    if with_do:
        do = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
        return q, k, v, do
    return q, k, v


def softmax_logits(rows=8 * 12 * 1024, cols=1024, seed=SEED_BASE + 1):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(2.0)
    qpos = (np.arange(rows) % cols)[:, None]
    x[np.arange(cols)[None, :] > qpos] = -np.inf
    return x


def layernorm_inputs(rows=8192, d=768, seed=SEED_BASE + 11):
    import ml_dtypes
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, d), dtype=np.float32).astype(ml_dtypes.bfloat16)
    gamma = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(d)).astype(np.float32)
    return x, gamma, beta


def calibration_batch(i, batch=8, heads=12, seq=1024, d=64, seed=SEED_BASE + 2):
    """Batch ``i`` of config 2: (q, k) fp32, q scaled by tau."""
    rng = np.random.default_rng([seed, i])
    q = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
    k = rng.standard_normal((batch, heads, seq, d), dtype=np.float32)
    q *= tau(heads)[None, :, None, None]
    return q, k


def to_bf16(x):
    import ml_dtypes
    return np.asarray(x, np.float32).astype(ml_dtypes.bfloat16)
