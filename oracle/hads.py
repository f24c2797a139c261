"""Oracle (test infrastructure): HADS calibration and block-mask construction.

Reference: kernels/hads/hads_pattern.py
  * ``compute_attention_entropy``  :36-50   clip(p, 1e-9, 1), H = -sum p log p over
    keys, mean over (batch, query)
  * ``entropy_to_sparsity``        :55-74   float32 min/max normalisation; note the
    span ``max_sparsity - min_sparsity`` is a Python-double subtraction that is
    rounded to float32 once (JAX weak typing; NumPy 2 follows the same NEP 50 rule)
  * ``_build_head_mask``           :79-113  window +/- w, then per row
    ``rng.choice(non-window columns, min(keep, len), replace=False)``, then the
    causal cut; ``rng = numpy.random.default_rng(seed)``
  * ``build_hads_profile``         :118-166 (mean of per-step entropies; seed = head)
  * ``dummy_hads_profile``         :169-206 (entropies = jnp.linspace(0.3, 2.5, H))
  * ``profile_summary``            :211-223
The "global KV block 0" rule is the documented one (README.md:166-169,
docs/hads_design.md:36-41) which the code lacks; ``apply_global_blocks`` adds it as
a separate step after the reference's mask so the reference's RNG draws are
unchanged.

Block masks depend on NumPy's PCG64 stream and ``Generator.choice``; they are
bit-exact for the NumPy version installed (recorded by the golden files).
"""

from __future__ import annotations

from typing import NamedTuple

import numpy as np

ENTROPY_EPS = 1e-9


class HADSProfile(NamedTuple):
    head_entropies: np.ndarray   # [H] float32
    head_sparsity: np.ndarray    # [H] float32
    block_masks: np.ndarray      # [H, nb, nb] bool


def compute_attention_entropy(attn_weights, compute_dtype=np.float64) -> np.ndarray:
    p = np.clip(np.asarray(attn_weights).astype(compute_dtype), ENTROPY_EPS, 1.0)
    h = -(p * np.log(p)).sum(axis=-1)          # [B, H, Sq]
    return h.mean(axis=(0, 2))                 # [H]


def entropy_head_sums(attn_weights) -> np.ndarray:
    """Per-head sum over (batch, query) of row entropies, float64 (un-normalised)."""
    p = np.clip(np.asarray(attn_weights).astype(np.float64), ENTROPY_EPS, 1.0)
    return (-(p * np.log(p)).sum(axis=-1)).sum(axis=(0, 2))


def entropy_to_sparsity(entropies, min_sparsity: float = 0.10, max_sparsity: float = 0.90):
    e = np.asarray(entropies, dtype=np.float32)
    e_min = e.min()
    e_max = e.max()
    e_range = np.maximum(e_max - e_min, np.float32(1e-6))
    norm = (e - e_min) / e_range
    span = np.float32(max_sparsity - min_sparsity)
    return (np.float32(max_sparsity) - norm * span).astype(np.float32)


def keep_margin(sparsity_ratio: float, num_blocks: int) -> float:
    """Distance of num_blocks*(1-rho) from the nearest integer (mask-parity safety margin)."""
    x = num_blocks * (1.0 - float(sparsity_ratio))
    return abs(x - round(x))


def build_head_mask(sparsity_ratio: float, num_blocks: int, window_size: int, seed: int,
                    causal: bool = False) -> np.ndarray:
    mask = np.zeros((num_blocks, num_blocks), dtype=bool)
    rng = np.random.default_rng(seed)
    keep = max(1, int(num_blocks * (1.0 - sparsity_ratio)))
    for i in range(num_blocks):
        lo = max(0, i - window_size)
        hi = min(num_blocks, i + window_size + 1)
        mask[i, lo:hi] = True
        cand = [j for j in range(num_blocks) if not mask[i, j]]
        if cand:
            mask[i, rng.choice(cand, size=min(keep, len(cand)), replace=False)] = True
    if causal:
        mask &= np.tri(num_blocks, num_blocks, dtype=bool)
    return mask


def apply_global_blocks(masks: np.ndarray, global_blocks: int) -> np.ndarray:
    m = np.array(masks, dtype=bool, copy=True)
    if global_blocks > 0:
        m[..., :, :global_blocks] = True
    return m


def jax_linspace_f32(start: float, stop: float, num: int) -> np.ndarray:
    """float32 ``jnp.linspace`` with x64 disabled: start*(1-t) + stop*t, t = i/(num-1),
    endpoint set exactly (JAX's linspace formulation)."""
    if num <= 0:
        return np.zeros((0,), np.float32)
    if num == 1:
        return np.array([start], np.float32)
    div = num - 1
    t = np.arange(div, dtype=np.float32) / np.float32(div)
    out = np.float32(start) * (np.float32(1) - t) + np.float32(stop) * t
    return np.concatenate([out, np.array([stop], np.float32)]).astype(np.float32)


def _masks(sparsity, num_blocks, window_size, causal, global_blocks):
    m = np.stack([build_head_mask(float(sparsity[h]), num_blocks, window_size, h, causal)
                  for h in range(len(sparsity))])
    return apply_global_blocks(m, global_blocks)


def build_hads_profile(calibration_attentions, seq_len: int, block_size: int,
                       min_sparsity: float = 0.10, max_sparsity: float = 0.90,
                       window_size: int = 2, causal: bool = False,
                       global_blocks: int = 0) -> HADSProfile:
    per_step = np.stack([compute_attention_entropy(a) for a in calibration_attentions])
    ent = per_step.mean(axis=0).astype(np.float32)
    return profile_from_entropies(ent, seq_len, block_size, min_sparsity, max_sparsity,
                                  window_size, causal, global_blocks)


def profile_from_entropies(ent, seq_len, block_size, min_sparsity=0.10, max_sparsity=0.90,
                           window_size=2, causal=False, global_blocks=0) -> HADSProfile:
    ent = np.asarray(ent, np.float32)
    sp = entropy_to_sparsity(ent, min_sparsity, max_sparsity)
    masks = _masks(sp, seq_len // block_size, window_size, causal, global_blocks)
    return HADSProfile(ent, sp, masks)


def dummy_hads_profile(n_heads: int, seq_len: int, block_size: int, min_sparsity: float = 0.10,
                       max_sparsity: float = 0.90, window_size: int = 2, causal: bool = False,
                       global_blocks: int = 0) -> HADSProfile:
    ent = jax_linspace_f32(0.3, 2.5, n_heads)
    return profile_from_entropies(ent, seq_len, block_size, min_sparsity, max_sparsity,
                                  window_size, causal, global_blocks)


def profile_summary(profile: HADSProfile) -> dict:
    sp = np.asarray(profile.head_sparsity)
    active = np.asarray(profile.block_masks).mean(axis=(-2, -1))
    return {
        "n_heads": int(np.asarray(profile.head_entropies).shape[0]),
        "mean_entropy": float(np.asarray(profile.head_entropies).mean()),
        "mean_sparsity": float(sp.mean()),
        "min_sparsity": float(sp.min()),
        "max_sparsity": float(sp.max()),
        "mean_active_frac": float(active.mean()),
        "overall_flop_ratio": float(active.mean()),
    }
