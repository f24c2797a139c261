"""HADS (head-adaptive dynamic sparsity) calibration and block masks.

Same API as the reference module kernels/hads/hads_pattern.py:
  * ``HADSProfile``                         :27-31
  * ``compute_attention_entropy``           :36-50   -> GPU kernel (xsake_entropy_rows)
  * ``entropy_to_sparsity``                 :55-74   -> host float32, same expression
  * ``_build_head_mask``                    :79-113  -> host NumPy, same RNG calls
  * ``build_hads_profile``                  :118-166
  * ``dummy_hads_profile``                  :169-206
  * ``profile_summary``                     :211-223
plus ``global_blocks`` (the documented "global KV block 0 always on" rule of README.md:166-169
and docs/hads_design.md:36-41, which the reference code lacks).  ``global_blocks=0`` (the
default) reproduces the reference's masks bit-exactly; it is applied after the reference's
draws so the seeded stream is unchanged.

The seeded mask draw stays on the host on purpose: it is O(heads * nb^2) NumPy work whose
result depends on NumPy's PCG64 ``Generator.choice`` stream, and bit-exact masks are the
contract.  The device work of mask handling (causal cut, compression into per-tile work
lists) happens in ``sparse_attention.compile_block_mask``.
"""

from __future__ import annotations

import ctypes as C
from typing import List, NamedTuple, Optional

import numpy as np
import torch

from . import _device as dev
from . import _lib

ENTROPY_EPS = 1e-9


class HADSProfile(NamedTuple):
    """Calibrated per-head sparsity configuration (hads_pattern.py:27-31)."""
    head_entropies: np.ndarray   # [n_heads] float32
    head_sparsity: np.ndarray    # [n_heads] float32
    block_masks: np.ndarray      # [n_heads, nb, nb] bool


# ----------------------------------------------------------------------------- entropy (GPU)
def entropy_head_sums(attn_weights) -> torch.Tensor:
    """float64 [H] sums over (batch, query) of row entropies of ``attn_weights``
    [B, H, Sq, Sk] (fp32).  Summable across ranks before dividing by B*Sq."""
    dev.require_cuda()
    p, _ = dev.to_device(attn_weights, torch.float32)
    p = p.contiguous()
    if p.dim() != 4:
        raise ValueError(f"attn_weights must be [batch, heads, seq_q, seq_k], got {tuple(p.shape)}")
    B, H, Sq, Sk = p.shape
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_entropy_workspace_size(B, H, Sq, C.byref(n)))
    ws = dev.workspace(n.value, p.device)
    sums = torch.empty(H, dtype=torch.float64, device=p.device)
    _lib.check(lib.xsake_entropy_rows(p.data_ptr(), B, H, Sq, Sk, sums.data_ptr(), ws.data_ptr(),
                                      ws.numel(), dev.stream_ptr()))
    return sums


def entropy_head_sums_qk(q, k, scale: Optional[float] = None) -> torch.Tensor:
    """float64 [H] sums over (batch, query) of the row entropies of softmax(q k^T * scale),
    without materialising the weights (fused on the GPU; q, k [B, H, S, D], fp32 or bf16)."""
    dev.require_cuda()
    q, _ = dev.to_device(q)
    k, _ = dev.to_device(k)
    q, k = q.contiguous(), k.contiguous()
    if q.dim() != 4 or k.shape != q.shape or k.dtype != q.dtype:
        raise ValueError(f"q and k must be [batch, heads, seq, d_head] of one dtype, got {tuple(q.shape)} "
                         f"{tuple(k.shape)}")
    B, H, S, D = q.shape
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_entropy_qk_workspace_size(B, H, S, C.byref(n)))
    ws = dev.workspace(n.value, q.device)
    sums = torch.empty(H, dtype=torch.float64, device=q.device)
    _lib.check(lib.xsake_entropy_qk(dev.xsake_dtype(q), q.data_ptr(), k.data_ptr(), B, H, S, D,
                                    float(scale) if scale else 0.0, sums.data_ptr(), ws.data_ptr(), ws.numel(),
                                    dev.stream_ptr()))
    return sums


def entropy_head_sums_attention(q, k, block_mask, block_size: int, scale: Optional[float] = None,
                                causal: bool = True) -> torch.Tensor:
    """float64 [H] sums over (batch, query) of the row entropies of the attention weights that
    ``sparse_attention(..., use_pallas=False)`` returns for this block mask (masked, causal cut,
    finfo.min fill), computed on the GPU without materialising them.  These are the weights
    the reference's calibration reduces (training/trainer.py:79-117 -> hads_pattern.py:36-50).
    q, k: CUDA [B, H, S, D] tensors, any strides with a unit last stride."""
    from .sparse_attention import _desc, _unit_last, compile_block_mask
    dev.require_cuda()
    q, k = (_unit_last(dev.to_device(t)[0]) for t in (q, k))
    if q.dim() != 4 or k.shape != q.shape or k.dtype != q.dtype:
        raise ValueError(f"q and k must be [batch, heads, seq, d_head] of one dtype, got {tuple(q.shape)} "
                         f"{tuple(k.shape)}")
    B, H, S, D = q.shape
    cm = compile_block_mask(block_mask, B, H, S, block_size, causal, q.device)
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_entropy_qk_workspace_size(B, H, S, C.byref(n)))
    ws = dev.workspace(n.value, q.device)
    sums = torch.empty(H, dtype=torch.float64, device=q.device)
    d = _desc(q, k, k, q, cm, scale)
    _lib.check(lib.xsake_attn_entropy(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(), sums.data_ptr(),
                                      ws.data_ptr(), ws.numel(), dev.stream_ptr()))
    return sums


def compute_attention_entropy_qk(q, k, scale: Optional[float] = None):
    """``compute_attention_entropy(softmax(q k^T * scale))`` (hads_pattern.py:36-50) fused: the
    calibration pass's entropies straight from q and k.  float32 [H] (NumPy for host input)."""
    was_host = not (isinstance(q, torch.Tensor) and q.is_cuda)
    B, _, S, _ = q.shape
    ent = (entropy_head_sums_qk(q, k, scale) / float(B * S)).to(torch.float32)
    return dev.to_host(ent) if was_host else ent


def compute_attention_entropy(attn_weights):
    """Mean Shannon entropy per head of softmax weights [B, H, Sq, Sk] (hads_pattern.py:36-50).
    Returns float32 [H]: NumPy for host input, a CUDA tensor for device input."""
    was_host = not (isinstance(attn_weights, torch.Tensor) and attn_weights.is_cuda)
    sums = entropy_head_sums(attn_weights)
    B, _, Sq, _ = attn_weights.shape
    ent = (sums / float(B * Sq)).to(torch.float32)
    return dev.to_host(ent) if was_host else ent


# ----------------------------------------------------------------------------- host mapping
def entropy_to_sparsity(entropies, min_sparsity: float = 0.10, max_sparsity: float = 0.90) -> np.ndarray:
    """Linear entropy -> sparsity map in float32 (hads_pattern.py:55-74).  The span is the
    Python-float difference ``max_sparsity - min_sparsity`` rounded once to float32, which is
    how the reference's weakly typed scalars combine with a float32 array."""
    if isinstance(entropies, torch.Tensor):
        entropies = entropies.detach().cpu().numpy()
    e = np.asarray(entropies, dtype=np.float32)
    e_min, e_max = e.min(), e.max()
    e_range = np.maximum(e_max - e_min, np.float32(1e-6))
    normalized = (e - e_min) / e_range
    return (np.float32(max_sparsity) - normalized * np.float32(max_sparsity - min_sparsity)).astype(np.float32)


def _build_head_mask(sparsity_ratio: float, num_blocks: int, window_size: int, seed: int,
                     causal: bool = False) -> np.ndarray:
    """One head's block mask (hads_pattern.py:79-113): local window of +/- window_size blocks,
    then per row ``min(keep, #free)`` distinct long-range blocks drawn with
    ``default_rng(seed).choice`` from the free columns in ascending order, then the causal cut.
    keep = max(1, int(num_blocks * (1 - sparsity_ratio))) in double precision."""
    mask = np.zeros((num_blocks, num_blocks), dtype=bool)
    rng = np.random.default_rng(seed)
    keep = max(1, int(num_blocks * (1.0 - sparsity_ratio)))
    cols = np.arange(num_blocks)
    for i in range(num_blocks):
        mask[i, max(0, i - window_size):min(num_blocks, i + window_size + 1)] = True
        free = cols[~mask[i]]
        if free.size:
            mask[i, rng.choice(free, size=min(keep, free.size), replace=False)] = True
    if causal:
        mask &= np.tri(num_blocks, dtype=bool)
    return mask


def _apply_global(masks: np.ndarray, global_blocks: int) -> np.ndarray:
    if global_blocks > 0:
        masks = masks.copy()
        masks[..., :global_blocks] = True
    return masks


def keep_margin(sparsity_ratio: float, num_blocks: int) -> float:
    """Distance of ``num_blocks * (1 - rho)`` from the nearest integer.  Masks can only differ
    from another implementation's when this is tiny (float rounding of rho), so profiles
    report it."""
    x = num_blocks * (1.0 - float(sparsity_ratio))
    return abs(x - round(x))


def profile_from_entropies(head_entropies, seq_len: int, block_size: int, min_sparsity: float = 0.10,
                           max_sparsity: float = 0.90, window_size: int = 2, causal: bool = False,
                           global_blocks: int = 0) -> HADSProfile:
    ent = np.asarray(head_entropies.detach().cpu().numpy() if isinstance(head_entropies, torch.Tensor)
                     else head_entropies, dtype=np.float32)
    sp = entropy_to_sparsity(ent, min_sparsity, max_sparsity)
    nb = seq_len // block_size
    masks = np.stack([_build_head_mask(float(sp[h]), nb, window_size, h, causal) for h in range(len(sp))])
    return HADSProfile(ent, sp, _apply_global(masks, global_blocks))


def build_hads_profile(calibration_attentions: List, seq_len: int, block_size: int,
                       min_sparsity: float = 0.10, max_sparsity: float = 0.90, window_size: int = 2,
                       causal: bool = False, global_blocks: int = 0) -> HADSProfile:
    """Profile from calibration attention weights (hads_pattern.py:118-166): per-step head
    entropies on the GPU, their float32 mean, the sparsity map and the per-head masks."""
    per_step = np.stack([np.asarray(dev.to_host(compute_attention_entropy(
        a if isinstance(a, torch.Tensor) else dev.to_device(a, torch.float32)[0])), np.float32)
        for a in calibration_attentions])
    head_entropies = per_step.mean(axis=0).astype(np.float32)
    return profile_from_entropies(head_entropies, seq_len, block_size, min_sparsity, max_sparsity,
                                  window_size, causal, global_blocks)


def jax_linspace_f32(start: float, stop: float, num: int) -> np.ndarray:
    """float32 linspace formulated as start*(1-t) + stop*t with the endpoint exact (the
    reference calls ``jnp.linspace`` with JAX's default 32-bit floats)."""
    if num == 1:
        return np.array([start], np.float32)
    t = np.arange(num - 1, dtype=np.float32) / np.float32(num - 1)
    head = np.float32(start) * (np.float32(1) - t) + np.float32(stop) * t
    return np.concatenate([head, np.array([stop], np.float32)]).astype(np.float32)


def dummy_hads_profile(n_heads: int, seq_len: int, block_size: int, min_sparsity: float = 0.10,
                       max_sparsity: float = 0.90, window_size: int = 2, causal: bool = False,
                       global_blocks: int = 0) -> HADSProfile:
    """Profile with linearly spaced synthetic entropies 0.3..2.5 (hads_pattern.py:169-206)."""
    return profile_from_entropies(jax_linspace_f32(0.3, 2.5, n_heads), seq_len, block_size,
                                  min_sparsity, max_sparsity, window_size, causal, global_blocks)


def profile_summary(profile: HADSProfile) -> dict:
    """Human-readable summary (hads_pattern.py:211-223)."""
    sp = np.asarray(profile.head_sparsity)
    active = np.asarray(profile.block_masks).mean(axis=(-2, -1))
    ent = np.asarray(profile.head_entropies)
    return {
        "n_heads": int(ent.shape[0]),
        "mean_entropy": float(ent.mean()),
        "mean_sparsity": float(sp.mean()),
        "min_sparsity": float(sp.min()),
        "max_sparsity": float(sp.max()),
        "mean_active_frac": float(active.mean()),
        "overall_flop_ratio": float(active.mean()),
    }


# ----------------------------------------------------------------------------- persistence
def save_profile(profile: HADSProfile, path) -> None:
    """Write a calibrated profile (entropies, rho, masks) with the NumPy version that drew the
    masks; the reference keeps its profile in memory only (training/checkpointing.py:9)."""
    np.savez(path, head_entropies=np.asarray(profile.head_entropies, np.float32),
             head_sparsity=np.asarray(profile.head_sparsity, np.float32),
             block_masks=np.asarray(profile.block_masks, bool), numpy_version=np.array(np.__version__))


def load_profile(path) -> HADSProfile:
    """Read a profile written by ``save_profile``.  The stored masks are used as they are, so a
    different NumPy version (whose Generator.choice stream may differ) does not change them."""
    z = np.load(path, allow_pickle=False)
    for key in ("head_entropies", "head_sparsity", "block_masks"):
        if key not in z.files:
            raise ValueError(f"{path}: not a HADS profile (missing {key})")
    return HADSProfile(z["head_entropies"].astype(np.float32), z["head_sparsity"].astype(np.float32),
                       z["block_masks"].astype(bool))


# ----------------------------------------------------------------------------- multi-rank
def allreduce_head_sums(sums: torch.Tensor, group: Optional[object] = None) -> torch.Tensor:
    """Sum per-head entropy partials over ranks (each rank's disjoint share of the calibration
    rows).  Deterministic for a fixed world size; a no-op without torch.distributed."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    return sums
