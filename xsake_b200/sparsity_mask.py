"""Block sparsity patterns other than HADS, for the same attention kernels.

Drop-in for kernels/pallas/sparsity_mask.py (make_block_mask :25-102, mask_to_token_level
:105-117, sparsity_ratio :120-124): host NumPy construction of bool [nq, nk] masks.  Any such mask
goes through ``sparse_attention`` / ``xsake_mask_compile`` unchanged; only HADS masks are per
head.  "dense", "local" and "bigbird" match the reference bit-exactly (pinned by golden vectors
from its own code); "random" takes an integer seed, because the reference draws its NumPy seed
from jax.random.randint, which is not available here.
"""

from __future__ import annotations

from typing import Optional

import numpy as np

SPARSITY_TYPES = ("dense", "local", "random", "bigbird")


def make_block_mask(seq_len: int, block_size: int, sparsity_type: str, sparsity_ratio: float = 0.5,
                    window_size: int = 3, global_blocks: int = 1, causal: bool = False,
                    rng: Optional[int] = None) -> np.ndarray:
    """bool [nb, nb] block mask of ``sparsity_type`` (sparsity_mask.py:25-102)."""
    if seq_len % block_size != 0:
        raise ValueError("seq_len must be divisible by block_size")
    nb = seq_len // block_size
    if sparsity_type == "dense":
        mask = np.ones((nb, nb), dtype=bool)
    elif sparsity_type == "local":
        mask = np.zeros((nb, nb), dtype=bool)
        for i in range(nb):
            mask[i, max(0, i - window_size):min(nb, i + window_size + 1)] = True
    elif sparsity_type == "random":
        keep = max(1, int(nb * (1.0 - sparsity_ratio)))
        mask = np.zeros((nb, nb), dtype=bool)
        gen = np.random.default_rng(0 if rng is None else int(rng))
        for i in range(nb):
            mask[i, gen.choice(nb, size=keep, replace=False)] = True
    elif sparsity_type == "bigbird":
        mask = np.zeros((nb, nb), dtype=bool)
        g = min(global_blocks, nb)
        rand_keep = max(1, int(nb * 0.15))
        gen = np.random.default_rng(42)
        for i in range(nb):
            mask[i, :g] = True                                            # global blocks
            mask[i, max(0, i - window_size):min(nb, i + window_size + 1)] = True   # local window
            candidates = np.where(~mask[i])[0]                            # random long range
            if len(candidates) > 0:
                mask[i, gen.choice(candidates, size=min(rand_keep, len(candidates)), replace=False)] = True
    else:
        raise ValueError(f"Unknown sparsity_type '{sparsity_type}'. For 'hads', use "
                         "xsake_b200.hads_pattern.build_hads_profile().")
    if causal:
        mask &= np.tri(nb, nb, dtype=bool)
    return mask


def mask_to_token_level(block_mask, block_size: int, seq_len: int) -> np.ndarray:
    """Token-level [seq, seq] expansion of a block mask (sparsity_mask.py:105-117)."""
    nb = seq_len // block_size
    bm = np.asarray(block_mask)[:nb, :nb]
    return np.repeat(np.repeat(bm, block_size, axis=0), block_size, axis=1)[:seq_len, :seq_len]


def sparsity_ratio(block_mask) -> float:
    """Fraction of blocks skipped (sparsity_mask.py:120-124)."""
    m = np.asarray(block_mask)
    return 1.0 - int(m.sum()) / m.size
