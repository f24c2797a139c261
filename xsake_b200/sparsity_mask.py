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


def _band(nb: int, half_width: int) -> np.ndarray:
    """bool [nb, nb]: |i - j| <= half_width."""
    idx = np.arange(nb)
    return np.abs(idx[:, None] - idx[None, :]) <= half_width


def make_block_mask(seq_len: int, block_size: int, sparsity_type: str, sparsity_ratio: float = 0.5,
                    window_size: int = 3, global_blocks: int = 1, causal: bool = False,
                    rng: Optional[int] = None) -> np.ndarray:
    """bool [nb, nb] block mask of ``sparsity_type`` (sparsity_mask.py:25-102).

    The seeded patterns draw with NumPy's ``Generator.choice`` row by row, in the reference's
    order and over the same candidate sets, so the masks are the reference's bit for bit."""
    if seq_len % block_size != 0:
        raise ValueError(f"block_size {block_size} does not divide seq_len {seq_len}")
    nb = seq_len // block_size
    if sparsity_type == "dense":
        mask = np.ones((nb, nb), dtype=bool)
    elif sparsity_type == "local":
        mask = _band(nb, window_size)
    elif sparsity_type == "random":
        per_row = max(1, int(nb * (1.0 - sparsity_ratio)))
        gen = np.random.default_rng(0 if rng is None else int(rng))
        mask = np.zeros((nb, nb), dtype=bool)
        for row in mask:
            row[gen.choice(nb, size=per_row, replace=False)] = True
    elif sparsity_type == "bigbird":
        # Fixed part first (leading columns + band around the diagonal), then per row a seeded
        # draw of up to 15% of the blocks among the columns the fixed part leaves out.
        mask = _band(nb, window_size)
        mask[:, :min(global_blocks, nb)] = True
        extra = max(1, int(nb * 0.15))
        gen = np.random.default_rng(42)
        for row in mask:
            free = np.flatnonzero(~row)
            if free.size:
                row[gen.choice(free, size=min(extra, free.size), replace=False)] = True
    else:
        raise ValueError(f"sparsity_type must be one of {SPARSITY_TYPES} (got {sparsity_type!r}); "
                         "HADS masks come from xsake_b200.hads_pattern.build_hads_profile()")
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
