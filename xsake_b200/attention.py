"""Multi-head HADS sparse attention layer: the caller of the attention kernels.

PyTorch counterpart of ``XSAKEAttention`` (model/attention.py:33-143): q, k, v projections of
d_model -> n_heads x d_head, block masks chosen as the reference does (a HADS profile, else the
configured pattern, else dense), sparse attention with causal=True and scale d_head^-0.5, output
projection, dropout.  The projections are plain GEMMs (torch.nn.Linear, cuBLAS); the attention is
this library's kernel.  The head split is a view: q, k, v stay in the projection's [B, S, H, D]
memory and are read through their strides, and the attention output is written in that layout,
so no [B, S, H, D] <-> [B, H, S, D] copy is made in either direction (the reference transposes,
model/attention.py:80,99).  Gradients flow through the library's backward kernels.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch
from torch import nn

from . import hads_pattern as hp
from . import sparsity_mask as sm
from .sparse_attention import attention_probabilities, sparse_attention_autograd


# Masks built from layer parameters alone (the uncalibrated HADS profile, the fixed patterns) are
# deterministic, so they are built once per parameter set and shared, read-only, by every layer
# and call.  The reference builds them on the host at trace time, i.e. once per compiled step;
# rebuilding the dummy profile on every call cost ~10 ms of host time per layer at S=4096.
_MASKS: dict = {}


def _cached_mask(key, build):
    m = _MASKS.get(key)
    if m is None:
        m = np.ascontiguousarray(build(), dtype=bool)
        m.setflags(write=False)
        _MASKS[key] = m
    return m


class XSAKEAttention(nn.Module):
    """Drop-in for model/attention.py's XSAKEAttention.

    Args mirror the reference's ModelConfig fields the layer reads: d_model, n_heads, n_layers
    (output-projection init scale), bias, dropout, dtype, and the kernel config: block_size
    (``block_size_q``), sparsity_type, and the HADS parameters used for the uncalibrated profile.
    """

    def __init__(self, d_model: int, n_heads: int, n_layers: int = 12, bias: bool = False,
                 dropout: float = 0.0, dtype=torch.bfloat16, block_size: int = 128,
                 sparsity_type: str = "hads", hads_profile: Optional[hp.HADSProfile] = None,
                 min_sparsity: float = 0.10, max_sparsity: float = 0.90, window_size: int = 2,
                 device=None):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        self.d_model, self.n_heads, self.d_head = d_model, n_heads, d_model // n_heads
        self.block_size, self.sparsity_type, self.hads_profile = block_size, sparsity_type, hads_profile
        self.min_sparsity, self.max_sparsity, self.window_size = min_sparsity, max_sparsity, window_size
        kw = dict(bias=bias, dtype=dtype, device=device)
        self.q_proj = nn.Linear(d_model, d_model, **kw)
        self.k_proj = nn.Linear(d_model, d_model, **kw)
        self.v_proj = nn.Linear(d_model, d_model, **kw)
        self.out_proj = nn.Linear(d_model, d_model, **kw)
        with torch.no_grad():
            for lin in (self.q_proj, self.k_proj, self.v_proj):
                nn.init.normal_(lin.weight, std=0.02)
            nn.init.normal_(self.out_proj.weight, std=0.02 / math.sqrt(2 * n_layers))
            for lin in (self.q_proj, self.k_proj, self.v_proj, self.out_proj):
                if lin.bias is not None:
                    nn.init.zeros_(lin.bias)
        self.drop = nn.Dropout(dropout)

    def _heads(self, t: torch.Tensor, batch: int, seq: int) -> torch.Tensor:
        # [B, S, d_model] -> [B, H, S, D] view of the same memory (strides S*H*D, D, H*D, 1)
        return t.view(batch, seq, self.n_heads, self.d_head).transpose(1, 2)

    def get_block_mask(self, seq: int) -> Tuple[np.ndarray, int]:
        """(block mask [H, nb, nb] or [nb, nb], block size) with the reference's priority
        (model/attention.py:107-143): HADS profile > sparsity_type > dense.  A sequence that is
        not a multiple of the block size attends densely, as the reference does."""
        bs = self.block_size
        if seq % bs != 0:
            bs = math.gcd(seq, bs)
            return np.ones((seq // bs, seq // bs), bool), bs
        if self.hads_profile is not None:
            return np.asarray(self.hads_profile.block_masks, bool), bs
        if self.sparsity_type == "hads":
            key = ("hads", self.n_heads, seq, bs, self.min_sparsity, self.max_sparsity, self.window_size)
            return _cached_mask(key, lambda: hp.dummy_hads_profile(
                self.n_heads, seq, bs, self.min_sparsity, self.max_sparsity, self.window_size,
                causal=True).block_masks), bs
        key = (self.sparsity_type, seq, bs)
        return _cached_mask(key, lambda: sm.make_block_mask(seq, bs, self.sparsity_type, sparsity_ratio=0.5,
                                                            causal=True)), bs

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None, training: Optional[bool] = None,
                collect_attn: bool = False):
        """x [B, S, d_model] -> (out [B, S, d_model], attention weights [B, H, S, S] fp32 or None).

        ``mask`` (a token mask) is accepted and, as in the reference, not used: causality is
        always applied.  ``training`` overrides the module's train/eval mode for dropout.
        ``collect_attn`` returns the attention weights that HADS calibration consumes."""
        del mask
        batch, seq, _ = x.shape
        q = self._heads(self.q_proj(x), batch, seq)
        k = self._heads(self.k_proj(x), batch, seq)
        v = self._heads(self.v_proj(x), batch, seq)
        block_mask, bs = self.get_block_mask(seq)
        scale = float(self.d_head ** -0.5)
        out = sparse_attention_autograd(q, k, v, block_mask, bs, scale, True)
        out = out.transpose(1, 2).reshape(batch, seq, self.d_model)   # a view when out is [B, S, H, D]
        out = self.out_proj(out)
        if training is None:
            out = self.drop(out)
        elif training:
            out = nn.functional.dropout(out, self.drop.p, True)
        weights = None
        if collect_attn:
            with torch.no_grad():
                weights = attention_probabilities(q.detach(), k.detach(), block_mask, bs, scale, True)
        return out, weights
