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


def _config_fields(cfg):
    """The layer's fields from a model config: the reference's ModelConfig with a nested
    ``kernel`` (model/config.py:18-58) or this package's flat ModelConfig."""
    k = getattr(cfg, "kernel", None)
    hads = getattr(k, "hads", None) if k is not None else None
    pick = lambda obj, name, flat: getattr(obj, name) if obj is not None else getattr(cfg, flat)   # noqa: E731
    dtype = torch.bfloat16 if getattr(cfg, "dtype", "bfloat16") == "bfloat16" else torch.float32
    return dict(d_model=cfg.d_model, n_heads=cfg.n_heads, n_layers=cfg.n_layers, bias=cfg.bias,
                dropout=cfg.dropout, dtype=dtype, block_size=pick(k, "block_size_q", "block_size"),
                sparsity_type=pick(k, "sparsity_type", "sparsity_type"),
                min_sparsity=pick(hads, "min_sparsity", "min_sparsity"),
                max_sparsity=pick(hads, "max_sparsity", "max_sparsity"),
                window_size=pick(hads, "window_size", "window_size"))


class XSAKEAttention(nn.Module):
    """Drop-in for model/attention.py's XSAKEAttention.

    Constructed like the reference, ``XSAKEAttention(config, hads_profile=None)``
    (model/attention.py:41-42, ``config`` a ModelConfig), or from the fields the layer reads:
    d_model, n_heads, n_layers (output-projection init scale), bias, dropout, dtype, and the
    kernel config: block_size (``block_size_q``), sparsity_type, and the HADS parameters used
    for the uncalibrated profile.  Keywords given next to a config override its fields (e.g.
    ``dtype=torch.float32`` for fp32 master weights under autocast)."""

    def __init__(self, d_model=None, n_heads=None, n_layers: int = 12, bias: bool = False,
                 dropout: float = 0.0, dtype=None, block_size: int = 128,
                 sparsity_type: str = "hads", hads_profile: Optional[hp.HADSProfile] = None,
                 min_sparsity: float = 0.10, max_sparsity: float = 0.90, window_size: int = 2,
                 device=None, config=None):
        if config is None and d_model is not None and not isinstance(d_model, int):
            config, d_model = d_model, None
        if config is not None:
            if n_heads is not None and not isinstance(n_heads, int):    # XSAKEAttention(config, profile)
                hads_profile, n_heads = n_heads, None
            f = _config_fields(config)
            d_model, n_heads, n_layers, bias, dropout = (f["d_model"], f["n_heads"], f["n_layers"], f["bias"],
                                                         f["dropout"])
            dtype = dtype if dtype is not None else f["dtype"]
            block_size, sparsity_type = f["block_size"], f["sparsity_type"]
            min_sparsity, max_sparsity, window_size = f["min_sparsity"], f["max_sparsity"], f["window_size"]
        if d_model is None or n_heads is None:
            raise TypeError("XSAKEAttention needs a model config or d_model and n_heads")
        dtype = dtype if dtype is not None else torch.bfloat16
        super().__init__()
        self.config = config
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

    @classmethod
    def from_config(cls, config, hads_profile: Optional[hp.HADSProfile] = None, **overrides):
        """``XSAKEAttention(config, hads_profile)`` of model/attention.py:41-42."""
        return cls(config=config, hads_profile=hads_profile, **overrides)

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
