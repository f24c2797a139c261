"""GPT-style transformer around the HADS attention layer: the model the reference trains.

PyTorch counterpart of XSAKETransformer (model/transformer.py:71-172), TransformerBlock
(:74-104), MLP (:33-46), the LayerNorm wrapper (:51-66), TransformerEmbedding
(model/embedding.py:63-90) and cross_entropy_loss (model/transformer.py:177-203):
token + learned position embeddings, pre-norm blocks (fused LayerNorm in fp32 as the reference
calls it, XSAKE attention, GELU MLP), final LayerNorm, logits tied to the token embedding.

Attention and LayerNorm run on this library's kernels; the dense projections, embeddings and the
optimizer are PyTorch.  The logits GEMM runs in the activation dtype with fp32 loss arithmetic
(the reference computes the logits GEMM itself in fp32).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
from torch import nn
from torch.nn import functional as F

from . import hads_pattern as hp
from .attention import XSAKEAttention
from .fused_layernorm import fused_layernorm


@dataclass
class ModelConfig:
    """The fields of model/config.py the model reads (defaults: GPT-2 small, the reference's)."""
    vocab_size: int = 50_257
    seq_len: int = 1_024
    n_layers: int = 12
    n_heads: int = 12
    d_model: int = 768
    d_ff: int = 3_072
    dropout: float = 0.0
    bias: bool = False
    block_size: int = 128
    sparsity_type: str = "hads"
    min_sparsity: float = 0.10
    max_sparsity: float = 0.90
    window_size: int = 2


class LayerNorm(nn.Module):
    """model/transformer.py:51-66: fp32 statistics and parameters, result in x's dtype."""

    def __init__(self, d_model: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(d_model, device=device))
        self.beta = nn.Parameter(torch.zeros(d_model, device=device))
        self.eps = eps

    def forward(self, x):
        return fused_layernorm(x.float(), self.gamma.float(), self.beta.float(), eps=self.eps).to(x.dtype)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig, device=None):
        super().__init__()
        self.fc1 = nn.Linear(cfg.d_model, cfg.d_ff, bias=cfg.bias, device=device)
        self.fc2 = nn.Linear(cfg.d_ff, cfg.d_model, bias=cfg.bias, device=device)
        nn.init.normal_(self.fc1.weight, std=0.02)
        nn.init.normal_(self.fc2.weight, std=0.02 / math.sqrt(2 * cfg.n_layers))
        for lin in (self.fc1, self.fc2):
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)
        self.drop = nn.Dropout(cfg.dropout)

    def forward(self, x):
        return self.drop(self.fc2(F.gelu(self.fc1(x), approximate="tanh")))   # flax nn.gelu default


class TransformerBlock(nn.Module):
    def __init__(self, cfg: ModelConfig, hads_profile: Optional[hp.HADSProfile] = None, device=None):
        super().__init__()
        self.ln1 = LayerNorm(cfg.d_model, device=device)
        self.attn = XSAKEAttention(cfg.d_model, cfg.n_heads, cfg.n_layers, cfg.bias, cfg.dropout,
                                   dtype=torch.float32, block_size=cfg.block_size,
                                   sparsity_type=cfg.sparsity_type, hads_profile=hads_profile,
                                   min_sparsity=cfg.min_sparsity, max_sparsity=cfg.max_sparsity,
                                   window_size=cfg.window_size, device=device)
        self.ln2 = LayerNorm(cfg.d_model, device=device)
        self.mlp = MLP(cfg, device=device)

    def forward(self, x, collect_attn: bool = False):
        a, w = self.attn(self.ln1(x), collect_attn=collect_attn)
        x = x + a
        x = x + self.mlp(self.ln2(x))
        return x, w


class XSAKETransformer(nn.Module):
    """Parameters are fp32 (master weights); run the forward under
    ``torch.autocast("cuda", torch.bfloat16)`` for bf16 arithmetic, as the reference's bf16 model."""

    def __init__(self, cfg: ModelConfig, hads_profile: Optional[hp.HADSProfile] = None, device=None):
        super().__init__()
        self.cfg = cfg
        self.tok = nn.Embedding(cfg.vocab_size, cfg.d_model, device=device)
        nn.init.normal_(self.tok.weight, std=0.02)
        self.pos = nn.Parameter(torch.randn(cfg.seq_len, cfg.d_model, device=device) * 0.01)
        self.drop = nn.Dropout(cfg.dropout)
        self.blocks = nn.ModuleList(TransformerBlock(cfg, hads_profile, device) for _ in range(cfg.n_layers))
        self.ln_f = LayerNorm(cfg.d_model, device=device)

    def set_hads_profile(self, profile: hp.HADSProfile) -> None:
        """Attach a (re)calibrated profile to every attention layer."""
        for blk in self.blocks:
            blk.attn.hads_profile = profile

    def forward(self, token_ids: torch.Tensor, collect_attn: bool = False
                ) -> Tuple[torch.Tensor, Optional[List[torch.Tensor]]]:
        """token_ids [B, S] -> (logits [B, S, vocab], per-layer attention weights or None)."""
        S = token_ids.shape[1]
        dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled() else torch.float32
        x = self.drop(self.tok(token_ids).to(dtype) + self.pos[:S].to(dtype))
        attn = [] if collect_attn else None
        for blk in self.blocks:
            x, w = blk(x, collect_attn)
            if collect_attn:
                attn.append(w)
        x = self.ln_f(x)
        logits = F.linear(x, self.tok.weight)    # tied to the token embedding
        return logits, attn


def cross_entropy_loss(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -1) -> torch.Tensor:
    """model/transformer.py:177-203: predict token t+1 from position t, mean over valid targets."""
    vocab = logits.shape[-1]
    flat_logits = logits[:, :-1].reshape(-1, vocab).float()
    flat_labels = labels[:, 1:].reshape(-1)
    valid = flat_labels != ignore_index
    nll = F.cross_entropy(flat_logits, flat_labels.clamp(0, vocab - 1), reduction="none")
    return (nll * valid).sum() / valid.sum().clamp(min=1)
