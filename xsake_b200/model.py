"""GPT-style transformer around the HADS attention layer: the model the reference trains.

PyTorch counterpart of XSAKETransformer (model/transformer.py:71-172), TransformerBlock
(:74-104), MLP (:33-46), the LayerNorm wrapper (:51-66), TransformerEmbedding
(model/embedding.py:63-90) and cross_entropy_loss (model/transformer.py:177-203):
token + learned position embeddings, pre-norm blocks (fused LayerNorm with fp32 statistics,
XSAKE attention, GELU MLP), final LayerNorm, logits tied to the token embedding.

Attention and LayerNorm run on this library's kernels; the dense projections, embeddings and the
optimizer are PyTorch.  The logits GEMM runs in the activation dtype with fp32 loss arithmetic
(the reference computes the logits GEMM itself in fp32).
"""

from __future__ import annotations

import math
import weakref
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
from torch import nn
from torch.nn import functional as F

from . import _device as dev
from . import _lib
from . import hads_pattern as hp
from .attention import XSAKEAttention
from .fused_layernorm import fused_layernorm


@dataclass
class HADSConfig:
    """model/config.py:8-15 (HADS calibration parameters)."""
    min_sparsity: float = 0.10
    max_sparsity: float = 0.90
    calibration_steps: int = 10
    block_size: int = 128
    window_size: int = 2
    entropy_temperature: float = 1.0


@dataclass
class KernelConfig:
    """model/config.py:18-31 (attention kernel parameters)."""
    block_size_q: int = 128
    block_size_kv: int = 128
    sparsity_type: str = "hads"
    use_pallas: bool = True
    hads: HADSConfig = field(default_factory=HADSConfig)


@dataclass
class ModelConfig:
    """The fields of model/config.py:34-58 the model reads (defaults: GPT-2 small, the
    reference's).  The kernel parameters can be given either as the reference's nested
    ``kernel=KernelConfig(...)`` or as the flat fields below; a ``kernel`` overrides them."""
    vocab_size: int = 50_257
    seq_len: int = 1_024
    n_layers: int = 12
    n_heads: int = 12
    d_model: int = 768
    d_ff: int = 3_072
    dropout: float = 0.0
    bias: bool = False
    dtype: str = "bfloat16"
    kernel: Optional[KernelConfig] = None
    block_size: int = 128
    sparsity_type: str = "hads"
    min_sparsity: float = 0.10
    max_sparsity: float = 0.90
    window_size: int = 2
    calibration_steps: int = 10

    def __post_init__(self):
        k = self.kernel
        if k is not None:
            self.block_size, self.sparsity_type = k.block_size_q, k.sparsity_type
            self.min_sparsity, self.max_sparsity = k.hads.min_sparsity, k.hads.max_sparsity
            self.window_size, self.calibration_steps = k.hads.window_size, k.hads.calibration_steps

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads


class LayerNorm(nn.Module):
    """model/transformer.py:51-66: fp32 statistics and parameters, result in x's dtype.

    The reference casts x to fp32, normalises and casts back.  The kernel reads x in its own
    dtype and does the same fp32 arithmetic on the upcast values, so the casts (two extra passes
    over the activations each way) are left out."""

    def __init__(self, d_model: int, eps: float = 1e-5, device=None):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(d_model, device=device))
        self.beta = nn.Parameter(torch.zeros(d_model, device=device))
        self.eps = eps

    def forward(self, x):
        return fused_layernorm(x, self.gamma, self.beta, eps=self.eps)


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
        self.attn = XSAKEAttention(cfg, hads_profile, dtype=torch.float32, device=device)
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
        """Attach a (re)calibrated profile to every attention layer (the reference rebuilds the
        model with the new profile, training/trainer.py:191-200)."""
        for blk in self.blocks:
            blk.attn.hads_profile = profile

    @torch.no_grad()
    def layer0_qk(self, token_ids: torch.Tensor):
        """The first attention layer's q and k for ``token_ids`` ([B, H, S, D] views of the
        projections), with its block mask and block size: what calibration reduces (the
        reference takes the first layer's weights, training/trainer.py:97-100).  Only the
        embedding, the first LayerNorm and two projections run."""
        S = token_ids.shape[1]
        dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled() else torch.float32
        x = self.tok(token_ids).to(dtype) + self.pos[:S].to(dtype)
        blk = self.blocks[0]
        h = blk.ln1(x)
        att = blk.attn
        B = token_ids.shape[0]
        q = att._heads(att.q_proj(h), B, S)
        k = att._heads(att.k_proj(h), B, S)
        mask, bs = att.get_block_mask(S)
        return q, k, mask, bs, float(att.d_head ** -0.5)

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
        # Logits tied to the token embedding.  The GEMM runs over the vocabulary padded to a
        # multiple of 64 rows (zeros) and the logits are the first vocab_size columns: with
        # 50,257 columns the rows of the logits and of their gradient are not 16-byte aligned,
        # and cuBLAS then falls back to kernels several times slower for all three GEMMs.
        w = self.tok.weight.to(x.dtype)
        vocab = w.shape[0]
        pad = -vocab % 64
        if pad:
            w = F.pad(w, (0, 0, 0, pad))
        logits = F.linear(x, w)
        if pad:
            logits = _VocabView.apply(logits, vocab)
        return logits, attn


# Gradient buffers written by _CrossEntropy.backward over whole padded rows (zeros past the
# vocabulary), keyed by data pointer until _VocabView.backward takes them (weakly held: an
# entry disappears with its buffer).
_PADDED_GRADS: "weakref.WeakValueDictionary" = weakref.WeakValueDictionary()


class _VocabView(torch.autograd.Function):
    """logits[..., :vocab] of the padded logits.  Its backward hands a gradient that already
    spans the padded rows (the fused cross entropy's) to the GEMM as it is, instead of a zero
    fill of the padded shape plus a strided copy (two passes over ~3 GB per step)."""

    @staticmethod
    def forward(ctx, padded, vocab):
        ctx.padded_shape = padded.shape
        return padded[..., :vocab]

    @staticmethod
    def backward(ctx, g):
        base = g._base
        if base is not None and _PADDED_GRADS.pop(base.data_ptr(), None) is base and \
                g.data_ptr() == base.data_ptr() and base.numel() == math.prod(ctx.padded_shape) and \
                g.stride()[-2] == ctx.padded_shape[-1]:
            return base.view(ctx.padded_shape), None
        out = g.new_zeros(ctx.padded_shape)
        out[..., :g.shape[-1]] = g
        return out, None


class _CrossEntropy(torch.autograd.Function):
    """Mean cross entropy over rows of logits [R, V] (unit column stride, any row stride) on the
    library's fused kernels: one pass over the logits for lse and nll, one pass that writes
    coef * (softmax - onehot) straight into the gradient; no fp32 copy of the logits is made."""

    @staticmethod
    def forward(ctx, logits, targets, ignore_index):
        rows, vocab = logits.shape
        lse = torch.empty(rows, dtype=torch.float32, device=logits.device)
        nll = torch.empty_like(lse)
        _lib.check(_lib.load().xsake_xent_fwd(
            dev.xsake_dtype(logits), rows, vocab, logits.stride(0), logits.data_ptr(), targets.data_ptr(),
            int(ignore_index), lse.data_ptr(), nll.data_ptr(), dev.stream_ptr()))
        n_valid = (targets != ignore_index).sum().clamp(min=1).float()
        ctx.save_for_backward(logits, targets, lse, n_valid)
        ctx.ignore_index = int(ignore_index)
        return nll.sum() / n_valid

    @staticmethod
    def backward(ctx, grad_out):
        logits, targets, lse, n_valid = ctx.saved_tensors
        rows, vocab = logits.shape
        ld = logits.stride(0)
        coef = (grad_out.float() / n_valid).reshape(1).contiguous()
        buf = torch.empty((rows, ld), dtype=logits.dtype, device=logits.device)
        _lib.check(_lib.load().xsake_xent_bwd(
            dev.xsake_dtype(logits), rows, vocab, ld, logits.data_ptr(), targets.data_ptr(), ctx.ignore_index,
            lse.data_ptr(), coef.data_ptr(), buf.data_ptr(), dev.stream_ptr()))
        if ld > vocab:
            _PADDED_GRADS[buf.data_ptr()] = buf
        return buf[:, :vocab], None, None


def _fused_rows(logits: torch.Tensor):
    """[B, S, V] logits as a [B*S, V] view with one row stride, or None."""
    if not logits.is_cuda or logits.dtype not in (torch.float32, torch.bfloat16) or logits.dim() != 3:
        return None
    if logits.stride(-1) != 1 or logits.stride(0) != logits.shape[1] * logits.stride(1):
        return None
    return logits.view(-1, logits.shape[-1])


def cross_entropy_loss(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -1) -> torch.Tensor:
    """model/transformer.py:177-203: predict token t+1 from position t, mean over valid targets.

    CUDA logits go through the library's fused kernels (fp32 arithmetic on the logits' own
    dtype): every position is a row and the last one's target is ignore_index, which is the
    reference's [:, :-1] / [:, 1:] shift without slicing the logits."""
    rows = _fused_rows(logits)
    if rows is not None:
        targets = torch.full_like(labels, ignore_index, dtype=torch.int64)
        targets[:, :-1] = labels[:, 1:]
        return _CrossEntropy.apply(rows, targets.reshape(-1).contiguous(), ignore_index)
    vocab = logits.shape[-1]
    flat_logits = logits[:, :-1].reshape(-1, vocab).float()
    flat_labels = labels[:, 1:].reshape(-1)
    valid = flat_labels != ignore_index
    nll = F.cross_entropy(flat_logits, flat_labels.clamp(0, vocab - 1), reduction="none")
    return (nll * valid).sum() / valid.sum().clamp(min=1)
