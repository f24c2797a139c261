"""HADS calibration of a model from its own activations, and the recalibration step.

Reference: training/trainer.py
  * ``_calibrate_hads(model, params, data_iter, model_config, n_steps)``        :79-117
  * recalibration every ``hads_recalibrate_every`` steps, then a model with the
    new profile                                                                  :191-200

The reference collects the first attention layer's weights over ``n_steps`` batches (on GPU its
Pallas path returns none, so it silently falls back to the dummy profile) and hands them to
``build_hads_profile``.  Here the same entropies come from the first layer's q and k through the
fused masked-entropy kernel (``xsake_attn_entropy``): no [B, H, S, S] weights are formed.  The
calibration batches are split round-robin over the ranks of a process group (or an
``xsake_b200.comm.Comm``) and the per-head float64 sums are all-reduced, so every rank builds the
same masks; with equal batch sizes the mean over all rows equals the reference's mean of
per-step means.
"""

from __future__ import annotations

from typing import Iterator, Optional

import torch

from . import calibration as cal
from . import hads_pattern as hp


def _ids(batch):
    return batch["input_ids"] if isinstance(batch, dict) else batch


def calibrate_hads(model, data_iter: Iterator, model_config=None, n_steps: Optional[int] = None,
                   global_blocks: int = 0, group=None, comm=None) -> hp.HADSProfile:
    """A fresh HADS profile from ``n_steps`` calibration batches (training/trainer.py:79-117).

    ``model``: an ``XSAKETransformer`` (or a DistributedDataParallel wrapping one).  Each rank
    draws its share of the batches (steps i with i % world == rank) from its own ``data_iter``
    (dicts with ``input_ids`` or token-id tensors [B, S]).  ``n_steps`` defaults to the config's
    calibration_steps; with no steps the uncalibrated (dummy) profile is returned, as the
    reference does when it collects no weights."""
    net = getattr(model, "module", model)
    cfg = model_config if model_config is not None else net.cfg
    n_steps = getattr(cfg, "calibration_steps", 10) if n_steps is None else int(n_steps)
    attn0 = net.blocks[0].attn
    if n_steps <= 0:
        return hp.dummy_hads_profile(cfg.n_heads, cfg.seq_len, attn0.block_size, attn0.min_sparsity,
                                     attn0.max_sparsity, attn0.window_size, causal=True)
    device = next(net.parameters()).device
    bf16 = getattr(cfg, "dtype", "bfloat16") == "bfloat16"
    seq = {}

    def batch_sums(i):
        ids = _ids(next(data_iter)).to(device)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
            q, k, mask, bs, scale = net.layer0_qk(ids)
        seq["S"], seq["bs"] = ids.shape[1], bs
        return hp.entropy_head_sums_attention(q, k, mask, bs, scale, causal=True), ids.shape[0] * ids.shape[1]

    was_training = net.training
    net.eval()
    try:
        return cal.calibrate_sums(batch_sums, n_steps, cfg.seq_len, attn0.block_size, attn0.min_sparsity,
                                  attn0.max_sparsity, attn0.window_size, causal=True, global_blocks=global_blocks,
                                  group=group, comm=comm)
    finally:
        net.train(was_training)


def maybe_recalibrate(step: int, every: int, model, data_iter: Iterator, model_config=None,
                      **kwargs) -> Optional[hp.HADSProfile]:
    """training/trainer.py:191-200: at a step > 0 that is a multiple of ``every``, calibrate and
    attach the new profile to every attention layer; returns it (None on other steps).  Every
    rank must call this at the same steps (the calibration exchange is a collective)."""
    if every <= 0 or step <= 0 or step % every:
        return None
    prof = calibrate_hads(model, data_iter, model_config, **kwargs)
    getattr(model, "module", model).set_hads_profile(prof)
    return prof
