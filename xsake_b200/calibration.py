"""HADS calibration across ranks, and the work split of the attention path.

Reference: ``_calibrate_hads`` (training/trainer.py:79-117) runs ``n_steps`` calibration forward
passes on one device and hands their attention weights to ``build_hads_profile``
(kernels/hads/hads_pattern.py:118-166).  Here the calibration batches are split round-robin over
ranks; every rank accumulates float64 per-head entropy sums over its batches (on the GPU, with
``hads_pattern.entropy_head_sums``), the sums and row counts are summed over ranks (one small
all-reduce: the only exchange of the path), and every rank then builds the same masks on the
host.  With equal batch sizes the global mean equals the reference's mean of per-step means.

The attention itself needs no exchange: (batch, head) units are independent.  ``lpt_shard``
assigns units to ranks by longest-processing-time first when a fixed job is split over ranks.
"""

from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

from . import hads_pattern as hp


def local_batches(n_batches: int, world: int, rank: int) -> List[int]:
    """Calibration batch indices this rank processes (round-robin)."""
    return [i for i in range(n_batches) if i % world == rank]


def _dist():
    import torch.distributed as dist
    return dist if (dist.is_available() and dist.is_initialized()) else None


def _world(group=None, comm=None):
    if comm is not None:
        return comm.nranks, comm.rank
    dist = _dist()
    return (dist.get_world_size(group), dist.get_rank(group)) if dist else (1, 0)


def calibrate_sums(batch_sums: Callable[[int], tuple], n_batches: int, seq_len: int, block_size: int,
                   min_sparsity: float = 0.10, max_sparsity: float = 0.90, window_size: int = 2,
                   causal: bool = True, global_blocks: int = 0, group: Optional[object] = None, device=None,
                   comm=None) -> hp.HADSProfile:
    """Build a HADS profile from ``n_batches`` calibration batches split round-robin over the
    ranks of ``group`` (or ``comm``, or one process).  ``batch_sums(i)`` returns batch i's float64
    per-head entropy sums over its rows and the row count; the sums and counts are summed over
    ranks (one fp64 all-reduce each) and every rank builds the same masks."""
    world, rank = _world(group, comm)
    sums, rows = None, 0
    for i in local_batches(n_batches, world, rank):
        s, r = batch_sums(i)
        s = s.to(torch.float64)
        sums = s if sums is None else sums + s
        rows += int(r)
    if sums is None:
        raise ValueError("every rank needs at least one calibration batch")
    if device is not None:
        sums = sums.to(device)
    total = torch.tensor([float(rows)], dtype=torch.float64, device=sums.device)
    if comm is not None:
        sums, total = comm.allreduce_sum_f64(sums.contiguous()), comm.allreduce_sum_f64(total)
    else:
        sums = hp.allreduce_head_sums(sums, group)
        total = hp.allreduce_head_sums(total, group)
    ent = (sums / total).to(torch.float32).cpu().numpy()
    return hp.profile_from_entropies(ent, seq_len, block_size, min_sparsity, max_sparsity, window_size,
                                     causal, global_blocks)


def calibrate(batch_attn: Callable[[int], torch.Tensor], n_batches: int, seq_len: int, block_size: int,
              min_sparsity: float = 0.10, max_sparsity: float = 0.90, window_size: int = 2,
              causal: bool = True, global_blocks: int = 0,
              head_sums: Callable[[torch.Tensor], torch.Tensor] = hp.entropy_head_sums,
              group: Optional[object] = None, device=None, comm=None) -> hp.HADSProfile:
    """``calibrate_sums`` for callers that hold the attention weights: ``batch_attn(i)`` returns
    the weights [B, H, Sq, Sk] of batch i and ``head_sums`` reduces them to float64 per-head
    entropy sums.  With ``comm`` (an ``xsake_b200.comm.Comm``) the exchange runs through the
    library's NCCL entry points instead of torch.distributed."""
    def batch_sums(i):
        p = batch_attn(i)
        return head_sums(p), int(p.shape[0]) * int(p.shape[2])
    return calibrate_sums(batch_sums, n_batches, seq_len, block_size, min_sparsity, max_sparsity, window_size,
                          causal, global_blocks, group, device, comm)


def unit_costs(block_masks: np.ndarray, batch: int, causal: bool = True) -> np.ndarray:
    """Active-block count of every (batch, head) unit: the forward's work per unit."""
    m = np.asarray(block_masks, bool)
    if m.ndim == 2:
        m = m[None]
    if causal:
        m = m & np.tri(m.shape[-2], m.shape[-1], dtype=bool)
    per_head = m.reshape(m.shape[0], -1).sum(axis=1)
    return np.tile(per_head, batch)                     # unit u = b * H + h


def pair_shard(block_masks: np.ndarray, batch: int, world: int, causal: bool = True) -> List[List[int]]:
    """Units ``b * H + h`` of each rank when one job's batch x heads is split over ``world``
    ranks, for per-head masks ``[H, nq, nk]`` shared by the batch.  Such a mask lets the forward
    compute two batch units of one head per work item, so units are assigned two at a time
    ((b, b+1) of one head, a lone unit when the batch is odd), longest first by active blocks
    (heads differ ~5x in density); each rank's list is ascending."""
    m = np.asarray(block_masks, bool)
    if m.ndim != 3:
        raise ValueError(f"pair_shard needs per-head masks [H, nq, nk], got shape {m.shape}")
    heads = m.shape[0]
    costs = unit_costs(m, batch, causal)
    jobs = [[b * heads + h for b in range(b0, min(b0 + 2, batch))]
            for h in range(heads) for b0 in range(0, batch, 2)]
    out: List[List[int]] = [[] for _ in range(world)]
    for r, idx in enumerate(lpt_shard([float(sum(costs[u] for u in j)) for j in jobs], world)):
        for i in idx:
            out[r].extend(jobs[i])
    return [sorted(x) for x in out]


def lpt_shard(costs: Sequence[float], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of units to ``world`` ranks (deterministic:
    ties broken by unit index and rank index)."""
    order = sorted(range(len(costs)), key=lambda u: (-float(costs[u]), u))
    heap = [(0.0, r) for r in range(world)]
    out: List[List[int]] = [[] for _ in range(world)]
    for u in order:
        load, r = heapq.heappop(heap)
        out[r].append(u)
        heapq.heappush(heap, (load + float(costs[u]), r))
    return [sorted(x) for x in out]
