"""Multi-rank host logic on CPU with the gloo backend (world size 2): calibration batches split
over ranks, the per-head entropy sums all-reduced, identical masks on every rank, equal to the
single-process profile; and the LPT split of (batch, head) attention units.

The GPU entropy reduction is replaced here by the oracle's float64 sums so that the test needs
no GPU; it exercises the exchange and the bookkeeping around it."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import hads as oh
from oracle import rowops as orow

H, S, BS, NB = 4, 256, 64, 5


def _batch(i):
    rng = np.random.default_rng(100 + i)
    q = rng.standard_normal((2, H, S, 16)).astype(np.float32) * np.linspace(0.5, 3, H)[None, :, None, None]
    k = rng.standard_normal((2, H, S, 16)).astype(np.float32)
    return torch.from_numpy(orow.softmax(np.einsum("bhqd,bhkd->bhqk", q, k) / 4.0).astype(np.float32))


def _sums(p):
    return torch.from_numpy(oh.entropy_head_sums(p.numpy()))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from xsake_b200 import calibration as cal
        prof = cal.calibrate(_batch, NB, S, BS, causal=True, global_blocks=1, head_sums=_sums)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ent=prof.head_entropies, rho=prof.head_sparsity,
                 mask=prof.block_masks, mine=np.array(cal.local_batches(NB, world, rank)))
    finally:
        dist.destroy_process_group()


def test_two_rank_calibration_matches_single_process(tmp_path):
    from xsake_b200 import calibration as cal
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0, r1 = (np.load(tmp_path / f"r{r}.npz") for r in range(2))
    assert sorted(list(r0["mine"]) + list(r1["mine"])) == list(range(NB))
    np.testing.assert_array_equal(r0["mask"], r1["mask"])
    np.testing.assert_array_equal(r0["ent"], r1["ent"])
    single = cal.calibrate(_batch, NB, S, BS, causal=True, global_blocks=1, head_sums=_sums)
    np.testing.assert_allclose(r0["ent"], single.head_entropies, rtol=1e-6)
    np.testing.assert_array_equal(r0["mask"], single.block_masks)
    # the reference's own path: mean of per-batch entropies, then the map and the masks
    ref = oh.build_hads_profile([_batch(i).numpy() for i in range(NB)], S, BS, causal=True, global_blocks=1)
    np.testing.assert_allclose(r0["ent"], ref.head_entropies, rtol=1e-5)
    np.testing.assert_array_equal(r0["mask"], ref.block_masks)


def test_lpt_shard_balances_hads_units():
    from xsake_b200 import calibration as cal
    masks = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1).block_masks
    costs = cal.unit_costs(masks, batch=4)
    assert costs.shape == (48,)
    for world in (1, 2, 4, 8):
        parts = cal.lpt_shard(costs, world)
        assert sorted(u for p in parts for u in p) == list(range(48))
        loads = [costs[p].sum() for p in parts]
        assert max(loads) <= 1.05 * costs.sum() / world + costs.max()
        assert parts == cal.lpt_shard(costs, world)            # deterministic


def test_pair_shard_keeps_unit_pairs_and_balances():
    from xsake_b200 import calibration as cal
    masks = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1).block_masks
    costs = cal.unit_costs(masks, batch=4)
    for world in (1, 2, 4, 8):
        parts = cal.pair_shard(masks, 4, world)
        assert sorted(u for p in parts for u in p) == list(range(48))
        for p in parts:                     # batch units (0, 1) and (2, 3) of a head stay together
            for u in p:
                b, h = divmod(u, 12)
                assert (b ^ 1) * 12 + h in p
        loads = [costs[p].sum() for p in parts]
        assert max(loads) <= 1.1 * costs.sum() / world
    odd = cal.pair_shard(masks, 3, 2)       # odd batch: the last batch unit of a head runs alone
    assert sorted(u for p in odd for u in p) == list(range(36))
