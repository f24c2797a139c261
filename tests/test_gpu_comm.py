"""The calibration exchange through the library's NCCL entry points (xsake_comm_*).

One GPU: a single-rank communicator (the all-reduce is the identity), argument errors, and
calibration through the communicator equal to calibration without it.  Two GPUs (skipped when
fewer are visible): two processes sum per-rank vectors and build identical masks."""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import hads as oh  # noqa: E402
from oracle import rowops as orow  # noqa: E402

H, S = 4, 256


def _batch(i):
    rng = np.random.default_rng(300 + i)
    q = rng.standard_normal((2, H, S, 16)).astype(np.float32) * np.linspace(0.5, 3, H)[None, :, None, None]
    k = rng.standard_normal((2, H, S, 16)).astype(np.float32)
    return torch.from_numpy(orow.softmax(np.einsum("bhqd,bhkd->bhqk", q, k) / 4.0).astype(np.float32)).cuda()


def test_single_rank_allreduce_is_identity():
    from xsake_b200 import comm
    with comm.Comm(comm.unique_id(), 1, 0, device=0) as c:
        t = torch.arange(12, dtype=torch.float64, device="cuda") * 0.5
        ref = t.clone()
        c.allreduce_sum_f64(t)
        torch.cuda.synchronize()
        assert torch.equal(t, ref)


def test_comm_argument_errors():
    from xsake_b200 import comm
    with pytest.raises(ValueError):
        comm.Comm(b"\0" * 127, 1, 0)
    with comm.Comm(comm.unique_id(), 1, 0) as c:
        with pytest.raises(ValueError):
            c.allreduce_sum_f64(torch.zeros(4, device="cuda"))           # float32
        with pytest.raises(ValueError):
            c.allreduce_sum_f64(torch.zeros(4, dtype=torch.float64))     # host tensor


def test_calibration_through_comm_matches_plain():
    from xsake_b200 import calibration as cal, comm
    plain = cal.calibrate(_batch, 3, S, 64, causal=True, global_blocks=1)
    with comm.Comm(comm.unique_id(), 1, 0) as c:
        via = cal.calibrate(_batch, 3, S, 64, causal=True, global_blocks=1, comm=c)
    np.testing.assert_array_equal(plain.head_entropies, via.head_entropies)
    np.testing.assert_array_equal(plain.block_masks, via.block_masks)
    ref = oh.build_hads_profile([_batch(i).cpu().numpy() for i in range(3)], S, 64, causal=True, global_blocks=1)
    np.testing.assert_allclose(via.head_entropies, ref.head_entropies, rtol=1e-5)
    np.testing.assert_array_equal(via.block_masks, ref.block_masks)


def _two_rank_worker(rank, uid, out_dir):
    import torch as T
    from xsake_b200 import calibration as cal, comm
    T.cuda.set_device(rank)
    with comm.Comm(uid, 2, rank) as c:
        t = T.full((12,), float(rank + 1), dtype=T.float64, device="cuda")
        c.allreduce_sum_f64(t)
        prof = cal.calibrate(_batch, 5, S, 64, causal=True, global_blocks=1, comm=c)
        T.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), t=t.cpu().numpy(), mask=prof.block_masks,
                 ent=prof.head_entropies)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_calibration_exchange(tmp_path):
    import torch.multiprocessing as mp
    from xsake_b200 import comm
    uid = comm.unique_id()
    mp.start_processes(_two_rank_worker, args=(uid, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0, r1 = (np.load(tmp_path / f"r{r}.npz") for r in range(2))
    np.testing.assert_array_equal(r0["t"], np.full(12, 3.0))
    np.testing.assert_array_equal(r0["mask"], r1["mask"])
    ref = oh.build_hads_profile([_batch(i).cpu().numpy() for i in range(5)], S, 64, causal=True, global_blocks=1)
    np.testing.assert_allclose(r0["ent"], ref.head_entropies, rtol=1e-5)
    np.testing.assert_array_equal(r0["mask"], ref.block_masks)


def test_rank_that_never_joins_times_out():
    """A two-rank communicator whose second rank never calls init: rank 0's init returns
    XSAKE_ETIMEOUT within its deadline (bootstrap only, no collective in flight), the
    communicator is aborted, and the process goes on to use a new communicator."""
    import time
    from xsake_b200 import _lib, comm
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    uid = comm.unique_id()
    t0 = time.monotonic()
    with pytest.raises(_lib.XsakeError) as e:
        comm.Comm(uid, 2, 0, device=0, timeout_s=2.0)
    assert e.value.code == _lib.XSAKE_ETIMEOUT
    assert time.monotonic() - t0 < 30.0
    with comm.Comm(comm.unique_id(), 1, 0, device=0, timeout_s=30.0) as c:
        t = torch.ones(12, dtype=torch.float64, device="cuda")
        c.allreduce_sum_f64(t)
        c.wait(10.0)
        assert torch.equal(t, torch.ones_like(t))
