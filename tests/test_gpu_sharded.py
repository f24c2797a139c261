"""A job's batch x heads split over ranks: plans restricted to a rank's (b, h) units, and the
forward's split pieces (a long kv walk cut into pieces whose partials the last piece merges).

Each rank of a sharded job compiles a plan of its own units; the attention kernels then write
only those units' rows.  The ranks are emulated one after another on one GPU.  Tolerances as in
test_gpu_attention.py: bf16 max|out - ref| <= 2e-2 * max|ref| against the float64 oracle,
fp32 <= 1e-5 * max(1, max|ref|); unsplit work is bit-identical to the full plan's.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402
from oracle import inputs as oi  # noqa: E402

BF16_TOL = 2e-2
F32_TOL = 1e-5


def _sa():
    from xsake_b200 import sparse_attention as sa
    return sa


def _cal():
    from xsake_b200 import calibration as cal
    return cal


def _bf16(x):
    return oi.to_bf16(x).astype(np.float32)


def _err(got, ref):
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)))


@pytest.mark.parametrize("world", [2, 8])
def test_config3_sharded_forward(world):
    """Config 3 (bf16 B=4 H=12 S=4096 D=64, HADS masks) split over `world` ranks: every rank's
    units match the oracle on sampled units, other units' rows are left untouched, and at 8 ranks
    the plans split long kv walks into pieces."""
    sa, cal = _sa(), _cal()
    B, H, S = 4, 12, 4096
    masks = oh.dummy_hads_profile(H, S, 64, causal=True, global_blocks=1).block_masks
    q, k, v = (_bf16(x) for x in oi.qkv(B, H, S, 64, seed=oi.SEED_BASE + 3))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    full, full_lse = sa.attention_forward(tq, tk, tv, masks, 64, None, True)
    shards = cal.pair_shard(masks, B, world)
    assert sorted(u for s in shards for u in s) == list(range(B * H))
    splits = 0
    for rank, units in enumerate(shards):
        cm = sa.compile_block_mask(masks, B, H, S, 64, True, units=units)
        st = cm.stats()
        assert st["selected_units"] == len(units)
        assert st["active_blocks"] == int(cal.unit_costs(masks, B)[units].sum())
        splits += st["split_items"]
        o = torch.full_like(tq, float("nan"))
        lse = torch.full((B, H, S), float("nan"), device="cuda")
        from xsake_b200 import _lib
        import ctypes as C
        d = sa._desc(tq, tk, tv, o, cm, None)
        n = C.c_size_t(0)
        _lib.check(_lib.load().xsake_attn_fwd_workspace_size(C.byref(d), C.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        for _ in range(2):   # a second call reuses the workspace (counters reset per call)
            _lib.check(_lib.load().xsake_attn_fwd(C.byref(d), cm.plan.data_ptr(), tq.data_ptr(), tk.data_ptr(),
                                                  tv.data_ptr(), o.data_ptr(), lse.data_ptr(), ws.data_ptr(),
                                                  ws.numel(), sa.dev.stream_ptr()))
        torch.cuda.synchronize()
        mine = set(units)
        for u in range(B * H):
            b, h = divmod(u, H)
            if u in mine:
                assert torch.isfinite(o[b, h].float()).all() and torch.isfinite(lse[b, h]).all()
                err = (o[b, h].float() - full[b, h].float()).abs().max().item()
                assert err <= BF16_TOL * full[b, h].float().abs().max().item(), (rank, u, err)
                assert (lse[b, h] - full_lse[b, h]).abs().max().item() <= 2e-2
            else:
                assert torch.isnan(o[b, h].float()).all() and torch.isnan(lse[b, h]).all(), (rank, u)
        # the oracle on the rank's first and last unit
        for u in (units[0], units[-1]):
            b, h = divmod(u, H)
            ref, _, lref = oa.sparse_attention_reference(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                                         v[b:b + 1, h:h + 1], masks[h:h + 1], 64, causal=True,
                                                         return_weights=False, return_lse=True)
            got = o[b, h].float().cpu().numpy()
            assert _err(got, ref[0, 0]) <= BF16_TOL * np.abs(ref).max(), (rank, u)
            np.testing.assert_allclose(lse[b, h].cpu().numpy(), lref[0, 0], atol=2e-2)
    if world == 8:
        assert splits > 0, "8 ranks of config 3 should split the longest kv walks"


@pytest.mark.parametrize("B,global_blocks", [(1, 1), (2, 1), (3, 0)])
def test_forced_split_pieces_match_oracle(B, global_blocks):
    """A plan that assumes many workers cuts every kv walk longer than 4 chunks into pieces;
    the merged result matches the oracle, including fully masked rows and a lone unit (B=3)
    and both pairings (B=1: query-chunk pairs; B>=2: unit pairs)."""
    sa = _sa()
    H, S = 3, 1024
    m = oh.dummy_hads_profile(H, S, 64, causal=True, global_blocks=global_blocks).block_masks.copy()
    m[1, 5, :] = False           # a q-block that attends nothing
    q, k, v = (_bf16(np.random.default_rng(200 + i).standard_normal((B, H, S, 64)).astype(np.float32))
               for i in range(3))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    cm = sa.compile_block_mask(m, B, H, S, 64, True, workers=100000)
    st = cm.stats()
    assert st["split_items"] > 0 and st["split_cap"] == 4
    out, lse = sa.attention_forward(tq, tk, tv, cm, 64, None, True)
    ref, _, lref = oa.sparse_attention_reference(q, k, v, m, 64, causal=True, return_weights=False,
                                                 return_lse=True)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    assert _err(o, ref) <= BF16_TOL * np.abs(ref).max()
    live = lref > -1e30
    np.testing.assert_allclose(lse.cpu().numpy()[live], lref[live], atol=2e-2)
    np.testing.assert_array_equal(lse.cpu().numpy()[~live], lref[~live])
    out2, lse2 = sa.attention_forward(tq, tk, tv, cm, 64, None, True)
    assert torch.equal(out, out2) and torch.equal(lse, lse2)      # merge order is fixed


def test_sharded_backward_writes_only_its_units():
    """The backward with a unit-restricted plan: the rank's gradients are bit-identical to the
    full plan's (no split in the backward) and other units' rows are untouched."""
    sa, cal = _sa(), _cal()
    B, H, S = 2, 4, 1024
    masks = oh.dummy_hads_profile(H, S, 64, causal=True, global_blocks=1).block_masks
    q, k, v, do = (torch.randn(B, H, S, 64, device="cuda").to(torch.bfloat16) for _ in range(4))
    o, lse = sa.attention_forward(q, k, v, masks, 64, None, True)
    g_full = sa.attention_backward(q, k, v, o, lse, do, masks, 64, None, True)
    for units in cal.pair_shard(masks, B, 2):
        cm = sa.compile_block_mask(masks, B, H, S, 64, True, units=units)
        import ctypes as C
        from xsake_b200 import _lib
        grads = [torch.full_like(q, float("nan")) for _ in range(3)]
        d = sa._desc(q, k, v, grads[0], cm, None)
        n = C.c_size_t(0)
        _lib.check(_lib.load().xsake_attn_bwd_workspace_size(C.byref(d), C.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        _lib.check(_lib.load().xsake_attn_bwd(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(),
                                              v.data_ptr(), o.data_ptr(), lse.data_ptr(), do.data_ptr(),
                                              grads[0].data_ptr(), grads[1].data_ptr(), grads[2].data_ptr(),
                                              ws.data_ptr(), ws.numel(), sa.dev.stream_ptr()))
        torch.cuda.synchronize()
        for g, gf in zip(grads, g_full):
            for u in range(B * H):
                b, h = divmod(u, H)
                if u in units:
                    assert torch.equal(g[b, h], gf[b, h]), u
                else:
                    assert torch.isnan(g[b, h].float()).all(), u


def test_sharded_cuda_core_path():
    """fp32 (the CUDA-core kernels) with a unit-restricted plan."""
    sa = _sa()
    B, H, S = 2, 3, 256
    m = oh.dummy_hads_profile(H, S, 64, causal=True).block_masks
    q, k, v = (np.random.default_rng(300 + i).standard_normal((B, H, S, 64)).astype(np.float32) for i in range(3))
    tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    units = [0, 4, 5]
    cm = sa.compile_block_mask(m, B, H, S, 64, True, units=units)
    o = torch.full_like(tq, float("nan"))
    lse = torch.full((B, H, S), float("nan"), device="cuda")
    import ctypes as C
    from xsake_b200 import _lib
    d = sa._desc(tq, tk, tv, o, cm, None)
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.load().xsake_attn_fwd(C.byref(d), cm.plan.data_ptr(), tq.data_ptr(), tk.data_ptr(),
                                          tv.data_ptr(), o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256,
                                          sa.dev.stream_ptr()))
    ref, _ = oa.sparse_attention_reference(q, k, v, m, 64, causal=True, return_weights=False)
    got = o.cpu().numpy()
    for u in range(B * H):
        b, h = divmod(u, H)
        if u in units:
            assert _err(got[b, h], ref[b, h]) <= F32_TOL * max(1.0, np.abs(ref[b, h]).max())
        else:
            assert np.isnan(got[b, h]).all()


def test_unit_list_is_validated():
    sa = _sa()
    m = oh.dummy_hads_profile(2, 256, 64, causal=True).block_masks
    with pytest.raises(ValueError):
        sa.compile_block_mask(m, 1, 2, 256, 64, True, units=[2])
    with pytest.raises(ValueError):
        sa.compile_block_mask(m, 1, 2, 256, 64, True, units=[])


def test_shard_api_with_host_buffers():
    """sparse_attention_shard on pinned host tensors copies only the rank's units' slices and
    returns them equal to the full job's output; other rows of `out` are left as they were."""
    sa, cal = _sa(), _cal()
    B, H, S = 2, 4, 512
    masks = oh.dummy_hads_profile(H, S, 64, causal=True, global_blocks=1).block_masks
    q, k, v = (torch.randn(B, H, S, 64).to(torch.bfloat16).pin_memory() for _ in range(3))
    full, _ = sa.attention_forward(q.cuda(), k.cuda(), v.cuda(), masks, 64, None, True)
    full = full.cpu()
    for units in cal.pair_shard(masks, B, 2):
        out = torch.full((B, H, S, 64), float("nan"), dtype=torch.bfloat16).pin_memory()
        got = sa.sparse_attention_shard(q, k, v, masks, units, 64, None, True, out=out)
        torch.cuda.synchronize()
        assert got is out
        for u in range(B * H):
            b, h = divmod(u, H)
            if u in units:
                assert torch.equal(out[b, h], full[b, h]), u
            else:
                assert torch.isnan(out[b, h].float()).all(), u
