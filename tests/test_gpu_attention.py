"""GPU parity of the attention path against the NumPy oracle (float64 on the same inputs).

Tolerances (written per test): fp32 max|out - ref| <= 1e-5 * max(1, max|ref|);
bf16 <= 2e-2 * max|ref| (inputs rounded to bf16 before the oracle sees them).
"""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402
from oracle import inputs as oi  # noqa: E402

G = os.path.join(os.path.dirname(__file__), "golden")
F32_TOL = 1e-5
BF16_TOL = 2e-2


def _sa():
    from xsake_b200 import sparse_attention as sa
    return sa


def _bf16_round(x):
    return oi.to_bf16(x).astype(np.float32)


def _err(got, ref):
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)))


def _rand(shape, seed, dtype=np.float32):
    return np.random.default_rng(seed).standard_normal(shape).astype(dtype)


@pytest.mark.parametrize("name,causal", [("hads_c1", True), ("hads_c0", False), ("bigbird32_c0", False),
                                         ("mask4d_c1", True), ("emptyrow_c1", True), ("dense16_c1", True)])
def test_fp32_matches_golden_reference(name, causal):
    z = np.load(os.path.join(G, "attention.npz"))
    sa = _sa()
    out, _ = sa.sparse_attention(z["q"], z["k"], z["v"], z[f"{name}_mask"], block_size=int(z[f"{name}_bs"]),
                                 causal=causal)
    ref = z[f"{name}_out"].astype(np.float64)
    assert _err(out, ref) <= F32_TOL * max(1.0, np.abs(ref).max())


def test_fp32_config0_calibrated_mask():
    """Config 0: fp32 B=1 H=12 S=1024 D=64, 64x64 blocks, calibrated HADS mask
    (rho in [0.1, 0.9], w=2, causal, global block 0)."""
    sa = _sa()
    from xsake_b200 import hads_pattern as hp
    q, k, v = oi.qkv(1, 12, 1024, 64, seed=oi.SEED_BASE + 0)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k) / 8.0
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ent = oh.compute_attention_entropy(p).astype(np.float32)
    prof = hp.profile_from_entropies(ent, 1024, 64, causal=True, global_blocks=1)
    ref_prof = oh.profile_from_entropies(ent, 1024, 64, causal=True, global_blocks=1)
    np.testing.assert_array_equal(prof.block_masks, ref_prof.block_masks)
    out, _ = sa.sparse_attention(q, k, v, prof.block_masks, block_size=64, causal=True)
    ref, _, lse_ref = oa.sparse_attention_reference(q, k, v, prof.block_masks, 64, causal=True,
                                                    return_weights=False, return_lse=True)
    assert _err(out, ref) <= F32_TOL * max(1.0, np.abs(ref).max())
    o2, lse = sa.attention_forward(q, k, v, prof.block_masks, 64, None, True)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, rtol=1e-5, atol=1e-5)


def _bf16_case(B, H, S, D, bs, causal, mask, seed, layout="bhsd", scale=None):
    sa = _sa()
    q, k, v = (_bf16_round(_rand((B, H, S, D), seed + i)) for i in range(3))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    if layout == "bshd":
        tq, tk, tv = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (tq, tk, tv))
    out, lse = sa.attention_forward(tq, tk, tv, mask, bs, scale, causal)
    ref, _, lse_ref = oa.sparse_attention_reference(q, k, v, mask, bs, scale=scale, causal=causal,
                                                    return_weights=False, return_lse=True)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    assert _err(o, ref) <= BF16_TOL * np.abs(ref).max(), _err(o, ref)
    live = lse_ref > -1e30
    np.testing.assert_allclose(lse.cpu().numpy()[live], lse_ref[live], rtol=0, atol=2e-2)
    return out


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("global_blocks", [0, 1])
def test_bf16_tensor_core_hads(causal, global_blocks):
    prof = oh.dummy_hads_profile(4, 512, 64, causal=causal, global_blocks=global_blocks)
    _bf16_case(2, 4, 512, 64, 64, causal, prof.block_masks, seed=10)


def test_bf16_block128_and_shared_mask():
    prof = oh.dummy_hads_profile(3, 1024, 128, causal=True)
    _bf16_case(1, 3, 1024, 64, 128, True, prof.block_masks, seed=20)
    shared = oh.build_head_mask(0.5, 8, 1, 3, causal=True)
    _bf16_case(2, 2, 512, 64, 64, True, shared, seed=21)


def test_bf16_odd_chunk_count_and_empty_rows():
    # S = 320 -> five 64-row chunks: the last 128-row tile is half outside the sequence.
    m = oh.dummy_hads_profile(2, 320, 64, causal=True).block_masks.copy()
    m[1, 2, :] = False                      # q-block 2 of head 1 attends nothing
    m[0, 4, :4] = False                     # only the diagonal block left
    _bf16_case(1, 2, 320, 64, 64, True, m, seed=30)


def test_bf16_paired_units_odd_count_and_empty_rows():
    # Masks shared over the batch pair (b, h) units of one head; with three batches the third
    # runs alone.  S = 320 gives an odd chunk count; one q-block attends nothing.
    m = oh.dummy_hads_profile(2, 320, 64, causal=True).block_masks.copy()
    m[1, 2, :] = False
    m[0, 4, :4] = False
    _bf16_case(3, 2, 320, 64, 64, True, m, seed=31)
    _bf16_case(3, 2, 320, 64, 64, False, m, seed=32)


def test_bf16_mask_shared_over_heads():
    # A [B, 1, nq, nk] mask: one mask per batch, shared by the heads (units paired over heads,
    # three heads so one runs alone).
    m = np.stack([oh.build_head_mask(0.6, 8, 1, 5 + b, causal=True) for b in range(2)])[:, None]
    _bf16_case(2, 3, 512, 64, 64, True, m, seed=33)


def test_bf16_mask_per_unit():
    # A mask per (b, h) unit leaves nothing to pair: the query-chunk-pair kernel runs.
    m = np.stack([oh.dummy_hads_profile(3, 512, 64, causal=True, global_blocks=b).block_masks
                  for b in range(2)])
    _bf16_case(2, 3, 512, 64, 64, True, m, seed=34)
    _bf16_case(2, 3, 512, 64, 64, False, m, seed=35)


def test_bf16_dense_mask_several_units():
    # A dense causal mask leaves (almost) nothing masked in query-chunk pairs: the plan keeps the
    # query-chunk pairing even with several units sharing the mask.
    _bf16_case(2, 2, 512, 64, 64, True, np.ones((8, 8), bool), seed=36)


def test_forward_pairing_follows_the_mask():
    # Unit pairing for HADS masks shared by 4 units, query-chunk pairing for one unit per mask
    # and for a dense causal mask, at block 64 and block 128 (the choice counts useful 64-row
    # halves, whatever the block size).
    sa = _sa()
    hads = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1).block_masks
    cases = [(hads, 4, 64, "unit"), (hads, 1, 64, "query_chunk"), (np.ones((64, 64), bool), 4, 64, "query_chunk"),
             (np.ones((32, 32), bool), 4, 128, "query_chunk")]
    for m, B, bs, want in cases:
        cm = sa.compile_block_mask(m, B, 12, 4096, bs, True)
        st = cm.stats()
        assert st["pairing"] == want, (B, bs, want)
        # computed tiles follow the chosen pairing: every useful half once for unit pairing
        if bs == 64 and want == "unit":
            assert st["computed_tiles"] == oa.active_block_count(m, B, 12, 4096 // bs, True)
        assert st["computed_tiles"] >= st["active_blocks"]


def _pairing_masks():
    """Masks for the forced-pairing tests: HADS causal and not, odd chunk counts with empty
    rows, a dense causal mask, block 128 and a mask per unit."""
    odd = oh.dummy_hads_profile(2, 320, 64, causal=True).block_masks.copy()
    odd[1, 2, :] = False
    odd[0, 4, :4] = False
    per_unit = np.stack([oh.dummy_hads_profile(3, 512, 64, causal=True, global_blocks=b).block_masks
                         for b in range(2)])
    return [
        (2, 4, 512, 64, True, oh.dummy_hads_profile(4, 512, 64, causal=True, global_blocks=1).block_masks),
        (2, 4, 512, 64, False, oh.dummy_hads_profile(4, 512, 64, causal=False, global_blocks=0).block_masks),
        (3, 2, 320, 64, True, odd),
        (3, 2, 320, 64, False, odd),
        (2, 2, 512, 64, True, np.ones((8, 8), bool)),
        (1, 3, 1024, 128, True, oh.dummy_hads_profile(3, 1024, 128, causal=True).block_masks),
        (2, 3, 512, 64, True, per_unit),
    ]


@pytest.mark.parametrize("case", range(7))
def test_every_forward_pairing_matches_oracle(case):
    # The plan option forces each of the tensor-core forward's role sets (query-chunk pairs, unit
    # pairs) on the same inputs, whatever the mask would choose: each matches the oracle, and
    # they agree with one another to bf16 output rounding.
    sa = _sa()
    B, H, S, bs, causal, mask = _pairing_masks()[case]
    q, k, v = (_bf16_round(_rand((B, H, S, 64), 700 + 10 * case + i)) for i in range(3))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    ref, _, lse_ref = oa.sparse_attention_reference(q, k, v, mask, bs, causal=causal, return_weights=False,
                                                    return_lse=True)
    live = lse_ref > -1e30
    outs = {}
    for pairing in ("query_chunk", "unit"):
        cm = sa.compile_block_mask(mask, B, H, S, bs, causal, pairing=pairing)
        assert cm.stats()["pairing"] == pairing
        out, lse = sa.attention_forward(tq, tk, tv, cm, bs, None, causal)
        o = out.float().cpu().numpy()
        assert np.isfinite(o).all(), pairing
        assert _err(o, ref) <= BF16_TOL * np.abs(ref).max(), (pairing, _err(o, ref))
        np.testing.assert_allclose(lse.cpu().numpy()[live], lse_ref[live], rtol=0, atol=2e-2)
        outs[pairing] = o
    for pairing, o in outs.items():
        assert _err(o, outs["query_chunk"]) <= 1e-2 * np.abs(ref).max(), pairing


def test_bf16_bshd_layout_and_scale():
    prof = oh.dummy_hads_profile(4, 256, 64, causal=True)
    _bf16_case(2, 4, 256, 64, 64, True, prof.block_masks, seed=40, layout="bshd", scale=0.2)


def test_bf16_simt_fallback_shapes():
    # head_dim 32 and block 32 are outside the tensor-core kernel: CUDA-core path.
    prof = oh.dummy_hads_profile(4, 256, 32, causal=True)
    _bf16_case(1, 4, 256, 32, 32, True, prof.block_masks, seed=50)


def test_forward_is_deterministic():
    sa = _sa()
    prof = oh.dummy_hads_profile(12, 2048, 64, causal=True, global_blocks=1)
    q, k, v = (torch.randn(2, 12, 2048, 64, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    o1, l1 = sa.attention_forward(q, k, v, prof.block_masks, 64, None, True)
    o2, l2 = sa.attention_forward(q, k, v, prof.block_masks, 64, None, True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_config3_full_size_slices():
    """Config 3 (bf16 B=4 H=12 S=4096 D=64) at full size; the dense oracle checks a sample of
    (b, h) slices (the full dense check would need ~200 GFLOP of float64 host work)."""
    sa = _sa()
    prof = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1)
    q, k, v = oi.qkv(4, 12, 4096, 64, seed=oi.SEED_BASE + 3)
    q, k, v = _bf16_round(q), _bf16_round(k), _bf16_round(v)
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    out, lse = sa.attention_forward(tq, tk, tv, prof.block_masks, 64, None, True)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    for (b, h) in [(0, 0), (1, 5), (3, 11), (2, 7)]:
        ref, _, lref = oa.sparse_attention_reference(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                                     v[b:b + 1, h:h + 1], prof.block_masks[h:h + 1], 64,
                                                     causal=True, return_weights=False, return_lse=True)
        assert _err(o[b:b + 1, h:h + 1], ref) <= BF16_TOL * np.abs(ref).max()
        np.testing.assert_allclose(lse.cpu().numpy()[b, h], lref[0, 0], atol=2e-2)
    cm = sa.compile_block_mask(prof.block_masks, 4, 12, 4096, 64, True)
    st = cm.stats()
    assert st["active_blocks"] == oa.active_block_count(prof.block_masks, 4, 12, 64, True)
    assert st["empty_qblocks"] == 0


def test_plan_stats_count_empty_blocks():
    sa = _sa()
    m = np.ones((2, 4, 4), bool)
    m[1, 2, :] = False
    cm = sa.compile_block_mask(m, 3, 2, 256, 64, True)
    st = cm.stats()
    assert st["active_blocks"] == oa.active_block_count(m, 3, 2, 4, True)
    assert st["empty_qblocks"] == 3


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_backward_matches_oracle(dtype):
    sa = _sa()
    B, H, S, D, bs = 1, 3, 256, 64, 64
    m = oh.dummy_hads_profile(H, S, bs, causal=True, global_blocks=1).block_masks.copy()
    m[2, 1, :] = False          # a fully masked q-block feeds dV only
    q, k, v, do = (_rand((B, H, S, D), 60 + i) for i in range(4))
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    if dtype == "bf16":
        q, k, v, do = (_bf16_round(x) for x in (q, k, v, do))
    tq, tk, tv, tdo = (torch.from_numpy(x).to(tdt).cuda() for x in (q, k, v, do))
    o, lse = sa.attention_forward(tq, tk, tv, m, bs, None, True)
    dq, dk, dv = sa.attention_backward(tq, tk, tv, o, lse, tdo, m, bs, None, True)
    rq, rk, rv = oa.sparse_attention_backward(q, k, v, do, m, bs, causal=True)
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        g = got.float().cpu().numpy()
        scale = max(1.0, np.abs(ref).max()) if dtype == "f32" else np.abs(ref).max()
        assert _err(g, ref) <= tol * scale, (_err(g, ref), scale)


def _bf16_bwd_case(B, H, S, D, bs, causal, mask, seed, layout="bhsd", scale=None):
    """bf16 backward (the tensor-core kernels for D=64 and 64-multiple blocks) against the
    float64 closed form on the same bf16-rounded inputs: max|err| <= 2e-2 * max|ref|."""
    sa = _sa()
    q, k, v, do = (_bf16_round(_rand((B, H, S, D), seed + i)) for i in range(4))
    tq, tk, tv, tdo = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v, do))
    if layout == "bshd":
        tq, tk, tv, tdo = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (tq, tk, tv, tdo))
    o, lse = sa.attention_forward(tq, tk, tv, mask, bs, scale, causal)
    if layout == "bshd":
        o = o.transpose(1, 2).contiguous().transpose(1, 2)
    dq, dk, dv = sa.attention_backward(tq, tk, tv, o, lse, tdo, mask, bs, scale, causal)
    rq, rk, rv = oa.sparse_attention_backward(q, k, v, do, mask, bs, scale=scale, causal=causal)
    for name, got, ref in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        g = got.float().cpu().numpy()
        assert np.isfinite(g).all(), name
        assert _err(g, ref) <= BF16_TOL * np.abs(ref).max(), (name, _err(g, ref), np.abs(ref).max())
    return dq, dk, dv


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("global_blocks", [0, 1])
def test_bf16_backward_tensor_core_hads(causal, global_blocks):
    prof = oh.dummy_hads_profile(4, 512, 64, causal=causal, global_blocks=global_blocks)
    _bf16_bwd_case(2, 4, 512, 64, 64, causal, prof.block_masks, seed=70)


def test_bf16_backward_block128_and_shared_mask():
    prof = oh.dummy_hads_profile(3, 1024, 128, causal=True)
    _bf16_bwd_case(1, 3, 1024, 64, 128, True, prof.block_masks, seed=80)
    shared = oh.build_head_mask(0.5, 8, 1, 3, causal=True)
    _bf16_bwd_case(2, 2, 512, 64, 64, True, shared, seed=81)


def test_bf16_backward_odd_chunk_count_and_empty_rows():
    # S = 320: the last 128-key and 128-query tiles are half outside the sequence; a fully
    # masked q-block sends dO/S to every key's dV and nothing to dQ/dK.
    m = oh.dummy_hads_profile(2, 320, 64, causal=True).block_masks.copy()
    m[1, 2, :] = False
    m[0, 4, :4] = False
    _bf16_bwd_case(1, 2, 320, 64, 64, True, m, seed=90)


def test_bf16_backward_bshd_layout_and_scale():
    prof = oh.dummy_hads_profile(4, 256, 64, causal=True)
    _bf16_bwd_case(2, 4, 256, 64, 64, True, prof.block_masks, seed=100, layout="bshd", scale=0.2)


def test_bf16_backward_simt_fallback_shapes():
    prof = oh.dummy_hads_profile(4, 256, 32, causal=True)
    _bf16_bwd_case(1, 4, 256, 32, 32, True, prof.block_masks, seed=110)


def test_backward_is_deterministic():
    sa = _sa()
    prof = oh.dummy_hads_profile(12, 2048, 64, causal=True, global_blocks=1)
    q, k, v, do = (torch.randn(2, 12, 2048, 64, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, lse = sa.attention_forward(q, k, v, prof.block_masks, 64, None, True)
    g1 = sa.attention_backward(q, k, v, o, lse, do, prof.block_masks, 64, None, True)
    g2 = sa.attention_backward(q, k, v, o, lse, do, prof.block_masks, 64, None, True)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_backward_config3_full_size_slices():
    """Backward at config 3 size (bf16 B=4 H=12 S=4096 D=64); the float64 closed form checks a
    sample of (b, h) slices."""
    sa = _sa()
    prof = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1)
    q, k, v = oi.qkv(4, 12, 4096, 64, seed=oi.SEED_BASE + 3)
    do = _rand((4, 12, 4096, 64), 123)
    q, k, v, do = (_bf16_round(x) for x in (q, k, v, do))
    tq, tk, tv, tdo = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v, do))
    o, lse = sa.attention_forward(tq, tk, tv, prof.block_masks, 64, None, True)
    dq, dk, dv = (t.float().cpu().numpy() for t in sa.attention_backward(tq, tk, tv, o, lse, tdo,
                                                                          prof.block_masks, 64, None, True))
    for (b, h) in [(0, 0), (3, 11), (2, 7)]:
        sl = (slice(b, b + 1), slice(h, h + 1))
        rq, rk, rv = oa.sparse_attention_backward(q[sl], k[sl], v[sl], do[sl], prof.block_masks[h:h + 1], 64,
                                                  causal=True)
        for name, got, ref in (("dq", dq[sl], rq), ("dk", dk[sl], rk), ("dv", dv[sl], rv)):
            assert _err(got, ref) <= BF16_TOL * np.abs(ref).max(), (name, b, h, _err(got, ref))


def test_autograd_function_matches_backward():
    sa = _sa()
    prof = oh.dummy_hads_profile(2, 256, 64, causal=True)
    q, k, v = (torch.randn(1, 2, 256, 64, device="cuda", requires_grad=True) for _ in range(3))
    out = sa.sparse_attention_autograd(q, k, v, prof.block_masks, 64, None, True)
    g = torch.randn_like(out)
    out.backward(g)
    o, lse = sa.attention_forward(q.detach(), k.detach(), v.detach(), prof.block_masks, 64, None, True)
    dq, dk, dv = sa.attention_backward(q.detach(), k.detach(), v.detach(), o, lse, g, prof.block_masks,
                                       64, None, True)
    assert torch.equal(q.grad, dq) and torch.equal(k.grad, dk) and torch.equal(v.grad, dv)


def test_plan_mismatch_is_reported_not_faulted():
    """A plan compiled for other dims is rejected on the host by the Python layer, and by the
    kernels' header check when the C ABI is called directly (status word, no fault)."""
    import ctypes as C
    from xsake_b200 import _lib
    sa = _sa()
    prof = oh.dummy_hads_profile(2, 256, 64, causal=True)
    cm = sa.compile_block_mask(prof.block_masks, 1, 2, 256, 64, True)
    q = torch.randn(2, 2, 256, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        sa.attention_forward(q, q, q, cm, 64, None, True)
    o = torch.empty_like(q)
    lse = torch.empty(2, 2, 256, device="cuda")
    d = sa._desc(q, q, q, o, cm, None)
    d.batch = 2                                          # the plan says batch 1
    lib = _lib.load()
    stream = sa.dev.stream_ptr()
    _lib.device_error(stream)                            # clear earlier words
    n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_fwd_workspace_size(C.byref(d), C.byref(n)))
    ws = torch.zeros(n.value, dtype=torch.uint8, device="cuda")
    _lib.check(lib.xsake_attn_fwd(C.byref(d), cm.plan.data_ptr(), q.data_ptr(), q.data_ptr(),
                                  q.data_ptr(), o.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), stream))
    code = _lib.device_error(stream)
    assert code >> 24 == 2


def test_cuda_mask_cache_follows_content():
    """Plans are cached by mask content: a freed bool CUDA mask whose address the caching
    allocator hands to a different mask, and a mask written in place through .data, each get the
    plan of their own content."""
    sa = _sa()
    B, H, S, bs = 1, 2, 256, 64
    q, k, v = (_bf16_round(_rand((B, H, S, 64), 400 + i)) for i in range(3))
    tq, tk, tv = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v))
    first = np.zeros((H, 4, 4), bool)
    first[:, :, 0] = True
    m1 = torch.from_numpy(first).cuda()
    o1, _ = sa.attention_forward(tq, tk, tv, m1, bs, None, True)
    del m1
    m2 = torch.ones((H, 4, 4), dtype=torch.bool, device="cuda")      # typically the freed address
    o2, _ = sa.attention_forward(tq, tk, tv, m2, bs, None, True)
    ref2, _ = oa.sparse_attention_reference(q, k, v, np.ones((H, 4, 4), bool), bs, causal=True,
                                            return_weights=False)
    assert _err(o2.float().cpu().numpy(), ref2) <= BF16_TOL * np.abs(ref2).max()
    m2.data.copy_(torch.from_numpy(first).cuda())                    # in place: _version unchanged
    o3, _ = sa.attention_forward(tq, tk, tv, m2, bs, None, True)
    assert torch.equal(o3, o1)
