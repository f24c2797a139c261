"""GPU parity of the calibration-side kernels against the NumPy oracle:

* attention weights (the second output of sparse_attention_reference, which the reference's
  calibration collects): fp32 max|P - ref| <= 1e-5 (weights are <= 1);
* fused QK -> entropy (compute_attention_entropy of softmax(q k^T * scale) without
  materialising P): |H - ref| / |ref| <= 1e-5 per head, against the oracle and against the
  drop-in path (materialised weights + xsake_entropy_rows).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402
from oracle import inputs as oi  # noqa: E402

P_TOL = 1e-5
ENT_RTOL = 1e-5


def _rand(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def _probs_case(B, H, S, D, bs, causal, mask, seed, dtype=np.float32, scale=None):
    from xsake_b200 import sparse_attention as sa
    q, k = _rand((B, H, S, D), seed), _rand((B, H, S, D), seed + 1)
    if dtype != np.float32:
        q, k = (oi.to_bf16(x).astype(np.float32) for x in (q, k))
    tq, tk = (torch.from_numpy(x).cuda() for x in (q, k))
    if dtype != np.float32:
        tq, tk = tq.to(torch.bfloat16), tk.to(torch.bfloat16)
    p = sa.attention_probabilities(tq, tk, mask, bs, scale, causal).cpu().numpy()
    _, ref = oa.sparse_attention_reference(q, k, k, mask, bs, scale=scale, causal=causal)
    assert p.shape == ref.shape
    assert np.abs(p - ref).max() <= P_TOL, np.abs(p - ref).max()
    np.testing.assert_allclose(p.sum(-1), 1.0, atol=1e-5)
    return p


@pytest.mark.parametrize("causal", [True, False])
def test_probs_hads_masks(causal):
    prof = oh.dummy_hads_profile(3, 256, 64, causal=causal, global_blocks=1)
    _probs_case(2, 3, 256, 64, 64, causal, prof.block_masks, seed=500)


def test_probs_fully_masked_rows_are_uniform():
    m = oh.dummy_hads_profile(2, 192, 64, causal=True).block_masks.copy()
    m[1, 1, :] = False
    p = _probs_case(1, 2, 192, 64, 64, True, m, seed=510)
    np.testing.assert_allclose(p[0, 1, 64:128], 1.0 / 192, rtol=1e-6)


def test_probs_batch_mask_head_dim_32_and_bf16():
    m = np.random.default_rng(3).random((2, 3, 8, 8)) < 0.5
    m[..., np.arange(8), np.arange(8)] = True
    _probs_case(2, 3, 256, 32, 32, True, m, seed=520)
    prof = oh.dummy_hads_profile(2, 128, 64, causal=False)
    _probs_case(1, 2, 128, 64, 64, False, prof.block_masks, seed=530, dtype="bf16", scale=0.3)


@pytest.mark.parametrize("dtype,bs,S,causal", [("f32", 32, 320, True), ("bf16", 64, 192, False),
                                               ("f32", 30, 210, True)])
def test_probs_entry_points_with_and_without_workspace(dtype, bs, S, causal):
    # xsake_attn_probs (no workspace: tensor cores for bf16 at head_dim 64, CUDA cores for fp32)
    # and xsake_attn_probs_ex (workspace: tensor cores for both) against the oracle's weights;
    # S = 210 leaves rows that do not start on 16-byte boundaries (scalar stores) and a partial
    # last 64-key chunk.
    import ctypes as C
    from xsake_b200 import sparse_attention as sa, _lib
    B, H, D = 1, 2, 64
    m = oh.dummy_hads_profile(H, S, bs, causal=causal, global_blocks=1).block_masks.copy()
    m[1, 2, :] = False
    q, k = _rand((B, H, S, D), 570), _rand((B, H, S, D), 571) * np.float32(1.5)
    if dtype == "bf16":
        q, k = (oi.to_bf16(x).astype(np.float32) for x in (q, k))
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    tq, tk = (torch.from_numpy(x).to(tdt).cuda() for x in (q, k))
    _, ref = oa.sparse_attention_reference(q, k, k, m, bs, causal=causal)
    cm = sa.compile_block_mask(m, B, H, S, bs, causal, tq.device)
    d = sa._desc(tq, tk, tk, tq, cm, None)
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_probs_workspace_size(C.byref(d), C.byref(n)))
    ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
    for with_ws in (False, True):
        p = torch.full((B, H, S, S), float("nan"), device="cuda")
        if with_ws:
            _lib.check(lib.xsake_attn_probs_ex(C.byref(d), cm.plan.data_ptr(), tq.data_ptr(), tk.data_ptr(),
                                               p.data_ptr(), ws.data_ptr(), ws.numel(), None))
        else:
            _lib.check(lib.xsake_attn_probs(C.byref(d), cm.plan.data_ptr(), tq.data_ptr(), tk.data_ptr(),
                                            p.data_ptr(), None))
        got = p.cpu().numpy()
        assert np.abs(got - ref).max() <= P_TOL, (with_ws, np.abs(got - ref).max())


def test_sparse_attention_use_pallas_false_returns_weights():
    from xsake_b200 import sparse_attention as sa
    prof = oh.dummy_hads_profile(2, 256, 64, causal=True)
    q, k, v = oi.qkv(1, 2, 256, 64, seed=540)
    out, w = sa.sparse_attention(q, k, v, prof.block_masks, block_size=64, causal=True, use_pallas=False)
    ref_o, ref_w = oa.sparse_attention_reference(q, k, v, prof.block_masks, 64, causal=True)
    assert isinstance(w, np.ndarray) and w.dtype == np.float32
    assert np.abs(w - ref_w).max() <= P_TOL
    assert np.abs(out - ref_o).max() <= 1e-5 * max(1.0, np.abs(ref_o).max())
    out2, none = sa.sparse_attention(q, k, v, prof.block_masks, block_size=64, causal=True)
    assert none is None


def _softmax64(q, k, scale):
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k.astype(np.float64)) * scale
    p = np.exp(s - s.max(-1, keepdims=True))
    return p / p.sum(-1, keepdims=True)


@pytest.mark.parametrize("S", [1024, 200, 48])
def test_entropy_qk_matches_oracle(S):
    from xsake_b200 import hads_pattern as hp
    q, k, _ = oi.qkv(2, 12, S, 64, seed=550)
    got = hp.compute_attention_entropy_qk(q, k, 0.125)
    ref = oh.compute_attention_entropy(_softmax64(q, k, 0.125))
    assert got.dtype == np.float32 and got.shape == (12,)
    assert np.max(np.abs(got - ref) / np.abs(ref)) <= ENT_RTOL, np.max(np.abs(got - ref) / np.abs(ref))


@pytest.mark.parametrize("dtype,D,S", [("bf16", 64, 320), ("f32", 32, 320), ("f32", 64, 129)])
def test_entropy_qk_dtypes_head_dims_and_tails(dtype, D, S):
    # bf16 inputs take one product on the tensor cores (bf16 products are exact); head_dim 32
    # stays on the CUDA cores; S = 129 leaves one live row in the second 128-row tile and one
    # live key in the last 64-key chunk.
    from xsake_b200 import hads_pattern as hp
    q, k = _rand((2, 3, S, D), 560), _rand((2, 3, S, D), 561)
    q *= np.linspace(0.5, 3.0, 3, dtype=np.float32)[None, :, None, None]
    tq, tk = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
    if dtype == "bf16":
        q, k = (oi.to_bf16(x).astype(np.float32) for x in (q, k))
        tq, tk = tq.to(torch.bfloat16), tk.to(torch.bfloat16)
    scale = D ** -0.5
    got = hp.compute_attention_entropy_qk(tq, tk, scale).cpu().numpy()
    ref = oh.compute_attention_entropy(_softmax64(q, k, scale))
    assert np.max(np.abs(got - ref) / np.abs(ref)) <= ENT_RTOL, np.max(np.abs(got - ref) / np.abs(ref))


def test_entropy_qk_matches_materialised_path_on_calibration_batch():
    """Config 2's calibration batch shape (B=8, H=12, S=1024, D=64, fp32, q scaled by tau):
    fused entropies == drop-in path (weights, then xsake_entropy_rows) == oracle on 2 batches."""
    from xsake_b200 import hads_pattern as hp, sparse_attention as sa
    q, k = oi.calibration_batch(0)
    tq, tk = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
    fused = hp.entropy_head_sums_qk(tq, tk, 0.125).cpu().numpy()
    full = np.ones((1, 16, 16), bool)
    w = sa.attention_probabilities(tq, tk, full, 64, 0.125, False)
    dropin = hp.entropy_head_sums(w).cpu().numpy()
    np.testing.assert_allclose(fused, dropin, rtol=ENT_RTOL)
    ref = oh.compute_attention_entropy(_softmax64(q[:2], k[:2], 0.125))
    got = hp.compute_attention_entropy_qk(tq[:2], tk[:2], 0.125).cpu().numpy()
    assert np.max(np.abs(got - ref) / np.abs(ref)) <= ENT_RTOL


def test_entropy_qk_rejects_bad_arguments():
    from xsake_b200 import hads_pattern as hp
    q = torch.zeros(1, 2, 64, 64, device="cuda")
    with pytest.raises(ValueError):
        hp.entropy_head_sums_qk(q, torch.zeros(1, 2, 32, 64, device="cuda"))
    with pytest.raises(Exception):
        hp.entropy_head_sums_qk(torch.zeros(1, 2, 64, 48, device="cuda"), torch.zeros(1, 2, 64, 48, device="cuda"))


@pytest.mark.parametrize("dtype,layout", [("f32", "bhsd"), ("bf16", "bshd")])
def test_masked_entropy_matches_weights_entropy(dtype, layout):
    """xsake_attn_entropy: the entropy of the masked causal weights (what the reference's
    calibration reduces) without materialising them, against the oracle's weights, 1e-5 relative;
    a fully masked q-block (uniform rows) included; [B, S, H, D] memory read through strides."""
    from xsake_b200 import hads_pattern as hp
    B, H, S, D, bs = 2, 3, 512, 64, 64
    m = oh.dummy_hads_profile(H, S, bs, causal=True, global_blocks=1).block_masks.copy()
    m[2, 3, :] = False
    q, k = _rand((B, H, S, D), 600), _rand((B, H, S, D), 601)
    q *= np.linspace(0.5, 3, H, dtype=np.float32)[None, :, None, None]
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    if dtype == "bf16":
        q, k = (oi.to_bf16(x).astype(np.float32) for x in (q, k))
    tq, tk = (torch.from_numpy(x).to(tdt).cuda() for x in (q, k))
    if layout == "bshd":
        tq, tk = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (tq, tk))
    sums = hp.entropy_head_sums_attention(tq, tk, m, bs, None, causal=True).cpu().numpy()
    _, ref_p = oa.sparse_attention_reference(q, k, k, m, bs, causal=True)
    ref = oh.entropy_head_sums(ref_p)
    assert np.max(np.abs(sums - ref) / np.abs(ref)) <= ENT_RTOL


@pytest.mark.parametrize("bs,causal,S", [(32, True, 320), (128, False, 384), (64, False, 192)])
def test_masked_entropy_block_sizes(bs, causal, S):
    # Block sizes below, at and above the 64-key chunk of the tensor-core kernel, with and
    # without the causal cut; one fully masked q-block.
    from xsake_b200 import hads_pattern as hp
    B, H, D = 2, 2, 64
    m = oh.dummy_hads_profile(H, S, bs, causal=causal, global_blocks=1).block_masks.copy()
    m[1, 1, :] = False
    q, k = _rand((B, H, S, D), 610 + bs), _rand((B, H, S, D), 611 + bs)
    q *= np.float32(2.0)
    sums = hp.entropy_head_sums_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), m, bs, None,
                                          causal=causal).cpu().numpy()
    _, ref_p = oa.sparse_attention_reference(q, k, k, m, bs, causal=causal)
    ref = oh.entropy_head_sums(ref_p)
    assert np.max(np.abs(sums - ref) / np.abs(ref)) <= ENT_RTOL, np.max(np.abs(sums - ref) / np.abs(ref))


def test_model_calibration_and_recalibration_step():
    """trainer.calibrate_hads (training/trainer.py:79-117): the first layer's masked causal
    weights over n_steps batches, reduced by the fused kernel, give the profile the reference's
    path builds from the materialised weights (entropies 1e-5 relative; masks bit-exact on heads
    whose keep margin is at least 1e-4); maybe_recalibrate attaches it at the multiples of
    `every` only."""
    from xsake_b200 import hads_pattern as hp
    from xsake_b200 import sparse_attention as sa
    from xsake_b200 import trainer
    from xsake_b200.model import ModelConfig, XSAKETransformer
    cfg = ModelConfig(vocab_size=512, seq_len=512, n_layers=2, n_heads=4, d_model=256, d_ff=512,
                      block_size=64, dtype="float32", calibration_steps=3)
    torch.manual_seed(0)
    model = XSAKETransformer(cfg, device="cuda")
    batches = [torch.randint(0, 512, (2, 512), device="cuda") for _ in range(3)]
    prof = trainer.calibrate_hads(model, iter(batches), cfg)
    per_step = []
    for ids in batches:
        q, k, mask, bs, scale = model.layer0_qk(ids)
        p = sa.attention_probabilities(q.float(), k.float(), mask, bs, scale, True).cpu().numpy()
        per_step.append(oh.compute_attention_entropy(p))
    ent_ref = np.mean(per_step, axis=0)
    assert np.max(np.abs(prof.head_entropies - ent_ref) / np.abs(ent_ref)) <= ENT_RTOL
    ref = oh.profile_from_entropies(ent_ref.astype(np.float32), 512, 64, causal=True)
    for h in range(4):
        if oh.keep_margin(ref.head_sparsity[h], 8) >= 1e-4:
            np.testing.assert_array_equal(prof.block_masks[h], ref.block_masks[h], err_msg=f"head {h}")
    assert trainer.maybe_recalibrate(5, 10, model, iter(batches), cfg) is None
    assert model.blocks[1].attn.hads_profile is None
    new = trainer.maybe_recalibrate(10, 10, model, iter(batches), cfg)
    assert new is not None and all(b.attn.hads_profile is new for b in model.blocks)
    np.testing.assert_array_equal(new.block_masks, prof.block_masks)
    assert hp.profile_summary(new)["n_heads"] == 4
