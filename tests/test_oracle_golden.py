"""Pin the NumPy oracle against golden vectors produced by the reference's own source.

The fixtures come from tests/golden/make_golden.py, which executes the reference
modules (kernels/hads/hads_pattern.py, kernels/pallas/sparse_attention.py,
fused_softmax.py, fused_layernorm.py, sparsity_mask.py) with NumPy standing in for
jax.numpy.  Masks must match bit-exactly; floats to the stated tolerances.
"""

import os

import numpy as np
import pytest

from oracle import attention as oa
from oracle import hads as oh
from oracle import rowops as orow

G = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(G, name + ".npz"), allow_pickle=False)


def test_golden_numpy_version_matches():
    z = _load("masks")
    assert str(z["_numpy_version"]) == np.__version__, (
        "block masks are bit-exact only for the NumPy version that made the fixtures")


@pytest.mark.parametrize("key", [
    "dummy_H8_S512_bs64_w2_c0", "dummy_H8_S512_bs64_w1_c0", "dummy_H4_S256_bs64_w2_c0",
    "dummy_H4_S128_bs32_w2_c0", "dummy_H12_S1024_bs64_w2_c1", "dummy_H12_S1024_bs128_w2_c1",
    "dummy_H12_S4096_bs64_w2_c1", "dummy_H12_S4096_bs128_w2_c1", "dummy_H12_S2048_bs64_w2_c0"])
def test_dummy_profile_bit_exact(key):
    z = _load("masks")
    H, nb, _ = z[key + "_shape"]
    parts = key.split("_")
    S, bs = int(parts[2][1:]), int(parts[3][2:])
    w, causal = int(parts[4][1:]), bool(int(parts[5][1:]))
    p = oh.dummy_hads_profile(int(H), S, bs, window_size=w, causal=causal)
    want = np.unpackbits(z[key + "_mask"], axis=-1, count=int(nb)).astype(bool)
    np.testing.assert_array_equal(p.head_entropies, z[key + "_ent"])
    np.testing.assert_array_equal(p.head_sparsity, z[key + "_rho"])
    np.testing.assert_array_equal(p.block_masks, want)
    # the parity margin of int(nb * (1 - rho)) must be comfortable
    for r in p.head_sparsity:
        assert oh.keep_margin(r, int(nb)) > 1e-4


def test_single_head_masks_bit_exact():
    z = _load("masks")
    i = 0
    while f"head_{i}_args" in z:
        rho, nb, w, seed, causal = z[f"head_{i}_args"]
        got = oh.build_head_mask(float(rho), int(nb), int(w), int(seed), bool(causal))
        np.testing.assert_array_equal(got, z[f"head_{i}_mask"])
        i += 1
    assert i >= 6


def test_global_block_step_keeps_reference_draws():
    p0 = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=0)
    p1 = oh.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1)
    assert p1.block_masks[:, :, 0].all()
    diff = p1.block_masks ^ p0.block_masks
    assert not diff[:, :, 1:].any()


@pytest.mark.parametrize("name", ["lin20", "rand12", "flat4", "near"])
def test_entropy_to_sparsity_exact(name):
    z = _load("entropy_to_sparsity")
    e = z[f"{name}_in"]
    np.testing.assert_array_equal(oh.entropy_to_sparsity(e), z[f"{name}_out"])
    np.testing.assert_array_equal(oh.entropy_to_sparsity(e, 0.2, 0.7), z[f"{name}_out_b"])


def test_entropy_and_calibrated_profile():
    z = _load("calibration")
    for a in ("attn", "attn2"):
        got = oh.compute_attention_entropy(z[a])
        want = z["entropy_" + a].astype(np.float64)
        assert np.max(np.abs(got - want) / np.abs(want)) <= 1e-5
    prof = oh.build_hads_profile([z["attn"], z["attn2"]], seq_len=128, block_size=16,
                                 causal=True)
    np.testing.assert_allclose(prof.head_entropies, z["profile_ent"], rtol=1e-5)
    np.testing.assert_allclose(prof.head_sparsity, z["profile_rho"], rtol=0, atol=1e-5)
    np.testing.assert_array_equal(prof.block_masks, z["profile_mask"])
    summ = oh.profile_summary(prof)
    assert sorted(summ) == [str(k) for k in z["summary_keys"]]
    np.testing.assert_allclose([summ[k] for k in sorted(summ)], z["summary_vals"], rtol=1e-5)


@pytest.mark.parametrize("name,causal", [("hads_c1", True), ("hads_c0", False),
                                         ("bigbird32_c0", False), ("mask4d_c1", True),
                                         ("emptyrow_c1", True), ("dense16_c1", True)])
def test_attention_reference_matches_golden(name, causal):
    z = _load("attention")
    out, w = oa.sparse_attention_reference(z["q"], z["k"], z["v"], z[f"{name}_mask"],
                                           block_size=int(z[f"{name}_bs"]), causal=causal)
    ref = z[f"{name}_out"]
    assert np.max(np.abs(out - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))
    np.testing.assert_allclose(w.sum(-1), z[f"{name}_wsum"], atol=1e-5)
    np.testing.assert_allclose(w[:, :, 37, :], z[f"{name}_w_row37"], atol=1e-6)


def test_attention_scale_override():
    z = _load("attention")
    out, _ = oa.sparse_attention_reference(z["q"], z["k"], z["v"], z["hads_c1_mask"],
                                           block_size=64, scale=0.3, causal=True)
    assert np.max(np.abs(out - z["scale03_out"])) <= 1e-5 * max(1.0, np.abs(out).max())


def test_rowops_match_golden():
    z = _load("rowops")
    np.testing.assert_allclose(orow.softmax(z["sm_x"]), z["sm_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(orow.softmax(z["sm_xm"]), z["sm_outm"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(orow.layernorm(z["ln_x"], z["ln_g"], z["ln_b"]), z["ln_out"],
                               rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(orow.layernorm(z["ln_x"], z["ln_g"], z["ln_b"], eps=1e-2),
                               z["ln_out_eps"], rtol=1e-4, atol=1e-5)


def test_patterns_are_bit_exact_inputs():
    """The non-HADS patterns (kernels/pallas/sparsity_mask.py) are plain bool masks that
    the CUDA path consumes unchanged; the fixture keeps them for the GPU tests."""
    z = _load("masks")
    for st in ["dense", "local", "bigbird"]:
        m = z[f"pattern_{st}_c1"]
        assert not np.triu(m, 1).any()
