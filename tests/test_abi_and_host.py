"""CPU-only checks: the C-ABI library loads and exports every symbol the header declares,
argument validation happens before any launch, and the host-side logic of the package
(HADS masks, entropy->sparsity map, mask broadcasting) equals the reference's."""

import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "xsake_hads.h")
G = os.path.join(ROOT, "tests", "golden")


def _declared():
    src = open(HDR).read()
    return sorted(set(re.findall(r"XSAKE_API\s+(?:const\s+char\*|int)\s+(xsake_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from xsake_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from xsake_b200 import build
        build.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from xsake_b200 import _lib
    declared = _declared()
    assert len(declared) >= 17
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == declared


def test_abi_version_and_host_only_queries(lib):
    from xsake_b200 import _lib
    assert lib.xsake_abi_version() == _lib.ABI_VERSION
    dims = _lib.MaskDims(4, 12, 4096, 1, 12, 64, 1)
    n = C.c_size_t(0)
    assert lib.xsake_mask_plan_bytes(C.byref(dims), C.byref(n)) == 0
    assert n.value > 12 * 64 * 64
    bad = _lib.MaskDims(4, 12, 4096, 2, 12, 64, 1)          # mask batch 2 vs batch 4
    assert lib.xsake_mask_plan_bytes(C.byref(bad), C.byref(n)) == _lib.XSAKE_EINVAL
    assert b"mask batch" in lib.xsake_last_error()
    bad = _lib.MaskDims(4, 12, 4000, 1, 12, 64, 1)           # block does not divide seq
    assert lib.xsake_mask_plan_bytes(C.byref(bad), C.byref(n)) == _lib.XSAKE_EINVAL


def test_validation_rejects_before_launch(lib):
    from xsake_b200 import _lib
    # NULL pointers / bad dtypes never reach a kernel.
    assert lib.xsake_softmax_fwd(7, 4, 4, None, None, None) == _lib.XSAKE_EINVAL
    assert lib.xsake_softmax_fwd(0, 4, 4, None, None, None) == _lib.XSAKE_EINVAL
    assert lib.xsake_softmax_fwd(0, 0, 4, None, None, None) == _lib.XSAKE_OK   # empty is a no-op
    assert lib.xsake_entropy_rows(None, 1, 1, 1, 1, None, None, 0, None) == _lib.XSAKE_EINVAL
    d = _lib.AttnDesc()
    d.dtype, d.batch, d.heads, d.seq, d.head_dim, d.block_size = 1, 1, 1, 128, 64, 64
    d.mask_batch = d.mask_heads = 1
    for f in ("q_stride", "k_stride", "v_stride", "o_stride"):
        setattr(d, f, (C.c_int64 * 3)(8192, 8192, 64))
    assert lib.xsake_attn_fwd(C.byref(d), None, None, None, None, None, None, None, 0, None) == _lib.XSAKE_EINVAL
    d.dtype = 5
    assert lib.xsake_attn_fwd(C.byref(d), C.c_void_p(256), None, None, None, None, None, None, 0,
                              None) == _lib.XSAKE_EINVAL
    n = C.c_size_t(0)
    d.dtype = 1
    assert lib.xsake_attn_bwd_workspace_size(C.byref(d), C.byref(n)) == 0 and n.value >= 128 * 4


def test_operators_fail_loudly_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from xsake_b200 import XsakeError
    from xsake_b200.fused_softmax import fused_softmax
    with pytest.raises(XsakeError):
        fused_softmax(np.zeros((2, 8), np.float32))


@pytest.mark.parametrize("key", ["dummy_H8_S512_bs64_w2_c0", "dummy_H12_S1024_bs64_w2_c1",
                                 "dummy_H12_S4096_bs64_w2_c1", "dummy_H12_S4096_bs128_w2_c1",
                                 "dummy_H4_S128_bs32_w2_c0"])
def test_product_masks_equal_reference(key):
    from xsake_b200 import hads_pattern as hp
    z = np.load(os.path.join(G, "masks.npz"))
    H, nb, _ = z[key + "_shape"]
    parts = key.split("_")
    S, bs = int(parts[2][1:]), int(parts[3][2:])
    w, causal = int(parts[4][1:]), bool(int(parts[5][1:]))
    p = hp.dummy_hads_profile(int(H), S, bs, window_size=w, causal=causal)
    np.testing.assert_array_equal(p.head_sparsity, z[key + "_rho"])
    np.testing.assert_array_equal(p.block_masks, np.unpackbits(z[key + "_mask"], axis=-1, count=int(nb)).astype(bool))
    i = 0
    while f"head_{i}_args" in z:
        rho, nbb, ww, seed, c = z[f"head_{i}_args"]
        np.testing.assert_array_equal(hp._build_head_mask(float(rho), int(nbb), int(ww), int(seed), bool(c)),
                                      z[f"head_{i}_mask"])
        i += 1


def test_product_entropy_to_sparsity_exact():
    from xsake_b200 import hads_pattern as hp
    z = np.load(os.path.join(G, "entropy_to_sparsity.npz"))
    for name in ("lin20", "rand12", "flat4", "near"):
        np.testing.assert_array_equal(hp.entropy_to_sparsity(z[f"{name}_in"]), z[f"{name}_out"])
        np.testing.assert_array_equal(hp.entropy_to_sparsity(z[f"{name}_in"], 0.2, 0.7), z[f"{name}_out_b"])


def test_product_profile_from_reference_entropies():
    from xsake_b200 import hads_pattern as hp
    z = np.load(os.path.join(G, "calibration.npz"))
    p = hp.profile_from_entropies(z["profile_ent"], 128, 16, causal=True)
    np.testing.assert_array_equal(p.block_masks, z["profile_mask"])
    summ = hp.profile_summary(p)
    assert sorted(summ) == [str(k) for k in z["summary_keys"]]


def test_global_blocks_default_is_reference_behaviour():
    from xsake_b200 import hads_pattern as hp
    p0 = hp.dummy_hads_profile(12, 4096, 64, causal=True)
    p1 = hp.dummy_hads_profile(12, 4096, 64, causal=True, global_blocks=1)
    assert p1.block_masks[..., 0].all()
    assert not (p0.block_masks ^ p1.block_masks)[..., 1:].any()


def test_broadcast_mask_semantics():
    from xsake_b200.sparse_attention import broadcast_mask
    m = np.eye(4, dtype=bool)
    assert broadcast_mask(m, 2, 3, 4).shape == (2, 3, 4, 4)
    assert broadcast_mask(m[None].repeat(3, 0), 2, 3, 4).shape == (2, 3, 4, 4)
