"""The C ABI driven by a C program with no Python and no PyTorch in its process
(tests/c_abi/xsake_c_client.c): device memory from the CUDA runtime, a compiled mask plan, the
attention forward, softmax and LayerNorm on one stream.  Its outputs are checked against the
oracle: bf16 attention 2e-2 * max|ref|, lse 2e-2 absolute, fp32 softmax rtol 1e-5, fp32
LayerNorm max|x - ref| <= 1e-5 * max(1, max|ref|)."""

import os
import shutil
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402
from oracle import inputs as oi  # noqa: E402
from oracle import rowops as orow  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    out = tmp_path_factory.mktemp("c_abi") / "xsake_c_client"
    lib = os.path.join(ROOT, "xsake_b200", "lib")
    subprocess.run([nvcc, "-O2", "-x", "cu", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "c_abi", "xsake_c_client.c"),
                    "-o", str(out), "-L", lib, "-lxsake_hads", "-Xlinker", "-rpath", "-Xlinker", lib],
                   check=True, capture_output=True)
    return str(out)


def test_c_client_matches_oracle(client, tmp_path):
    B, H, S, D, bs = 2, 3, 256, 64, 64
    rng = np.random.default_rng(77)
    q, k, v = (oi.to_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32)).astype(np.float32) for _ in range(3))
    mask = oh.dummy_hads_profile(H, S, bs, causal=True, global_blocks=1).block_masks
    sx = (rng.standard_normal((37, 100)) * 3).astype(np.float32)
    lx = (rng.standard_normal((19, 768)) * 2 + 1).astype(np.float32)
    lg = (1 + 0.1 * rng.standard_normal(768)).astype(np.float32)
    lb = (0.1 * rng.standard_normal(768)).astype(np.float32)
    inp, outp = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        np.array([B, H, S, D, bs, 1, H, 37, 100, 19, 768], np.int32).tofile(f)
        for a in (q, k, v):
            a.tofile(f)
        mask.astype(np.uint8).tofile(f)
        for a in (sx, lx, lg, lb):
            a.tofile(f)
    r = subprocess.run([client, str(inp), str(outp)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(outp, np.float32)
    n = B * H * S * D
    o, lse = got[:n].reshape(B, H, S, D), got[n:n + B * H * S].reshape(B, H, S)
    rest = got[n + B * H * S:]
    sy, ly = rest[:37 * 100].reshape(37, 100), rest[37 * 100:].reshape(19, 768)
    ref, _, lref = oa.sparse_attention_reference(q, k, v, mask, bs, causal=True, return_weights=False,
                                                 return_lse=True)
    assert np.abs(o - ref).max() <= 2e-2 * np.abs(ref).max()
    np.testing.assert_allclose(lse, lref, atol=2e-2)
    np.testing.assert_allclose(sy, orow.softmax(sx), rtol=1e-5, atol=1e-6)
    lref_y = orow.layernorm(lx, lg, lb)
    assert np.abs(ly - lref_y).max() <= 1e-5 * max(1.0, np.abs(lref_y).max())
