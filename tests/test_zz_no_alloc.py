"""The allocation-free entropy entry point, called through the C ABI.

xsake_entropy_rows_noalloc serves callers that cannot give the library a device workspace and
cannot allocate one (framework plugins restricted to their framework's allocator, processes
whose device memory is held by a pool allocator, loops that cannot pay for cudaMalloc's
synchronisation).  Its scratch is a static device array inside the library, so this test
checks that two calls in a row (the second one seeing the first one's leftovers, with a
different shape in between) match the workspace-based xsake_entropy_rows within the entropy
tolerance used elsewhere (1e-5 relative), and that oversized requests are refused before any
launch.  The file is named to be collected last.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _probs(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.softmax(torch.randn(*shape, device="cuda", generator=g) * 3, dim=-1).contiguous()


def _with_workspace(lib, p):
    B, H, Sq, Sk = p.shape
    n = C.c_size_t(0)
    assert lib.xsake_entropy_workspace_size(B, H, Sq, C.byref(n)) == 0
    ws = torch.empty(max(n.value, 16), dtype=torch.uint8, device="cuda")
    out = torch.zeros(H, dtype=torch.float64, device="cuda")
    st = lib.xsake_entropy_rows(p.data_ptr(), B, H, Sq, Sk, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.xsake_last_error()
    return out


def _no_alloc(lib, p):
    B, H, Sq, Sk = p.shape
    out = torch.full((H,), float("nan"), dtype=torch.float64, device="cuda")
    st = lib.xsake_entropy_rows_noalloc(p.data_ptr(), B, H, Sq, Sk, out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.xsake_last_error()
    return out


def test_noalloc_entropy_matches_workspace_version_twice():
    from xsake_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(0)
    p1 = _probs((2, 12, 512, 512), 1)
    p2 = _probs((3, 5, 256, 384), 2)
    ref1, ref2 = _with_workspace(lib, p1), _with_workspace(lib, p2)
    for _ in range(2):                      # second round reuses the static scratch as left behind
        got1 = _no_alloc(lib, p1)
        got2 = _no_alloc(lib, p2)
        torch.cuda.synchronize()
        for got, ref in ((got1, ref1), (got2, ref2)):
            g, r = got.cpu().numpy(), ref.cpu().numpy()
            assert np.all(np.isfinite(g))
            assert np.max(np.abs(g - r) / np.abs(r)) <= 1e-5
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    from xsake_b200 import _lib
    lib = _lib.load()
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    p = torch.zeros(16, dtype=torch.float32, device="cuda")
    # 2048 * 64 slices of 64 query rows, 16 rows per partial -> 524,288 partial sums > 65,536:
    # refused, nothing launched
    st = lib.xsake_entropy_rows_noalloc(p.data_ptr(), 2048, 64, 64, 4, out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert st == _lib.XSAKE_EUNSUPPORTED
    assert b"static limit" in lib.xsake_last_error()
