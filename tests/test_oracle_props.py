"""Oracle self-checks that need no fixtures: closed-form backwards against central
finite differences in float64 (the reference has no VJP of its own, so this is how
the gradient oracle is pinned), plus the dense-mask identity of
tests/test_kernel_correctness.py:46-57 in the reference."""

import numpy as np
import pytest

from oracle import attention as oa
from oracle import hads as oh
from oracle import rowops as orow


def _fd(f, x, dy, eps=1e-6, n=12, seed=0):
    rng = np.random.default_rng(seed)
    idx = [tuple(rng.integers(0, s) for s in x.shape) for _ in range(n)]
    out = []
    for i in idx:
        xp = x.copy(); xp[i] += eps
        xm = x.copy(); xm[i] -= eps
        out.append(((f(xp) - f(xm)) * dy).sum() / (2 * eps))
    return idx, np.array(out)


@pytest.mark.parametrize("causal", [True, False])
def test_attention_backward_matches_finite_differences(causal):
    rng = np.random.default_rng(3)
    B, H, S, D, bs = 1, 2, 64, 8, 16
    q, k, v, do = (rng.standard_normal((B, H, S, D)) for _ in range(4))
    mask = oh.dummy_hads_profile(H, S, bs, window_size=1, causal=causal).block_masks
    mask = mask.copy(); mask[1, 3, :] = False       # one fully masked q-block
    dq, dk, dv = oa.sparse_attention_backward(q, k, v, do, mask, bs, causal=causal)
    for name, x, g in (("q", q, dq), ("k", k, dk), ("v", v, dv)):
        def f(xx, name=name):
            args = {"q": q, "k": k, "v": v}
            args[name] = xx
            return oa.sparse_attention_reference(args["q"], args["k"], args["v"], mask, bs,
                                                 causal=causal, return_weights=False)[0]
        idx, num = _fd(f, x, do)
        np.testing.assert_allclose([g[i] for i in idx], num, rtol=1e-5, atol=1e-7)


def test_dense_mask_equals_plain_attention():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 4, 256, 32)).astype(np.float32) for _ in range(3))
    out, _ = oa.sparse_attention_reference(q, k, v, np.ones((4, 4), bool), 64)
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k) / np.sqrt(32)
    ref = np.einsum("bhqk,bhkd->bhqd", orow.softmax(s), v)
    assert float(np.sqrt(np.mean((out - ref) ** 2))) < 1e-4


def test_softmax_and_layernorm_backward_fd():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 17))
    dy = rng.standard_normal((3, 17))
    y = orow.softmax(x)
    idx, num = _fd(lambda xx: orow.softmax(xx), x, dy)
    g = orow.softmax_backward(y, dy)
    np.testing.assert_allclose([g[i] for i in idx], num, rtol=1e-6, atol=1e-8)
    gam = rng.standard_normal(17)
    bet = rng.standard_normal(17)
    dx, dg, db = orow.layernorm_backward(x, gam, dy)
    idx, num = _fd(lambda xx: orow.layernorm(xx, gam, bet), x, dy)
    np.testing.assert_allclose([dx[i] for i in idx], num, rtol=1e-5, atol=1e-7)
    idx, num = _fd(lambda gg: orow.layernorm(x, gg, bet), gam, dy)
    np.testing.assert_allclose([dg[i] for i in idx], num, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(db, dy.sum(0))


def test_fully_masked_row_is_uniform_mean_of_v():
    rng = np.random.default_rng(2)
    q, k, v = (rng.standard_normal((1, 1, 128, 8)) for _ in range(3))
    mask = np.ones((2, 2), bool); mask[1, :] = False
    out, w, lse = oa.sparse_attention_reference(q, k, v, mask, 64, causal=True, return_lse=True)
    np.testing.assert_allclose(out[0, 0, 64:], np.broadcast_to(v[0, 0].mean(0), (64, 8)),
                               rtol=1e-12)
    assert np.all(lse[0, 0, 64:] < -1e38)
