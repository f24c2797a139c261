"""Config 3 at full size (bf16 B=4 H=12 S=4096 D=64, 64x64 blocks) checked on every (b, h)
slice, and config 3 with masks calibrated from its own tau-scaled Q, K.

Tolerances: bf16 outputs and gradients max|x - ref| <= 2e-2 * max|ref| per slice against the
oracle on the same bf16-rounded inputs (computed in float32 here: its rounding is ~1e-6, far
under the bound); entropies 1e-5 relative; masks bit-exact; lse 2e-2 absolute.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402
from oracle import inputs as oi  # noqa: E402

B, H, S, D, BS = 4, 12, 4096, 64, 64
BF16_TOL = 2e-2
MARGIN_MIN = 1e-4


def _sa():
    from xsake_b200 import sparse_attention as sa
    return sa


def _bf16(x):
    return oi.to_bf16(x).astype(np.float32)


def _inputs():
    q, k, v, do = oi.qkv(B, H, S, D, seed=oi.SEED_BASE + 3, with_do=True)
    return tuple(_bf16(x) for x in (q, k, v, do))


def _check_all_slices(masks, q, k, v, do, what):
    sa = _sa()
    tq, tk, tv, tdo = (torch.from_numpy(x).to(torch.bfloat16).cuda() for x in (q, k, v, do))
    out, lse = sa.attention_forward(tq, tk, tv, masks, BS, None, True)
    dq, dk, dv = sa.attention_backward(tq, tk, tv, out, lse, tdo, masks, BS, None, True)
    o, l = out.float().cpu().numpy(), lse.cpu().numpy()
    g = [t.float().cpu().numpy() for t in (dq, dk, dv)]
    worst = {"out": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    for b in range(B):
        for h in range(H):
            sl = (slice(b, b + 1), slice(h, h + 1))
            args = (q[sl], k[sl], v[sl])
            ref, _, lref = oa.sparse_attention_reference(*args, masks[h:h + 1], BS, causal=True,
                                                         compute_dtype=np.float32, return_weights=False,
                                                         return_lse=True)
            e = np.abs(o[sl] - ref).max() / np.abs(ref).max()
            worst["out"] = max(worst["out"], e)
            assert e <= BF16_TOL, (what, "out", b, h, e)
            np.testing.assert_allclose(l[b, h], lref[0, 0], atol=2e-2)
            grads = oa.sparse_attention_backward(*args, do[sl], masks[h:h + 1], BS, causal=True,
                                                 compute_dtype=np.float32)
            for name, got, ref_g in zip(("dq", "dk", "dv"), g, grads):
                e = np.abs(got[sl] - ref_g).max() / np.abs(ref_g).max()
                worst[name] = max(worst[name], e)
                assert e <= BF16_TOL, (what, name, b, h, e)
    print(f"{what}: worst relative error over 48 slices {worst}")


def test_config3_every_slice_forward_and_backward():
    masks = oh.dummy_hads_profile(H, S, BS, causal=True, global_blocks=1).block_masks
    _check_all_slices(masks, *_inputs(), "dummy profile")


def test_config3_calibrated_masks():
    """Masks as in config 0 but at S = 4096: entropies of the config's own tau-scaled Q, K (full
    non-causal softmax, scale 1/8) computed on the GPU from Q, K, checked against the float64
    oracle at 1e-5 relative; per head, the margin of nb * (1 - rho) to the nearest integer is
    reported.  Heads whose margin is at least 1e-4 must get bit-exact masks from the GPU
    entropies; a head under that margin could flip on any rounding difference, so the masks
    are then built from the oracle's entropies.  Forward and backward then run on those masks
    and are checked on every slice."""
    from xsake_b200 import hads_pattern as hp
    q, k, v, do = _inputs()
    sums_gpu = hp.entropy_head_sums_qk(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), 0.125)
    ent_gpu = sums_gpu.cpu().numpy() / (B * S)
    sums = np.zeros(H)
    for b in range(B):
        for h in range(H):
            s_ = (q[b, h].astype(np.float64) @ k[b, h].astype(np.float64).T) / 8.0
            p = np.exp(s_ - s_.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            sums[h] += oh.entropy_head_sums(p[None, None])[0]
    ent_ref = sums / (B * S)
    rel = np.abs(ent_gpu - ent_ref) / np.abs(ent_ref)
    assert rel.max() <= 1e-5, rel
    rho = oh.entropy_to_sparsity(ent_ref.astype(np.float32))
    margins = [oh.keep_margin(r, S // BS) for r in rho]
    low = [h for h, mg in enumerate(margins) if mg < MARGIN_MIN]
    print("per-head keep margins:", [f"{m:.2e}" for m in margins], "under 1e-4:", low)
    prof_gpu = hp.profile_from_entropies(ent_gpu.astype(np.float32), S, BS, causal=True, global_blocks=1)
    prof_ref = oh.profile_from_entropies(ent_ref.astype(np.float32), S, BS, causal=True, global_blocks=1)
    for h in range(H):
        if h not in low:
            np.testing.assert_array_equal(prof_gpu.block_masks[h], prof_ref.block_masks[h], err_msg=f"head {h}")
    _check_all_slices(prof_ref.block_masks, q, k, v, do, "calibrated profile")
