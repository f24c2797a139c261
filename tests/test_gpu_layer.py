"""XSAKEAttention (model/attention.py:33-143) end to end on the GPU: projections, HADS masks,
the sparse attention kernels reading the projection's [B, S, H, D] memory through strides, the
output projection, and autograd through the library's backward.

Reference: the same composition in float64 on the CPU with a dense masked softmax (token mask
from the oracle).  Tolerances: fp32 layer 1e-4 * max(1, max|ref|) (two GEMMs and the attention
compose their fp32 rounding); bf16 layer 3e-2 * max|ref| (q, k, v and the attention output are
rounded to bf16 between the stages, on top of the attention kernels' 2e-2)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import attention as oa  # noqa: E402
from oracle import hads as oh  # noqa: E402


def _reference(layer, x, block_mask, bs):
    """float64 CPU forward of the layer's math; returns (out, tensors needing grad)."""
    W = {n: p.detach().double().cpu().requires_grad_(True) for n, p in layer.named_parameters()}
    xr = x.detach().double().cpu().requires_grad_(True)
    B, S, _ = xr.shape
    H, D = layer.n_heads, layer.d_head

    def proj(name, t):
        y = t @ W[f"{name}.weight"].T
        return y + W[f"{name}.bias"] if f"{name}.bias" in W else y

    q, k, v = (proj(n, xr).view(B, S, H, D).transpose(1, 2) for n in ("q_proj", "k_proj", "v_proj"))
    bm = oa.broadcast_mask(np.asarray(block_mask), B, H, S // bs)
    tm = torch.from_numpy(np.stack([np.stack([oa.token_mask(bm[b, h], bs, S, True) for h in range(H)])
                                    for b in range(B)]))
    s = (q @ k.transpose(-1, -2)) * D ** -0.5
    s = torch.where(tm, s, torch.tensor(np.finfo(np.float32).min, dtype=torch.float64))
    o = torch.softmax(s, -1) @ v
    out = proj("out_proj", o.transpose(1, 2).reshape(B, S, H * D))
    return out, xr, W


def _check(got, ref, tol, rel_to_max=True):
    g, r = got.detach().float().cpu().double(), ref.detach()
    scale = r.abs().max().item() if rel_to_max else max(1.0, r.abs().max().item())
    err = (g - r).abs().max().item()
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_layer_forward_backward_matches_float64(dtype, tol):
    from xsake_b200.attention import XSAKEAttention
    torch.manual_seed(0)
    layer = XSAKEAttention(256, 4, n_layers=2, bias=True, dtype=dtype, block_size=64, device="cuda")
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.15)
    x = torch.randn(2, 512, 256, device="cuda", dtype=dtype, requires_grad=True)
    out, w = layer(x)
    assert w is None and out.shape == (2, 512, 256) and out.dtype == dtype
    g = torch.randn_like(out)
    out.backward(g)
    bm, bs = layer.get_block_mask(512)
    ref, xr, W = _reference(layer, x, bm, bs)
    ref.backward(g.detach().double().cpu())
    f32 = dtype == torch.float32
    _check(out, ref, tol, rel_to_max=not f32)
    _check(x.grad, xr.grad, tol, rel_to_max=not f32)
    # Parameter gradients against the layer's largest one: the key bias has gradient exactly 0
    # (it shifts a whole score row by q.b_k, which softmax ignores), so only rounding noise shows.
    gmax = max(W[n].grad.abs().max().item() for n in W)
    for n, p in layer.named_parameters():
        err = (p.grad.detach().double().cpu() - W[n].grad).abs().max().item()
        assert err <= tol * gmax, (n, err, gmax)
    assert W["k_proj.bias"].grad.abs().max().item() <= 1e-9 * gmax


def test_layer_keeps_projection_layout_and_collects_weights():
    from xsake_b200 import sparse_attention as sa
    from xsake_b200.attention import XSAKEAttention
    layer = XSAKEAttention(256, 4, dtype=torch.bfloat16, block_size=64, device="cuda",
                           hads_profile=oh.dummy_hads_profile(4, 256, 64, causal=True, global_blocks=1))
    x = torch.randn(2, 256, 256, device="cuda", dtype=torch.bfloat16)
    q = layer._heads(layer.q_proj(x), 2, 256)
    o, _ = sa.attention_forward(q, q, q, layer.hads_profile.block_masks, 64, None, True)
    assert o.stride() == q.stride()            # written in [B, S, H, D] memory
    assert o.transpose(1, 2).is_contiguous()   # so the merge of the heads is a view
    out, w = layer(x, collect_attn=True)
    assert w.shape == (2, 4, 256, 256) and w.dtype == torch.float32
    torch.testing.assert_close(w.sum(-1), torch.ones(2, 4, 256, device="cuda"))
    k = layer._heads(layer.k_proj(x), 2, 256)
    ref = sa.attention_probabilities(q, k, layer.hads_profile.block_masks, 64, 0.125, True)
    assert torch.equal(w, ref)


@pytest.mark.parametrize("stype", ["local", "bigbird", "dense"])
def test_layer_non_hads_patterns(stype):
    from xsake_b200.attention import XSAKEAttention
    torch.manual_seed(1)
    layer = XSAKEAttention(128, 2, dtype=torch.float32, block_size=64, sparsity_type=stype, device="cuda")
    x = torch.randn(1, 256, 128, device="cuda")
    out, _ = layer(x)
    bm, bs = layer.get_block_mask(256)
    ref, _, _ = _reference(layer, x, bm, bs)
    _check(out, ref, 1e-4, rel_to_max=False)
