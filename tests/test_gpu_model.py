"""The transformer of model/transformer.py built on this library's attention and LayerNorm
kernels: loss and gradients against a torch-only composition of the same math (dense masked
softmax attention, torch LayerNorm), and a few bf16 AdamW steps that lower the loss.
Tolerance (fp32 model): 1e-4 relative on the loss, 1e-3 of the largest gradient."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
F = torch.nn.functional

from oracle import attention as oa  # noqa: E402


def _cfg():
    from xsake_b200.model import ModelConfig
    return ModelConfig(vocab_size=97, seq_len=256, n_layers=2, n_heads=2, d_model=128, d_ff=256,
                       block_size=64, bias=True)


def _torch_forward(model, ids):
    """Same math with dense torch ops (fp32)."""
    cfg = model.cfg
    B, S = ids.shape
    x = model.tok(ids) + model.pos[:S]
    for blk in model.blocks:
        h = F.layer_norm(x, (cfg.d_model,), blk.ln1.gamma, blk.ln1.beta, 1e-5)
        at = blk.attn
        q, k, v = (lin(h).view(B, S, cfg.n_heads, -1).transpose(1, 2) for lin in (at.q_proj, at.k_proj, at.v_proj))
        bm, bs = at.get_block_mask(S)
        bm = oa.broadcast_mask(np.asarray(bm), B, cfg.n_heads, S // bs)
        tm = torch.from_numpy(np.stack([np.stack([oa.token_mask(bm[b, hh], bs, S, True)
                                                  for hh in range(cfg.n_heads)]) for b in range(B)])).cuda()
        s = (q @ k.transpose(-1, -2)) * at.d_head ** -0.5
        s = torch.where(tm, s, torch.tensor(torch.finfo(torch.float32).min, device="cuda"))
        o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B, S, cfg.d_model)
        x = x + at.out_proj(o)
        h = F.layer_norm(x, (cfg.d_model,), blk.ln2.gamma, blk.ln2.beta, 1e-5)
        x = x + blk.mlp.fc2(F.gelu(blk.mlp.fc1(h), approximate="tanh"))
    x = F.layer_norm(x, (cfg.d_model,), model.ln_f.gamma, model.ln_f.beta, 1e-5)
    return F.linear(x, model.tok.weight)


def _torch_xent(logits, labels, ignore_index=-1):
    """cross_entropy_loss of model/transformer.py:177-203 with plain torch ops (fp32)."""
    vocab = logits.shape[-1]
    fl = logits[:, :-1].reshape(-1, vocab).float()
    lb = labels[:, 1:].reshape(-1)
    valid = lb != ignore_index
    nll = F.cross_entropy(fl, lb.clamp(0, vocab - 1), reduction="none")
    return (nll * valid).sum() / valid.sum().clamp(min=1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("vocab,ld", [(97, 128), (50257, 50304), (33, 33)])
def test_fused_cross_entropy_matches_torch(dtype, vocab, ld):
    # Logits as a [..., :vocab] view of a padded buffer (the model's layout; 16-byte vector
    # path) and a contiguous buffer with an odd row length (scalar path), with ignored targets.
    from xsake_b200.model import cross_entropy_loss
    torch.manual_seed(3)
    B, S = 2, (96 if vocab > 1000 else 300)
    buf = (3 * torch.randn(B, S, ld, device="cuda")).to(dtype)
    labels = torch.randint(0, vocab, (B, S), device="cuda")
    labels[0, 5] = -1
    labels[1, 7] = -1
    src = buf.clone().requires_grad_(True)
    loss = cross_entropy_loss(src[..., :vocab], labels)
    loss.backward()
    ref_src = buf.float().clone().requires_grad_(True)
    ref = _torch_xent(ref_src[..., :vocab], labels)
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-5 * abs(ref.item()), (loss.item(), ref.item())
    g, rg = src.grad.float(), ref_src.grad
    tol = 1e-6 if dtype == torch.float32 else 1e-2 * rg.abs().max().item()
    assert (g - rg).abs().max().item() <= tol, (g - rg).abs().max().item()


def test_model_loss_and_grads_match_torch_composition():
    from xsake_b200.model import XSAKETransformer, cross_entropy_loss
    torch.manual_seed(0)
    model = XSAKETransformer(_cfg(), device="cuda")
    ids = torch.randint(0, 97, (2, 256), device="cuda")
    ids[0, 10] = -1                                    # an ignored target
    logits, attn = model(ids.clamp(min=0))
    assert attn is None and logits.shape == (2, 256, 97)
    loss = cross_entropy_loss(logits, ids)
    loss.backward()
    got = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    ref_loss = _torch_xent(_torch_forward(model, ids.clamp(min=0)), ids)
    ref_loss.backward()
    assert abs(loss.item() - ref_loss.item()) <= 1e-4 * abs(ref_loss.item())
    gmax = max(p.grad.abs().max().item() for p in model.parameters())
    for n, p in model.named_parameters():
        err = (got[n] - p.grad).abs().max().item()
        assert err <= 1e-3 * gmax, (n, err, gmax)


def test_model_bf16_training_steps_reduce_loss_and_collect_attention():
    from xsake_b200.model import XSAKETransformer, cross_entropy_loss
    torch.manual_seed(1)
    model = XSAKETransformer(_cfg(), device="cuda")
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3, fused=True)
    ids = torch.randint(0, 97, (4, 256), device="cuda")
    losses = []
    for _ in range(8):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, _ = model(ids)
            loss = cross_entropy_loss(logits, ids)
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in model.parameters())
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 0.5
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        _, attn = model(ids, collect_attn=True)
    assert len(attn) == 2 and attn[0].shape == (4, 2, 256, 256)
    torch.testing.assert_close(attn[0].sum(-1), torch.ones(4, 2, 256, device="cuda"))
