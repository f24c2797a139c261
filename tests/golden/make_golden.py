"""Generate the golden fixtures in this folder by running the REFERENCE's own source.

The reference (Hridambiswas/XSAKE) is JAX code and JAX cannot be installed in
this environment, so the reference modules are executed against a small
NumPy-backed stand-in for ``jax`` / ``jax.numpy`` defined below.  What that pins:

* block masks: bit-exact -- ``_build_head_mask`` uses NumPy's RNG alone;
* the entropy -> sparsity map: the reference's float32 expression structure
  (JAX weak typing and NumPy 2's NEP 50 promote Python scalars the same way);
* ``sparse_attention_reference``: its token-mask expansion, causal cut, finfo.min
  fill, broadcast rules and softmax, evaluated in float32 NumPy arithmetic;
* the CPU branches of ``fused_softmax`` / ``fused_layernorm``.
What it cannot pin: XLA's exact float32 rounding/reduction order, and
``jnp.linspace`` (the stand-in restates JAX's formulation).

Run from the repository root (needs the reference checkout), giving its location as the
first argument or in XSAKE_REFERENCE:
    python tests/golden/make_golden.py /path/to/reference
"""

from __future__ import annotations

import functools
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("XSAKE_REFERENCE", "")
if __name__ == "__main__" and not (REF and os.path.isdir(REF)):
    sys.exit("usage: make_golden.py /path/to/reference  (or set XSAKE_REFERENCE)")


# ----------------------------------------------------------------------------- stand-in jax
def _linspace(start, stop, num=50, dtype=None):
    if num == 1:
        return np.array([start], np.float32)
    div = num - 1
    t = np.arange(div, dtype=np.float32) / np.float32(div)
    out = np.float32(start) * (np.float32(1) - t) + np.float32(stop) * t
    return np.concatenate([out, np.array([stop], np.float32)]).astype(dtype or np.float32)


def _f32_default(fn):
    @functools.wraps(fn)
    def wrap(*a, dtype=None, **kw):
        return fn(*a, dtype=np.float32 if dtype is None else dtype, **kw)
    return wrap


def _array(x, dtype=None):
    arr = np.array(x, dtype=dtype)
    if dtype is None and arr.dtype == np.float64:
        arr = arr.astype(np.float32)
    return arr


def _softmax(x, axis=-1):
    x = np.asarray(x)
    with np.errstate(invalid="ignore"):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / np.sum(e, axis=axis, keepdims=True)


def _jit(fn=None, **_):
    if fn is None:
        return lambda f: f
    return fn


def install_stub():
    import ml_dtypes
    jnp = types.ModuleType("jax.numpy")
    for name in ["clip", "log", "exp", "sqrt", "sum", "mean", "min", "max", "maximum", "stack",
                 "repeat", "tril", "einsum", "where", "finfo", "broadcast_to", "concatenate",
                 "diff", "all", "isfinite", "float32", "bool_", "ndarray", "abs", "eye"]:
        setattr(jnp, name, getattr(np, name))
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.linspace = _linspace
    jnp.ones = _f32_default(np.ones)
    jnp.zeros = _f32_default(np.zeros)
    jnp.full = lambda shape, fill, dtype=None: np.full(shape, fill, dtype or np.float32)
    jnp.array = _array
    jnp.asarray = _array
    jax = types.ModuleType("jax")
    jax.numpy = jnp
    jax.nn = types.SimpleNamespace(softmax=_softmax)
    jax.jit = _jit
    jax.default_backend = lambda: "cpu"
    jax.Array = np.ndarray
    jax.lax = types.SimpleNamespace()
    exp = types.ModuleType("jax.experimental")
    pallas = types.ModuleType("jax.experimental.pallas")
    exp.pallas = pallas
    jax.experimental = exp
    sys.modules.update({"jax": jax, "jax.numpy": jnp, "jax.experimental": exp,
                        "jax.experimental.pallas": pallas})


def load_ref(relpath, name):
    path = os.path.join(REF, relpath)
    mod = types.ModuleType(name)
    mod.__file__ = path
    with open(path) as f:
        src = f.read()
    exec(compile(src, path, "exec"), mod.__dict__)
    return mod


# ----------------------------------------------------------------------------- fixtures
def main():
    install_stub()
    hp = load_ref("kernels/hads/hads_pattern.py", "ref_hads_pattern")
    sa = load_ref("kernels/pallas/sparse_attention.py", "ref_sparse_attention")
    fs = load_ref("kernels/pallas/fused_softmax.py", "ref_fused_softmax")
    fl = load_ref("kernels/pallas/fused_layernorm.py", "ref_fused_layernorm")
    sm = load_ref("kernels/pallas/sparsity_mask.py", "ref_sparsity_mask")
    meta = {"numpy_version": np.__version__}

    # 1. dummy HADS profiles (masks bit-exact) -----------------------------------------
    masks = {}
    cases = [(8, 512, 64, 2, False), (8, 512, 64, 1, False), (4, 256, 64, 2, False),
             (4, 128, 32, 2, False), (12, 1024, 64, 2, True), (12, 1024, 128, 2, True),
             (12, 4096, 64, 2, True), (12, 4096, 128, 2, True), (12, 2048, 64, 2, False)]
    for (H, S, bs, w, causal) in cases:
        p = hp.dummy_hads_profile(H, S, bs, window_size=w, causal=causal)
        key = f"dummy_H{H}_S{S}_bs{bs}_w{w}_c{int(causal)}"
        masks[key + "_mask"] = np.packbits(np.asarray(p.block_masks, bool), axis=-1)
        masks[key + "_shape"] = np.array(np.asarray(p.block_masks).shape)
        masks[key + "_ent"] = np.asarray(p.head_entropies, np.float32)
        masks[key + "_rho"] = np.asarray(p.head_sparsity, np.float32)
    # per-head masks at awkward sparsities straight from _build_head_mask
    for i, (rho, nb, w, seed, causal) in enumerate(
            [(0.0, 16, 2, 0, False), (1.0, 16, 2, 1, True), (0.37, 64, 3, 7, True),
             (0.9, 64, 0, 3, False), (0.5, 5, 1, 11, False), (0.25, 1, 2, 0, True)]):
        masks[f"head_{i}_args"] = np.array([rho, nb, w, seed, int(causal)], np.float64)
        masks[f"head_{i}_mask"] = hp._build_head_mask(rho, nb, w, seed, causal)
    # non-HADS patterns through the reference's make_block_mask
    for st in ["dense", "local", "bigbird"]:
        for causal in (False, True):
            masks[f"pattern_{st}_c{int(causal)}"] = np.asarray(
                sm.make_block_mask(1024, 64, st, causal=causal), bool)

    # 2. entropy -> sparsity ------------------------------------------------------------
    ent_cases = {
        "lin20": np.asarray(_linspace(0.1, 3.0, 20), np.float32),
        "rand12": np.random.default_rng(5).uniform(1.0, 7.0, 12).astype(np.float32),
        "flat4": np.full(4, 2.5, np.float32),
        "near": np.array([3.0, 3.0000002, 3.0000005, 3.1], np.float32),
    }
    e2s = {}
    for name, e in ent_cases.items():
        e2s[f"{name}_in"] = e
        e2s[f"{name}_out"] = np.asarray(hp.entropy_to_sparsity(e), np.float32)
        e2s[f"{name}_out_b"] = np.asarray(hp.entropy_to_sparsity(e, 0.2, 0.7), np.float32)

    # 3. entropy + calibrated profile (focused vs diffuse, test_hads_pattern.py:223-249) -
    rng = np.random.default_rng(7)
    H, S = 8, 128
    focused = _softmax(np.repeat(np.repeat(np.eye(S, dtype=np.float32)[None, None], 2, 0),
                                 H // 2, 1) * np.float32(10.0))
    diffuse = _softmax(rng.standard_normal((2, H // 2, S, S), dtype=np.float32))
    attn = np.concatenate([focused, diffuse], axis=1).astype(np.float32)
    attn2 = _softmax(rng.standard_normal((2, H, S, S), dtype=np.float32) * np.float32(3.0))
    cal = {"attn": attn, "attn2": attn2,
           "entropy_attn": np.asarray(hp.compute_attention_entropy(attn), np.float32),
           "entropy_attn2": np.asarray(hp.compute_attention_entropy(attn2), np.float32)}
    prof = hp.build_hads_profile([attn, attn2], seq_len=S, block_size=16, causal=True)
    cal["profile_ent"] = np.asarray(prof.head_entropies, np.float32)
    cal["profile_rho"] = np.asarray(prof.head_sparsity, np.float32)
    cal["profile_mask"] = np.asarray(prof.block_masks, bool)
    summ = hp.profile_summary(prof)
    cal["summary_keys"] = np.array(sorted(summ))
    cal["summary_vals"] = np.array([summ[k] for k in sorted(summ)], np.float64)

    # 4. sparse_attention_reference ----------------------------------------------------
    rng = np.random.default_rng(11)
    B, H, S, D = 1, 4, 256, 32
    q = rng.standard_normal((B, H, S, D), dtype=np.float32)
    k = rng.standard_normal((B, H, S, D), dtype=np.float32)
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    att = {"q": q, "k": k, "v": v}
    prof64 = hp.dummy_hads_profile(H, S, 64, causal=True)
    m3 = np.asarray(prof64.block_masks, bool)
    m2 = np.asarray(sm.make_block_mask(S, 32, "bigbird", causal=False), bool)
    m4 = m3[None]
    empty = m3.copy()
    empty[1, 2, :] = False         # q-block 2 of head 1 fully masked
    for name, mask, bs, causal in [("hads_c1", m3, 64, True), ("hads_c0", m3, 64, False),
                                   ("bigbird32_c0", m2, 32, False), ("mask4d_c1", m4, 64, True),
                                   ("emptyrow_c1", empty, 64, True), ("dense16_c1",
                                   np.ones((S // 16, S // 16), bool), 16, True)]:
        out, w = sa.sparse_attention_reference(q, k, v, mask, block_size=bs, causal=causal)
        att[f"{name}_mask"] = mask
        att[f"{name}_bs"] = np.array(bs)
        att[f"{name}_out"] = np.asarray(out, np.float32)
        att[f"{name}_wsum"] = np.asarray(w, np.float32).sum(-1)
        att[f"{name}_w_row37"] = np.asarray(w, np.float32)[:, :, 37, :]
    out, _ = sa.sparse_attention(q, k, v, m3, block_size=64, scale=0.3, causal=True)
    att["scale03_out"] = np.asarray(out, np.float32)

    # 5. row kernels (CPU branches) ------------------------------------------------------
    rng = np.random.default_rng(13)
    x = rng.standard_normal((8, 512), dtype=np.float32) * np.float32(2.0)
    xm = x.copy()
    xm[np.arange(512)[None, :] > (np.arange(8) * 60)[:, None]] = -np.inf
    xl = rng.standard_normal((4, 16, 128), dtype=np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    b = (0.1 * rng.standard_normal(128)).astype(np.float32)
    rows = {"sm_x": x, "sm_out": np.asarray(fs.fused_softmax(x, use_pallas=False)),
            "sm_xm": xm, "sm_outm": np.asarray(fs.fused_softmax(xm, use_pallas=False)),
            "ln_x": xl, "ln_g": g, "ln_b": b,
            "ln_out": np.asarray(fl.fused_layernorm(xl, g, b, use_pallas=False)),
            "ln_out_eps": np.asarray(fl.fused_layernorm(xl, g, b, eps=1e-2, use_pallas=False))}

    for fname, d in [("masks", masks), ("entropy_to_sparsity", e2s), ("calibration", cal),
                     ("attention", att), ("rowops", rows)]:
        np.savez_compressed(os.path.join(HERE, f"{fname}.npz"), **d, **{"_" + k: v for k, v in
                                                                          meta.items()})
        print("wrote", fname)


if __name__ == "__main__":
    main()
