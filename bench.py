#!/usr/bin/env python
"""Benchmark of the HADS block-sparse attention forward on B200.

Default workload (one "step" = one forward over one batch):
  bf16 B=4 H=12 S=4096 D=64, 64x64 blocks, HADS masks from dummy_hads_profile (the profile the
  reference's own attention benchmark uses) with causal cut and global KV block 0, per rank.
Metric: effective TFLOP/s over active blocks, 4*D*64*64 FLOPs per active (q-block, kv-block)
pair after the causal cut (n_a), whole job (all ranks).  Multi-GPU: one process per GPU, each
rank runs its own batch of 4 (weak scaling), no collective on the data path; timing is the max
over ranks of CUDA-event time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl xsake|reference]
                    [--workload attn|attn_bwd|calib|train|softmax|layernorm|entropy]

--impl reference times the CPU reference semantics (the NumPy port of
sparse_attention_reference, the reference's own CPU path, dense O(S^2)) on a bounded sample
of the same workload on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, H, S, D, BS = 4, 12, 4096, 64, 64
FLOP_PER_BLOCK = 4 * D * 64 * 64          # QK^T + PV of one 64x64 active tile
L2_BYTES = 126 * 2 ** 20


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops"), d.get("hbm_gbs"), "measured"
    return 1590.0, 6650.0, "fallback"


def _traffic(workload):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(workload)
    return None


# ----------------------------------------------------------------------------- clocks
REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(index), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 3:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                bits = int(parts[2], 16)
            except ValueError:
                continue
            reasons |= {n for b, n in REASONS.items() if bits & b and n != "gpu_idle"}
        os.unlink(self.f.name)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed
def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _init_pg(world, local):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def _barrier(dist):
    if dist is not None:
        dist.barrier()


def _max_over_ranks(x: float, dist):
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, dist):
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- masks / inputs
def hads_masks():
    from xsake_b200 import hads_pattern as hp
    prof = hp.dummy_hads_profile(H, S, BS, causal=True, global_blocks=1)
    return prof.block_masks


def n_active(masks, batch):
    return int(np.tril(masks).sum()) * batch


# ----------------------------------------------------------------------------- reference arm
_TMASK = {}


def cpu_reference_step(q, k, v, masks, h, t):
    """One step of the reference CPU path (sparse_attention_reference: dense scores, token mask,
    softmax, P.V) for the 128 query rows [128t, 128t+128) of head h against all S keys, float32
    NumPy (oracle port).  Returns the active-block FLOPs of those rows."""
    from oracle import attention as oa
    tm = _TMASK.get(h)
    if tm is None:
        tm = _TMASK[h] = oa.token_mask(masks[h], BS, S, True)
    rows = slice(128 * t, 128 * t + 128)
    oa._slice_forward(q[0, h, rows], k[0, h], v[0, h], tm[rows], D ** -0.5, np.float32)
    return int(np.tril(masks[h])[2 * t:2 * t + 2].sum()) * FLOP_PER_BLOCK


def _ref_schedule(i):
    """(head, 128-row tile) of reference step i: heads cycle fastest, tiles advance by a stride
    coprime with S/128 so short runs still sample early and late (short and long) rows."""
    return i % H, (7 * (i // H) + 3) % (S // 128)


def cpu_inputs():
    from oracle import inputs as oi
    q, k, v = oi.qkv(1, H, S, D, seed=oi.SEED_BASE + 3)
    return oi.to_bf16(q).astype(np.float32), oi.to_bf16(k).astype(np.float32), oi.to_bf16(v).astype(np.float32)


def cpu_baseline(masks, budget_s=10.0):
    q, k, v = cpu_inputs()
    cpu_reference_step(q, k, v, masks, 0, 0)
    flops, n, t0 = 0, 0, time.perf_counter()
    while True:
        flops += cpu_reference_step(q, k, v, masks, *_ref_schedule(n))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} tiles of 128 query rows x all 4096 keys of the bf16 B=4 H=12 S=4096 D=64 "
                      f"workload (dense float32 NumPy port of sparse_attention_reference), {dt:.1f} s"}


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    masks = hads_masks()
    q, k, v = cpu_inputs()
    for i in range(args.warmup):
        cpu_reference_step(q, k, v, masks, *_ref_schedule(i))
    flops, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        flops += cpu_reference_step(q, k, v, masks, *_ref_schedule(i))
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    line = {"metric": "HADS attn fwd active-block TFLOP/s (bf16 B=4 H=12 S=4096 D=64)", "value": value,
            "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "hads_attn_fwd_bf16_B4_H12_S4096_D64_block64", "batch_per_rank": B,
                       "heads": H, "seq_len": S, "head_dim": D, "block": BS,
                       "mask": "dummy_hads_profile rho 0.1-0.9, window 2, causal, global block 0",
                       "active_blocks_per_rank": n_active(masks, B),
                       "flops_per_step_per_rank": n_active(masks, B) * FLOP_PER_BLOCK,
                       "parallelism": "reference CPU path on the host cores of rank 0",
                       "step": "128 query rows x 4096 keys of one head, dense float32 (reference CPU path); "
                               "value counts the active-block FLOPs of those rows"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": f"{args.steps} tiles of 128 query rows x 4096 keys, dense float32 "
                                       "NumPy port of sparse_attention_reference"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def run_attention(args, dist, rank, world, local):
    import ctypes as C
    import torch
    from xsake_b200 import _lib, sparse_attention as sa
    from xsake_b200 import _device as dev

    masks = hads_masks()
    cm = sa.compile_block_mask(masks, B, H, S, BS, True)
    set_bytes = 4 * B * H * S * D * 2
    nsets = max(2, math.ceil(3 * L2_BYTES / set_bytes) + 1)
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    sets = []
    tau = torch.linspace(0.25, 4.0, H, device="cuda").view(1, H, 1, 1)
    for _ in range(nsets):
        q = (torch.randn(B, H, S, D, device="cuda", generator=g) * tau).to(torch.bfloat16)
        k = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)
        lse = torch.empty(B, H, S, device="cuda")
        sets.append((q, k, v, o, lse))
    lib = _lib.load()
    desc = sa._desc(sets[0][0], sets[0][1], sets[0][2], sets[0][3], cm, None)
    ws_n = C.c_size_t(0)
    _lib.check(lib.xsake_attn_fwd_workspace_size(C.byref(desc), C.byref(ws_n)))
    ws = torch.empty(max(ws_n.value, 16), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step(i):
        q, k, v, o, lse = sets[i % nsets]
        st = lib.xsake_attn_fwd(C.byref(desc), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                o.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), sp)
        if st:
            _lib.check(st)

    step(0)
    torch.cuda.synchronize()
    assert _lib.device_error(sp) == 0
    clocks = ClockSampler(local)
    time.sleep(0.3)              # the sampler's first readings; the warm-up follows right before timing
    for i in range(args.warmup):
        step(i)
    _barrier(dist)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        ev[2 * i].record(stream)
        step(i)
        ev[2 * i + 1].record(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    _barrier(dist)
    ck = clocks.stop()
    total_ms = e0.elapsed_time(e1)
    kernel_ms = float(np.mean([ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)]))
    assert _lib.device_error(sp) == 0
    total_ms_max = _max_over_ranks(total_ms, dist)

    na = n_active(masks, B)
    flops_rank = na * FLOP_PER_BLOCK
    value = world * flops_rank * args.steps / (total_ms_max * 1e-3) / 1e12
    peak_tf, _, peak_kind = _peaks()
    achieved = flops_rank / (kernel_ms * 1e-3) / 1e12

    # End to end through the public API: pinned host q/k/v -> GPU -> attention -> pinned host
    # out, every step.  Steps alternate between two streams, as a serving loop would issue them,
    # so the upload of step i+1 overlaps the download of step i (the copies are PCIe-bound; the
    # kernel is ~7% of a step).
    e2e_steps = max(3, min(args.steps, 50))
    hq, hk, hv = (t.cpu().pin_memory() for t in sets[0][:3])
    houts = [torch.empty_like(hq).pin_memory() for _ in range(2)]
    e2e_streams = [torch.cuda.Stream(), torch.cuda.Stream()]

    def e2e_step(i):
        with torch.cuda.stream(e2e_streams[i % 2]):
            out = sa.sparse_attention_pallas(hq.cuda(non_blocking=True), hk.cuda(non_blocking=True),
                                             hv.cuda(non_blocking=True), masks, BS, BS, None, True)
            houts[i % 2].copy_(out, non_blocking=True)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    _barrier(dist)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for s_ in e2e_streams:
        s_.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    for s_ in e2e_streams:
        stream.wait_stream(s_)
    a1.record(stream)
    torch.cuda.synchronize()
    _barrier(dist)
    e2e_ms = _max_over_ranks(a0.elapsed_time(a1), dist)
    e2e_value = world * flops_rank * e2e_steps / (e2e_ms * 1e-3) / 1e12

    cpu = cpu_baseline(masks) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    st = cm.stats()
    if rank == 0:
        line = {
            "metric": "HADS attn fwd active-block TFLOP/s (bf16 B=4 H=12 S=4096 D=64)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "hads_attn_fwd_bf16_B4_H12_S4096_D64_block64", "batch_per_rank": B,
                       "heads": H, "seq_len": S, "head_dim": D, "block": BS,
                       "mask": "dummy_hads_profile rho 0.1-0.9, window 2, causal, global block 0",
                       "active_blocks_per_rank": na, "computed_tiles_per_rank": st["computed_tiles"],
                       "flops_per_step_per_rank": flops_rank,
                       "l2": f"{nsets} rotating input sets of {set_bytes / 1e6:.0f} MB (> 126 MB L2)",
                       "parallelism": f"weak, {world} rank(s) x batch {B}, no collective"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "peak_source": f"bf16_tflops ({peak_kind}, burst)",
                         "kernel": "tc_fwd_kernel (unit pairing)", "kernel_ms": kernel_ms, "traffic": _traffic("attn")},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 3 * B * H * S * D * 2, "d2h_bytes_per_step": B * H * S * D * 2,
                    "steps": e2e_steps, "api": "xsake_b200.sparse_attention.sparse_attention_pallas",
                    "streams": 2},
            "gpu_launches": args.steps,
            "clocks": ck,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def run_train(args, dist, rank, world, local):
    """The config-4 training step (a "next" row, not the headline): 12-layer, d=768 XSAKE
    transformer, batch 8 per GPU of uniform random token ids, S=4096, bf16 autocast over fp32
    master weights, fused AdamW; under torch.distributed.run the gradients are all-reduced by
    DDP (NCCL, bucketed and overlapped with the backward).  Value: whole-job tokens/s."""
    import torch
    from xsake_b200.model import ModelConfig, XSAKETransformer, cross_entropy_loss
    cfg = ModelConfig(seq_len=4096, block_size=64)
    torch.manual_seed(1234 + rank)
    model = XSAKETransformer(cfg, device="cuda")
    if dist is not None:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=64)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    Bt, St = 8, cfg.seq_len
    batches = [torch.randint(0, cfg.vocab_size, (Bt, St), device="cuda") for _ in range(2)]
    host = [torch.randint(0, cfg.vocab_size, (Bt, St)).pin_memory() for _ in range(2)]

    def step(ids):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, _ = model(ids)
            loss = cross_entropy_loss(logits, ids)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for i in range(args.warmup):
        step(batches[i % 2])
    torch.cuda.synchronize()
    _barrier(dist)
    clocks = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        loss = step(batches[i % 2])
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), dist) / args.steps
    # end to end: token ids copied from pinned host memory and the loss read back every step
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(2, args.steps // 2)
    _barrier(dist)
    f0.record()
    for i in range(n_e2e):
        ids = host[i % 2].to("cuda", non_blocking=True)
        lv = float(step(ids).detach().cpu())
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1), dist) / n_e2e
    ck = clocks.stop()
    _barrier(dist)
    if rank == 0:
        tokens = world * Bt * St
        line = {"metric": "XSAKE transformer training tokens/s (12L d768 H12, S=4096, batch 8 per GPU)",
                "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "train_xsake_12L_d768_S4096", "global_batch": world * Bt, "seq_len": St,
                           "mask": "uncalibrated HADS profile (dummy_hads_profile), block 64",
                           "optimizer": "AdamW fused, fp32 master weights", "parallelism": f"dp{world}",
                           "loss": float(loss.detach().cpu()), "last_e2e_loss": lv},
                "note": "secondary row; not the headline",
                "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": Bt * St * 8,
                        "d2h_bytes_per_step": 4, "steps": n_e2e},
                "clocks": ck}
        print(json.dumps(line), flush=True)


def run_rowop(args, dist, rank, world, local):
    """Secondary rows (not the headline): softmax / LayerNorm / entropy / attention backward.

    The row kernels are microseconds long, so each is timed as a CUDA graph of 20 direct C-ABI
    calls on preallocated buffers (no Python or allocation between launches); inputs rotate over
    enough buffers to exceed the 126 MB L2."""
    import ctypes as C
    import torch
    from xsake_b200 import _lib, sparse_attention as sa
    lib = _lib.load()
    wl = args.workload
    sp = lambda: torch.cuda.current_stream().cuda_stream
    if wl == "softmax":
        rows, cols = 8 * 12 * 1024, 1024
        x = torch.randn(rows, cols, device="cuda") * 2
        x.masked_fill_(torch.arange(cols, device="cuda")[None] > (torch.arange(rows, device="cuda") % cols)[:, None],
                       float("-inf"))
        y = torch.empty_like(x)
        nbytes = rows * cols * 8
        calls = [lambda: lib.xsake_softmax_fwd(0, rows, cols, x.data_ptr(), y.data_ptr(), sp())]
        unit, metric = "GB/s", "fused softmax fp32 [98304,1024] HBM GB/s"
    elif wl == "layernorm":
        xs = [torch.randn(8192, 768, device="cuda").to(torch.bfloat16) for _ in range(12)]
        g = (1 + 0.1 * torch.randn(768, device="cuda"))
        b = 0.1 * torch.randn(768, device="cuda")
        ys = [torch.empty_like(x) for x in xs]
        nbytes = 8192 * 768 * 4 + 2 * 768 * 4
        calls = [lambda i=i: lib.xsake_layernorm_fwd(1, 8192, 768, xs[i].data_ptr(), g.data_ptr(), b.data_ptr(),
                                                     1e-5, ys[i].data_ptr(), None, None, sp()) for i in range(12)]
        unit, metric = "GB/s", "fused layernorm bf16 [8192,768] HBM GB/s"
    elif wl == "entropy":
        p = torch.softmax(torch.randn(8, 12, 1024, 1024, device="cuda") * 2, -1)
        n = C.c_size_t(0)
        lib.xsake_entropy_workspace_size(8, 12, 1024, C.byref(n))
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        sums = torch.empty(12, dtype=torch.float64, device="cuda")
        nbytes = p.numel() * 4
        calls = [lambda: lib.xsake_entropy_rows(p.data_ptr(), 8, 12, 1024, 1024, sums.data_ptr(), ws.data_ptr(),
                                                ws.numel(), sp())]
        unit, metric = "GB/s", "HADS entropy over materialised P fp32 [8,12,1024,1024] HBM GB/s"
    elif wl == "calib":
        # one config-2 calibration batch: B=8 H=12 S=1024 D=64 fp32, q scaled per head, no mask
        Bc, Hc, Sc, Dc = 8, 12, 1024, 64
        tau = torch.linspace(0.25, 4.0, Hc, device="cuda")
        q = torch.randn(Bc, Hc, Sc, Dc, device="cuda") * tau[None, :, None, None]
        k = torch.randn(Bc, Hc, Sc, Dc, device="cuda")
        n = C.c_size_t(0)
        lib.xsake_entropy_qk_workspace_size(Bc, Hc, Sc, C.byref(n))
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        sums = torch.empty(Hc, dtype=torch.float64, device="cuda")
        nbytes = None
        calls = [lambda: lib.xsake_entropy_qk(0, q.data_ptr(), k.data_ptr(), Bc, Hc, Sc, Dc, 0.125, sums.data_ptr(),
                                              ws.data_ptr(), ws.numel(), sp())]
        # the drop-in path for comparison: materialised weights, then the entropy reduction
        full = np.ones((1, 16, 16), bool)
        cm = sa.compile_block_mask(full, Bc, Hc, Sc, 64, False, q.device)
        dsc = sa._desc(q, k, k, q, cm, 0.125)
        pw = torch.empty(Bc, Hc, Sc, Sc, device="cuda")
        n2 = C.c_size_t(0)
        lib.xsake_entropy_workspace_size(Bc, Hc, Sc, C.byref(n2))
        ws2 = torch.empty(n2.value, dtype=torch.uint8, device="cuda")
        def dropin():
            st = lib.xsake_attn_probs(C.byref(dsc), cm.plan.data_ptr(), q.data_ptr(), k.data_ptr(), pw.data_ptr(), sp())
            return st or lib.xsake_entropy_rows(pw.data_ptr(), Bc, Hc, Sc, Sc, sums.data_ptr(), ws2.data_ptr(),
                                                ws2.numel(), sp())
        unit, metric = "TFLOP/s", "HADS calibration entropy fused from Q,K (fp32, B=8 H=12 S=1024 D=64) TFLOP/s"
    elif wl == "attn_bwd":
        masks = hads_masks()
        # two input sets of 151 MB (q, k, v, o, do bf16 + lse) alternate, so each call reads
        # operands that are not L2-resident from the previous call
        sets = []
        for _ in range(2):
            q, k, v, do = (torch.randn(B, H, S, D, device="cuda").to(torch.bfloat16) for _ in range(4))
            o, lse = sa.attention_forward(q, k, v, masks, BS, None, True)
            sets.append((q, k, v, o, lse, do, torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)))
        cm = sa.compile_block_mask(masks, B, H, S, BS, True, sets[0][0].device)
        d = sa._desc(sets[0][0], sets[0][1], sets[0][2], sets[0][6], cm, None)
        n = C.c_size_t(0)
        _lib.check(lib.xsake_attn_bwd_workspace_size(C.byref(d), C.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device="cuda")
        nbytes = None
        calls = [lambda t=t: lib.xsake_attn_bwd(C.byref(d), cm.plan.data_ptr(), *(x.data_ptr() for x in t),
                                                ws.data_ptr(), ws.numel(), sp()) for t in sets]
        unit, metric = "TFLOP/s", "HADS attn bwd active-block TFLOP/s (bf16 B=4 H=12 S=4096 D=64)"
    else:
        raise SystemExit(f"unknown workload {wl}")
    use_graph = True

    def run_all():
        for i in range(20):
            st = calls[i % len(calls)]()
            if st:
                _lib.check(st)
    for _ in range(args.warmup):
        run_all()
    torch.cuda.synchronize()
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run_all()
        replay = graph.replay
    else:
        replay = run_all
    replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (args.steps * 20)
    extra = {}
    if wl == "attn_bwd":
        value = n_active(hads_masks(), B) * 10 * D * 64 * 64 / (ms * 1e-3) / 1e12
    elif wl == "calib":
        value = 2 * 2 * 8 * 12 * 1024 * 1024 * 64 / (ms * 1e-3) / 1e12
        for _ in range(3):
            _lib.check(dropin())
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(10):
            _lib.check(dropin())
        f1.record()
        torch.cuda.synchronize()
        extra = {"dropin_ms_per_batch": f0.elapsed_time(f1) / 10, "fused_ms_per_batch": ms,
                 "dropin": "xsake_attn_probs (403 MB of fp32 weights) + xsake_entropy_rows"}
    else:
        value = nbytes / (ms * 1e-3) / 1e9
    _, hbm, kind = _peaks()
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps * 20,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "config": {"workload": wl, "timing": "CUDA graph of 20 calls" if use_graph else "eager"},
            "note": "secondary row; not the headline"}
    line.update(extra)
    if wl == "calib":
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        line["roofline"] = {"bound": "fp32 CUDA cores", "achieved": value, "peak": fp32_peak, "unit": "TFLOP/s",
                            "frac": value / fp32_peak,
                            "peak_source": "nominal fp32 FMA rate (148 SMs x 128 lanes x 2 x 1.965 GHz); "
                                           "not in the measured peaks"}
    elif unit == "GB/s":
        line["roofline"] = {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s", "frac": value / hbm,
                            "peak_source": f"hbm_gbs ({kind})"}
    else:
        peak_tf = _peaks()[0]
        line["roofline"] = {"bound": "tensor", "achieved": value, "peak": peak_tf, "unit": "TFLOP/s",
                            "frac": value / peak_tf, "peak_source": f"bf16_tflops ({kind}, burst)",
                            "work": "10 * D * 64 * 64 FLOPs per active block (dQ, dK, dV, dP, S)"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="xsake", choices=["xsake", "reference"])
    ap.add_argument("--workload", default="attn", choices=["attn", "attn_bwd", "calib", "train", "softmax", "layernorm", "entropy"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
        return
    world, rank, local = _dist()
    dist = _init_pg(world, local)
    try:
        if args.workload == "attn":
            run_attention(args, dist, rank, world, local)
        elif args.workload == "train":
            run_train(args, dist, rank, world, local)
        else:
            run_rowop(args, dist, rank, world, local)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
