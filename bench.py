#!/usr/bin/env python
"""Benchmark of the fused NeRF training step (BASELINE metric: trained samples/s, fwd+bwd+Adam).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg3|cfg2|cfg1] [--impl reference]

Default workload cfg3: 16384 rays x 64 samples = 2^20 samples per step, split by ray across the
N ranks (strong scaling), hash grid L=16 F=2 T=2^19 fp32, finest resolution 2048, density MLP
32-64-16, colour MLP 32-64-64-3, occupancy grid 128^3 in a warmed-up state (~5% of sub-cells
occupied, proposals on, maintenance every 32 steps), on the seeded 56-camera 450x800 Gaussian
blob scene (synthetic data: rays through random pixels, targets rendered analytically and
quantised to 8 bits).  Every step is the full training step: forward, backward, MLP Adam and the
hash-table SGD update -- on one GPU applied inside the fused kernel as the reference does
(Hogwild), on N GPUs by the fused exchange kernel (cross-rank gradient sum, table SGD of each
rank's shard and broadcast of the new table over NVLink peer memory, or NVSwitch multicast from 4
ranks up).  The MLPs run on the tensor cores (--mlp fp16, the default): fp16 operand pairs with
fp32 accumulation (a compensated hi/lo forward, fp16 backward operands); the table is fp32.
--mlp fp32 runs the CUDA-core fp32 MLP instead.  L2 is flushed between timed steps; ``l2_warm``
repeats the steps back to back without the flush.

For N > 1 run under torchrun (one process per GPU, NCCL).  Rank 0 prints one JSON line:
  value       -- samples/s of the whole job, inputs resident on the device, CUDA events, max
                 over ranks;
  e2e         -- the same through the public API (ffnerf_tools.RayBatch uploads from pinned host
                 memory, Nerf.step, non-blocking read-back of the rendered colours) per step, the
                 steps pipelined as a user runs them (the host takes step i's colours after
                 enqueueing step i+1) and bracketed by one pair of events, L2 flushes included;
  roofline    -- the fused forward/backward kernel: algorithmic bytes per launch / its average
                 duration (CUDA events on its stream) against the measured HBM copy bandwidth;
  cpu_baseline-- the reference kernels compiled for the CPU (oracle/_ref) on the host cores.
``--impl reference`` times the reference's own kernels compiled for the CPU (oracle/_ref) on the
same workload -- the same batches, occupancy grid, initial parameters and schedules -- on all host
cores (rank 0 only) and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ffnerf-experimental_b200"))

import numpy as np

METRIC = "train samples/s (fwd+bwd+Adam)"
WORKLOADS = {
    "cfg3": dict(rays=16384, spr=64, F=2, ND=1, NC=2, log2T=19, rmax=2048.0, G=128, n_cams=56, W=800, H=450,
                 maint=32, desc="cfg3: 16384 rays x 64 samples (2^20 samples/step) split by ray across GPUs; "
                                "hash L=16 F=2 T=2^19 fp32 replicated, Rmax 2048; MLP 32-64-16 / 32-64-64-3; "
                                "occupancy 128^3 ~5% occupied; 56-camera 450x800 synthetic blob scene"),
    "cfg2": dict(rays=512, spr=64, F=2, ND=1, NC=2, log2T=19, rmax=2048.0, G=128, n_cams=56, W=800, H=450,
                 maint=16, desc="cfg2: 512 rays x 64 samples; hash L=16 F=2 T=2^19, Rmax 2048; occupancy 128^3, "
                                "maintenance every 16 steps; 56-camera 450x800 synthetic blob scene"),
    "cfg1": dict(rays=512, spr=64, F=2, ND=1, NC=2, log2T=14, rmax=512.0, G=64, n_cams=8, W=64, H=64,
                 maint=32, desc="cfg1: 512 rays x 64 samples; hash L=16 F=2 T=2^14, Rmax 512; occupancy 64^3; "
                                "8 cameras at 64x64"),
}
# Kernel microbenchmarks (BASELINE configs 4 and 5): one JSON line each, own metric.
MICRO = {
    "cfg4": dict(kind="hash", points=1 << 22, F=2, log2T=19, rmax=2048.0,
                 desc="cfg4: hash encode fwd+bwd, 2^22 points U[0,1]^3, L=16 F=2 T=2^19 fp32 table, "
                      "upstream grads N(0,1) [2^22, 32] fp32"),
    "cfg4-T22": dict(kind="hash", points=1 << 22, F=2, log2T=22, rmax=2048.0,
                     desc="cfg4: hash encode fwd+bwd, 2^22 points U[0,1]^3, L=16 F=2 T=2^22 fp32 table, "
                          "upstream grads N(0,1) [2^22, 32] fp32"),
    "cfg4-f16": dict(kind="hash", points=1 << 22, F=2, log2T=19, rmax=2048.0, table="f16",
                     desc="cfg4: hash encode fwd+bwd, 2^22 points U[0,1]^3, L=16 F=2 T=2^19 fp16 table "
                          "(fp16 encoding out), upstream grads N(0,1) [2^22, 32] fp32"),
    "cfg4-T22-f16": dict(kind="hash", points=1 << 22, F=2, log2T=22, rmax=2048.0, table="f16",
                         desc="cfg4: hash encode fwd+bwd, 2^22 points U[0,1]^3, L=16 F=2 T=2^22 fp16 table "
                              "(fp16 encoding out), upstream grads N(0,1) [2^22, 32] fp32"),
    "cfg5-mlp": dict(kind="mlp", n=1 << 22, desc="cfg5: density (32-64-16) and colour (32-64-64-3) MLPs forward and "
                                                  "backward with weight gradients on 2^22 samples of N(0,1) fp16 inputs, "
                                                  "fp16 operands / fp32 accumulation"),
    "cfg5-adam": dict(kind="adam", n=1 << 24, desc="cfg5: Adam over 2^24 fp32 parameters, grads N(0,1e-3), "
                                                    "beta1 0.9 beta2 0.99 eps 1e-15 lr 1e-2"),
}


def hash_bytes_per_point(F: int, s_tab: int = 4):
    """Algorithmic bytes per point for table entries of s_tab bytes per feature (4: fp32, 2: fp16;
    the encoding is written in the table's type): forward = xyz + 16 levels x 8 corners x F x s_tab
    gathered + 16 F x s_tab written; backward = xyz + 16 F x 4 B fp32 upstream + 16 x 8 x F x s_tab
    atomic read-modify-write (fp32: 1164 / 2188 B at F=2; fp16: 588 / 1164 B)."""
    gather = 16 * 8 * F * s_tab
    return 12 + gather + 16 * F * s_tab, 12 + 16 * F * 4 + 2 * gather


MLP_FLOP_PER_SAMPLE = 56448   # forward 18,816 (6,144 density + 12,672 colour) x 3 with the backward


def run_mlp_micro(args, wl, dev, st, gen, timed) -> dict:
    """cfg5's MLP half on the tensor cores over 2^22 packed fp16 inputs: the headline is the plain
    fp16-operand form (ffn_mlp_bench_f16: the configuration's fp16 inputs, fp32 accumulation, one MMA
    per product); `compensated` is the training step's form (ffn_mlp_bench: every product from fp16
    operand pairs), timed the same way."""
    import torch
    import ffn_native as fn
    from ffn_config import make_geometry, param_layout, param_shapes
    hbm, tflops_peak, peak_kind = peaks()
    g = make_geometry(F=2, ND=1, NC=2, spr=64, G=16, log2_entries=12, rmax=512.0)
    ctx = fn.Context(g, device=0, mlp_precision="fp16")
    lay, total = param_layout(2, 1, 2)
    shapes = param_shapes(2, 1, 2)
    rng = np.random.default_rng(0)
    blob = np.zeros(total, np.float32)
    for name, (off, size) in lay.items():          # He-normal hidden layers, N(0, 0.01) heads, zero biases
        if size and name.startswith("W"):
            out_, in_ = shapes[name]
            blob[off:off + size] = rng.normal(0.0, 0.01 if out_ <= 16 else np.sqrt(2.0 / in_), size)
    ctx.tensor(fn.BUF_PARAMS).copy_(torch.from_numpy(blob))
    n = wl["n"]
    x16 = torch.randn((n, 32), device=dev, generator=gen).half()
    tiles = torch.empty(ctx.x0_tile_bytes(n), dtype=torch.uint8, device=dev)
    ctx.pack_x0(x16, tiles, n, stream=st)
    step = lambda: ctx.mlp_bench_f16(tiles, n, stream=st)       # noqa: E731
    step_cp = lambda: ctx.mlp_bench(tiles, n, stream=st)        # noqa: E731
    for _ in range(args.warmup):
        with torch.cuda.stream(st):
            step()
            step_cp()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    with ClockSampler(0) as clk:
        (t,) = timed([step], flush=False)             # inputs (268 MB) exceed L2
        launches = ctx.launches - launches0
        h_x = x16.cpu().pin_memory()
        h_g = torch.empty(total).pin_memory()

        def e2e():
            x16.copy_(h_x, non_blocking=True)
            ctx.pack_x0(x16, tiles, n, stream=st)
            step()
            h_g.copy_(ctx.tensor(fn.BUF_GRADS)[-total:], non_blocking=True)
        (t_e2e,) = timed([e2e], flush=False)
        (t_cp,) = timed([step_cp], flush=False)
    ms = t / args.steps
    ms_cp = t_cp / args.steps
    tf_cp = MLP_FLOP_PER_SAMPLE * n / (ms_cp * 1e-3) / 1e12
    tf = MLP_FLOP_PER_SAMPLE * n / (ms * 1e-3) / 1e12
    # CPU: the same MLP forward/backward in fp32 with torch on the host cores, a bounded sample
    m = 1 << 16
    xc = x16[:m].float().cpu()
    P = {k: torch.tensor(blob[o:o + s].reshape(shapes[k]), requires_grad=True) for k, (o, s) in lay.items() if s}
    sh = torch.tensor([0.28209479177387814] + [0.0] * 15).expand(m, 16)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < 5.0:
        h1 = torch.relu(xc @ P["Wd_in"].T + P["bd_0"])
        dout = h1 @ P["Wd_out"].T + P["bd_out"]
        c1 = torch.relu(torch.cat([dout, sh], 1) @ P["Wc_in"].T + P["bc_0"])
        c2 = torch.relu(c1 @ P["Wc_01"].T + P["bc_1"])
        rgb = torch.sigmoid(0.5 * (c2 @ P["Wc_out"].T + P["bc_out"]))
        (0.5 * (rgb - 0.5) ** 2).sum().backward()
        reps += 1
    cpu_tf = MLP_FLOP_PER_SAMPLE * m * reps / (time.perf_counter() - t0) / 1e12
    ctx.close()
    return {
        "metric": "MLP TFLOP/s (fwd+bwd+weight gradients, 56,448 flop/sample)", "value": tf, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f16 operands, f32 accumulation", "data": "synthetic",
        "config": {"workload": wl["desc"], "samples": n, "l2": "inputs (268 MB) exceed L2; no flush"},
        "e2e": {"value": MLP_FLOP_PER_SAMPLE * n / (t_e2e / args.steps * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": n * 64, "d2h_bytes_per_step": total * 4},
        "gpu_launches": launches,
        "compensated": {"value": tf_cp, "unit": "TFLOP/s", "ms_per_step": ms_cp, "frac": tf_cp / tflops_peak,
                        "note": "the training step's form: every product from compensated fp16 operand pairs "
                                "(three MMAs per counted product, lo tiles stored by every epilogue)"},
        "roofline": {"bound": "tensor", "kernel": "fused_step_tc_kernel<2,1,staged,mlp,plain> + reduce_partials",
                     "achieved": tf, "peak": tflops_peak, "unit": "TFLOP/s", "frac": tf / tflops_peak,
                     "traffic": None, "peak_source": peak_kind,
                     "note": "peak = measured cuBLAS bf16 burst; the MLP is 128-row tiles of 32-64 wide layers"},
        "clocks": clk.summary(),
        "cpu_baseline": {"value": cpu_tf, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{m} samples fwd+bwd in fp32 with torch on the host, repeated for 5 s"},
    }


def run_micro(args, name: str) -> dict:
    import torch
    import ffn_native as fn
    from ffn_config import make_geometry
    wl = MICRO[name]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    st = torch.cuda.Stream()
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    hbm, _, peak_kind = peaks()

    def timed(fns, flush=True):
        """Per-iteration CUDA events on stream st around each callable; L2 flushed before each."""
        sums = [0.0] * len(fns)
        for _ in range(args.steps):
            with torch.cuda.stream(st):
                if flush:
                    flush_buf.zero_()
                for k, f in enumerate(fns):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(st)
                    f()
                    b.record(st)
                    torch.cuda.synchronize()
                    sums[k] += a.elapsed_time(b)
        return sums

    if wl["kind"] == "hash":
        g = make_geometry(F=wl["F"], ND=1, NC=2, spr=64, G=16, log2_entries=wl["log2T"], rmax=wl["rmax"])
        ctx = fn.Context(g, device=0)
        n = wl["points"]
        f16 = wl.get("table") == "f16"
        s_tab = 2 if f16 else 4
        ctx.tensor(fn.BUF_TABLE).uniform_(-1e-4, 1e-4, generator=gen)
        pts = torch.rand((n, 3), device=dev, generator=gen)
        enc = torch.empty((n, 16 * wl["F"]), device=dev, dtype=torch.float16 if f16 else torch.float32)
        denc = torch.randn((n, 16 * wl["F"]), device=dev, generator=gen)
        if f16:
            table16 = ctx.tensor(fn.BUF_TABLE).half()
            grad16 = torch.zeros_like(table16)
            fwd = lambda: ctx.hash_encode_f16(table16, pts, enc, n, stream=st)       # noqa: E731
            bwd = lambda: ctx.hash_encode_bwd_f16(grad16, pts, denc, n, stream=st)   # noqa: E731
        else:
            fwd = lambda: ctx.hash_encode(pts, enc, n, stream=st)            # noqa: E731
            bwd = lambda: ctx.hash_encode_bwd(pts, denc, n, stream=st)       # noqa: E731
        for _ in range(args.warmup):
            with torch.cuda.stream(st):
                fwd(); bwd()
        torch.cuda.synchronize()
        with ClockSampler(0) as clk:
            t_fwd, t_bwd = timed([fwd, bwd])
            # end to end: pinned-host points and upstream grads in, encoding out, every iteration
            h_pts = pts.cpu().pin_memory()
            h_denc = denc.cpu().pin_memory()
            h_enc = torch.empty(enc.shape, dtype=enc.dtype).pin_memory()

            def e2e():
                pts.copy_(h_pts, non_blocking=True)
                denc.copy_(h_denc, non_blocking=True)
                fwd(); bwd()
                h_enc.copy_(enc, non_blocking=True)
            (t_e2e,) = timed([e2e])
        ceil = random_access_ceiling(g["table_entries"] * wl["F"] * s_tab, 16 * 8 * n, dev, st)
        bf, bb = hash_bytes_per_point(wl["F"], s_tab)
        gbs_f = bf * n / (t_fwd / args.steps * 1e-3) / 1e9
        gbs_b = bb * n / (t_bwd / args.steps * 1e-3) / 1e9
        gbs = (bf + bb) * n / ((t_fwd + t_bwd) / args.steps * 1e-3) / 1e9
        e2e_gbs = (bf + bb) * n / (t_e2e / args.steps * 1e-3) / 1e9
        # CPU: the oracle's hash encode / scatter on a bounded sample (one thread)
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as orc
        o = orc.Oracle()
        m = 1 << 15
        table_h = ctx.tensor(fn.BUF_TABLE).cpu().numpy()
        p_h, d_h = pts[:m].cpu().numpy(), denc[:m].cpu().numpy()
        e_h, tg_h = np.zeros((m, 16 * wl["F"]), np.float32), np.zeros_like(table_h)
        cfg = orc.make_orc_config(g)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 10.0:
            o.hash_fwd(cfg, table_h, p_h, e_h)
            o.hash_bwd(cfg, p_h, d_h, tg_h)
            reps += 1
        bf32, bb32 = hash_bytes_per_point(wl["F"])          # the oracle works on an fp32 table
        cpu_gbs = (bf32 + bb32) * m * reps / (time.perf_counter() - t0) / 1e9
        ctx.close()
        line = {
            "metric": "hash-grid GB/s (encode fwd+bwd, algorithmic bytes)", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": (t_fwd + t_bwd) / args.steps, "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "f16 table, f32 accumulation" if f16 else "f32", "data": "synthetic",
            "config": {"workload": wl["desc"], "points": n, "l2": "flushed between iterations (256 MB write)",
                       "table_bytes": g["table_entries"] * wl["F"] * s_tab},
            "fwd": {"ms": t_fwd / args.steps, "GB/s": gbs_f, "points/s": n / (t_fwd / args.steps * 1e-3),
                    "bytes_per_point": bf},
            "bwd": {"ms": t_bwd / args.steps, "GB/s": gbs_b, "points/s": n / (t_bwd / args.steps * 1e-3),
                    "bytes_per_point": bb},
            "e2e": {"value": e2e_gbs, "unit": "GB/s", "h2d_bytes_per_step": n * (12 + 16 * wl["F"] * 4),
                    "d2h_bytes_per_step": n * 16 * wl["F"] * s_tab},
            "gpu_launches": args.steps * 2,
            "roofline": {"bound": "hbm" if g["table_entries"] * wl["F"] * s_tab > 100e6 else "l2",
                         "kernel": "hash_fwd_f16_kernel + hash_bwd_f16_kernel" if f16
                         else "hash_fwd_kernel + hash_bwd_kernel", "achieved": gbs, "peak": hbm,
                         "unit": "GB/s", "frac": gbs / hbm, "traffic": None, "peak_source": peak_kind,
                         "note": "peak = measured HBM copy bandwidth; random 8 B gathers move 32 B sectors"},
            "achievable": {
                "what": "fully random 8-byte accesses over a buffer of the table's size (ffn_probe_random_access: "
                        "float2 loads on the read-only path / red.global.add.v2.f32), 8 in flight per thread",
                "gather_ops_per_s": ceil["gather_ops_per_s"], "red_ops_per_s": ceil["red_ops_per_s"],
                "fwd_gathers_per_s": 128 * n / (t_fwd / args.steps * 1e-3),
                "fwd_frac": 128 * n / (t_fwd / args.steps * 1e-3) / ceil["gather_ops_per_s"],
                "bwd_reds_per_s": 128 * n / (t_bwd / args.steps * 1e-3),
                "bwd_frac": 128 * n / (t_bwd / args.steps * 1e-3) / ceil["red_ops_per_s"],
                "note": "16 levels x 8 corners = 128 random accesses per point each way; coarse levels share "
                        "cells between points, so a kernel can exceed the fully random rate"},
            "clocks": clk.summary(),
            "cpu_baseline": {"value": cpu_gbs, "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"{m} points fwd+bwd, oracle restatement (fp32 table; its GB/s counts "
                                       f"fp32 bytes), repeated for 10 s"},
        }
        return line
    if wl["kind"] == "mlp":
        return run_mlp_micro(args, wl, dev, st, gen, timed)
    # Adam
    n = wl["n"]
    p = torch.randn(n, device=dev, generator=gen)
    gr = torch.randn(n, device=dev, generator=gen) * 1e-3
    m_ = torch.zeros(n, device=dev)
    v_ = torch.zeros(n, device=dev)
    step = lambda: fn.adam(p, gr, m_, v_, n, 1e-2, 0.9, 0.99, 1e-15, stream=st)   # noqa: E731
    for _ in range(args.warmup):
        with torch.cuda.stream(st):
            step()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        (t,) = timed([step], flush=False)
        h_g = gr.cpu().pin_memory()
        h_p = torch.empty(n).pin_memory()

        def e2e():
            gr.copy_(h_g, non_blocking=True)
            step()
            h_p.copy_(p, non_blocking=True)
        (t_e2e,) = timed([e2e], flush=False)
    gbs = 28 * n / (t / args.steps * 1e-3) / 1e9
    # CPU: numpy Adam on a bounded slice (same update, vectorised, one thread)
    mm = 1 << 22
    ph, gh = p[:mm].cpu().numpy(), gr[:mm].cpu().numpy()
    mh, vh = np.zeros(mm, np.float32), np.zeros(mm, np.float32)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < 5.0:
        mh = 0.9 * mh + 0.1 * gh
        vh = 0.99 * vh + 0.01 * gh * gh
        ph -= 1e-2 * mh / (np.sqrt(vh) + 1e-15)
        reps += 1
    cpu_gbs = 28 * mm * reps / (time.perf_counter() - t0) / 1e9
    return {
        "metric": "Adam GB/s (28 B per parameter)", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl["desc"], "params": n, "l2": "working set 470 MB exceeds L2; no flush"},
        "e2e": {"value": 28 * n / (t_e2e / args.steps * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * n,
                "d2h_bytes_per_step": 4 * n},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "kernel": "adam_kernel", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "traffic": None, "peak_source": peak_kind},
        "clocks": clk.summary(),
        "cpu_baseline": {"value": cpu_gbs, "unit": "GB/s", "cores": 1, "kind": "port",
                         "sample": f"numpy Adam over {mm} parameters, repeated for 5 s"},
    }
# Algorithmic bytes per sample of the fused forward/backward kernel (F=2): trilinear gather
# 16 levels x 8 corners x F x 4 B, atomic scatter read+write of the same, ray/target/colour I/O
# (64 B per ray / spr) and one occupancy word per sample.
def fused_bytes_per_sample(F: int, spr: int) -> float:
    gather = 16 * 8 * F * 4
    return gather + 2 * gather + 64.0 / spr + 4


def random_access_ceiling(table_bytes: int, n_ops: int, dev, st, reps: int = 5) -> dict:
    """Achievable rates of fully random 8-byte loads and vector reductions over a buffer of
    table_bytes (ffn_probe_random_access): median of reps launches of n_ops each, CUDA events on st."""
    import torch
    import ffn_native as fn
    buf = torch.zeros(max(table_bytes // 4, 4), dtype=torch.float32, device=dev)
    out = {}
    for mode, name in ((fn.PROBE_GATHER, "gather"), (fn.PROBE_RED, "red")):
        with torch.cuda.stream(st):
            fn.probe_random_access(buf, mode, n_ops, seed=7, stream=st)
        ms = []
        for r in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            with torch.cuda.stream(st):
                fn.probe_random_access(buf, mode, n_ops, seed=11 + r, stream=st)
            b.record(st)
            torch.cuda.synchronize()
            ms.append(a.elapsed_time(b))
        out[name + "_ops_per_s"] = n_ops / (statistics.median(ms) * 1e-3)
        out[name + "_ms"] = statistics.median(ms)
    out["table_bytes"] = int(table_bytes)
    out["ops"] = int(n_ops)
    del buf
    return out


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ shared inputs
BATCH_POOL = 4          # global batches drawn once and cycled through the steps
BASE_LR = 5e-5 * 8      # base learning rate of the timed steps (schedules.lr_schedule)
START_STEP = 3000       # steps_trained before the first step: the schedules' steady state


def build_inputs(wl: dict, n_glob: int, rank: int, world: int, device):
    """The workload's synthetic batches and occupancy grid, the same on both arms: BATCH_POOL global
    batches of n_glob rays through random pixels of the seeded scene's cameras (targets rendered by
    quadrature, quantised to 8 bits), this rank's contiguous slice of each; the scene's occupancy
    grid with ~5% of sub-cells occupied."""
    import torch
    from synthetic_scene import BlobScene, cameras_ring, cameras_sphere, intrinsics, pixel_rays
    scene = BlobScene(0)
    cams = cameras_ring(wl["n_cams"], 2.5, 0) if wl["n_cams"] > 8 else cameras_sphere(wl["n_cams"], 2.0, 0)
    K = intrinsics(wl["W"], wl["H"], 50.0)
    n_loc = n_glob // world
    rng = np.random.default_rng(1234)
    pool_rays, pool_tg = [], []
    for _ in range(BATCH_POOL):
        ci = rng.integers(0, cams.shape[0], n_glob)
        u = rng.integers(0, wl["W"], n_glob)
        v = rng.integers(0, wl["H"], n_glob)
        rays = np.zeros((n_glob, 8), np.float32)
        for c in np.unique(ci):
            sel = ci == c
            rays[sel] = pixel_rays(cams[c], K, u[sel], v[sel])
        rays_t = torch.from_numpy(rays).to(device)
        rgb = scene.render_torch(rays_t, n_quad=192)
        tg = torch.zeros((n_glob, 4), device=device)
        tg[:, :3] = torch.round(rgb * 255.0) / 255.0
        sl = slice(rank * n_loc, (rank + 1) * n_loc)
        pool_rays.append(rays_t[sl].contiguous())
        pool_tg.append(tg[sl].contiguous())
    return pool_rays, pool_tg, scene.occupancy_grid_torch(wl["G"], device)


def reference_init(g: dict, seed: int = 777):
    """Fresh parameters with the reference's draws in the reference's order (Nerf._init_fresh,
    ffnerf_tools.py:836-898), as the public host class makes them for our arm: table U(-1e-4, 1e-4),
    weights N(0, 0.01) for heads of <= 16 outputs else He N(0, sqrt(2/fan_in)), biases 0 except
    bd_out[0] = -2.  Returns (param blob, table, the generator -- it draws the per-step seeds next)."""
    from ffn_config import param_layout, param_shapes
    rng = np.random.default_rng(seed)
    lay, total = param_layout(g["F"], g["ND"], g["NC"])
    shapes = param_shapes(g["F"], g["ND"], g["NC"])
    table = rng.uniform(-1e-4, 1e-4, size=g["table_entries"] * g["F"]).astype(np.float32)
    blob = np.zeros(total, np.float32)
    for name in ("Wd_in", "Wd_01", "Wd_12", "Wd_out", "Wc_in", "Wc_01", "Wc_12", "Wc_23", "Wc_out"):
        if name not in shapes:
            continue
        sh = shapes[name]
        std = 0.01 if sh[0] <= 16 else np.sqrt(2.0 / int(sh[1]))
        off, size = lay[name]
        blob[off:off + size] = rng.normal(0.0, std, size=sh).astype(np.float32).reshape(-1)
    blob[lay["bd_out"][0]] = -2.0
    return blob, table, rng


# ------------------------------------------------------------------------------ reference arm
def run_reference_arm(args, wl, n_rays: int | None = None, steps: int | None = None, warmup: int | None = None) -> dict:
    """The reference's own kernels, compiled for the CPU from their sources (oracle/_ref), timed on
    all host cores on the same workload as our arm: the same batches (n_rays of each, default the
    whole global batch), occupancy grid, initial parameters, per-step seeds and schedules, and the
    reference's step order (fused kernel, occupancy decay every 32nd step, weight update + Adam).
    The oracle port stands in when the compiled reference is absent."""
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    import schedules as sch
    from ffn_config import make_geometry, param_layout, param_shapes
    g = make_geometry(F=wl["F"], ND=wl["ND"], NC=wl["NC"], spr=wl["spr"], G=wl["G"], log2_entries=wl["log2T"],
                      rmax=wl["rmax"], dt_min=2.0 / 8192, dt_max=12.8 / wl["spr"] / 6 * 2.0)
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    n_glob, spr = wl["rays"], wl["spr"]
    n_rays = n_glob if n_rays is None else min(n_rays, n_glob)
    pool_rays, pool_tg, occ_grid = build_inputs(wl, n_glob, 0, 1, "cpu")
    rays_pool = [r[:n_rays].numpy().copy() for r in pool_rays]
    tg_pool = [t[:n_rays].numpy().copy() for t in pool_tg]
    blob, table, rng = reference_init(g)
    occ_in, occ_st = occ_grid.copy(), occ_grid.copy()
    lay, total = param_layout(g["F"], g["ND"], g["NC"])
    variant = {"cfg3": "cfg3", "cfg2": "cfg3", "cfg1": "cfg1"}[args.workload]
    kind = "reference"
    try:
        ref = orc.RefKernels(variant)
    except (FileNotFoundError, OSError):
        ref, kind = None, "port"
    lmbda = sch.lr_lambda(1e-4, n_glob, spr)
    b1, b2 = np.float32(0.9), np.float32(0.999)
    state = {"t": START_STEP}
    out = np.zeros((n_rays, 4), np.float32)
    if ref is not None:
        shapes = param_shapes(g["F"], g["ND"], g["NC"])
        params = {n: (blob[o:o + s].view(np.int32).copy() if n in shapes else np.zeros(0, np.int32))
                  for n, (o, s) in lay.items()}
        m = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
        v = {k: np.zeros(v.size, np.float32) for k, v in params.items()}
        scr = ref.alloc_scratch(n_rays * spr)
        table_i = table.view(np.int32)

        def step(i):
            lr_f = sch.lr_schedule(state["t"], BASE_LR, lmbda, n_glob, spr)
            seed = int(np.uint32(rng.integers(0, 2**32, dtype=np.uint32)))
            state["t"] += 1
            t = np.float32(state["t"])
            lr_t = float(np.float32(lr_f) * np.sqrt(1.0 - b2 ** t) / (1.0 - b1 ** t))
            b = i % BATCH_POOL
            ref.train(params, table_i, rays_pool[b], tg_pool[b], out, scr, occ_in, occ_st, g, float(lr_f), 1.0, 1.0,
                      seed, True, cores)
            if state["t"] % 32 == 0:
                ref.decay(occ_in, occ_st, 15099494, seed)
            ref.weight_update(params, m, v, scr, n_rays * spr, lr_t, 1.0, 0.9, 0.999, 1e-6, cores)
    else:
        o_ = orc.Oracle()
        cfg = orc.make_orc_config(g)
        m, v = np.zeros_like(blob), np.zeros_like(blob)
        tgr, mg = np.zeros_like(table), np.zeros_like(blob)
        cores = 1

        def step(i):
            lr_f = sch.lr_schedule(state["t"], BASE_LR, lmbda, n_glob, spr)
            seed = int(np.uint32(rng.integers(0, 2**32, dtype=np.uint32)))
            state["t"] += 1
            t = np.float32(state["t"])
            lr_t = np.float32(np.float32(lr_f) * np.sqrt(1.0 - b2 ** t) / (1.0 - b1 ** t))
            b = i % BATCH_POOL
            tgr[:] = 0
            o_.forward_backward(cfg, orc.OrcStep(lr_f, 1.0, 1.0, seed, 1, 0), blob, table, occ_in, occ_st,
                                rays_pool[b], tg_pool[b], out, tgr, mg)
            if state["t"] % 32 == 0:
                o_.decay(occ_in, occ_st, 15099494, seed)
            o_.mlp_adam(cfg, blob, mg, m, v, lr_t, 1.0, b1, b2, np.float32(1e-6))
            o_.table_apply(cfg, table, tgr, lr_f)
    for i in range(warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(steps):
        step(warmup + i)
    dt = time.perf_counter() - t0
    samples = n_rays * spr * steps
    val = samples / dt
    same = n_rays == n_glob
    sample_desc = (f"{'the whole global batch' if same else 'a bounded sample'}: {n_rays} rays x {spr} samples per "
                   f"step ({n_rays * spr} of the workload's {n_glob * spr}), {steps} timed steps after {warmup}; "
                   f"fused step + occupancy decay + weight update + Adam on the workload's batches, occupancy "
                   f"grid, initial parameters and schedules")
    return {"metric": METRIC, "value": val, "unit": "samples/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": dt / steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": {"workload": wl["desc"], "global_batch_rays": n_glob, "samples_per_ray": spr,
                                            "samples_per_step": n_glob * spr, "rays_timed_per_step": n_rays},
            "cpu_baseline": {"value": val, "unit": "samples/s", "cores": cores, "kind": kind, "sample": sample_desc},
            "e2e": {"value": val, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_baseline_sample(args, wl) -> dict:
    """A bounded run (~10-20 s) of the reference kernels compiled for the CPU: the whole global
    batch, 3 timed steps after 1."""
    class A:
        pass
    a = A()
    a.gpus, a.workload = 1, args.workload
    r = run_reference_arm(a, WORKLOADS[args.workload], steps=3, warmup=1)
    return r["cpu_baseline"]


# ------------------------------------------------------------------------------ our arm
def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(MICRO), default="cfg3")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end loop (profiling runs)")
    ap.add_argument("--rays", type=int, default=0, help="override the global batch (profiling a small case)")
    ap.add_argument("--mlp", choices=["fp16", "fp32"], default="fp16",
                    help="MLP arithmetic: fp16 operands / fp32 accumulation on the tensor cores, or fp32 CUDA cores")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in MICRO:
        if int(os.environ.get("RANK", "0")) == 0:
            if args.impl == "reference":
                print(json.dumps({"impl": "reference", "unavailable": "kernel microbenchmark: the reference has no "
                                  "standalone kernel for it; the CPU figure is in this arm's cpu_baseline"}), flush=True)
            else:
                print(json.dumps(run_micro(args, args.workload)), flush=True)
        return
    wl = dict(WORKLOADS[args.workload])
    if args.rays:
        wl["rays"] = int(args.rays)
        wl["desc"] += f" [reduced to {args.rays} rays per step]"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and not (world == 1 and args.gpus == 1):
        if world == 1:
            sys.exit(f"--gpus {args.gpus} needs torchrun with {args.gpus} processes")

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference_arm(args, wl)), flush=True)
        return

    import torch
    import ffn_native
    import ffnerf_tools as ft
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    # ---- synthetic data: a pool of global batches (same on every rank) and the occupancy grid
    n_glob, spr = wl["rays"], wl["spr"]
    n_loc = n_glob // world
    pool = BATCH_POOL
    pool_rays, pool_tg, occ_grid = build_inputs(wl, n_glob, rank, world, dev)

    # ---- the model through the public host API
    ctx = ft.Context([ft.Device(local)])
    queue = ft.CommandQueue(ctx)
    occ = ft.OccParams(G_occ=wl["G"], box_min=np.array([-1, -1, -1], np.float32), box_max=np.array([1, 1, 1], np.float32),
                       rho_min=np.float32(1.0), rho_max=np.float32(16.0), dt_min=np.float32(2.0 / 8192),
                       dt_max=np.float32(12.8 / spr / 6 * 2.0), t_near_clip=np.float32(0.3),
                       t_far_clip=np.float32(1e9), occ_update_strength0=np.float32(1.0)).finalize()
    tmp = tempfile.mkdtemp(prefix="ffn_bench_")

    def make_nerf(mlp_precision: str):
        m = ft.Nerf(ctx, queue, training_dir=tmp, model_id="bench", transfer_fmt="fp32",
                    table_size_entries=16 << wl["log2T"], f_per_level=wl["F"], occ=occ, rng_seed=777,
                    background="random", finest_resolution=wl["rmax"], nd=wl["ND"], nc=wl["NC"],
                    mlp_precision=mlp_precision, verbose=False)
        m.state_i32["occ_grid_in_u32"] = occ_grid.view(np.int32).copy()
        m.state_i32["occ_grid_st_u32"] = occ_grid.view(np.int32).copy()
        m.steps_trained = START_STEP           # steady-state schedules (past the warm-up phases)
        if world > 1:
            m.enable_data_parallel(ray_offset=rank * n_loc)
        m.setup_buffers(n_loc, spr)
        return m

    nerf = make_nerf(args.mlp)
    io = ft.RayBatch.init(ctx, queue, n_loc, spr)
    import schedules as sch
    lmbda = sch.lr_lambda(1e-4, n_glob, spr)

    def one_step(i, host=False, model=None):
        model = model or nerf
        b = i % pool
        stp = model.steps_trained
        lr_f = sch.lr_schedule(stp, BASE_LR, lmbda, n_glob, spr)
        if host:
            io.upload_rays(host_rays[b])
            io.upload_targets(host_tg[b])
        else:
            io.rays_buf, io.targets_buf = pool_rays[b], pool_tg[b]
        out = model.step(io, lr_f=float(lr_f), do_train=True, return_output=host, sh_multiplier=1.0,
                         color_MLP_rel_lr=1.0, occ_update_strength=1.0)[0]
        return out

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- timing.  Every timed step is bracketed by its own CUDA events on the queue's stream; L2 is
    # flushed (a 256 MB write, twice the L2) between steps, outside the brackets, so no step starts
    # with the previous step's table lines in L2.
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    host_s = []

    def timed_steps(n_steps: int, start: int, host: bool, flush: bool = True, model=None):
        pairs, outs = [], []
        for i in range(n_steps):
            if flush:
                with torch.cuda.stream(queue.stream):
                    flush_buf.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(queue.stream)
            h0 = time.perf_counter()
            out = one_step(start + i, host=host, model=model)
            host_s.append(time.perf_counter() - h0)
            b.record(queue.stream)
            pairs.append((a, b))
            outs.append(out)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in pairs), outs

    def exchange_alone(k: int):
        """Device time of ffn_dp_reduce_apply with no forward/backward skew between the ranks (k
        back-to-back calls between one event pair, max over ranks), and the bytes that cross NVLink per
        direction per rank: peer form, its shard of every peer's gradients in and the updated shard
        out to every peer, 2 (W - 1) / W of the buffer; NVSwitch form, the reduced shard in and every
        peer's stored shard in, about the buffer once."""
        nat = nerf.native
        stp = ffn_native.make_step(lr_f=0.0, lr_t=0.0, rng_u32=1, spr=spr)
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(queue.stream)
        for _ in range(k):
            nat.dp_reduce_apply(stp, queue.stream)
        b.record(queue.stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(a.elapsed_time(b) / k)
        buf = nat.grad_buffer()[1] * 4          # bytes of [table | MLP] gradients
        per_dir = buf if nerf.dp.nvls else 2.0 * (world - 1) / world * buf
        return {"form": "nvls" if nerf.dp.nvls else "p2p", "alone_ms": ms, "in_step_ms": None,
                "bytes_per_direction": per_dir, "gbs_per_direction": per_dir / (ms * 1e-3) / 1e9,
                "link_gbs": 770.0, "frac_of_link": per_dir / (ms * 1e-3) / 1e9 / 770.0,
                "note": "link_gbs: measured peer-copy rate per direction per GPU on this pool"}

    def e2e_steps(n_steps: int):
        """End to end through the public API, as a user pipelines it: per step the L2 flush, the
        pinned-host uploads of the step's rays and targets, Nerf.step and the non-blocking colour
        read-back (into one of two pinned host arrays) are enqueued without waiting for the previous
        step; the host takes step i's colours (waits for its read-back) after enqueueing step i+1.
        One pair of CUDA events on the queue's stream brackets all n_steps steps, so every copy, the
        flushes and any device idle time between steps are inside the interval."""
        slots = [torch.zeros((n_loc, 4), dtype=torch.float32).pin_memory().numpy() for _ in range(2)]
        outs, pending = [], None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(queue.stream)
        for i in range(n_steps):
            with torch.cuda.stream(queue.stream):
                flush_buf.zero_()
            io.out_host = slots[i % 2]
            io.upload_rays(host_rays[i % pool])
            io.upload_targets(host_tg[i % pool])
            lr_f = sch.lr_schedule(nerf.steps_trained, BASE_LR, lmbda, n_glob, spr)
            out, ev = nerf.step(io, lr_f=float(lr_f), do_train=True, return_output=True, sh_multiplier=1.0,
                                color_MLP_rel_lr=1.0, occ_update_strength=1.0)
            if pending is not None:
                pending[1].wait()
                outs.append(pending[0].copy())
            pending = (out, ev)
        b.record(queue.stream)
        pending[1].wait()
        outs.append(pending[0].copy())
        torch.cuda.synchronize()
        return a.elapsed_time(b), outs

    for i in range(args.warmup):
        one_step(i)
    queue.finish()
    barrier()
    torch.cuda.synchronize()
    host_rays = [r.cpu().numpy().view(ft.ray_dtype).reshape(-1) for r in pool_rays]
    host_tg = [t.cpu().numpy() for t in pool_tg]
    io_dev = io
    with ClockSampler(local) as clk:
        # (1) device-resident inputs: value, and the fused kernel's own events (roofline)
        nerf.fb_events = []
        nerf.ex_events = []
        launches0 = nerf.native.launches
        ms_sum, _ = timed_steps(args.steps, args.warmup, host=False)
        host_ms = 1e3 * statistics.median(host_s)
        barrier()
        ms_total = max_over_ranks(ms_sum)
        launches = nerf.native.launches - launches0
        fb_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in nerf.fb_events))
        ex_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in nerf.ex_events)) if nerf.ex_events else 0.0
        nerf.fb_events = None
        # (2) the same steps back to back without the flush (the table stays in L2 across steps)
        barrier()
        ms_warm, _ = timed_steps(args.steps, args.warmup, host=False, flush=False)
        barrier()
        ms_warm = max_over_ranks(ms_warm)
        # (2b) the fused exchange alone: back-to-back calls, every rank arriving at once, with a zero
        # learning rate (the table does not change; the gradients are recomputed by the next step)
        ex_alone = exchange_alone(10) if (nerf.dp is not None and nerf.dp.fused) else None
        # (3) end to end through the public API: pinned-host uploads, Nerf.step, colour download
        if not args.no_e2e:
            io = ft.RayBatch.init(ctx, queue, n_loc, spr)
            for i in range(3):
                one_step(i, host=True)
            queue.finish()
            barrier()
            e2e_sum, outs = e2e_steps(args.steps)
            barrier()
            e2e_ms = max_over_ranks(e2e_sum)
            losses = [float(np.mean((o[:, :3] - host_tg[i % pool][:, :3]) ** 2)) for i, o in enumerate(outs)]
            io = io_dev
        # (4) the same device-resident steps with the fp32 CUDA-core MLP (one GPU)
        fp32_line = None
        if world == 1 and args.mlp == "fp16" and not args.no_e2e:
            nerf32 = make_nerf("fp32")
            for i in range(args.warmup):
                one_step(i, model=nerf32)
            torch.cuda.synchronize()
            ms32, _ = timed_steps(args.steps, args.warmup, host=False, model=nerf32)
            fp32_line = {"value": n_glob * spr * args.steps / (ms32 * 1e-3), "unit": "samples/s",
                         "ms_per_step": ms32 / args.steps,
                         "note": "same steps with mlp_precision fp32 (fp32 MLP on the CUDA cores)"}
            nerf32.native.close()
        # (5) the random-access ceiling at the step's table size: as many random gathers as the encoder
        # makes and as many random reductions as the scatter would make without its coarse-level merging
        ceil = None
        if world == 1 and not args.no_e2e:
            ceil = random_access_ceiling((16 << wl["log2T"]) * wl["F"] * 4, 16 * 8 * n_loc * spr, dev, queue.stream)
    clocks = clk.summary()
    if args.no_e2e:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": n_glob * spr * args.steps / (ms_total * 1e-3),
                              "unit": "samples/s", "note": "profiling run (no e2e, no baseline)",
                              "gpu_launches": launches, "fused_ms": fb_ms, "exchange_ms": ex_ms,
                              "exchange": (dict(ex_alone, in_step_ms=ex_ms) if ex_alone else
                                           "nccl" if nerf.dp is not None else None),
                              "host_ms_per_step": host_ms,
                              "ms_per_step": ms_total / args.steps}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    # ---- report (rank 0)
    samples_per_step = n_glob * spr
    value = samples_per_step * args.steps / (ms_total * 1e-3)
    e2e_val = samples_per_step * args.steps / (e2e_ms * 1e-3)
    hbm, bf16, peak_kind = peaks()
    bytes_launch = fused_bytes_per_sample(wl["F"], spr) * n_loc * spr
    achieved = bytes_launch / (fb_ms * 1e-3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / f"fused_step_{args.workload}_traffic.json"
    if tfile.exists() and world == 1 and nerf.table_immediate:   # captured on one GPU, immediate update
        t = json.loads(tfile.read_text())
        traffic = t.get("bytes_per_launch_at_samples", {}).get(str(n_loc * spr))
        if traffic is None and "bytes_per_sample" in t:
            traffic = t["bytes_per_sample"] * n_loc * spr
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("f16 operands / f32 accumulation (MLP on tensor cores, compensated hi/lo f16 forward); "
                      "f32 table" if args.mlp == "fp16" else "f32"),
            "data": "synthetic",
            "config": {"workload": wl["desc"], "global_batch_rays": n_glob, "samples_per_ray": spr,
                       "mlp": ("tensor cores: f16 hi/lo operand pairs in the forward, f16 backward operands, "
                               "f32 accumulation" if args.mlp == "fp16" else "fp32 on the CUDA cores"),
                       "samples_per_step": samples_per_step, "parallelism": f"dp{world}",
                       "table_update": "immediate (Hogwild, in the fused kernel)" if nerf.table_immediate
                                       else ("deferred; fused exchange kernel over NVSwitch multicast (multimem "
                                             "ld_reduce gradient sum + table SGD + multimem st broadcast)"
                                             if (nerf.dp is not None and nerf.dp.nvls) else
                                             "deferred; fused exchange kernel over NVLink peer loads/stores (gradient "
                                             "sum + table SGD + broadcast)" if (nerf.dp is not None and nerf.dp.fused)
                                             else "deferred; NCCL all-reduce + table SGD pass"),
                       "l2": "flushed between timed steps (256 MB write outside the step's events)"},
            "l2_warm": {"value": samples_per_step * args.steps / (ms_warm * 1e-3), "ms_per_step": ms_warm / args.steps,
                        "note": "same steps back to back, no flush: the table stays in L2 across steps"},
            "e2e": {"value": e2e_val, "unit": "samples/s", "h2d_bytes_per_step": n_loc * (32 + 16) * world,
                    "d2h_bytes_per_step": n_loc * 16 * world, "final_mse": losses[-1],
                    "timing": "all steps pipelined between one pair of events on the queue's stream; "
                              "L2 flush before every step inside the interval"},
            "gpu_launches": launches,
            "mlp_fp32": fp32_line,
            "host_ms_per_step": host_ms,
            "exchange_ms": ex_ms,
            "exchange": dict(ex_alone, in_step_ms=ex_ms) if ex_alone else None,
            "roofline": {"bound": "hbm", "kernel": ("forward/backward group: sample_stage_kernel + encode_stage_kernel + "
                                                    "fused_step_tc_kernel<staged> + reduce_partials" if args.mlp == "fp16"
                                                    else "fused_step_kernel + reduce_partials"),
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": traffic, "peak_source": peak_kind,
                         "algorithmic_bytes_per_sample": fused_bytes_per_sample(wl["F"], spr),
                         "launch_ms": fb_ms,
                         "binding": "random 32-byte sector requests (trilinear gathers in L1/L2, vector "
                                    "reductions at L2; the table is L2-resident), not DRAM bandwidth: see achievable"},
            "clocks": clocks,
        }
        if ceil is not None:
            floor_ms = ceil["gather_ms"] + ceil["red_ms"]
            line["roofline"]["achievable"] = {
                "what": "the step's random accesses at the measured fully random rates over a buffer of the "
                        "table's size: 128 gathers + 128 vector reductions per sample (ffn_probe_random_access)",
                "gather_ops_per_s": ceil["gather_ops_per_s"], "red_ops_per_s": ceil["red_ops_per_s"],
                "floor_ms": floor_ms, "frac": floor_ms / fb_ms}
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline_sample(args, wl)
            except Exception as exc:   # the baseline is a side measurement; report why it is missing
                line["cpu_baseline"] = {"value": None, "unit": "samples/s", "cores": os.cpu_count(),
                                        "kind": "reference", "sample": f"not run: {exc}"}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
