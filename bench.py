#!/usr/bin/env python3
"""Benchmark: 1F1B MLP training samples/s on N B200s (one pipeline stage per GPU), plus the
contraction and bandwidth-op figures at N = 1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun (N > 1) every rank builds one stage; rank 0 prints one JSON line.

Workload (the reference's pipeline benchmark configuration): 32 x Linear 8192->8192 + ReLU, bf16 compute weights with f32
masters initialised N(0, 1/8192), global batch 2048 = 32 microbatches x 64 rows, synthetic
N(0, 1) inputs and targets (seeded SplitMix64), MSE loss, SGD lr 1e-3; layers split evenly by
contiguous placement across the N stages.

`value` times K steps with inputs already on the device (CUDA events on the stage's compute
stream, barrier + synchronize on both sides, max over ranks).  `e2e` times K more steps through
the same public call with the inputs in pinned host memory: every step copies its inputs to the
device and its loss back.  `--impl reference` times the reference's CPU path (the C oracle
restating crates/cpu's gemm, on every host thread) on a bounded sample of the same workload and
extrapolates it to the step; it also times one whole training step of the oracle on a reduced
configuration, and says so.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "pipeline-parallelism-deep-learning-library_b200"))

LAYERS, WIDTH, MB, MBS, LR = 32, 8192, 64, 32, 1e-3
BATCH = MB * MBS
STEP_FLOP = 6 * BATCH * WIDTH * WIDTH * LAYERS
METRIC = "1F1B MLP training samples/s (32 x 8192 Linear+ReLU, bf16, batch 2048 = 32 x 64)"
WORKLOAD = "1F1B MLP training step: 32 x Linear 8192->8192 + ReLU, bf16 weights / f32 master, " \
           "global batch 2048 = 32 microbatches x 64, MSE, SGD lr 1e-3"


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, kind) measured on this pool."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms during a timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1", "0x1"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------------
# reference arm: the reference's CPU gemm path (the oracle port), bounded sample
# ----------------------------------------------------------------------------------------------

def cpu_sample(threads: int):
    """Times one microbatch through one layer ([64, 8192] x [8192, 8192], bf16 in, f32 accumulate)
    with the CPU backend's sequential k-order loop, and scales it to the full training step:
    forward, weight-gradient and input-gradient products are each this size, for 32 layers and
    32 microbatches.  Returns (samples/s, seconds of the sample)."""
    import numpy as np
    from linalg_b200 import data
    from oracle import oracle as O

    x = O.f32_to_bf16(data.normal(1, (MB, WIDTH)))
    w = O.f32_to_bf16(data.normal(2, (WIDTH, WIDTH), scale=WIDTH ** -0.5))
    out = np.zeros((MB, WIDTH), np.float32)
    t0 = time.perf_counter()
    O.gemm3(O.DT_BF16, O.DT_BF16, O.DT_F32, x, w, out, 1.0, 0.0, threads=threads)
    dt = time.perf_counter() - t0
    step_s = dt * 3 * LAYERS * MBS
    return BATCH / step_s, dt


def config_dict(world: int) -> dict:
    """The workload, identical in both arms' lines."""
    return {"workload": WORKLOAD, "layers": LAYERS, "width": WIDTH, "global_batch": BATCH, "microbatch": MB,
            "microbatches": MBS, "stages": world, "parallelism": f"pp{world}",
            "l2": "inputs larger than L2: every GEMM streams a 128 MiB weight matrix from HBM"}


def reduced_step_seconds():
    """One whole training step of the oracle (crates/cpu's gemm and training ops, the sequential
    pipeline reference) on a reduced configuration: d = 512, 4 layers, 8 microbatches of 16."""
    from linalg_b200 import data
    from oracle import oracle as O

    L, d, mbs, mb = 4, 512, 8, 16
    master = np.stack([data.normal(100 + l, (d, d), scale=d ** -0.5) for l in range(L)])
    x = data.normal(1, (mbs * mb, d))
    t = data.normal(2, (mbs * mb, d))
    t0 = time.perf_counter()
    O.mlp_step(master, x, t, mb, LR)
    return time.perf_counter() - t0, {"layers": L, "width": d, "microbatches": mbs, "microbatch": mb}


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_sample(threads)
    vals, secs = [], []
    for _ in range(args.steps):
        v, s = cpu_sample(threads)
        vals.append(v)
        secs.append(s)
    value = statistics.median(vals)
    red_s, red_cfg = reduced_step_seconds()
    sample = (f"one microbatch x one layer ([64,8192]x[8192,8192] bf16, f32 k-order accumulate) per step on "
              f"{threads} threads, median {statistics.median(secs):.3f} s, scaled by 3 products x 32 layers x "
              f"32 microbatches (activation, loss and SGD work not counted); the Rust reference cannot be "
              f"built here, the C oracle restates crates/cpu")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * BATCH / value, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(world),
        "extrapolated": True,
        "sampled_seconds_per_step": statistics.median(secs),
        "timed_seconds": sum(secs),
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port", "sample": sample},
        "reduced_step": {"config": red_cfg, "seconds": red_s, "samples_per_s": red_cfg["microbatches"] *
                         red_cfg["microbatch"] / red_s, "threads": 1,
                         "what": "one whole training step of the CPU oracle, measured, not extrapolated"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------------------------
# GPU measurements
# ----------------------------------------------------------------------------------------------

def time_launches(fn, stream, iters: int, warm: int = 3):
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.ExternalStream(stream) if isinstance(stream, int) else stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def op_figures(hbm_peak, tc_peak):
    """Contraction and bandwidth-op numbers at N = 1 (rank 0): the metric's first half."""
    import numpy as np
    import torch
    import linalg_b200 as lb
    from linalg_b200 import data

    ctx = lb.Context(torch.cuda.current_device())
    st = ctx.stream
    out = {}
    # 8192^3 bf16 (inputs 128 MiB each, larger than L2)
    n = 8192
    a = torch.randn(n, n, device="cuda").bfloat16()
    b = torch.randn(n, n, device="cuda").bfloat16()
    c = torch.empty(n, n, device="cuda", dtype=torch.bfloat16)
    ms = time_launches(lambda: lb.encode_gemm(ctx, st, 1.0, a, b, 0.0, c), st, 20)
    tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
    out["gemm_bf16_8192"] = {"ms": ms, "tflops": tf, "frac_of_measured_bf16": tf / tc_peak}
    del a, b, c
    # The f32 path's denominator: the tensor cores' tf32 rate, measured here as cuBLAS's tf32
    # 8192^3 product (the same kind of figure as the measured bf16 peak).  3xTF32 issues three
    # tf32 products per f32 product, so an f32 figure's roofline is a third of it.
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    c = torch.empty(n, n, device="cuda")
    ms = time_launches(lambda: torch.matmul(a, b, out=c), torch.cuda.current_stream(), 10)
    torch.backends.cuda.matmul.allow_tf32 = prev
    tf32_peak = 2 * n ** 3 / (ms * 1e-3) / 1e12
    out["tf32_peak_cublas_8192"] = {"ms": ms, "tflops": tf32_peak,
                                    "what": "cuBLAS tf32 8192^3, the denominator of the f32 (3xTF32) figures"}
    del a, b, c
    # f32 1024^3 (3xTF32) and the permuting contraction
    a = torch.rand(1024, 1024, device="cuda") * 2 - 1
    b = torch.rand(1024, 1024, device="cuda") * 2 - 1
    c = torch.empty(1024, 1024, device="cuda")
    ms = time_launches(lambda: lb.encode_contract(ctx, st, 1.0, (a, "ik"), (b, "kj"), 0.0, (c, "ij")), st, 50)
    out["contract_f32_1024"] = {"ms": ms, "tflops": 2 * 1024 ** 3 / (ms * 1e-3) / 1e12}
    A = torch.rand(32, 64, 128, 256, device="cuda") * 2 - 1
    B = torch.rand(128, 256, 512, device="cuda") * 2 - 1
    C = torch.empty(32, 64, 512, device="cuda")
    ms = time_launches(lambda: lb.encode_contract(ctx, st, 1.0, (A, "abcd"), (B, "cde"), 0.0, (C, "abe")), st, 20)
    out["contract_f32_permuting"] = {"ms": ms, "tflops": 2 * 2048 * 512 * 32768 / (ms * 1e-3) / 1e12}
    del A, B, C
    K = 262144
    a = (torch.randn(256, K, device="cuda") / K ** 0.5)
    b = (torch.randn(K, 256, device="cuda") / K ** 0.5)
    c = torch.empty(256, 256, device="cuda")
    ms = time_launches(lambda: lb.encode_contract(ctx, st, 1.0, (a, "ik"), (b, "kj"), 0.0, (c, "ij")), st, 20)
    out["contract_f32_splitk_256x256x262144"] = {"ms": ms, "tflops": 2 * 256 * 256 * K / (ms * 1e-3) / 1e12}
    ab, bb, cb = a.bfloat16(), b.bfloat16(), c.bfloat16()
    ms = time_launches(lambda: lb.encode_contract(ctx, st, 1.0, (ab, "ik"), (bb, "kj"), 0.0, (cb, "ij")), st, 20)
    gbs = (2 * 256 * K * 2) / (ms * 1e-3) / 1e9
    out["contract_bf16_splitk_256x256x262144"] = {"ms": ms, "tflops": 2 * 256 * 256 * K / (ms * 1e-3) / 1e12,
                                                  "gbs": gbs, "frac_of_measured_hbm": gbs / hbm_peak}
    del a, b, c, ab, bb, cb
    # bandwidth ops on f32 [64, 128, 128, 64]
    x = torch.randn(64, 128, 128, 64, device="cuda")
    xp = x.abs() + 1e-3
    nbytes = x.numel() * 4
    perm = lb.permute_view(x, [0, 3, 1, 2])
    dst = torch.empty(perm.shape, device="cuda")
    ms = time_launches(lambda: lb.encode_materialize(ctx, st, perm, dst), st, 20)
    out["permute_0312"] = {"ms": ms, "gbs": 2 * nbytes / (ms * 1e-3) / 1e9}
    sl = lb.slice(x, [range(0, 64), range(32, 96), range(0, 128), range(16, 48)])
    dst2 = torch.empty(sl.shape, device="cuda")
    ms = time_launches(lambda: lb.encode_pack(ctx, st, sl, dst2), st, 20)
    out["slice_pack"] = {"ms": ms, "gbs": 2 * dst2.numel() * 4 / (ms * 1e-3) / 1e9}
    am = torch.empty(64, 128, 128, dtype=torch.uint32, device="cuda")
    ms = time_launches(lambda: lb.encode_argmax_rows(ctx, st, x, am), st, 20)
    out["argmax_last_axis"] = {"ms": ms, "gbs": (nbytes + am.numel() * 4) / (ms * 1e-3) / 1e9}
    y = torch.empty_like(x)
    ms = time_launches(lambda: lb.encode_sqrt(ctx, st, xp, y), st, 20)
    out["sqrt"] = {"ms": ms, "gbs": 2 * nbytes / (ms * 1e-3) / 1e9}
    ms = time_launches(lambda: lb.encode_reciprocal(ctx, st, xp, y), st, 20)
    out["reciprocal"] = {"ms": ms, "gbs": 2 * nbytes / (ms * 1e-3) / 1e9}
    for k, v in out.items():
        if "gbs" in v:
            v["frac_of_measured_hbm"] = v["gbs"] / hbm_peak
        if k.startswith("contract_f32"):
            v["frac_of_tf32x3_roofline"] = 3 * v["tflops"] / tf32_peak
    del x, xp, dst, dst2, am, y
    ctx.close()
    torch.cuda.empty_cache()
    return out


# dram__bytes_read.sum + dram__bytes_write.sum of one launch, from the ncu captures of the
# profiling drivers below (`--profile group` and `--profile gemm`); None until captured
TRAFFIC_GROUP_GEMM = None
TRAFFIC_FWD_GEMM = 140_140_544


def product_roofline(hbm_peak, tc_peak, rows: int, grouped: bool):
    """One forward product of the step, timed alone with CUDA events on its launch stream over 4
    rotating weight matrices (512 MiB, 4x L2, so every launch streams its weights from HBM).
    grouped: the one-stage step's product over four microbatches, [256, 8192] x [8192, 8192] with
    the fused ReLU, pinned as the pipeline pins it (2-way split over a CTA pair, C^T = W^T H^T,
    256-wide tile); otherwise one microbatch [64, 8192] x [8192, 8192], the product every stage of
    a multi-GPU run streams.  Algorithmic bytes: the weights once plus activations in and out."""
    import torch
    import linalg_b200 as lb

    ctx = lb.Context(torch.cuda.current_device())
    st = ctx.stream
    ws = [torch.randn(WIDTH, WIDTH, device="cuda").bfloat16() for _ in range(4)]
    x = torch.randn(rows, WIDTH, device="cuda").bfloat16()
    y = torch.empty(rows, WIDTH, device="cuda", dtype=torch.bfloat16)
    i = [0]
    pin = dict(tile_n=256, splits=2, swap=1) if grouped else {}

    def one():
        lb.encode_gemm_fused(ctx, st, 1.0, x, ws[i[0] % 4], 0.0, y, lb.EPI_RELU, **pin)
        i[0] += 1

    ms = time_launches(one, st, 64)
    name = ctx.debug_launches()[-1]
    algo_bytes = WIDTH * WIDTH * 2 + 2 * rows * WIDTH * 2
    flops = 2 * rows * WIDTH * WIDTH
    del ws, x, y
    ctx.close()
    torch.cuda.empty_cache()
    t_hbm = algo_bytes / (hbm_peak * 1e9)
    t_tc = flops / (tc_peak * 1e12)
    gbs = algo_bytes / (ms * 1e-3) / 1e9
    tfs = flops / (ms * 1e-3) / 1e12
    out = {"kernel": name, "rows": rows, "algorithmic_bytes_per_launch": algo_bytes, "flop_per_launch": flops,
           "ms_per_launch": ms, "gbs": gbs, "tflops": tfs,
           "frac_of_roofline": max(t_hbm, t_tc) / (ms * 1e-3)}
    if t_hbm >= t_tc:
        out.update({"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak})
    else:
        out.update({"bound": "tensor", "achieved": tfs, "peak": tc_peak, "unit": "TFLOP/s", "frac": tfs / tc_peak})
    out["traffic"] = TRAFFIC_GROUP_GEMM if grouped else TRAFFIC_FWD_GEMM
    return out


def run_profile(args):
    """Minimal drivers for ncu: no extras, no CPU work, a known number of launches."""
    import torch
    import linalg_b200 as lb
    from linalg_b200 import data
    from linalg_b200.pipeline import Pipeline

    torch.cuda.set_device(0)
    if args.profile in ("gemm", "group"):
        # --steps forward products as product_roofline times them: one microbatch ('gemm') or the
        # one-stage step's group of four ('group'), fused ReLU, 4 rotating weight matrices
        ctx = lb.Context(0)
        rows = MB if args.profile == "gemm" else 4 * MB
        pin = dict(tile_n=256, splits=2, swap=1) if args.profile == "group" else {}
        ws = [torch.randn(WIDTH, WIDTH, device="cuda").bfloat16() for _ in range(4)]
        x = torch.randn(rows, WIDTH, device="cuda").bfloat16()
        y = torch.empty(rows, WIDTH, device="cuda", dtype=torch.bfloat16)
        for i in range(args.steps):
            lb.encode_gemm_fused(ctx, None, 1.0, x, ws[i % 4], 0.0, y, lb.EPI_RELU, **pin)
        ctx.sync()
        print(json.dumps({"profile": args.profile, "launches": ctx.debug_launches()[-8:]}))
        return 0
    if args.profile == "square":
        # --warmup + --steps back-to-back 8192^3 bf16 products (the gemm_bf16_8192 figure)
        ctx = lb.Context(0)
        n = 8192
        a = torch.randn(n, n, device="cuda").bfloat16()
        b = torch.randn(n, n, device="cuda").bfloat16()
        c = torch.empty(n, n, device="cuda", dtype=torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            lb.encode_gemm(ctx, ctx.stream, 1.0, a, b, 0.0, c)
        ctx.sync()
        print(json.dumps({"profile": "square", "launches": ctx.debug_launches()[-1:]}))
        return 0
    if args.profile == "ops":
        # one round = slice+pack, bf16 split-K, f32 split-K (3xTF32), argmax over the last axis,
        # permute (0,3,1,2), sqrt: the configs of the op figures, in that launch order
        ctx = lb.Context(0)
        st = ctx.stream
        x = torch.randn(64, 128, 128, 64, device="cuda")
        sl = lb.slice(x, [range(0, 64), range(32, 96), range(0, 128), range(16, 48)])
        packed = torch.empty(sl.shape, device="cuda")
        K = 262144
        a = torch.randn(256, K, device="cuda") / K ** 0.5
        b = torch.randn(K, 256, device="cuda") / K ** 0.5
        c = torch.empty(256, 256, device="cuda")
        ab, bb, cb = a.bfloat16(), b.bfloat16(), c.bfloat16()
        am = torch.empty(64, 128, 128, dtype=torch.uint32, device="cuda")
        perm = lb.permute_view(x, [0, 3, 1, 2])
        permuted = torch.empty(perm.shape, device="cuda")
        xp = x.abs() + 1e-3
        y = torch.empty_like(x)
        for _ in range(args.warmup + args.steps):
            lb.encode_pack(ctx, st, sl, packed)
            lb.encode_contract(ctx, st, 1.0, (ab, "ik"), (bb, "kj"), 0.0, (cb, "ij"))
            lb.encode_contract(ctx, st, 1.0, (a, "ik"), (b, "kj"), 0.0, (c, "ij"))
            lb.encode_argmax_rows(ctx, st, x, am)
            lb.encode_materialize(ctx, st, perm, permuted)
            lb.encode_sqrt(ctx, st, xp, y)
        ctx.sync()
        print(json.dumps({"profile": "ops", "launches": ctx.debug_launches()[-9:]}))
        return 0
    p = Pipeline(args.layers, WIDTH, MB, MBS, lr=LR)
    p.init_weights(1234, WIDTH ** -0.5)
    x = torch.from_numpy(data.normal(1, (BATCH, WIDTH))).cuda()
    t = torch.from_numpy(data.normal(2, (BATCH, WIDTH))).cuda()
    torch.cuda.synchronize()
    n0 = p.debug_launches()
    for _ in range(args.warmup + args.steps):
        loss = p.step(x, t, on_device=True)
    print(json.dumps({"profile": "step", "launches_per_step": (p.debug_launches() - n0) // (args.warmup + args.steps),
                      "init_launches": n0, "loss": loss, "last_step_ms": p.last_step_ms}))
    p.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the N=1 contraction/op figures")
    ap.add_argument("--layers", type=int, default=LAYERS, help="profiling driver only: pipeline depth")
    ap.add_argument("--profile", choices=["step", "gemm", "group", "ops", "square"], default=None,
                    help="profiling driver: 'step' runs --warmup + --steps pipeline steps and nothing else; "
                         "'gemm' runs --steps forward-shaped GEMMs ([64,8192] x [8192,8192] bf16); "
                         "'group' runs --steps grouped forward products ([256,8192] x [8192,8192]); "
                         "'ops' runs --warmup + --steps rounds of the op-figure configs (pack, bf16 and "
                         "f32 split-K, argmax rows, permute, sqrt); 'square' runs --warmup + --steps "
                         "8192^3 bf16 products")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile is not None:
        return run_profile(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=300))
    import linalg_b200 as lb
    from linalg_b200 import data
    from linalg_b200.pipeline import Pipeline, unique_id

    hbm_peak, tc_peak, tc_sustained, peak_kind = peaks()
    extras = None
    roof = None
    if rank == 0 and world == 1 and not args.no_extras:
        extras = op_figures(hbm_peak, tc_peak)
    roof_one = None
    if rank == 0:
        # the dominant kernel: every stage runs its microbatches in groups of four, one product per
        # layer over 256 rows; the one-microbatch product is reported beside it
        roof_one = product_roofline(hbm_peak, tc_peak, MB, grouped=False)
        roof = product_roofline(hbm_peak, tc_peak, 4 * MB, grouped=True)

    uid = None
    if world > 1:
        obj = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    p = Pipeline(LAYERS, WIDTH, MB, MBS, lr=LR, rank=rank, world=world, device=local, uid=uid, timeout_ms=120000)
    p.init_weights(1234, WIDTH ** -0.5)
    first = rank == 0
    last = rank == world - 1
    x_host = torch.from_numpy(data.normal(1, (BATCH, WIDTH))).pin_memory() if first else None
    t_host = torch.from_numpy(data.normal(2, (BATCH, WIDTH))).pin_memory() if last else None
    x_dev = x_host.cuda() if first else None
    t_dev = t_host.cuda() if last else None
    stream = torch.cuda.ExternalStream(p.stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def timed(k, on_device):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        losses = []
        for _ in range(k):
            if on_device:
                losses.append(p.step(x_dev, t_dev, on_device=True))
            else:
                losses.append(p.step(x_host, t_host, on_device=False))
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        barrier()
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, losses

    for _ in range(args.warmup):
        p.step(x_dev, t_dev, on_device=True)
    launches0 = p.debug_launches()
    with Clocks(local) as clk:
        ms, losses = timed(args.steps, True)
    launches = p.debug_launches() - launches0
    ms_e2e, losses_e2e = timed(args.steps, False)
    clocks = clk.summary()
    # one more step, untimed, with every op's compute bracketed by CUDA events: where each stage
    # spends the step (its busy time against the 1F1B fill/drain and transfer waits)
    p.set_trace(True)
    p.step(x_dev, t_dev, on_device=True)
    from linalg_b200.pipeline import trace_summary
    stage_trace = trace_summary(p.trace(), p.last_step_ms)
    p.set_trace(False)
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, stage_trace)
    else:
        gathered = [stage_trace]
    value = args.steps * BATCH / (ms * 1e-3)
    e2e = args.steps * BATCH / (ms_e2e * 1e-3)
    if world > 1:
        lt = torch.tensor([float(launches)], dtype=torch.float64)
        dist.all_reduce(lt, op=dist.ReduceOp.SUM)
        launches = int(lt.item())
        ls = torch.tensor([losses[-1] if last else 0.0], dtype=torch.float64)
        dist.all_reduce(ls, op=dist.ReduceOp.SUM)
        final_loss = float(ls.item())
    else:
        final_loss = losses[-1]
    p.close()

    if rank == 0:
        cpu_v, cpu_s = (None, None)
        if world == 1:
            cpu_v, cpu_s = cpu_sample(1)
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded SplitMix64 N(0,1) inputs/targets, "
                                                          "N(0,1/8192) weights on device)",
            "config": config_dict(world),
            "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": (BATCH * WIDTH * 4) * 2,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "clocks": clocks,
            "loss": final_loss,
            "roofline": roof,
            "peaks": {"kind": peak_kind, "hbm_gbs": hbm_peak, "bf16_tflops": tc_peak,
                      "bf16_tflops_sustained": tc_sustained},
            # 6 B d^2 L flop per step (forward, data and weight gradients) against the sustained
            # bf16 peak: the whole step, inside which every kernel runs under the power cap
            "step_tflops": STEP_FLOP / (ms / args.steps * 1e-3) / 1e12,
            "step_frac_of_sustained_bf16": STEP_FLOP / (ms / args.steps * 1e-3) / 1e12 / tc_sustained,
        }
        line["roofline_one_microbatch"] = roof_one
        line["stage_trace"] = gathered
        if cpu_v is not None:
            line["cpu_baseline"] = {"value": cpu_v, "unit": "samples/s", "cores": 1, "kind": "port",
                                    "sample": f"one microbatch x one layer bf16 product ({cpu_s:.2f} s, 1 thread), "
                                              f"scaled by 3 products x 32 layers x 32 microbatches"}
        if extras is not None:
            line["contraction_and_ops"] = extras
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
