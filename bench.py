"""Benchmark of the MoE block hot path (one JSON line on rank 0).

Workload: 8K-token prefill -- 16 chunks of 512 tokens whose tokens share
each expert's weight pass -- through 40 stacked Qwen3.6-35B-A3B MoE layers with 8-bit group-64
weights (256 experts, top-8, intermediate 512, sigmoid-gated shared expert), bf16 activations
~N(0,1), weights ~N(0,0.02) quantised by the min/max affine rule and generated on the device.
A step is one pass of the 40-layer residual stack x += block_l(RMSNorm(x)) over the 8192 tokens.
The batch-1 decode of configs[1] (same 40 layers, one token) is reported in "decode".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's CPU path for this block, restated in C in its own loop
shape (oracle/cpu_block.c: Qwen36Model.Moe over CpuMatrix.Multiply's Vector<float> row dots,
src/DeepInfer.Backends/Models/Qwen36Model.cs:218-262, Compute/MatVec.cs:44-54; .NET is not on the
machine), on all host cores with the same metric: each step is BASELINE configs[0] (one full-size
8-bit layer, 512 tokens) timed whole; the per-token path makes the 8K x 40-layer time 16 x 40 of it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "infer.net_b200"))

LAYERS, TOKENS, D, E, I = 40, 8192, 2048, 256, 512
SEED = 20261201
# algorithmic counts (per token per layer): routed 8 x 6,291,456 + shared 6,291,456 + router 1,048,576
# + shared-route gate 4,096 FLOPs; decode weight bytes per layer: 9 experts + router + gate
FLOPS_TOKEN_LAYER = 8 * 6291456 + 6291456 + 1048576 + 4096
GATE_UP_FLOPS_PER_ROUTE = 2 * 2 * I * D  # gate and up rows, 2 FLOPs per MAC
DECODE_BYTES_LAYER = 9 * 3342336 + 557056 + 2176
METRIC = "MoE-block prefill tokens/s @8K (16x512-token chunks, 40 layers, 8-bit g64)"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed regions."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([v.strip() for v in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows for k in range(4) if len(r) > 5 + k and r[5 + k] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------------- reference arm

_CPU = {}


def _cpu_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def cpu_layers(n: int):
    """n full-size 8-bit layers of the benchmark's weights on the host, prepared for the CPU path
    (generated once per process and kept)."""
    O = _cpu_oracle()
    layers = _CPU.setdefault("layers", [])
    while len(layers) < n:
        layers.append(O.CpuLayer(O.Layer(SEED, layer=len(layers), bits=8)))
    return layers[:n]


def cpu_cfg0(threads: int, tokens: int = 512):
    """Seconds for one pass of BASELINE configs[0] (`tokens` tokens through one full-size 8-bit
    layer) on the CPU path with `threads` threads."""
    O = _cpu_oracle()
    cl = cpu_layers(1)[0]
    x = O.gen_bf16(SEED, O.ACT_STREAM, tokens * D).reshape(tokens, D)
    t0 = time.perf_counter()
    rc, *_ = O.cpu_block(cl, x, threads)
    dt = time.perf_counter() - t0
    assert rc == 0
    return dt


def cpu_decode_us(threads: int, layers: int, steps: int = 5):
    """Microseconds per token of batch-1 decode through `layers` distinct full-size layers."""
    O = _cpu_oracle()
    import numpy as np
    cls = cpu_layers(layers)
    norms = np.ones((layers, D), np.float32)
    x0 = O.bf16_to_f32(O.gen_bf16(SEED, O.ACT_STREAM + 1, D)).reshape(1, D)
    O.cpu_stack(cls, norms, x0, 1e-6, threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        rc, _, _ = O.cpu_stack(cls, norms, x0, 1e-6, threads)
        assert rc == 0
    return (time.perf_counter() - t0) / steps * 1e6


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline_block(threads: int, steps: int, warmup: int, decode_layers: int = 8):
    """The CPU baseline: configs[0] timed whole on all cores (mean of `steps` after `warmup`), the
    prefill metric derived from it, the same on one core (64 tokens), and batch-1 decode."""
    O = _cpu_oracle()
    for _ in range(warmup):
        cpu_cfg0(threads)
    t = sum(cpu_cfg0(threads) for _ in range(steps)) / steps
    t1 = cpu_cfg0(1, 64)
    dec = cpu_decode_us(threads, decode_layers)
    return t, {
        "value": 512 / (t * LAYERS), "unit": "tokens/s", "cores": threads, "kind": "port",
        "isa": O.cpu_isa(), "cpu": cpu_model(),
        "sample": ("configs[0] timed whole per step: 512 tokens through one full-size 8-bit layer "
                   f"({t * 1e3:.1f} ms on {threads} threads); the reference's per-token path makes the "
                   "8192-token x 40-layer step 16 x 40 such passes"),
        "single_core": {"value": 64 / (t1 * LAYERS), "unit": "tokens/s", "cores": 1,
                        "sample": f"64 tokens through one layer in {t1 * 1e3:.1f} ms on one core, x40 layers"},
        "decode": {"us_per_token": dec / decode_layers * LAYERS, "cores": threads,
                   "sample": f"batch-1 decode through {decode_layers} distinct layers "
                             f"({dec:.0f} us), scaled to 40 layers"},
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    t, cpu = cpu_baseline_block(threads, args.steps, args.warmup, args.cpu_decode_layers)
    value = cpu["value"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "prefill 8192 tokens x 40 MoE layers, 8-bit g64 (CPU: configs[0] per step)",
                   "tokens": TOKENS, "layers": LAYERS, "bits": 8, "experts": E, "top_k": 8},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------------- our arm

def run_ours(args):
    global LAYERS, TOKENS
    LAYERS, TOKENS = args.layers, args.tokens
    import numpy as np
    import torch

    import deepinfer_cuda as di

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        return run_expert_parallel(args, di, torch, rank, local, world)
    ctx = di.Context(resident=0)
    layers = [di.MoeLayer.generated(ctx, SEED, l, bits=8) for l in range(LAYERS)]
    norms = torch.ones((LAYERS, D), dtype=torch.float32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(SEED)
    x0 = torch.randn((TOKENS, D), generator=gen, device="cuda").to(torch.bfloat16).float()
    x = torch.empty_like(x0)
    arr = (di.C.c_void_p * LAYERS)(*[l.h for l in layers])
    err = di.C.create_string_buffer(2048)

    def stack(xptr, T, flags):
        ms = di.C.c_double()
        rc = di.lib().di_moe_stack(ctx.h, di.C.cast(arr, di.C.c_void_p), norms.data_ptr() if flags & di.DEVICE_IO
                                   else norms_host.ctypes.data, LAYERS, 1e-6, xptr, T, None, None, flags,
                                   di.C.byref(ms), err, 2048)
        if rc:
            raise RuntimeError(err.value.decode())
        return ms.value

    norms_host = np.ones((LAYERS, D), np.float32)
    if args.only_decode:  # profiling case: the batch-1 decode stack alone
        x1 = x0[:1].clone()
        for _ in range(args.warmup):
            x1.copy_(x0[:1])
            stack(x1.data_ptr(), 1, di.DEVICE_IO | di.PATH_GEMV)
        dms = []
        for _ in range(args.steps):
            x1.copy_(x0[:1])
            dms.append(stack(x1.data_ptr(), 1, di.DEVICE_IO | di.PATH_GEMV))
        print(json.dumps({"decode_us_per_token": 1e3 * sum(dms) / len(dms), "layers": LAYERS, "steps": args.steps}))
        return
    flags = di.DEVICE_IO | di.PATH_GROUPED
    # ---- device-resident timed region (value): no per-stage events, so the kernels run as the
    # product runs them (one programmatically dependent chain)
    for _ in range(args.warmup):
        x.copy_(x0)
        torch.cuda.synchronize()
        stack(x.data_ptr(), TOKENS, flags)
    torch.cuda.synchronize()
    stage_tot = {}
    step_ms = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            x.copy_(x0)
            torch.cuda.synchronize()
            step_ms.append(stack(x.data_ptr(), TOKENS, flags))
        torch.cuda.synchronize()
        # ---- the same steps again with CUDA events at every stage boundary (DI_MOE_PROFILE): the
        # stage times and the dominant kernel's duration for the roofline
        prof_ms = []
        for _ in range(args.steps):
            x.copy_(x0)
            torch.cuda.synchronize()
            prof_ms.append(stack(x.data_ptr(), TOKENS, flags | di.PROFILE))
            for k, v in ctx.last_profile().items():
                stage_tot[k] = stage_tot.get(k, 0.0) + v
        torch.cuda.synchronize()
        # ---- end to end through the public API with pinned host buffers, then batch-1 decode
        e2e, dec_us = None, None
        if not args.only_prefill:
            e2e, dec_us = e2e_and_decode(args, di, torch, ctx, stack, x0)
    ms = sum(step_ms) / len(step_ms)
    value = TOKENS / (ms / 1e3)
    pk = peaks()

    # ---- roofline of the dominant kernel: grouped gate/up + SwiGLU
    gate_up_ms = stage_tot.get("gate_up", 0.0) / (args.steps * LAYERS)
    gu_flops = (8 * TOKENS + TOKENS) * GATE_UP_FLOPS_PER_ROUTE
    achieved = gu_flops / (gate_up_ms * 1e-3) / 1e12 if gate_up_ms > 0 else None
    cpu = None
    if rank == 0 and not args.no_cpu:
        _, cpu = cpu_baseline_block(os.cpu_count() or 1, 2, 1, args.cpu_decode_layers)
    total_flops = FLOPS_TOKEN_LAYER * TOKENS * LAYERS
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "prefill 8192 tokens (16 x 512 chunks) x 40 MoE layers, 8-bit g64",
                   "tokens": TOKENS, "layers": LAYERS, "experts": E, "top_k": 8, "intermediate": I, "hidden": D,
                   "parallelism": "ep1", "l2": "inputs larger than L2 (34.4 GB of weights per step)"},
        "tensor_frac_step": total_flops / (ms * 1e-3) / (pk["bf16_tflops"] * 1e12),
        "roofline": {"kernel": "grouped_gemm<gate_up,8bit>", "bound": "tensor", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": (achieved / pk["bf16_tflops"]) if achieved else None,
                     "frac_of_sustained": (achieved / pk["bf16_tflops_sustained"]) if achieved else None,
                     "traffic": None,
                     "peak_source": pk["source"] + " burst bf16"},
        "stage_ms_per_step": {k: v / args.steps for k, v in stage_tot.items()},
        "ms_per_step_profiled": sum(prof_ms) / len(prof_ms),
        "cpu_baseline": cpu,
        "e2e": None if e2e is None else {
            "value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": TOKENS * D * 4 + LAYERS * D * 4,
            "d2h_bytes_per_step": TOKENS * D * 4},
        "decode": None if dec_us is None else {
            "workload": "batch-1 decode, 40 layers (configs[1])", "us_per_token": dec_us,
            "gbs": DECODE_BYTES_LAYER * LAYERS / (dec_us * 1e-6) / 1e9,
            "hbm_frac": DECODE_BYTES_LAYER * LAYERS / (dec_us * 1e-6) / 1e9 / pk["hbm_gbs"]},
        "clocks": clk.summary(),
        # per layer: router tiles, router GEMM, router select, scan, scatter + row permutation, gate_up,
        # down, combine (+ next RMSNorm); one RMSNorm before the first layer (router norms are cached
        # per layer)
        "gpu_launches": args.steps * (LAYERS * 8 + 1),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    for l in layers:
        l.close()
    ctx.close()


def run_expert_parallel(args, di, torch, rank, local, world):
    """configs[2] at N GPUs: 256/N experts per GPU, the 8192 tokens sharded 8192/N per GPU,
    token rows dispatched to the experts' GPUs and partial rows returned by the library's own
    peer-memory stores over NVLink (di_moe_ep_stack; NCCL only bootstraps the group)."""
    import datetime

    import numpy as np
    import torch.distributed as dist

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = di.Context(resident=0)
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(di.ExpertParallel.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    ep = di.ExpertParallel(ctx, bytes(uid.cpu().numpy().tobytes()), rank, world)
    layers = [ep.layer(di.generate_layer_matrices(ctx, SEED, l, 8, E, D, I, shard=(rank, world)))
              for l in range(LAYERS)]
    Tl = TOKENS // world
    norms = torch.ones((LAYERS, D), dtype=torch.float32, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(SEED)
    x0 = torch.randn((TOKENS, D), generator=gen, device="cuda").to(torch.bfloat16).float()[rank * Tl:(rank + 1) * Tl]
    x = torch.empty_like(x0)
    for _ in range(args.warmup):
        x.copy_(x0)
        torch.cuda.synchronize()
        ep.stack(layers, norms, x, Tl, 1e-6, di.DEVICE_IO)
    total = 0.0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            x.copy_(x0)
            torch.cuda.synchronize()
            dist.barrier()
            total += ep.stack(layers, norms, x, Tl, 1e-6, di.DEVICE_IO)
            torch.cuda.synchronize()
    t = torch.tensor([total], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    value = TOKENS / (ms / 1e3)
    # one profiled call after the timed ones: this rank's per-stage milliseconds over the 40 layers
    x.copy_(x0)
    torch.cuda.synchronize()
    dist.barrier()
    ep.stack(layers, norms, x, Tl, 1e-6, di.DEVICE_IO | di.PROFILE)
    prof = list(ctx.last_profile().values())
    ep_stage_names = ["router_logits", "top8_dispatch", "receive_scan", "scatter", "gate_up", "down", "send",
                      "combine"]
    ep_stages = dict(zip(ep_stage_names, prof[:len(ep_stage_names)]))
    # end to end through the host-buffer API
    xh = x0.cpu().pin_memory()
    xo = torch.empty_like(xh).pin_memory()
    nh = np.ones((LAYERS, D), np.float32)
    e2e_total = 0.0
    for i in range(args.warmup + args.steps):
        xo.copy_(xh)
        dist.barrier()
        t0 = time.perf_counter()
        ep.stack(layers, nh, xo, Tl, 1e-6, 0)
        if i >= args.warmup:
            e2e_total += time.perf_counter() - t0
    et = torch.tensor([e2e_total], dtype=torch.float64, device="cuda")
    dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e = TOKENS / (float(et.item()) / args.steps)
    pk = peaks()
    total_flops = FLOPS_TOKEN_LAYER * TOKENS * LAYERS
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "prefill 8192 tokens (16 x 512 chunks) x 40 MoE layers, 8-bit g64",
                   "tokens": TOKENS, "layers": LAYERS, "experts": E, "top_k": 8, "intermediate": I, "hidden": D,
                   "parallelism": f"ep{world} (dispatch and combine by peer-memory stores over NVLink; NCCL bootstraps the group)", "tokens_per_gpu": Tl,
                   "l2": "inputs larger than L2 (34.4 GB of weights per step over the node)"},
        "tensor_frac_step": total_flops / (ms * 1e-3) / (world * pk["bf16_tflops"] * 1e12),
        "roofline": {"kernel": "whole expert-parallel step", "bound": "tensor",
                     "achieved": total_flops / (ms * 1e-3) / 1e12 / world, "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s per GPU", "frac": total_flops / (ms * 1e-3) / (world * pk["bf16_tflops"] * 1e12),
                     "traffic": None, "peak_source": pk["source"] + " burst bf16"},
        "cpu_baseline": None,
        "stage_ms_rank0": ep_stages,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": Tl * D * 4 * world + LAYERS * D * 4 * world,
                "d2h_bytes_per_step": Tl * D * 4 * world},
        "clocks": clk.summary(),
        # per layer: router tiles, router GEMM, router select, layout, dispatch, receive, scan, scatter +
        # row permutation, gate_up, down, partial-row send, combine; one RMSNorm before the first layer
        "gpu_launches": args.steps * (LAYERS * 10 + 1),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    for l in layers:
        l.close()
    ep.close()
    ctx.close()
    dist.destroy_process_group()


def e2e_and_decode(args, di, torch, ctx, stack, x0):
    """End-to-end prefill through the host-buffer API, then the batch-1 decode stack."""
    xh = x0.cpu().pin_memory()
    xo = torch.empty_like(xh).pin_memory()
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        xo.copy_(xh)
        t0 = time.perf_counter()
        stack(xo.data_ptr(), TOKENS, di.PATH_GROUPED)
        dt = (time.perf_counter() - t0) * 1e3
        if i >= args.warmup:
            e2e_ms.append(dt)
    e2e = TOKENS / (sum(e2e_ms) / len(e2e_ms) / 1e3)
    x1 = x0[:1].clone()
    dflags = di.DEVICE_IO | di.PATH_GEMV  # one token: all layers in one persistent kernel
    for _ in range(args.warmup):
        stack(x1.data_ptr(), 1, dflags)
    n = max(args.steps, 10)
    dms = []
    for _ in range(n):
        x1.copy_(x0[:1])
        dms.append(stack(x1.data_ptr(), 1, dflags))
    return e2e, 1e3 * sum(dms) / len(dms)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-decode-layers", type=int, default=8,
                    help="distinct layers the CPU decode leg runs (its time is scaled to 40 layers)")
    ap.add_argument("--layers", type=int, default=LAYERS, help="profiling case: fewer stacked layers")
    ap.add_argument("--tokens", type=int, default=TOKENS, help="profiling case: fewer prefill tokens")
    ap.add_argument("--only-prefill", action="store_true", help="profiling case: skip the e2e and decode legs")
    ap.add_argument("--only-decode", action="store_true", help="profiling case: only the batch-1 decode stack")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
