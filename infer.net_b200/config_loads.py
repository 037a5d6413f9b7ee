"""Throughput and realised expert loads of BASELINE configs[3] and configs[4] on one GPU (a
measurement tool, not used by the library; parity of both configs is in tests/test_gpu_block.py).

    python infer.net_b200/config_loads.py            (on a B200)

32K tokens through one full-geometry 5-bit layer (a one-layer stack: RMSNorm, block,
residual) whose router logits carry the bias
-1.1 ln(e + 1) (the Zipf(1.1)-shaped popularity of the parity test), timed per layer; the realised
per-expert route histogram and, for expert-parallel shards of 256/G contiguous experts, the
max/mean routes per GPU at G = 2, 4, 8.
the ragged packed batch (16 request lengths drawn uniform in [1, 4096] from seed 4, plus
48 single-token rows) through 40 stacked 8-bit layers, timed per call.

Device times are the library's own CUDA-event stage times (DI_MOE_PROFILE), so host copies are
excluded; every input is synthetic from fixed seeds.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import deepinfer_cuda as di  # noqa: E402

E, D, I = 256, 2048, 512


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def loads(ids: np.ndarray) -> dict:
    counts = np.bincount(ids.reshape(-1), minlength=E)
    out = {"routes": int(counts.sum()), "expert_max_over_mean": float(counts.max() / counts.mean()),
           "top8_experts_share": float(np.sort(counts)[::-1][:8].sum() / counts.sum()),
           "histogram_first16": counts[:16].tolist(), "histogram_last16": counts[-16:].tolist()}
    for G in (2, 4, 8):
        per = counts.reshape(G, E // G).sum(axis=1)
        out[f"gpu_routes_G{G}"] = per.tolist()
        out[f"gpu_max_over_mean_G{G}"] = float(per.max() / per.mean())
    return out


def config3(ctx, reps=5):
    T = 32768
    layer = di.MoeLayer.generated(ctx, 20261203, 0, bits=5)
    layer.set_router_bias((-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32))
    xb = bf16_bits(np.random.default_rng(19).standard_normal((T, D), dtype=np.float32))
    x0 = (xb.astype(np.uint32) << 16).view(np.float32)
    norms = np.ones((1, D), np.float32)
    times = []
    for r in range(reps + 2):
        # a one-layer stack: x + block(RMSNorm(x)), with per-stage events
        _, _, it, _ = di.moe_stack(ctx, [layer], norms, x0, 1e-6, di.PATH_GROUPED | di.PROFILE, trace=(r == 0))
        prof = ctx.last_profile()
        if r == 0:
            ids = it[0]
        if r >= 2:
            times.append(sum(prof.values()))
    ms = float(np.median(times))
    res = {"config": "configs[3]: 32K tokens, 5-bit g64, Zipf-biased router, one layer on 1 GPU",
           "ms_per_layer": ms, "tokens_per_s_per_layer": T / (ms / 1e3),
           "tokens_per_s_40_layers": T / (40 * ms / 1e3), "stage_ms": prof}
    res.update(loads(ids))
    layer.close()
    return res


def config4(ctx, reps=3):
    rng = np.random.default_rng(4)
    lengths = [int(n) for n in rng.integers(1, 4097, 16)] + [1] * 48
    T = sum(lengths)
    layers = [di.MoeLayer.generated(ctx, 20261204, l, bits=8) for l in range(40)]
    norms = np.ones((40, D), np.float32)
    xb = bf16_bits(np.random.default_rng(20).standard_normal((T, D), dtype=np.float32))
    x0 = (xb.astype(np.uint32) << 16).view(np.float32)
    _, ids0, _, _ = di.moe_block(layers[0], xb, di.PATH_GROUPED)  # the first layer's routes (norm weights 1)
    times = []
    for r in range(reps + 1):
        di.moe_stack(ctx, layers, norms, x0, 1e-6, di.PATH_GROUPED | di.PROFILE)
        if r:
            times.append(sum(ctx.last_profile().values()))
    ms = float(np.median(times))
    res = {"config": "configs[4]: ragged packed batch (16 requests U[1,4096] + 48 single rows), 40 8-bit layers, 1 GPU",
           "tokens": T, "lengths": lengths[:16], "ms_per_call": ms, "tokens_per_s": T / (ms / 1e3)}
    res.update({f"layer0_input_{k}": v for k, v in loads(ids0).items() if k.startswith(("expert_max", "gpu_max"))})
    for layer in layers:
        layer.close()
    return res


def main():
    ctx = di.Context(resident=0)
    print(json.dumps(config3(ctx)))
    print(json.dumps(config4(ctx)))
    ctx.close()


if __name__ == "__main__":
    main()
