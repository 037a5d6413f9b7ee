"""Per-layer timeline of the one-token decode stack kernel (a profiling tool, not used by the library).

Builds a copy of libdeepinfer_cuda.so with -DDI_DECODE_TIMELINE into infer.net_b200/_build/
(the product build has the timeline compiled out), runs the batch-1 decode of BASELINE configs[1]
(40 stacked 8-bit layers, 256 experts, hidden 2048) and prints, for a routed-unit CTA (CTA 0)
and a shared-expert-unit CTA (CTA 143), the mean %globaltimer offset of every step of a layer
from the layer's start, over layers 2-39 of the last call:

    python infer.net_b200/decode_timeline.py            (on a B200)

Steps: the previous layer's output complete, h ready, this CTA's logits published, top-8 known,
copies requested, the first gate/up group landed, every copy landed, act complete, the output
vector complete, the reduction and arrival done.
"""
import ctypes as C
import os
import shutil
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(HERE, "_build", "timeline")
STEPS = ["previous output", "h ready", "logits out", "top-8", "copies issued", "group 0 landed",
         "all copies", "act", "output vector", "reduced"]


def build() -> str:
    src = os.path.join(BUILD, "infer.net_b200")
    if os.path.exists(BUILD):
        shutil.rmtree(BUILD)
    shutil.copytree(os.path.join(HERE, "csrc"), os.path.join(src, "csrc"))
    shutil.copytree(os.path.join(ROOT, "include"), os.path.join(BUILD, "include"))
    subprocess.run(["make", "-C", os.path.join(src, "csrc"), "EXTRA=-DDI_DECODE_TIMELINE"], check=True,
                   stdout=subprocess.DEVNULL)
    return os.path.join(src, "libdeepinfer_cuda.so")


def main():
    lib_path = build()
    sys.path[:0] = [HERE, os.path.join(ROOT, "oracle")]
    import deepinfer_cuda as di
    di.LIB_PATH = lib_path
    import oracle as O
    lib = di.lib()
    lib.di_debug_decode_timeline.argtypes = [C.c_void_p]
    ctx = di.Context(resident=0)
    n, D, seed = 40, 2048, 20261201
    layers = [di.MoeLayer.generated(ctx, seed, l, bits=8) for l in range(n)]
    norms = np.ones((n, D), np.float32)
    x0 = O.bf16_to_f32(O.gen_bf16(seed, O.ACT_STREAM + 7, D)).reshape(1, D)
    ms = [di.moe_stack(ctx, layers, norms, x0.copy(), 1e-6, di.PATH_GEMV)[3] for _ in range(12)]
    print(f"decode: {1e3 * np.mean(ms[2:]):.1f} us per token (timeline build)")
    tl = np.zeros((2, 64, 11), np.uint64)
    if lib.di_debug_decode_timeline(tl.ctypes.data) != 0:
        raise RuntimeError("timeline read failed")
    for c, name in ((0, "CTA 0 (routed unit)"), (1, "CTA 143 (shared-expert unit)")):
        t = tl[c, :n].astype(np.int64)
        d = t - t[:, :1]
        print(f"{name}: layer period {np.diff(t[:, 0])[1:].mean():.0f} ns")
        for e, step in enumerate(STEPS, start=1):
            print(f"  {step:16s} +{d[2:, e].mean():6.0f} ns   (step {np.mean(d[2:, e] - d[2:, e - 1]):5.0f})")
    for G in layers:
        G.close()
    ctx.close()


if __name__ == "__main__":
    main()
