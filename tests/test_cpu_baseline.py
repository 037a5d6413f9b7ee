"""The timed CPU baseline (oracle/cpu_block.c) against the oracle.

The CPU baseline restates the reference's CPU loop shape (Qwen36Model.Moe over CpuMatrix's
Vector<float> row dots, src/DeepInfer.Backends/Models/Qwen36Model.cs:218-262,
Compute/MatVec.cs:44-54) with the host's SIMD width; it is what bench.py's reference arm times.
Before its time means anything it must compute the block: routing ids equal the oracle's (its
router keeps the canonical order), probabilities equal, and outputs within the block tolerance --
in practice within float rounding, since only the GEMV summation order differs. Every SIMD width
the host offers is checked (OC_CPU_ISA narrows it in a subprocess).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("bits,E,D,I,T", [(8, 64, 256, 128, 9), (5, 64, 512, 128, 5), (8, 256, 2048, 512, 3)])
@pytest.mark.parametrize("threads", [1, 4])
def test_cpu_block_matches_oracle(bits, E, D, I, T, threads):
    L = O.Layer(11, bits=bits, E=E, D=D, I=I)
    x = O.gen_bf16(3, O.ACT_STREAM + T, T * D).reshape(T, D)
    cl = O.CpuLayer(L)
    rc, out, ids, probs = O.cpu_block(cl, x, threads)
    orc, oout, oids, oprobs, _ = O.moe_block(L, x, O.MODE_F32)
    assert rc == 0 and orc == 0
    assert np.array_equal(ids, oids)
    assert np.array_equal(probs, oprobs)
    ma, rl = O.tolerance_report(out, oout)
    assert ma <= 1e-4 and rl <= 1e-5, (ma, rl)
    cl.close()


def test_cpu_block_rejects_non_finite_logits():
    L = O.Layer(12, bits=8, E=64, D=256, I=128)
    x = O.gen_bf16(4, O.ACT_STREAM, 4 * 256).reshape(4, 256)
    x[2, 7] = 0x7FC0  # NaN
    cl = O.CpuLayer(L)
    for threads in (1, 8):
        rc, *_ = O.cpu_block(cl, x, threads)
        assert rc == -1
    cl.close()


def test_cpu_stack_matches_oracle_stack():
    n, D = 2, 256
    layers = [O.Layer(13, layer=l, bits=8, E=64, D=D, I=128) for l in range(n)]
    norms = (1.0 + 0.1 * np.sin(np.arange(n * D))).astype(np.float32).reshape(n, D)
    x0 = O.bf16_to_f32(O.gen_bf16(5, O.ACT_STREAM, 6 * D)).reshape(6, D)
    cls = [O.CpuLayer(L) for L in layers]
    rc, xc, ids = O.cpu_stack(cls, norms, x0, 1e-6, 0, trace=True)
    xo = x0.copy()
    oids = np.zeros((n, 6, 8), np.int32)
    orc = O.lib().oc_moe_stack(O.C.cast((O.LayerC * n)(*[L.c() for L in layers]), O.C.c_void_p), O.ptr(norms), n,
                               1e-6, O.ptr(xo), 6, O.MODE_F32, O.ptr(oids), 0)
    assert rc == 0 and orc == 0
    assert np.array_equal(ids[0], oids[0])  # layer 0 sees identical inputs
    ma, rl = O.tolerance_report(xc, xo)
    assert ma <= 1e-3 and rl <= 1e-5, (ma, rl)


@pytest.mark.parametrize("isa", ["avx2", "scalar"])
def test_narrower_simd_paths_agree(isa):
    code = ("import sys; sys.path[:0] = ['oracle']; import numpy as np, oracle as O; "
            "L = O.Layer(14, bits=5, E=64, D=512, I=128); x = O.gen_bf16(6, O.ACT_STREAM, 5 * 512).reshape(5, 512); "
            "rc, out, ids, pr = O.cpu_block(O.CpuLayer(L), x, 2); r2, o2, i2, p2, _ = O.moe_block(L, x, O.MODE_F32); "
            "ma, rl = O.tolerance_report(out, o2); "
            "assert rc == 0 and np.array_equal(ids, i2) and ma <= 1e-4 and rl <= 1e-5, (ma, rl); print(O.cpu_isa())")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       env=dict(os.environ, OC_CPU_ISA=isa), timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() in (isa, "scalar")
