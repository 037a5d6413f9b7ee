"""Golden known-answer vectors taken from the reference's own tests for this path.

Each case restates one reference test's inputs and its independent double-precision
expectation (not our oracle), so the oracle and the CUDA library can both be checked
against the reference's own known answers:

  gemv_*     TiledGemvMatchesIndependentScalarWithTailRowsAndEightExperts
             (tests/DeepInfer.Tests/QuantizedTests.cs:49-70), tolerance 3e-4
  fused_*    FusedExpertsMatchScalarSwiGluAndDownAcrossChangedInputs (:71-117), 3e-4
  mixed_*    IndependentMixedGemvsPreserveOutputsWithOneBatchWait (:166-209), 2e-4
  selected_* SelectedExpertGemvMatchesScalarQuantization (:228-256), 4e-3
  route_*    RoutingSelectsAndRenormalizesTopEight (:280-288) and the five graph_top8
             logit patterns of native/DeepInfer.Metal/graph_checks.mm:63-77 (sorted with
             ties to the lower index), probabilities to 1e-6
  selftest_* the CUDA selftest operator check (native/DeepInfer.Cuda/split_prefix.cu:614-649):
             w = q/256 - 0.25, routed ids {1, 0}

Run `python tests/golden/make_golden.py` to regenerate tests/golden/reference_kats.npz.
Inputs are rebuilt by the functions below; the .npz holds the expected outputs.
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "reference_kats.npz")

GEMV_CASES = [(5, 512, True), (8, 512, False), (5, 2048, False), (8, 2048, True), (5, 4096, True),
              (8, 4096, False), (5, 64, True), (8, 64, False), (5, 192, False), (8, 192, True),
              (5, 256, True), (8, 256, False)]
FUSED_CASES = [(5, 128), (8, 128), (5, 256), (8, 256)]
EXPERT_ORDER = [8, 0, 6, 2, 5, 1, 7, 3]


def f32(x):
    return np.float32(x)


def scalar_weight_f64(bits, expert, row, col, seed):
    """ScalarWeight (QuantizedTests.cs:136-141); exact in float32, returned as float64."""
    col = np.asarray(col)
    group = col // 64
    q = (col * 7 + expert * 3 + row * 5 + seed * 11) & ((1 << bits) - 1)
    return q * (((group + seed) % 3 + 1) / 512.0) + ((row + group + seed) % 5 - 2) / 32.0


def sinf_series(n, step, amp, cos=False):
    i = np.arange(n, dtype=np.float32)
    arg = (i * f32(step)).astype(np.float32)
    v = (np.cos(arg) if cos else np.sin(arg)).astype(np.float32)
    return (v * f32(amp)).astype(np.float32)


def gemv_inputs(bits, columns, batched):
    return sinf_series(columns * (8 if batched else 1), 0.013, 0.1)


def gemv_expected(bits, columns, batched):
    x = gemv_inputs(bits, columns, batched).astype(np.float64)
    out = np.zeros(8 * 129)
    cols = np.arange(columns)
    for slot, e in enumerate(EXPERT_ORDER):
        xs = x[slot * columns:(slot + 1) * columns] if batched else x[:columns]
        for row in range(129):
            out[slot * 129 + row] = np.dot(scalar_weight_f64(bits, e, row, cols, 3), xs)
    return out


def fused_inputs(columns, npass):
    """State of (input, sharedInput, ids) after `npass`+1 iterations of the test loop."""
    inp = sinf_series(columns, 0.13, 0.1)
    sinp = sinf_series(64, 0.07, 0.2, cos=True)
    ids = list(EXPERT_ORDER)
    for _ in range(npass + 1):
        inp[0] = f32(inp[0] + f32(0.15))
        sinp[0] = f32(sinp[0] - f32(0.2))
        ids.reverse()
    return inp, sinp, ids


def fused_expected(bits, columns, npass):
    inp, sinp, ids = fused_inputs(columns, npass)
    x = inp.astype(np.float64)
    sx = sinp.astype(np.float64)
    down_bits = 8 if bits == 5 else 5
    out = np.zeros(8 * columns)
    cols = np.arange(columns)
    for slot, e in enumerate(ids):
        act = np.zeros(192)
        for row in range(192):
            g = np.dot(scalar_weight_f64(bits, e, row, cols, 1), x)
            u = np.dot(scalar_weight_f64(bits, e, row, cols, 2), x)
            act[row] = (g / (1 + np.exp(-g))) * u
        c192 = np.arange(192)
        for row in range(columns):
            out[slot * columns + row] = np.dot(scalar_weight_f64(down_bits, e, row, c192, 3), act)
    shared = np.zeros(columns)
    c64 = np.arange(64)
    for row in range(columns):
        shared[row] = np.dot(scalar_weight_f64(5, 0, row, c64, 4), sx)
    return out, shared


def mixed_inputs(npass):
    inp = ((np.arange(64) - 20) * f32(0.01)).astype(np.float32)
    batched = ((np.arange(256) - 100) * f32(0.005)).astype(np.float32)
    for _ in range(npass + 1):
        inp[0] = f32(inp[0] + f32(0.25))
        batched[0] = f32(batched[0] - f32(0.5))
    return inp, batched


# (experts, rows, cols, bits), job experts, batched -- QuantizedTests.cs:173-190
MIXED_MATRICES = [(1, 3, 64, 5), (3, 7, 128, 8), (2, 5, 64, 5), (1, 4, 64, 8)]
MIXED_JOBS = [([0], False), ([2, 0], True), ([1, 0], False), ([0], False)]


def mixed_expected(npass):
    inp, batched = mixed_inputs(npass)
    outs = []
    for j, ((E, R, Cc, bits), (experts, bat)) in enumerate(zip(MIXED_MATRICES, MIXED_JOBS)):
        src = batched if bat else inp
        y = np.zeros(len(experts) * R, np.float32)
        for slot, expert in enumerate(experts):
            for row in range(R):
                w = f32((j + 1) + (expert * R + row) * f32(0.25))
                acc = f32(0)
                for k in range(Cc):
                    acc = f32(acc + f32(w * src[(slot * Cc if bat else 0) + k]))
                y[slot * R + row] = acc
        outs.append(y)
    return outs


def selected_inputs():
    return np.sin((np.arange(256, dtype=np.float32) * f32(0.17)).astype(np.float32)).astype(np.float32)


def selected_expected(bits):
    x = selected_inputs()
    y = np.zeros(14, np.float32)
    for slot in range(2):
        e = 2 if slot == 0 else 0
        for r in range(7):
            acc = f32(0)
            for c in range(128):
                q = (c * 7 + e * 3 + r) & ((1 << bits) - 1)
                acc = f32(acc + f32((f32(q) + f32(0.5)) * x[slot * 128 + c]))
            y[slot * 7 + r] = acc
    return y


def top8_patterns():
    """graph_checks.mm:63-66 logit patterns plus the RoutingSelects case (i*0.01)."""
    i = np.arange(256)
    pats = [np.zeros(256, np.float32),
            (i.astype(np.float32) * f32(0.01)).astype(np.float32),
            np.where((i % 32 == 0) | (i == 255), 3, -1).astype(np.float32),
            ((i - 128).astype(np.float32) * f32(100.0)).astype(np.float32),
            (((i * 7919) % 97 - 48).astype(np.float32) * f32(0.07)).astype(np.float32)]
    return pats


def top8_expected(values):
    order = sorted(range(256), key=lambda k: (-float(values[k]), k))[:8]
    v = np.array([float(values[k]) for k in order])
    p = np.exp(v - v[0])
    return np.array(order, np.int32), p / p.sum()


def selftest_matrix():
    """split_prefix.cu:618-627: codes (i*17+3)%256, scale 0x3b80, bias 0xbe80."""
    w = ((np.arange(2 * 13 * 256) * 17 + 3) % 256).astype(np.uint8)
    x = (((np.arange(256) * 11) % 23 - 11) / np.float32(23)).astype(np.float32)
    return w, x


def selftest_expected():
    w, x = selftest_matrix()
    chosen = [1, 0]
    out = np.zeros(26)
    for e in range(2):
        for r in range(13):
            q = w[(chosen[e] * 13 + r) * 256:(chosen[e] * 13 + r + 1) * 256].astype(np.float64)
            out[e * 13 + r] = np.dot(q / 256 - 0.25, x.astype(np.float64))
    return out


def build():
    data = {}
    for bits, cols, bat in GEMV_CASES:
        data[f"gemv_{bits}_{cols}_{int(bat)}"] = gemv_expected(bits, cols, bat)
    for bits, cols in FUSED_CASES:
        for npass in range(2):
            o, s = fused_expected(bits, cols, npass)
            data[f"fused_{bits}_{cols}_{npass}_out"] = o
            data[f"fused_{bits}_{cols}_{npass}_shared"] = s
    for npass in range(2):
        for j, y in enumerate(mixed_expected(npass)):
            data[f"mixed_{npass}_{j}"] = y
    for bits in (5, 8):
        data[f"selected_{bits}"] = selected_expected(bits)
    for k, v in enumerate(top8_patterns()):
        ids, p = top8_expected(v)
        data[f"route_{k}_ids"] = ids
        data[f"route_{k}_probs"] = p
    data["selftest_out"] = selftest_expected()
    np.savez_compressed(FIXTURE, **data)
    return FIXTURE


def load():
    return dict(np.load(FIXTURE))


if __name__ == "__main__":
    print(build())
