"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline legs import this
module. It wraps oracle/libmoe_oracle.so (built by oracle/Makefile) and provides the
synthetic-input helpers used to build identical inputs for the oracle and the CUDA
library, plus the reference tests' deterministic weight formula
(tests/DeepInfer.Tests/QuantizedTests.cs:136-165).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_oracle.so")

MODE_F32, MODE_F64, MODE_BF16OPS = 0, 1, 2

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class QMatrixC(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("experts", C.c_int32), ("rows", C.c_int32), ("cols", C.c_int32), ("bits", C.c_int32)]


class LayerC(C.Structure):
    _fields_ = [(n, QMatrixC) for n in ("router", "gate", "up", "down", "shared_gate", "shared_up",
                                        "shared_down", "shared_route")] + [("router_bias", C.c_void_p)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, I64, U64, F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float
        sig = {
            "oc_abi_version": (I, []),
            "oc_bf16_to_f32": (F, [C.c_uint16]),
            "oc_f32_to_bf16": (C.c_uint16, [F]),
            "oc_mix64": (U64, [U64]),
            "oc_stream_base": (U64, [U64, U64]),
            "oc_normal_scale": (F, [F]),
            "oc_normal": (F, [U64, U64, F]),
            "oc_gen_bf16": (None, [U64, U64, I64, F, P]),
            "oc_gen_quant_matrix": (None, [U64, U64, I, I, I, I, F, P, P, P]),
            "oc_quantize_rows": (None, [P, I64, I, I, P, P, P]),
            "oc_code": (C.c_uint32, [P, I, I, I]),
            "oc_weight": (F, [P, I, I, I]),
            "oc_dot_canonical": (F, [P, I, I, P]),
            "oc_dot_f64": (C.c_double, [P, I, I, P, I]),
            "oc_gemv": (None, [P, P, P, P, I, I, I]),
            "oc_select_experts": (I, [P, I, P, P]),
            "oc_force_route": (I, [P, P, P, P]),
            "oc_permute": (None, [P, I, I, P, P, P]),
            "oc_moe_block": (I, [P, P, I, I, P, P, P, P, P, I]),
            "oc_moe_stack": (I, [P, P, I, F, P, I, I, P, I]),
            "oc_rmsnorm_bf16": (None, [P, P, I, F, P]),
            "oc_cpu_prepare": (P, [P]),
            "oc_cpu_release": (None, [P]),
            "oc_cpu_isa": (C.c_char_p, []),
            "oc_cpu_block": (I, [P, P, I, P, P, P, I]),
            "oc_cpu_stack": (I, [P, P, I, F, P, I, P, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------------ bf16

def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits (uint16); NaN preserved."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------- matrices

class QMatrix:
    """Host copy of one affine-quantised [experts, rows, cols] stack in MLX layout."""

    def __init__(self, experts: int, rows: int, cols: int, bits: int):
        assert cols % 64 == 0 and bits in (5, 8)
        self.experts, self.rows, self.cols, self.bits = experts, rows, cols, bits
        self.packed = np.zeros((experts, rows, cols * bits // 32), np.uint32)
        self.scales = np.zeros((experts, rows, cols // 64), np.uint16)
        self.biases = np.zeros((experts, rows, cols // 64), np.uint16)

    def c(self) -> QMatrixC:
        return QMatrixC(self.packed.ctypes.data, self.scales.ctypes.data, self.biases.ctypes.data,
                        self.experts, self.rows, self.cols, self.bits)

    @classmethod
    def generate(cls, seed: int, stream: int, experts: int, rows: int, cols: int, bits: int,
                 stddev: float = 0.02) -> "QMatrix":
        m = cls(experts, rows, cols, bits)
        lib().oc_gen_quant_matrix(seed, stream, experts, rows, cols, bits, stddev,
                                  ptr(m.packed), ptr(m.scales), ptr(m.biases))
        return m

    def dequant(self) -> np.ndarray:
        """Float32 [experts, rows, cols] with w = fma(q, scale, bias) (single rounding)."""
        codes = unpack_codes(self.packed, self.cols, self.bits).astype(np.float64)
        s = np.repeat(bf16_to_f32(self.scales), 64, axis=-1).astype(np.float64)
        b = np.repeat(bf16_to_f32(self.biases), 64, axis=-1).astype(np.float64)
        return (codes * s + b).astype(np.float32)  # exact product then one rounding == fmaf


def unpack_codes(packed: np.ndarray, cols: int, bits: int) -> np.ndarray:
    """LSB-first codes crossing word boundaries (QuantizedTests.cs:155-161)."""
    words = packed.reshape(-1, packed.shape[-1]).astype(np.uint64)
    c = np.arange(cols)
    bit = c * bits
    at, shift = bit // 32, (bit % 32).astype(np.uint64)
    lo = words[:, at] >> shift
    hi_at = np.minimum(at + 1, packed.shape[-1] - 1)
    hi = np.where(shift + np.uint64(bits) > 32, (words[:, hi_at] << (np.uint64(32) - shift)) & 0xFFFFFFFF, 0)
    q = ((lo | hi) & ((1 << bits) - 1)).astype(np.uint32)
    return q.reshape(packed.shape[:-1] + (cols,))


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    cols = codes.shape[-1]
    flat = codes.reshape(-1, cols).astype(np.uint64)
    out = np.zeros((flat.shape[0], cols * bits // 32), np.uint64)
    for c in range(cols):
        bit = c * bits
        at, shift = bit // 32, bit % 32
        out[:, at] |= (flat[:, c] << np.uint64(shift)) & np.uint64(0xFFFFFFFF)
        if shift + bits > 32:
            out[:, at + 1] |= flat[:, c] >> np.uint64(32 - shift)
    return out.astype(np.uint32).reshape(codes.shape[:-1] + (cols * bits // 32,))


def populate(m: QMatrix, seed: int) -> QMatrix:
    """Deterministic weights of the reference tests (QuantizedTests.cs:136-165):
    q = (c*7 + e*3 + r*5 + seed*11) & mask, scale = ((g+seed)%3+1)/512,
    bias = ((r+g+seed)%5-2)/32, truncated to bf16 by >>16."""
    e = np.arange(m.experts)[:, None, None]
    r = np.arange(m.rows)[None, :, None]
    c = np.arange(m.cols)[None, None, :]
    q = (c * 7 + e * 3 + r * 5 + seed * 11) & ((1 << m.bits) - 1)
    m.packed[...] = pack_codes(q.astype(np.uint32), m.bits)
    g = np.arange(m.cols // 64)[None, None, :]
    scale = (((g + seed) % 3 + 1) / 512.0).astype(np.float32) + np.zeros((m.experts, m.rows, 1), np.float32)
    bias = (((r + g + seed) % 5 - 2) / 32.0).astype(np.float32) + np.zeros((m.experts, 1, 1), np.float32)
    m.scales[...] = (scale.view(np.uint32) >> 16).astype(np.uint16)
    m.biases[...] = (np.broadcast_to(bias, m.scales.shape).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return m


def scalar_weight(bits: int, expert, row, col, seed: int):
    """ScalarWeight (QuantizedTests.cs:136-141) in float32 arithmetic as C# evaluates it."""
    group = col // 64
    q = (col * 7 + expert * 3 + row * 5 + seed * 11) & ((1 << bits) - 1)
    scale = np.float32(((group + seed) % 3 + 1) / np.float32(512))
    bias = np.float32(((row + group + seed) % 5 - 2) / np.float32(32))
    return np.float32(q) * scale + bias


# ------------------------------------------------------------------ layers

# geometry of Qwen3.6-35B-A3B's MoE block (Qwen36Weights.cs:8, :91-100)
D_MODEL, N_EXPERTS, TOP_K, D_INTER = 2048, 256, 8, 512

LAYER_MATRICES = ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down", "shared_route")


class Layer:
    """Synthetic MoE layer: W ~ N(0, 0.02) quantised by our min/max affine g64 quantiser.
    Stream ids: layer*16 + matrix index, so every matrix of every layer is independent."""

    def __init__(self, seed: int, layer: int = 0, bits: int = 8, E: int = N_EXPERTS, D: int = D_MODEL,
                 I: int = D_INTER, stddev: float = 0.02, router_bias: np.ndarray | None = None):
        self.seed, self.layer, self.bits, self.E, self.D, self.I = seed, layer, bits, E, D, I
        shapes = {
            "router": (1, E, D, 8), "gate": (E, I, D, bits), "up": (E, I, D, bits), "down": (E, D, I, bits),
            "shared_gate": (1, I, D, bits), "shared_up": (1, I, D, bits), "shared_down": (1, D, I, bits),
            "shared_route": (1, 1, D, 8),
        }
        self.m = {}
        for k, name in enumerate(LAYER_MATRICES):
            e, r, c, b = shapes[name]
            self.m[name] = QMatrix.generate(seed, layer * 16 + k, e, r, c, b, stddev)
        self.router_bias = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)

    def c(self) -> LayerC:
        return LayerC(*[self.m[n].c() for n in LAYER_MATRICES],
                      None if self.router_bias is None else self.router_bias.ctypes.data)


def gen_bf16(seed: int, stream: int, n: int, stddev: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().oc_gen_bf16(seed, stream, n, stddev, ptr(out))
    return out


# activation streams live far above weight streams
ACT_STREAM = 1 << 40


def moe_block(layer: Layer, x_bf16: np.ndarray, mode: int = MODE_F32, forced: np.ndarray | None = None,
              threads: int = 0):
    x_bf16 = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1, layer.D)
    T = x_bf16.shape[0]
    out = np.zeros((T, layer.D), np.float32)
    ids = np.zeros((T, 8), np.int32)
    probs = np.zeros((T, 8), np.float32)
    logits = np.zeros((T, layer.E + 1), np.float32)
    lc = layer.c()
    f = None if forced is None else np.ascontiguousarray(forced, np.int32)
    rc = lib().oc_moe_block(C.byref(lc), ptr(x_bf16), T, mode, ptr(f), ptr(out), ptr(ids), ptr(probs),
                            ptr(logits), threads)
    return rc, out, ids, probs, logits


def select_experts(logits: np.ndarray):
    logits = np.ascontiguousarray(logits, np.float32)
    ids = np.zeros(8, np.int32)
    probs = np.zeros(8, np.float32)
    rc = lib().oc_select_experts(ptr(logits), logits.shape[0], ptr(ids), ptr(probs))
    return rc, ids, probs


def permute(ids: np.ndarray, n_experts: int):
    ids = np.ascontiguousarray(ids, np.int32)
    T = ids.size // 8
    counts = np.zeros(n_experts, np.int32)
    offsets = np.zeros(n_experts, np.int32)
    routes = np.zeros(T * 8, np.int32)
    lib().oc_permute(ptr(ids), T, n_experts, ptr(counts), ptr(offsets), ptr(routes))
    return counts, offsets, routes


def gemv(m: QMatrix, x: np.ndarray, experts, batched: bool, mode: int = MODE_F32) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    ex = np.ascontiguousarray(experts, np.int32)
    y = np.zeros(len(ex) * m.rows, np.float32)
    mc = m.c()
    lib().oc_gemv(C.byref(mc), ptr(x), ptr(y), ptr(ex), len(ex), int(batched), mode)
    return y


def rmsnorm_bf16(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(x.shape, np.uint16)
    D = x.shape[-1]
    for t in range(x.size // D):
        lib().oc_rmsnorm_bf16(ptr(x[t] if x.ndim > 1 else x), ptr(w), D, eps,
                              ptr(out[t] if out.ndim > 1 else out))
    return out


def tolerance_report(actual: np.ndarray, expected: np.ndarray):
    """max-abs and relative-L2 error, the block's parity metrics."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    max_abs = float(np.max(np.abs(a - e))) if a.size else 0.0
    rel_l2 = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
    return max_abs, rel_l2


# ------------------------------------------------------------------ CPU baseline (reference loop shape)

class CpuLayer:
    """A layer prepared for the CPU baseline (cpu_block.c): router rows dequantised once, the
    expert GEMVs in CpuMatrix's Vector<float> row-dot shape. Keeps the Layer alive."""

    def __init__(self, layer: Layer):
        self.layer = layer
        self._lc = layer.c()
        self.h = lib().oc_cpu_prepare(C.byref(self._lc))
        if not self.h:
            raise MemoryError("oc_cpu_prepare failed")

    def close(self):
        if self.h:
            lib().oc_cpu_release(self.h)
            self.h = None

    def __del__(self):
        self.close()


def cpu_isa() -> str:
    return lib().oc_cpu_isa().decode()


def cpu_block(cl: CpuLayer, x_bf16: np.ndarray, threads: int = 0):
    D = cl.layer.D
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1, D)
    T = x.shape[0]
    out = np.zeros((T, D), np.float32)
    ids = np.zeros((T, 8), np.int32)
    probs = np.zeros((T, 8), np.float32)
    rc = lib().oc_cpu_block(cl.h, ptr(x), T, ptr(out), ptr(ids), ptr(probs), threads)
    return rc, out, ids, probs


def cpu_stack(layers, norms: np.ndarray, x: np.ndarray, eps: float = 1e-6, threads: int = 0, trace: bool = False):
    x = np.ascontiguousarray(x, np.float32).copy()
    D = x.shape[-1]
    T = x.size // D
    arr = (C.c_void_p * len(layers))(*[l.h for l in layers])
    norms = np.ascontiguousarray(norms, np.float32)
    ids = np.zeros((len(layers), T, 8), np.int32) if trace else None
    rc = lib().oc_cpu_stack(C.cast(arr, C.c_void_p), ptr(norms), len(layers), eps, ptr(x), T, ptr(ids), threads)
    return rc, x, ids
