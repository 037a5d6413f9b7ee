"""ctypes binding of libdeepinfer_cuda.so (the C ABI declared in include/deepinfer_cuda.h).

The Python side is a thin driver, like the reference's own ctypes benchmark driver
(scripts/benchmark-metal-quant.py:22-31): every computation runs in the CUDA library.
There is no fallback: if the library is missing or no sm_100 device is present, calls
fail loudly.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdeepinfer_cuda.so")
CSRC = os.path.join(HERE, "csrc")

DEVICE_IO, FORCE_ROUTES, PATH_GEMV, PATH_GROUPED, PROFILE, ROUTER_EXACT = 1, 2, 4, 8, 16, 32
STAGES = ("router", "top8", "scan", "scatter", "gate_up", "down", "combine", "rmsnorm")

_lib = None


def build(force: bool = False) -> str:
    """Compile the library for sm_100a in-tree (nvcc cross-compiles without a GPU)."""
    args = ["make", "-s", "-C", CSRC]
    if force:
        args.append("-B")
    subprocess.run(args, check=True)
    return LIB_PATH


class QuantJob(C.Structure):
    _fields_ = [("matrix", C.c_void_p), ("input", C.c_void_p), ("output", C.c_void_p), ("experts", C.c_void_p),
                ("count", C.c_int32), ("batched", C.c_int32)]


SIGNATURES = {
    "di_abi_version": (C.c_int, []),
    "di_quant_create": (C.c_void_p, [C.c_char_p, C.c_int]),
    "di_quant_create_configured": (C.c_void_p, [C.c_int, C.c_int, C.c_char_p, C.c_int]),
    "di_quant_destroy": (None, [C.c_void_p]),
    "di_quant_residency_bytes": (C.c_uint64, [C.c_void_p]),
    "di_quant_residency_prepare": (None, [C.c_void_p]),
    "di_quant_matrix_create": (C.c_void_p, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p,
                                            C.c_int]),
    "di_quant_matrix_buffer": (C.c_void_p, [C.c_void_p, C.c_int]),
    "di_quant_matrix_destroy": (None, [C.c_void_p]),
    "di_quant_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_quant_matvec": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                  C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_quant_experts": (C.c_int, [C.c_void_p] * 5 + [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                                      C.c_void_p, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_quant_embedding": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "di_quant_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_quant_matrix_device_buffer": (C.c_void_p, [C.c_void_p, C.c_int]),
    "di_quant_matrix_upload": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_uint64, C.c_char_p, C.c_int]),
    "di_quant_matrix_generate": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.c_float, C.c_int, C.c_char_p,
                                           C.c_int]),
    "di_moe_layer_create": (C.c_void_p, [C.c_void_p] * 9 + [C.c_char_p, C.c_int]),
    "di_moe_layer_destroy": (None, [C.c_void_p]),
    "di_moe_checkpoint_probe": (C.c_int, [C.c_char_p, C.c_int, C.c_void_p, C.c_char_p, C.c_int]),
    "di_moe_layer_load": (C.c_void_p, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_char_p, C.c_int]),
    "di_moe_layer_set_router_bias": (C.c_int, [C.c_void_p, C.c_void_p, C.c_char_p, C.c_int]),
    "di_moe_block": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                               C.c_int, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_moe_stack": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_int,
                               C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_moe_last_profile": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.c_int]),
    "di_moe_last_routes": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_char_p, C.c_int]),
    "di_moe_ep_unique_id": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int]),
    "di_moe_ep_create": (C.c_void_p, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_int]),
    "di_moe_ep_destroy": (None, [C.c_void_p]),
    "di_moe_ep_layer_create": (C.c_void_p, [C.c_void_p] * 9 + [C.c_char_p, C.c_int]),
    "di_moe_ep_stack": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_int,
                                  C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
    "di_moe_block_static": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.POINTER(C.c_double), C.c_char_p, C.c_int]),
}


def header_symbols() -> list[str]:
    """Every function the public header declares (used by the ABI export test)."""
    import re
    hdr = os.path.join(os.path.dirname(HERE), "include", "deepinfer_cuda.h")
    text = re.sub(r"/\*.*?\*/", "", open(hdr).read(), flags=re.S)
    return sorted(set(re.findall(r"\b(di_[a-z0-9_]+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class DeepInferError(RuntimeError):
    pass


def _p(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class Context:
    def __init__(self, resident: int | None = None, refresh_ms: int = 1000):
        err = C.create_string_buffer(2048)
        if resident is None:
            h = lib().di_quant_create(err, 2048)
        else:
            h = lib().di_quant_create_configured(resident, refresh_ms, err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        self.h = h

    def close(self):
        if self.h:
            lib().di_quant_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def matrix(self, experts, rows, cols, bits, group=64) -> "Matrix":
        return Matrix(self, experts, rows, cols, bits, group)

    @property
    def residency_bytes(self) -> int:
        return lib().di_quant_residency_bytes(self.h)

    def prepare_residency(self):
        lib().di_quant_residency_prepare(self.h)

    def batch(self, jobs):
        """jobs: list of (matrix, x f32, y f32, experts uint32, batched)."""
        arr = (QuantJob * len(jobs))()
        keep = []
        for i, (m, x, y, ex, bat) in enumerate(jobs):
            ex = np.ascontiguousarray(ex, np.uint32)
            keep.append(ex)
            arr[i] = QuantJob(m.h if m is not None else None, _p(x), _p(y), _p(ex), len(ex), int(bat))
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        rc = lib().di_quant_batch(self.h, C.cast(arr, C.c_void_p), len(jobs), C.byref(ms), err, 2048)
        if rc:
            raise DeepInferError(err.value.decode())
        return ms.value

    def experts(self, gate, up, down, shared, x, sx, ids, y, sy):
        ids = np.ascontiguousarray(ids, np.uint32)
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        rc = lib().di_quant_experts(self.h, gate.h, up.h, down.h, shared.h, _p(x), _p(sx), _p(ids), len(ids),
                                    _p(y), _p(sy), C.byref(ms), err, 2048)
        if rc:
            raise DeepInferError(err.value.decode())
        return ms.value

    def last_routes(self, tokens: int, experts: int):
        """(perm_route [8T], seg_offsets [E+1], seg_counts [E+1]) of the last grouped-path block."""
        perm = np.zeros(8 * tokens, np.int32)
        off = np.zeros(experts + 1, np.int32)
        cnt = np.zeros(experts + 1, np.int32)
        err = C.create_string_buffer(2048)
        n = lib().di_moe_last_routes(self.h, _p(perm), _p(off), _p(cnt), perm.size, err, 2048)
        if n < 0:
            raise DeepInferError(err.value.decode())
        return perm[:n], off, cnt

    def last_profile(self):
        out = (C.c_double * len(STAGES))()
        n = lib().di_moe_last_profile(self.h, out, len(STAGES))
        return dict(zip(STAGES[:n], list(out)[:n]))


class Matrix:
    def __init__(self, ctx: Context, experts, rows, cols, bits, group=64):
        err = C.create_string_buffer(2048)
        h = lib().di_quant_matrix_create(ctx.h, experts, rows, cols, bits, group, err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        self.ctx, self.h = ctx, h
        self.experts, self.rows, self.cols, self.bits = experts, rows, cols, bits

    def nbytes(self, index):
        n = self.experts * self.rows
        return n * self.cols * self.bits // 8 if index == 0 else n * (self.cols // 64) * 2

    def write(self, index, data: np.ndarray):
        """QuantMatrix.Write (QuantizedMetal.cs:171-176) through the host staging buffer."""
        data = np.ascontiguousarray(data)
        if data.nbytes != self.nbytes(index):
            raise ValueError("Quantized buffer length mismatch.")
        p = lib().di_quant_matrix_buffer(self.h, index)
        if not p:
            raise DeepInferError("Missing quantized buffer.")
        C.memmove(p, data.ctypes.data, data.nbytes)

    def upload(self, index, data: np.ndarray):
        data = np.ascontiguousarray(data)
        err = C.create_string_buffer(2048)
        if lib().di_quant_matrix_upload(self.h, index, data.ctypes.data, data.nbytes, err, 2048):
            raise DeepInferError(err.value.decode())

    def load(self, q):
        """Upload an oracle QMatrix (packed, scales, biases)."""
        self.upload(0, q.packed)
        self.upload(1, q.scales)
        self.upload(2, q.biases)
        return self

    def generate(self, seed, stream, stddev=0.02, first_expert=0):
        err = C.create_string_buffer(2048)
        if lib().di_quant_matrix_generate(self.h, seed, stream, stddev, first_expert, err, 2048):
            raise DeepInferError(err.value.decode())
        return self

    def device_buffer(self, index):
        return lib().di_quant_matrix_device_buffer(self.h, index)

    def matvec(self, x, y, experts, batched=False):
        ex = np.ascontiguousarray(experts, np.uint32)
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        rc = lib().di_quant_matvec(self.ctx.h, self.h, _p(x), _p(y), _p(ex), len(ex), int(batched), C.byref(ms),
                                   err, 2048)
        if rc:
            raise DeepInferError(err.value.decode())
        return ms.value

    def gemm(self, x, expert: int = 0, flags: int = 0, y=None):
        """Dense projection of a bf16 token batch: returns (y bf16 [T, rows], ms)."""
        T = (x.numel() if hasattr(x, "numel") else x.size) // self.cols
        if y is None:
            y = np.zeros((T, self.rows), np.uint16)
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        if lib().di_quant_gemm(self.ctx.h, self.h, expert, _p(x), T, _p(y), flags, C.byref(ms), err, 2048):
            raise DeepInferError(err.value.decode())
        return y, ms.value

    def embedding(self, token):
        out = np.zeros(self.cols, np.float32)
        if lib().di_quant_embedding(self.h, token, _p(out)):
            raise DeepInferError("Embedding lookup failed.")
        return out

    def close(self):
        if self.h:
            lib().di_quant_matrix_destroy(self.h)
            self.h = None


LAYER_ORDER = ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down", "shared_route")


class MoeLayer:
    """One bound MoE block (router, experts, shared expert) on a context."""

    def __init__(self, ctx: Context, mats: dict):
        err = C.create_string_buffer(2048)
        h = lib().di_moe_layer_create(ctx.h, *[mats[n].h for n in LAYER_ORDER], err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        self.ctx, self.h, self.mats = ctx, h, mats
        self.D = mats["gate"].cols

    @classmethod
    def from_oracle(cls, ctx: Context, layer) -> "MoeLayer":
        """Upload the matrices of an oracle.Layer."""
        mats = {}
        for n in LAYER_ORDER:
            q = layer.m[n]
            mats[n] = Matrix(ctx, q.experts, q.rows, q.cols, q.bits).load(q)
        obj = cls(ctx, mats)
        if layer.router_bias is not None:
            obj.set_router_bias(layer.router_bias)
        return obj

    @classmethod
    def generated(cls, ctx: Context, seed: int, layer: int, bits: int = 8, E=256, D=2048, I=512, stddev=0.02):
        """Synthetic weights generated on the device (same bits as oracle.Layer(seed, layer, ...))."""
        return cls(ctx, generate_layer_matrices(ctx, seed, layer, bits, E, D, I, stddev))

    @classmethod
    def load(cls, ctx: Context, directory: str, layer: int):
        """Layer `layer` of an MLX checkpoint directory: (MoeLayer, RMSNorm weights f32 [D])."""
        geo = probe_checkpoint(directory, layer)
        norm = np.zeros(geo["D"], np.float32)
        err = C.create_string_buffer(2048)
        h = lib().di_moe_layer_load(ctx.h, directory.encode(), layer, _p(norm), err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        obj = cls.__new__(cls)
        obj.ctx, obj.h, obj.mats, obj.D = ctx, h, {}, geo["D"]
        return obj, norm

    def set_router_bias(self, bias):
        err = C.create_string_buffer(2048)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        if lib().di_moe_layer_set_router_bias(self.h, _p(b), err, 2048):
            raise DeepInferError(err.value.decode())

    def block(self, x, tokens, y, ids=None, probs=None, flags=0):
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        rc = lib().di_moe_block(self.ctx.h, self.h, _p(x), tokens, _p(y), _p(ids), _p(probs), flags, C.byref(ms),
                                err, 2048)
        if rc:
            raise DeepInferError(err.value.decode())
        return ms.value

    def close(self, matrices=True):
        if self.h:
            lib().di_moe_layer_destroy(self.h)
            self.h = None
        if matrices:
            for m in self.mats.values():
                m.close()


def probe_checkpoint(directory: str, layer: int) -> dict:
    """Validate layer `layer` of an MLX checkpoint without a GPU: {E, D, I, bits}."""
    geo = np.zeros(4, np.int32)
    err = C.create_string_buffer(2048)
    if lib().di_moe_checkpoint_probe(directory.encode(), layer, _p(geo), err, 2048):
        raise DeepInferError(err.value.decode())
    return dict(zip(("E", "D", "I", "bits"), (int(v) for v in geo)))


def generate_layer_matrices(ctx, seed, layer, bits=8, E=256, D=2048, I=512, stddev=0.02, shard=(0, 1)):
    """Device-generated matrices of one layer; with shard=(rank, world) the routed experts are the
    rank's contiguous share [rank*E/world, (rank+1)*E/world) of the same full layer."""
    rank, world = shard
    El = E // world
    shapes = {"router": (1, E, D, 8, 0), "gate": (El, I, D, bits, rank * El), "up": (El, I, D, bits, rank * El),
              "down": (El, D, I, bits, rank * El), "shared_gate": (1, I, D, bits, 0),
              "shared_up": (1, I, D, bits, 0), "shared_down": (1, D, I, bits, 0), "shared_route": (1, 1, D, 8, 0)}
    mats = {}
    for k, n in enumerate(LAYER_ORDER):
        e, r, c, b, first = shapes[n]
        mats[n] = Matrix(ctx, e, r, c, b).generate(seed, layer * 16 + k, stddev, first)
    return mats


class ExpertParallel:
    """NCCL expert-parallel group of one process per GPU (di_moe_ep_*)."""

    def __init__(self, ctx: Context, unique_id: bytes, rank: int, world: int):
        err = C.create_string_buffer(2048)
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        h = lib().di_moe_ep_create(ctx.h, buf, rank, world, err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        self.ctx, self.h, self.rank, self.world = ctx, h, rank, world

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        err = C.create_string_buffer(2048)
        if lib().di_moe_ep_unique_id(buf, err, 2048):
            raise DeepInferError(err.value.decode())
        return bytes(buf)

    def layer(self, mats: dict) -> "MoeLayer":
        err = C.create_string_buffer(2048)
        h = lib().di_moe_ep_layer_create(self.h, *[mats[n].h for n in LAYER_ORDER], err, 2048)
        if not h:
            raise DeepInferError(err.value.decode())
        obj = MoeLayer.__new__(MoeLayer)
        obj.ctx, obj.h, obj.mats, obj.D = self.ctx, h, mats, mats["gate"].cols
        return obj

    def stack(self, layers, norms, x, tokens, eps=1e-6, flags=0, h_trace=None, ids_trace=None):
        arr = (C.c_void_p * len(layers))(*[l.h for l in layers])
        ms = C.c_double()
        err = C.create_string_buffer(2048)
        rc = lib().di_moe_ep_stack(self.h, C.cast(arr, C.c_void_p), _p(norms), len(layers), eps, _p(x), tokens,
                                   _p(h_trace), _p(ids_trace), flags, C.byref(ms), err, 2048)
        if rc:
            raise DeepInferError(err.value.decode())
        return ms.value

    def close(self):
        if self.h:
            lib().di_moe_ep_destroy(self.h)
            self.h = None


def moe_block(layer: MoeLayer, x_bf16: np.ndarray, flags: int = 0, forced: np.ndarray | None = None):
    """Host-buffer convenience call: returns (y bf16 [T,D], ids [T,8], probs [T,8], ms)."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T = x.size // layer.D
    y = np.zeros_like(x)
    ids = np.zeros((T, 8), np.int32) if forced is None else np.ascontiguousarray(forced, np.int32).copy()
    probs = np.zeros((T, 8), np.float32)
    ms = layer.block(x, T, y, ids, probs, flags | (FORCE_ROUTES if forced is not None else 0))
    return y, ids, probs, ms


def moe_stack(ctx: Context, layers, norms: np.ndarray, x: np.ndarray, eps: float = 1e-6, flags: int = 0,
              trace: bool = False):
    x = np.ascontiguousarray(x, np.float32).copy()
    D = x.shape[-1]
    T = x.size // D
    n = len(layers)
    arr = (C.c_void_p * n)(*[l.h for l in layers])
    norms = np.ascontiguousarray(norms, np.float32)
    ht = np.zeros((n, T, D), np.uint16) if trace else None
    it = np.zeros((n, T, 8), np.int32) if trace else None
    ms = C.c_double()
    err = C.create_string_buffer(2048)
    rc = lib().di_moe_stack(ctx.h, C.cast(arr, C.c_void_p), _p(norms), n, eps, _p(x), T, _p(ht), _p(it), flags,
                            C.byref(ms), err, 2048)
    if rc:
        raise DeepInferError(err.value.decode())
    return x, ht, it, ms.value
