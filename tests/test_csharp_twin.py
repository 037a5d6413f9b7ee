"""The C# binding (src/DeepInfer.Backends/Compute/QuantizedCuda.cs) against include/deepinfer_cuda.h.

QuantizedCuda.cs is the twin of the reference's QuantizedMetal.cs (its QuantNative table,
src/DeepInfer.Backends/Compute/QuantizedMetal.cs:242-274) for libdeepinfer_cuda. No .NET SDK is
installed here, so the file is checked textually: every function the header declares is bound by
exactly one LibraryImport, with the same parameter count, the same pointer/scalar shape per
parameter and a matching return kind; the Job struct mirrors di_quant_job; the flag values equal
the header's macros.
"""
import os
import re

import deepinfer_cuda as di

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CS = os.path.join(ROOT, "src", "DeepInfer.Backends", "Compute", "QuantizedCuda.cs")
HDR = os.path.join(ROOT, "include", "deepinfer_cuda.h")


def _header():
    text = re.sub(r"/\*.*?\*/", "", open(HDR).read(), flags=re.S)
    decls = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w \t\*]*?)\b(di_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        ps = [p.strip() for p in params.split(",")]
        ps = [] if ps == ["void"] else ps
        decls[name] = (ret.strip(), ps)
    return text, decls


def _csharp():
    text = open(CS).read()
    binds = {}
    for name, ret, params in re.findall(
            r'EntryPoint = "(di_[a-z0-9_]+)"[^\]]*\]\s*internal static partial (\w+) \w+\(([^)]*)\);', text, flags=re.S):
        ps = [" ".join(p.split()) for p in params.split(",") if p.strip()]
        assert name not in binds, f"{name} bound twice"
        binds[name] = (ret, ps)
    return text, binds


def _c_kind(param: str) -> str:
    if "*" in param:
        return "ptr"
    t = param.rsplit(" ", 1)[0]
    return {"int": "i32", "int32_t": "i32", "uint64_t": "u64", "float": "f32"}[t]


def _cs_kind(param: str) -> str:
    t = param.rsplit(" ", 1)[0]
    if t.startswith("out ") or "*" in t or t in ("CudaHandle", "nint", "string"):
        return "ptr"
    return {"int": "i32", "ulong": "u64", "float": "f32"}[t]


def test_every_header_entry_is_bound_once_with_matching_parameters():
    _, decls = _header()
    _, binds = _csharp()
    assert set(decls) == set(di.header_symbols())
    assert set(binds) == set(decls), (sorted(set(decls) - set(binds)), sorted(set(binds) - set(decls)))
    for name, (cret, cps) in decls.items():
        ret, ps = binds[name]
        assert len(ps) == len(cps), name
        assert [_cs_kind(p) for p in ps] == [_c_kind(p) for p in cps], name
        assert len(di.SIGNATURES[name][1]) == len(cps), name
        want = {"void": "void", "int": "int", "uint64_t": "ulong"}.get(cret, "nint" if "*" in cret else None)
        assert ret == want, (name, cret, ret)


def test_job_struct_mirrors_the_header():
    text, _ = _csharp()
    hdr = open(HDR).read()
    job = re.search(r"typedef struct di_quant_job \{(.*?)\} di_quant_job;", hdr, flags=re.S).group(1)
    assert [l.split("/*")[0].strip() for l in job.strip().splitlines()] == [
        "void *matrix;", "const float *input;", "float *output;", "const uint32_t *experts;", "int32_t count, batched;"]
    cs = re.search(r"internal struct Job\s*\{(.*?)\}", text, flags=re.S).group(1)
    assert [l.strip() for l in cs.strip().splitlines()] == [
        "public nint Matrix;", "public float* Input;", "public float* Output;", "public int* Experts;",
        "public int Count, Batched;"]


def test_flag_values_equal_the_header_macros():
    text, _ = _csharp()
    hdr = open(HDR).read()
    macros = {m: int(v) for m, v in re.findall(r"#define (DI_MOE_[A-Z_]+) (\d+)\b", hdr)}
    flags = {m: int(v) for _, v, m in re.findall(r"(\w+) = (\d+),\s*// (DI_MOE_[A-Z_]+)", text)}
    for m in ("DI_MOE_DEVICE_IO", "DI_MOE_FORCE_ROUTES", "DI_MOE_PATH_GEMV", "DI_MOE_PATH_GROUPED",
              "DI_MOE_PROFILE", "DI_MOE_ROUTER_EXACT"):
        assert flags[m] == macros[m], m
    assert "const string Lib = \"deepinfer_cuda\"" in text
