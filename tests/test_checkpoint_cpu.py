"""MLX checkpoint validation on the CPU (di_moe_checkpoint_probe; no GPU needed).

The loader must accept the layout the reference loads (Qwen36Weights.cs:55-100, SafeTensors.cs:13-46)
and reject, before anything is allocated, what the reference rejects: bad header lengths,
unsupported dtypes, shape mismatches, byte ranges outside the data area or overlapping, duplicate
names, shard names that leave the directory, missing tensors, and quantisation overrides that
disagree with the expected bits.
"""
import json
import os
import struct

import numpy as np
import pytest

import deepinfer_cuda as di
import mlx_checkpoint as M
import oracle as O


def _ckpt(tmp_path, bits=8, n=2, overrides=None):
    layers = [O.Layer(70 + l, layer=l, bits=bits, E=16, D=256, I=128) for l in range(n)]
    norms = (1.0 + 0.25 * np.arange(n * 256).reshape(n, 256) % 3).astype(np.float32)
    d = str(tmp_path / "ckpt")
    wm = M.write_checkpoint(d, layers, norms, bits, overrides)
    return d, wm


def test_probe_reads_the_geometry(tmp_path):
    for bits in (8, 5):
        d, _ = _ckpt(tmp_path / str(bits), bits)
        for l in (0, 1):
            assert di.probe_checkpoint(d, l) == {"E": 16, "D": 256, "I": 128, "bits": bits}
        with pytest.raises(di.DeepInferError, match="Layer index"):
            di.probe_checkpoint(d, 2)


def _rewrite_shard(path, mutate):
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    header, data = mutate(header, data)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + data)


def _first_tensor(header):
    return next(k for k in header if k != "__metadata__")


@pytest.mark.parametrize("case,msg", [
    ("dtype", "Unsupported safetensors dtype"),
    ("shape", "offsets"),
    ("overlap", "Overlapping"),
    ("beyond", "offsets"),
    ("header_len", "header length"),
])
def test_corrupt_shards_are_rejected(tmp_path, case, msg):
    d, _ = _ckpt(tmp_path)
    shard = os.path.join(d, "model-00001-of-00002.safetensors")
    if case == "header_len":
        with open(shard, "r+b") as f:
            f.write(struct.pack("<Q", 1 << 40))
    else:
        def mutate(h, data):
            names = [k for k in h if k != "__metadata__"]
            t = h[names[0]]
            if case == "dtype":
                t["dtype"] = "F16"
            elif case == "shape":
                t["shape"] = [t["shape"][0] + 1] + t["shape"][1:]
            elif case == "overlap":
                h[names[1]]["data_offsets"] = [t["data_offsets"][0], t["data_offsets"][0] + (
                    h[names[1]]["data_offsets"][1] - h[names[1]]["data_offsets"][0])]
            elif case == "beyond":
                span = t["data_offsets"][1] - t["data_offsets"][0]
                t["data_offsets"] = [len(data) - span + 16, len(data) + 16]
            return h, data
        _rewrite_shard(shard, mutate)
    with pytest.raises(di.DeepInferError, match=msg):
        di.probe_checkpoint(d, 0)


def test_unsafe_shard_name_and_missing_tensor(tmp_path):
    d, wm = _ckpt(tmp_path)
    idx = os.path.join(d, "model.safetensors.index.json")
    name = "language_model.model.layers.0.mlp.switch_mlp.up_proj.scales"
    for bad in ("../model-00001-of-00002.safetensors", "sub/x.safetensors", ".."):
        m = dict(wm)
        m[name] = bad
        with open(idx, "w") as f:
            json.dump({"weight_map": m}, f)
        with pytest.raises(di.DeepInferError, match="Unsafe shard path"):
            di.probe_checkpoint(d, 0)
    m = dict(wm)
    del m[name]
    with open(idx, "w") as f:
        json.dump({"weight_map": m}, f)
    with pytest.raises(di.DeepInferError, match="Missing"):
        di.probe_checkpoint(d, 0)


def test_wrong_expected_shape_and_dtype(tmp_path):
    d, wm = _ckpt(tmp_path)
    # a routed matrix stored without its expert dimension: shape mismatch against [E, rows, width]
    name = "language_model.model.layers.0.mlp.switch_mlp.gate_proj.weight"
    shard = os.path.join(d, wm[name])

    def flatten(h, data):
        h[name]["shape"] = [h[name]["shape"][0] * h[name]["shape"][1], h[name]["shape"][2]]
        return h, data
    _rewrite_shard(shard, flatten)
    with pytest.raises(di.DeepInferError, match="shape mismatch"):
        di.probe_checkpoint(d, 0)
    # scales stored as F32 instead of BF16 (same element count, twice the bytes: rewrite the bytes)
    d2, wm2 = _ckpt(tmp_path / "b")
    sname = "language_model.model.layers.1.mlp.shared_expert.up_proj.scales"
    shard2 = os.path.join(d2, wm2[sname])

    def to_f32(h, data):
        t = h[sname]
        a, b = t["data_offsets"]
        t["dtype"] = "F32"
        f32 = np.frombuffer(data[a:b], np.uint16).astype(np.uint32) << 16
        new = data[:a] + f32.tobytes() + data[b:]
        grow = (b - a)
        for k, v in h.items():
            if k != "__metadata__" and k != sname and v["data_offsets"][0] >= b:
                v["data_offsets"] = [v["data_offsets"][0] + grow, v["data_offsets"][1] + grow]
        t["data_offsets"] = [a, b + grow]
        return h, new
    _rewrite_shard(shard2, to_f32)
    with pytest.raises(di.DeepInferError, match="BF16"):
        di.probe_checkpoint(d2, 1)


def test_quantization_override_must_match(tmp_path):
    d, _ = _ckpt(tmp_path, overrides={"language_model.model.layers.0.mlp.switch_mlp.down_proj":
                                      {"group_size": 64, "bits": 5}})
    with pytest.raises(di.DeepInferError, match="override"):
        di.probe_checkpoint(d, 0)
    # the router forced to 8-bit by an override of another width is refused too
    d2, _ = _ckpt(tmp_path / "r", overrides={"language_model.model.layers.1.mlp.gate": {"group_size": 64, "bits": 5}})
    with pytest.raises(di.DeepInferError, match="override"):
        di.probe_checkpoint(d2, 1)
    di.probe_checkpoint(d2, 0)


def test_config_geometry_checks(tmp_path):
    d, _ = _ckpt(tmp_path)
    cfg_path = os.path.join(d, "config.json")
    cfg = json.load(open(cfg_path))
    for key, val, msg in (("num_experts_per_tok", 4, "top-8"), ("norm_topk_prob", False, "renormalised")):
        bad = json.loads(json.dumps(cfg))
        bad["text_config"][key] = val
        json.dump(bad, open(cfg_path, "w"))
        with pytest.raises(di.DeepInferError, match=msg):
            di.probe_checkpoint(d, 0)
    bad = json.loads(json.dumps(cfg))
    bad["quantization"]["group_size"] = 32
    json.dump(bad, open(cfg_path, "w"))
    with pytest.raises(di.DeepInferError, match="group64"):
        di.probe_checkpoint(d, 0)
    open(cfg_path, "w").write("{\"text_config\": {")
    with pytest.raises(di.DeepInferError, match="Invalid JSON"):
        di.probe_checkpoint(d, 0)
