"""Writes a synthetic checkpoint in the MLX layout the reference loads (test infrastructure).

The layout is the one Qwen36Weights reads (src/DeepInfer.Backends/Models/Qwen36Weights.cs:55-100):
config.json with a text_config and a quantization block, model.safetensors.index.json whose
weight_map names the shard of every tensor, and safetensors shards (an 8-byte little-endian header
length, a JSON header of {dtype, shape, data_offsets}, then the tensor bytes). Each matrix is
stored as .weight (U32 packed codes), .scales and .biases (BF16), with [experts, rows, width]
shapes for the routed experts and [rows, width] otherwise; the router and the shared-route gate
are 8-bit. The layers come from oracle.Layer, so a loaded layer can be checked against the
oracle. Tensors are spread over two shards, alternating, so the index is exercised.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

MATRICES = (  # (tensor prefix after "language_model.model.layers.{l}.", oracle matrix name, per-expert)
    ("mlp.gate", "router", False),
    ("mlp.switch_mlp.gate_proj", "gate", True),
    ("mlp.switch_mlp.up_proj", "up", True),
    ("mlp.switch_mlp.down_proj", "down", True),
    ("mlp.shared_expert.gate_proj", "shared_gate", False),
    ("mlp.shared_expert.up_proj", "shared_up", False),
    ("mlp.shared_expert.down_proj", "shared_down", False),
    ("mlp.shared_expert_gate", "shared_route", False),
)


def write_shard(path: str, tensors: dict, metadata: dict | None = None):
    """tensors: name -> (dtype string, numpy array)."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dtype, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_checkpoint(directory: str, layers, norms: np.ndarray, bits: int, overrides: dict | None = None):
    """layers: oracle.Layer objects (one per model layer); norms: f32 [n_layers, D] written as BF16
    post_attention_layernorm weights (values must be exact in bf16)."""
    os.makedirs(directory, exist_ok=True)
    L0 = layers[0]
    config = {
        "model_type": "qwen3_5_moe",
        "text_config": {"hidden_size": L0.D, "num_experts": L0.E, "moe_intermediate_size": L0.I,
                        "num_experts_per_tok": 8, "num_hidden_layers": len(layers), "norm_topk_prob": True},
        "quantization": {"group_size": 64, "bits": bits, "mode": "affine"},
    }
    for l in range(len(layers)):
        for prefix in ("mlp.gate", "mlp.shared_expert_gate"):
            config["quantization"][f"language_model.model.layers.{l}.{prefix}"] = {"group_size": 64, "bits": 8}
    if overrides:
        config["quantization"].update(overrides)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f)
    shards = [{}, {}]
    weight_map = {}
    k = 0
    for l, L in enumerate(layers):
        pre = f"language_model.model.layers.{l}."
        for prefix, name, per_expert in MATRICES:
            q = L.m[name]
            for suffix, dtype, arr in ((".weight", "U32", q.packed), (".scales", "BF16", q.scales),
                                       (".biases", "BF16", q.biases)):
                a = arr if per_expert else arr.reshape(arr.shape[1:])
                tname = pre + prefix + suffix
                shards[k % 2][tname] = (dtype, a)
                weight_map[tname] = f"model-0000{k % 2 + 1}-of-00002.safetensors"
                k += 1
        nb = (np.ascontiguousarray(norms[l], np.float32).view(np.uint32) >> 16).astype(np.uint16)
        tname = pre + "post_attention_layernorm.weight"
        shards[k % 2][tname] = ("BF16", nb)
        weight_map[tname] = f"model-0000{k % 2 + 1}-of-00002.safetensors"
        k += 1
    for i, t in enumerate(shards):
        write_shard(os.path.join(directory, f"model-0000{i + 1}-of-00002.safetensors"), t, {"format": "mlx"})
    with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return weight_map
