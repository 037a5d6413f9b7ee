"""Loading MoE blocks straight from an MLX checkpoint (di_moe_layer_load) against the oracle.

A synthetic checkpoint in the layout the reference reads (tests/mlx_checkpoint.py) is loaded layer
by layer; each loaded block must route and compute exactly like the same weights uploaded through
the matrix API (bit for bit), and like the oracle within the block tolerance; the RMSNorm weights
come back as written. Real checkpoints are not on this machine; the layout, names, dtypes and
shapes are the ones Qwen36Weights.cs:55-100 reads.
"""
import numpy as np
import pytest

import deepinfer_cuda as di
import mlx_checkpoint as M
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = di.Context(resident=0)
    yield c
    c.close()


@pytest.mark.parametrize("bits", [8, 5])
def test_loaded_layers_match_uploaded_and_oracle(ctx, tmp_path, bits):
    n, E, D, I = 2, 64, 256, 128
    layers = [O.Layer(80 + l, layer=l, bits=bits, E=E, D=D, I=I) for l in range(n)]
    norms = (1.0 + 0.125 * (np.arange(n * D).reshape(n, D) % 5)).astype(np.float32)
    d = str(tmp_path / "ckpt")
    M.write_checkpoint(d, layers, norms, bits)
    for l, L in enumerate(layers):
        G, nw = di.MoeLayer.load(ctx, d, l)
        assert np.array_equal(nw, norms[l])
        U = di.MoeLayer.from_oracle(ctx, L)
        for T, flags in ((37, di.PATH_GROUPED), (3, di.PATH_GEMV)):
            x = O.gen_bf16(81, O.ACT_STREAM + T + l, T * D).reshape(T, D)
            y, ids, probs, _ = di.moe_block(G, x, flags)
            yu, idu, pu, _ = di.moe_block(U, x, flags)
            assert np.array_equal(ids, idu) and np.array_equal(y, yu) and np.array_equal(probs, pu)
            rc, out, oids, _, _ = O.moe_block(L, x, O.MODE_F32)
            assert rc == 0 and np.array_equal(ids, oids)
            ma, rl = O.tolerance_report(O.bf16_to_f32(y).reshape(T, D), out)
            assert ma <= 2e-2 and rl <= 5e-3, (ma, rl)
        U.close()
        G.close(matrices=False)


def test_loaded_full_geometry_layer(ctx, tmp_path):
    L = O.Layer(83, bits=8)  # 256 experts, hidden 2048, intermediate 512
    norms = np.ones((1, 2048), np.float32)
    d = str(tmp_path / "full")
    M.write_checkpoint(d, [L], norms, 8)
    G, nw = di.MoeLayer.load(ctx, d, 0)
    assert np.array_equal(nw, norms[0])
    x = O.gen_bf16(84, O.ACT_STREAM, 96 * 2048).reshape(96, 2048)
    y, ids, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    rows = np.arange(0, 96, 8)
    rc, out, oids, _, _ = O.moe_block(L, x[rows], O.MODE_F32)
    assert rc == 0 and np.array_equal(ids[rows], oids)
    ma, rl = O.tolerance_report(O.bf16_to_f32(y[rows]).reshape(len(rows), 2048), out)
    assert ma <= 2e-2 and rl <= 5e-3, (ma, rl)
    G.close(matrices=False)


def test_load_rejects_before_allocating(ctx, tmp_path):
    L = O.Layer(85, bits=8, E=16, D=256, I=128)
    d = str(tmp_path / "bad")
    M.write_checkpoint(d, [L], np.ones((1, 256), np.float32), 8,
                       overrides={"language_model.model.layers.0.mlp.switch_mlp.gate_proj": {"group_size": 64, "bits": 5}})
    err = di.C.create_string_buffer(2048)
    h = di.lib().di_moe_layer_load(ctx.h, d.encode(), 0, None, err, 2048)
    assert not h and b"override" in err.value
