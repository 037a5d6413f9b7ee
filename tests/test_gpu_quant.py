"""GPU tests of the di_quant_* operator table, ported from the reference's QuantizedTests.

Each test mirrors one test of tests/DeepInfer.Tests/QuantizedTests.cs with the same inputs
and the same tolerance, calling the CUDA library through its C ABI.
"""
import numpy as np
import pytest

import deepinfer_cuda as di
import make_golden as G
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = di.Context(resident=0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def kats():
    return G.load()


def populate(ctx, experts, rows, cols, bits, seed):
    q = O.populate(O.QMatrix(experts, rows, cols, bits), seed)
    m = ctx.matrix(experts, rows, cols, bits)
    # QuantMatrix.Write path: host staging buffers returned by di_quant_matrix_buffer
    m.write(0, q.packed)
    m.write(1, q.scales)
    m.write(2, q.biases)
    return m


@pytest.mark.parametrize("bits,columns,batched", G.GEMV_CASES)
def test_tiled_gemv_matches_independent_scalar(ctx, kats, bits, columns, batched):
    # QuantizedTests.cs:49-70
    m = populate(ctx, 9, 129, columns, bits, 3)
    x = G.gemv_inputs(bits, columns, batched)
    y = np.zeros(129 * 8, np.float32)
    m.matvec(x, y, G.EXPERT_ORDER, batched)
    assert np.max(np.abs(kats[f"gemv_{bits}_{columns}_{int(batched)}"] - y)) <= 3e-4
    m.close()


@pytest.mark.parametrize("bits,columns", G.FUSED_CASES)
def test_fused_experts_match_scalar_swiglu_and_down(ctx, kats, bits, columns):
    # QuantizedTests.cs:71-117 (two passes with changed inputs and reversed ids)
    gate = populate(ctx, 9, 192, columns, bits, 1)
    up = populate(ctx, 9, 192, columns, bits, 2)
    down = populate(ctx, 9, columns, 192, 8 if bits == 5 else 5, 3)
    shared = populate(ctx, 1, columns, 64, 5, 4)
    for npass in range(2):
        inp, sinp, ids = G.fused_inputs(columns, npass)
        y = np.zeros(columns * 8, np.float32)
        sy = np.zeros(columns, np.float32)
        ctx.experts(gate, up, down, shared, inp, sinp, ids, y, sy)
        assert np.max(np.abs(kats[f"fused_{bits}_{columns}_{npass}_out"] - y)) <= 3e-4
        assert np.max(np.abs(kats[f"fused_{bits}_{columns}_{npass}_shared"] - sy)) <= 3e-4
    for m in (gate, up, down, shared):
        m.close()


def test_invalid_fused_expert_call_does_not_submit_or_overwrite(ctx):
    # QuantizedTests.cs:118-135: validation before submission, outputs untouched
    other = di.Context(resident=0)
    gate = populate(ctx, 3, 64, 64, 5, 1)
    up = populate(ctx, 3, 64, 64, 5, 2)
    down = populate(ctx, 3, 64, 64, 8, 3)
    shared = populate(ctx, 1, 64, 64, 5, 4)
    foreign = populate(other, 3, 64, 64, 5, 5)
    x = np.zeros(64, np.float32)
    y = np.full(128, -2, np.float32)
    sy = np.zeros(64, np.float32)
    with pytest.raises(di.DeepInferError, match="out of bounds"):
        ctx.experts(gate, up, down, shared, x, x, [3, 0], y, sy)
    with pytest.raises(di.DeepInferError):
        ctx.experts(gate, foreign, down, shared, x, x, [1, 0], y, sy)
    with pytest.raises(di.DeepInferError):
        ctx.experts(gate, gate, down, shared, x, x, [1, 0], y, sy)
    up.close()
    with pytest.raises(di.DeepInferError):
        ctx.experts(gate, up, down, shared, x, x, [1, 0], y, sy)
    assert np.all(y == -2)
    for m in (gate, down, shared, foreign):
        m.close()
    other.close()


def _mixed(ctx, j, E, R, Cc, bits):
    m = ctx.matrix(E, R, Cc, bits)
    groups = Cc // 64
    i = np.arange(E * R * groups)
    m.write(0, np.zeros(E * R * Cc * bits // 32, np.uint32))
    m.write(1, np.full(E * R * groups, 0x3F80, np.uint16))
    b = (np.float32(j + 1) + (i // groups).astype(np.float32) * np.float32(0.25)).astype(np.float32)
    m.write(2, (b.view(np.uint32) >> 16).astype(np.uint16))
    return m


def test_independent_mixed_gemvs_preserve_outputs_with_one_batch(ctx, kats):
    # QuantizedTests.cs:166-209
    mats = [_mixed(ctx, j, *shape) for j, shape in enumerate(G.MIXED_MATRICES)]
    for npass in range(2):
        inp, bat = G.mixed_inputs(npass)
        outs = [np.zeros(len(ex) * m.rows, np.float32) for m, (ex, _) in zip(mats, G.MIXED_JOBS)]
        ctx.batch([(m, bat if b else inp, y, ex, b) for m, y, (ex, b) in zip(mats, outs, G.MIXED_JOBS)])
        for j, y in enumerate(outs):
            assert np.max(np.abs(kats[f"mixed_{npass}_{j}"] - y)) <= 2e-4
    for m in mats:
        m.close()


def test_invalid_batch_has_no_partial_submission_or_output(ctx):
    # QuantizedTests.cs:210-227
    other = di.Context(resident=0)
    a = populate(ctx, 1, 64, 64, 5, 1)
    b = populate(ctx, 1, 64, 64, 5, 2)
    foreign = populate(other, 1, 64, 64, 5, 3)
    inp = np.zeros(64, np.float32)
    out = np.full(64, -3, np.float32)
    with pytest.raises(di.DeepInferError, match="distinct"):
        ctx.batch([(a, inp, out, [0], False), (a, inp, np.zeros(64, np.float32), [0], False)])
    with pytest.raises(di.DeepInferError):
        ctx.batch([(a, inp, out, [0], False), (foreign, inp, np.zeros(64, np.float32), [0], False)])
    with pytest.raises(di.DeepInferError, match="out of bounds"):
        ctx.batch([(a, inp, out, [0], False), (b, inp, np.zeros(64, np.float32), [1], False)])
    b.close()
    with pytest.raises(di.DeepInferError):
        ctx.batch([(a, inp, out, [0], False), (b, inp, np.zeros(64, np.float32), [0], False)])
    assert np.all(out == -3)
    a.close()
    foreign.close()
    other.close()


@pytest.mark.parametrize("bits", [5, 8])
def test_selected_expert_gemv_matches_scalar_quantization(ctx, kats, bits):
    # QuantizedTests.cs:228-256
    m = ctx.matrix(3, 7, 128, bits)
    e, r, c = np.meshgrid(np.arange(3), np.arange(7), np.arange(128), indexing="ij")
    m.write(0, O.pack_codes(((c * 7 + e * 3 + r) & ((1 << bits) - 1)).astype(np.uint32), bits))
    m.write(1, np.full(42, 0x3F80, np.uint16))
    m.write(2, np.full(42, 0x3F00, np.uint16))
    y = np.zeros(14, np.float32)
    m.matvec(G.selected_inputs(), y, [2, 0], batched=True)
    assert np.max(np.abs(kats[f"selected_{bits}"] - y)) <= 4e-3
    m.close()


def test_cuda_selftest_operator_check(ctx, kats):
    # split_prefix.cu:614-649 operator check (w = q/256 - 0.25, ids {1, 0})
    w, x = G.selftest_matrix()
    m = ctx.matrix(2, 13, 256, 8)
    m.write(0, w.view(np.uint32))
    m.write(1, np.full(2 * 13 * 4, 0x3B80, np.uint16))
    m.write(2, np.full(2 * 13 * 4, 0xBE80, np.uint16))
    y = np.zeros(26, np.float32)
    m.matvec(x, y, [1, 0])
    assert np.max(np.abs(kats["selftest_out"] - y)) <= 1e-4
    m.close()


def test_residency_accounting_and_release():
    # QuantizedTests.cs:28-47: resident context accounts its weights, disabled one does not
    enabled = di.Context(resident=1, refresh_ms=20)
    disabled = di.Context(resident=0)
    ordinary = populate(disabled, 1, 64, 64, 8, 3)
    assert disabled.residency_bytes == 0
    matrix = populate(enabled, 1, 64, 64, 8, 3)
    assert enabled.residency_bytes >= 4096
    enabled.prepare_residency()
    enabled.prepare_residency()
    x = np.full(64, 0.125, np.float32)
    a, b = np.zeros(64, np.float32), np.zeros(64, np.float32)
    matrix.matvec(x, a, [0])
    ordinary.matvec(x, b, [0])
    assert np.array_equal(a, b)
    matrix.close()
    assert enabled.residency_bytes == 0
    ordinary.close()
    enabled.close()
    disabled.close()


def test_embedding_row_matches_dequant(ctx):
    q = O.populate(O.QMatrix(1, 9, 192, 5), 6)
    m = ctx.matrix(1, 9, 192, 5).load(q)
    for t in (0, 4, 8):
        assert np.array_equal(m.embedding(t), q.dequant()[0, t])
    with pytest.raises(di.DeepInferError):
        m.embedding(9)
    m.close()


@pytest.mark.parametrize("bits", [5, 8])
def test_device_generator_matches_oracle_bits(ctx, bits):
    q = O.QMatrix.generate(21, 7, 3, 40, 256, bits)
    m = ctx.matrix(3, 40, 256, bits).generate(21, 7)
    # read the device bytes back through the staging buffers
    import ctypes
    for idx, ref in ((0, q.packed), (1, q.scales), (2, q.biases)):
        p = di.lib().di_quant_matrix_buffer(m.h, idx)
        got = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint8)), shape=(ref.nbytes,)).copy()
        assert np.array_equal(got, ref.view(np.uint8).reshape(-1)), idx
    m.close()
