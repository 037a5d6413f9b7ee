"""Dense quantised projections on the tensor cores (di_quant_gemm) against the oracle.

The reference runs every non-expert projection of a prefill chunk as a batched GEMM with bf16
operands and f32 accumulation (native/DeepInfer.Metal/gpu_prefill.mm:603-614, prefill_bf16.mm:47-53;
native/DeepInfer.Cuda/prefill_batch.cuh:16-52). Checked here: against the oracle's canonical f32
GEMV (the reference semantics) within the block tolerance (max-abs 2e-2, relative L2 5e-3), and
against a bf16-operand double-precision product within twice the bf16 output rounding plus the
worst case of f32 accumulation (2^-12 of the sum of absolute products for K <= 2048).
"""
import numpy as np
import pytest

import deepinfer_cuda as di
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = di.Context(resident=0)
    yield c
    c.close()


@pytest.mark.parametrize("bits", [8, 5])
@pytest.mark.parametrize("rows,cols,experts,expert,T", [
    (512, 2048, 1, 0, 1), (512, 2048, 1, 0, 777), (2048, 1024, 1, 0, 300),
    (264, 256, 4, 2, 4096), (32, 2048, 1, 0, 65), (8192, 2048, 1, 0, 96)])
def test_dense_gemm_matches_oracle(ctx, bits, rows, cols, experts, expert, T):
    q = O.QMatrix.generate(70 + bits, rows + cols, experts, rows, cols, bits)
    m = di.Matrix(ctx, experts, rows, cols, bits).load(q)
    x = O.gen_bf16(71, O.ACT_STREAM + T, T * cols).reshape(T, cols)
    y, _ = m.gemm(x, expert)
    got = O.bf16_to_f32(y).reshape(T, rows).astype(np.float64)
    W = q.dequant()[expert].astype(np.float64)  # fma(q, s, b) in f32, exactly
    xf = O.bf16_to_f32(x).astype(np.float64)
    ref = xf @ W.T
    ma, rl = O.tolerance_report(got, ref)
    assert ma <= 2e-2 and rl <= 5e-3, (ma, rl)
    # bf16 operands, exact products, f32 accumulation: within the bf16 output rounding of the
    # double-precision product of the same operands
    Wb = O.bf16_to_f32(O.f32_to_bf16(W.astype(np.float32))).astype(np.float64)
    refb = xf @ Wb.T
    bound = 2.0 ** -8 * np.abs(refb) + 2.0 ** -12 * (np.abs(xf) @ np.abs(Wb).T)
    assert np.all(np.abs(got - refb) <= bound)
    # the oracle's canonical f32 GEMV (the reference arithmetic) on sampled tokens
    for t in np.random.default_rng(T).choice(T, min(T, 3), replace=False):
        yo = O.gemv(q, xf[t].astype(np.float32), [expert], batched=False)
        ma, rl = O.tolerance_report(got[t], yo)
        assert ma <= 2e-2 and rl <= 5e-3, (t, ma, rl)
    m.close()


def test_dense_gemm_device_io_and_rejections(ctx):
    import torch
    q = O.QMatrix.generate(80, 1, 1, 256, 512, 8)
    m = di.Matrix(ctx, 1, 256, 512, 8).load(q)
    T = 40
    x = O.gen_bf16(81, O.ACT_STREAM, T * 512).reshape(T, 512)
    y_host, _ = m.gemm(x)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    yd = torch.zeros((T, 256), dtype=torch.int16, device="cuda")
    m.gemm(xd, 0, di.DEVICE_IO, yd)
    assert np.array_equal(yd.cpu().numpy().view(np.uint16), y_host)
    with pytest.raises(di.DeepInferError, match="out of bounds"):
        m.gemm(x, 1)
    with pytest.raises(di.DeepInferError, match="device memory"):
        m.gemm(x, 0, di.DEVICE_IO, yd)  # host x with the device flag
    bad = di.Matrix(ctx, 1, 100, 512, 8)  # rows not a multiple of 8
    with pytest.raises(di.DeepInferError, match="Unsupported"):
        bad.gemm(x)
    bad.close()
    m.close()
