"""The allocation-free block entry (di_moe_block_static) against the allocating one.

di_moe_block_static serves callers that must not allocate GPU memory while running (graph
capture, no-allocation serving loops, memory already reserved by another allocator). This
test calls it through the C ABI twice in a row with different inputs and checks each result
against di_moe_block on the same inputs: routing ids exact, outputs within the block's
tolerance (max-abs 2e-2, relative L2 5e-3). It lives in its own file, collected last.
"""
import ctypes as C

import numpy as np
import pytest

import deepinfer_cuda as di
import oracle as O

pytestmark = pytest.mark.gpu


def _call_static(ctx, layer, x, T, y, ids, probs):
    ms = C.c_double()
    err = C.create_string_buffer(2048)
    rc = di.lib().di_moe_block_static(ctx.h, layer.h, x.data_ptr(), T, y.data_ptr(), ids.data_ptr(),
                                      probs.data_ptr(), C.byref(ms), err, 2048)
    return rc, err.value.decode()


@pytest.mark.parametrize("E,D,I", [(64, 256, 128), (256, 2048, 512)])
def test_static_entry_matches_allocating_entry_twice(E, D, I):
    import torch
    torch.cuda.init()
    ctx = di.Context(resident=0)
    try:
        L = O.Layer(91, bits=8, E=E, D=D, I=I)
        G = di.MoeLayer.from_oracle(ctx, L)
        for call, T in enumerate((5, 16)):
            xh = O.gen_bf16(92 + call, O.ACT_STREAM + call, T * D).reshape(T, D)
            x = torch.from_numpy(xh.view(np.int16)).cuda()
            y = torch.zeros_like(x)
            ids = torch.full((T, 8), -1, dtype=torch.int32, device="cuda")
            probs = torch.zeros((T, 8), dtype=torch.float32, device="cuda")
            rc, msg = _call_static(ctx, G, x, T, y, ids, probs)
            assert rc == 0, msg
            torch.cuda.synchronize()
            ref_y, ref_ids, ref_probs, _ = di.moe_block(G, xh, di.PATH_GEMV)
            assert np.array_equal(ids.cpu().numpy(), ref_ids)
            assert np.max(np.abs(probs.cpu().numpy() - ref_probs)) <= 1e-6
            got = O.bf16_to_f32(y.cpu().numpy().view(np.uint16)).reshape(T, D)
            ref = O.bf16_to_f32(ref_y).reshape(T, D)
            ma, rl = O.tolerance_report(got, ref)
            assert ma <= 2e-2 and rl <= 5e-3, (ma, rl)
        G.close()
    finally:
        ctx.close()


def test_static_entry_rejects_sizes_beyond_its_array():
    import torch
    ctx = di.Context(resident=0)
    try:
        L = O.Layer(93, bits=8, E=64, D=256, I=128)
        G = di.MoeLayer.from_oracle(ctx, L)
        T = 17
        x = torch.zeros((T, 256), dtype=torch.int16, device="cuda")
        y = torch.full_like(x, 7)
        ids = torch.zeros((T, 8), dtype=torch.int32, device="cuda")
        probs = torch.zeros((T, 8), dtype=torch.float32, device="cuda")
        rc, msg = _call_static(ctx, G, x, T, y, ids, probs)
        assert rc != 0 and "tokens" in msg
        assert bool((y == 7).all())
        G.close()
        # a geometry whose scratch exceeds the fixed array is refused before any GPU work
        W = O.Layer(94, bits=8, E=64, D=256, I=2048)
        H = di.MoeLayer.from_oracle(ctx, W)
        T = 16
        x, y = x[:T], y[:T]
        rc, msg = _call_static(ctx, H, x, T, y, ids[:T], probs[:T])
        assert rc != 0 and "scratch" in msg
        assert bool((y == 7).all())
        H.close()
    finally:
        ctx.close()
