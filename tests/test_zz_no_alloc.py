"""The allocation-free block entry (di_moe_block_static) against the allocating one and the oracle.

Some callers cannot call cudaMalloc once they are running: serving loops that forbid device
allocation after start-up, and processes whose device memory is already reserved by another
allocator. di_moe_block_static serves them from one fixed device array. This test calls it through
the C ABI twice in a row with different inputs, on one token (the fused one-token kernel with its
grid barrier) and on 5 and 16 tokens, and checks each result: bit for bit against di_moe_block on
the decode path (both run the same kernels in the same order), routing ids equal to the oracle's
and outputs within the block's tolerance of it (max-abs 2e-2, relative L2 5e-3). Free device
memory must not change across the calls. It lives in its own file, collected last.
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


@pytest.mark.parametrize("E,D,I,tokens", [(64, 256, 128, (5, 16)), (256, 2048, 512, (1, 1)),
                                          (256, 2048, 512, (16, 5))])
def test_static_entry_matches_allocating_entry_twice(E, D, I, tokens):
    import torch
    torch.cuda.init()
    ctx = di.Context(resident=0)
    try:
        L = O.Layer(91, bits=8, E=E, D=D, I=I)
        G = di.MoeLayer.from_oracle(ctx, L)
        inputs = [O.gen_bf16(92 + call, O.ACT_STREAM + 7 * call + T, T * D).reshape(T, D)
                  for call, T in enumerate(tokens)]
        # the allocating entry first: it may grow its workspace, the static one must not allocate
        refs = [di.moe_block(G, xh, di.PATH_GEMV) for xh in inputs]
        dev = [(torch.from_numpy(xh.view(np.int16)).cuda(), xh.shape[0]) for xh in inputs]
        outs = [(torch.zeros_like(x), torch.full((T, 8), -1, dtype=torch.int32, device="cuda"),
                 torch.zeros((T, 8), dtype=torch.float32, device="cuda")) for x, T in dev]
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for (x, T), (y, ids, probs) in zip(dev, outs):
            rc, msg = _call_static(ctx, G, x, T, y, ids, probs)
            assert rc == 0, msg
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, "the allocation-free entry changed free device memory"
        for xh, (ref_y, ref_ids, ref_probs, _), (y, ids, probs) in zip(inputs, refs, outs):
            T = xh.shape[0]
            got_y = y.cpu().numpy().view(np.uint16)
            assert np.array_equal(ids.cpu().numpy(), ref_ids)
            assert np.array_equal(probs.cpu().numpy().view(np.uint32), ref_probs.view(np.uint32))
            assert np.array_equal(got_y, ref_y)
            rc, out, oids, _, _ = O.moe_block(L, xh, O.MODE_F32)
            assert rc == 0 and np.array_equal(ids.cpu().numpy(), oids)
            ma, rl = O.tolerance_report(O.bf16_to_f32(got_y).reshape(T, D), out)
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
        # host memory is refused before any GPU work
        xh = torch.zeros((4, 256), dtype=torch.int16)
        rc, msg = _call_static(ctx, G, xh, 4, y, ids, probs)
        assert rc != 0 and "device memory" in msg
        assert bool((y == 7).all())
        G.close()
        # a geometry whose scratch exceeds the fixed array is refused before any GPU work
        W = O.Layer(94, bits=8, E=64, D=256, I=2048)
        H = di.MoeLayer.from_oracle(ctx, W)
        T = 16
        rc, msg = _call_static(ctx, H, x[:T], T, y[:T], ids[:T], probs[:T])
        assert rc != 0 and "scratch" in msg
        assert bool((y == 7).all())
        H.close()
        # so is one whose T input rows do not fit the route kernel's shared memory (T*D > 49152)
        V = O.Layer(95, bits=8, E=64, D=4096, I=128)
        K = di.MoeLayer.from_oracle(ctx, V)
        xw = torch.zeros((T, 4096), dtype=torch.int16, device="cuda")
        yw = torch.full_like(xw, 7)
        rc, msg = _call_static(ctx, K, xw, T, yw, ids[:T], probs[:T])
        assert rc != 0 and "T*D" in msg
        assert bool((yw == 7).all())
        K.close()
        # the context stays usable: a valid call afterwards succeeds
        L2 = O.Layer(96, bits=8, E=64, D=256, I=128)
        G2 = di.MoeLayer.from_oracle(ctx, L2)
        rc, msg = _call_static(ctx, G2, x[:4], 4, y[:4], ids[:4], probs[:4])
        assert rc == 0, msg
        G2.close()
    finally:
        ctx.close()
