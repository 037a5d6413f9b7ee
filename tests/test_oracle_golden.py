"""Pins the CPU oracle against the reference's own known-answer tests (CPU only).

The expected values come from tests/golden/reference_kats.npz, which restates the
reference tests' double-precision expectations (see tests/golden/make_golden.py).
"""
import numpy as np
import pytest

import make_golden as G
import oracle as O


@pytest.fixture(scope="module")
def kats():
    return G.load()


def test_oracle_library_loads():
    assert O.lib().oc_abi_version() == 1


@pytest.mark.parametrize("bits,columns,batched", G.GEMV_CASES)
def test_tiled_gemv_matches_independent_scalar(kats, bits, columns, batched):
    # QuantizedTests.cs:49-70: 9 experts x 129 rows (tail), 8 reordered experts, tol 3e-4
    m = O.populate(O.QMatrix(9, 129, columns, bits), 3)
    x = G.gemv_inputs(bits, columns, batched)
    y = O.gemv(m, x, G.EXPERT_ORDER, batched)
    exp = kats[f"gemv_{bits}_{columns}_{int(batched)}"]
    assert np.max(np.abs(exp - y)) <= 3e-4


def test_populate_matches_scalar_weight():
    # Populate packing (QuantizedTests.cs:142-165) decodes back to ScalarWeight exactly
    for bits in (5, 8):
        m = O.populate(O.QMatrix(3, 5, 192, bits), 2)
        w = m.dequant()
        e, r, c = np.meshgrid(np.arange(3), np.arange(5), np.arange(192), indexing="ij")
        ref = G.scalar_weight_f64(bits, e, r, c, 2)
        assert np.array_equal(w.astype(np.float64), ref)


@pytest.mark.parametrize("bits,columns", G.FUSED_CASES)
def test_fused_experts_match_scalar_swiglu_and_down(kats, bits, columns):
    # QuantizedTests.cs:71-117: gate/up -> SwiGLU -> down (other bit width) + shared down
    gate = O.populate(O.QMatrix(9, 192, columns, bits), 1)
    up = O.populate(O.QMatrix(9, 192, columns, bits), 2)
    down = O.populate(O.QMatrix(9, columns, 192, 8 if bits == 5 else 5), 3)
    shared = O.populate(O.QMatrix(1, columns, 64, 5), 4)
    for npass in range(2):
        inp, sinp, ids = G.fused_inputs(columns, npass)
        g = O.gemv(gate, inp, ids, False).reshape(8, 192)
        u = O.gemv(up, inp, ids, False).reshape(8, 192)
        act = (g * (1.0 / (1.0 + np.exp(-g))) * u).astype(np.float32)
        y = O.gemv(down, act.reshape(-1), ids, True)
        sy = O.gemv(shared, sinp, [0], False)
        assert np.max(np.abs(kats[f"fused_{bits}_{columns}_{npass}_out"] - y)) <= 3e-4
        assert np.max(np.abs(kats[f"fused_{bits}_{columns}_{npass}_shared"] - sy)) <= 3e-4


def _mixed_matrix(j, E, R, Cc, bits):
    m = O.QMatrix(E, R, Cc, bits)
    groups = Cc // 64
    i = np.arange(E * R * groups)
    m.scales[...] = 0x3F80
    b = (np.float32(j + 1) + (i // groups).astype(np.float32) * np.float32(0.25)).astype(np.float32)
    m.biases[...] = (b.view(np.uint32) >> 16).astype(np.uint16).reshape(m.biases.shape)
    return m


def test_independent_mixed_gemvs(kats):
    # QuantizedTests.cs:166-209: zero codes, unit scales, row-dependent biases, tol 2e-4
    mats = [_mixed_matrix(j, *shape) for j, shape in enumerate(G.MIXED_MATRICES)]
    for npass in range(2):
        inp, bat = G.mixed_inputs(npass)
        for j, (m, (experts, batched)) in enumerate(zip(mats, G.MIXED_JOBS)):
            y = O.gemv(m, bat if batched else inp, experts, batched)
            assert np.max(np.abs(kats[f"mixed_{npass}_{j}"] - y)) <= 2e-4


@pytest.mark.parametrize("bits", [5, 8])
def test_selected_expert_gemv_matches_scalar_quantization(kats, bits):
    # QuantizedTests.cs:228-256: scale 1.0 (0x3f80), bias 0.5 (0x3f00), tol 4e-3
    m = O.QMatrix(3, 7, 128, bits)
    e, r, c = np.meshgrid(np.arange(3), np.arange(7), np.arange(128), indexing="ij")
    m.packed[...] = O.pack_codes(((c * 7 + e * 3 + r) & ((1 << bits) - 1)).astype(np.uint32), bits)
    m.scales[...] = 0x3F80
    m.biases[...] = 0x3F00
    y = O.gemv(m, G.selected_inputs(), [2, 0], True)
    assert np.max(np.abs(kats[f"selected_{bits}"] - y)) <= 4e-3


def test_cuda_selftest_constants(kats):
    # split_prefix.cu:614-649: byte codes are the MLX 8-bit packing on little-endian
    w, x = G.selftest_matrix()
    m = O.QMatrix(2, 13, 256, 8)
    m.packed[...] = w.view(np.uint32).reshape(m.packed.shape)
    m.scales[...] = 0x3B80
    m.biases[...] = 0xBE80
    y = O.gemv(m, x, [1, 0], False)
    assert np.max(np.abs(kats["selftest_out"] - y)) <= 1e-4


@pytest.mark.parametrize("k", range(5))
def test_top8_patterns_ties_to_lower_index(kats, k):
    # graph_checks.mm:63-77 and QuantizedTests.cs:280-288
    values = G.top8_patterns()[k]
    rc, ids, probs = O.select_experts(values)
    assert rc == 0
    assert ids.tolist() == kats[f"route_{k}_ids"].tolist()
    assert np.max(np.abs(probs - kats[f"route_{k}_probs"])) <= 1e-6


def test_routing_selects_and_renormalizes_top_eight():
    # QuantizedTests.cs:280-288: logits i*0.01 -> ids 255..248, sum p = 1, p0 > p7
    rc, ids, probs = O.select_experts((np.arange(256, dtype=np.float32) * np.float32(0.01)))
    assert rc == 0 and ids.tolist() == list(range(255, 247, -1))
    assert abs(float(probs.sum()) - 1) <= 1e-6 and probs[0] > probs[7]


def test_non_finite_logits_rejected():
    # Qwen36Model.cs:252 / ModelTests.cs:24-29
    for bad in (np.nan, np.inf, -np.inf):
        v = np.zeros(256, np.float32)
        v[17] = bad
        assert O.select_experts(v)[0] != 0


@pytest.mark.parametrize("count", [64, 65, 127, 128, 129, 512, 513, 2048])
@pytest.mark.parametrize("pattern", [0, 1, 2])
def test_permutation_is_stable_and_complete(count, pattern):
    # prefill_expert_checks.mm:26-49: hot / scattered / skewed route patterns
    t = np.arange(count)[:, None]
    s = np.arange(8)[None, :]
    ids = [s + 0 * t, (t * 7 + s * 13) % 256, (t // 5 * 11 + s * 19) % 256][pattern].astype(np.int32)
    counts, offsets, routes = O.permute(ids, 256)
    flat = ids.reshape(-1)
    assert counts.sum() == count * 8
    seen = np.zeros(count * 8, bool)
    for e in range(256):
        seg = routes[offsets[e]:offsets[e] + counts[e]]
        assert np.all(flat[seg] == e) and np.all(np.diff(seg) > 0)
        seen[seg] = True
    assert seen.all()
    assert np.array_equal(routes, np.argsort(flat, kind="stable"))


def test_generator_is_normal_and_deterministic():
    a = O.gen_bf16(7, O.ACT_STREAM, 1 << 16)
    b = O.gen_bf16(7, O.ACT_STREAM, 1 << 16)
    assert np.array_equal(a, b)
    v = O.bf16_to_f32(a)
    assert abs(v.mean()) < 0.02 and abs(v.std() - 1) < 0.02


def test_quantizer_roundtrip_error_bounded():
    m = O.QMatrix.generate(3, 5, 2, 16, 256, 8)
    w = m.dequant()
    # regenerate the unquantised weights and compare: error <= scale/2 + bf16 slack
    base = O.lib().oc_stream_base(3, 5)
    sc = O.lib().oc_normal_scale(0.02)
    raw = np.array([O.lib().oc_normal(base, i, sc) for i in range(2 * 16 * 256)], np.float32).reshape(w.shape)
    step = np.repeat(O.bf16_to_f32(m.scales), 64, axis=-1)
    assert np.all(np.abs(w - raw) <= 0.5 * step + 4e-3 * np.abs(raw) + 1e-7)


def test_block_modes_agree_within_tolerance():
    # small geometry of the block: f32 reference semantics vs double vs bf16 operand path
    L = O.Layer(11, bits=8, E=64, D=256, I=128)
    x = O.gen_bf16(11, O.ACT_STREAM, 16 * 256).reshape(16, 256)
    rc0, out32, ids32, p32, lg = O.moe_block(L, x, O.MODE_F32)
    rc1, out64, ids64, _, _ = O.moe_block(L, x, O.MODE_F64)
    rc2, outbf, idsbf, _, _ = O.moe_block(L, x, O.MODE_BF16OPS)
    assert rc0 == rc1 == rc2 == 0
    # routing uses the canonical f32 router in every mode
    assert np.array_equal(ids32, ids64) and np.array_equal(ids32, idsbf)
    assert np.allclose(p32.sum(1), 1, atol=1e-6)
    ma, rl = O.tolerance_report(out32, out64)
    assert ma < 1e-4 and rl < 1e-5
    ma, rl = O.tolerance_report(outbf, out64)
    assert ma < 2e-2 and rl < 5e-3


def test_forced_routes_follow_given_ids():
    L = O.Layer(12, bits=5, E=64, D=256, I=64)
    x = O.gen_bf16(12, O.ACT_STREAM, 4 * 256).reshape(4, 256)
    forced = np.array([[(t * 7 + s * 13) % 64 for s in range(8)] for t in range(4)], np.int32)
    rc, out, ids, probs, lg = O.moe_block(L, x, O.MODE_F32, forced=forced)
    assert rc == 0 and np.array_equal(ids, forced)
    sel = np.take_along_axis(lg[:, :64], forced, 1)
    p = np.exp(sel - sel.max(1, keepdims=True))
    assert np.allclose(probs, p / p.sum(1, keepdims=True), atol=1e-6)
