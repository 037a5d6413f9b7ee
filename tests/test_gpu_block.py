"""GPU parity of the MoE block (di_moe_block / di_moe_stack) against the CPU oracle.

Bar (north star): routing ids and the permutation bit-exact, ties to the lower expert id;
block outputs within max-abs 2e-2 and relative-L2 5e-3 of the oracle's f32 reference
semantics (Qwen36Model.cs:218-262) in bf16.
"""
import numpy as np
import pytest

import deepinfer_cuda as di
import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 5e-3


@pytest.fixture(scope="module")
def ctx():
    c = di.Context(resident=0)
    yield c
    c.close()


_layers = {}


def layer_pair(ctx, seed, bits, E, D, I, layer=0):
    key = (seed, bits, E, D, I, layer)
    if key not in _layers:
        L = O.Layer(seed, layer=layer, bits=bits, E=E, D=D, I=I)
        _layers[key] = (L, di.MoeLayer.from_oracle(ctx, L))
    return _layers[key]


def check_block(ctx, L, G, T, flags, seed=5, forced=None):
    x = O.gen_bf16(seed, O.ACT_STREAM + T, T * L.D).reshape(T, L.D)
    y, ids, probs, ms = di.moe_block(G, x, flags, forced=forced)
    rc, out, oids, oprobs, logits = O.moe_block(L, x, O.MODE_F32, forced=forced)
    assert rc == 0
    assert np.array_equal(ids, oids), "routing ids differ"
    assert np.max(np.abs(probs - oprobs)) <= 1e-6
    yf = O.bf16_to_f32(y).reshape(T, L.D)
    ma, rl = O.tolerance_report(yf, out)
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)
    return yf, out, ids


@pytest.mark.parametrize("bits", [8, 5])
@pytest.mark.parametrize("T", [1, 3])
def test_decode_gemv_path_small_geometry(ctx, bits, T):
    L, G = layer_pair(ctx, 31, bits, 64, 256, 128)
    check_block(ctx, L, G, T, di.PATH_GEMV)


@pytest.mark.parametrize("bits", [8, 5])
@pytest.mark.parametrize("T", [1, 17, 64, 65, 200])
def test_grouped_path_small_geometry(ctx, bits, T):
    L, G = layer_pair(ctx, 32, bits, 64, 256, 128)
    check_block(ctx, L, G, T, di.PATH_GROUPED)


def test_grouped_path_row_tail(ctx):
    # intermediate 192 = one full and one half 128-row tile of the grouped GEMM
    L, G = layer_pair(ctx, 33, 8, 32, 512, 192)
    check_block(ctx, L, G, 100, di.PATH_GROUPED)


def test_grouped_matches_bf16_operand_oracle_tightly(ctx):
    L, G = layer_pair(ctx, 34, 8, 64, 256, 128)
    T = 96
    x = O.gen_bf16(9, O.ACT_STREAM, T * L.D).reshape(T, L.D)
    y, ids, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    _, out, _, _, _ = O.moe_block(L, x, O.MODE_BF16OPS)
    ma, rl = O.tolerance_report(O.bf16_to_f32(y).reshape(T, L.D), out)
    assert rl < 2e-3, (ma, rl)


@pytest.mark.parametrize("pattern", [0, 1, 2])
def test_forced_route_patterns(ctx, pattern):
    # prefill_expert_checks.mm:26-27 hot / scattered / skewed route patterns
    L, G = layer_pair(ctx, 35, 8, 256, 256, 64)
    T = 129
    t = np.arange(T)[:, None]
    s = np.arange(8)[None, :]
    forced = [s + 0 * t, (t * 7 + s * 13) % 256, (t // 5 * 11 + s * 19) % 256][pattern].astype(np.int32)
    check_block(ctx, L, G, T, di.PATH_GROUPED, forced=forced)


def test_full_geometry_cfg0_prefill_512_tokens(ctx):
    # T=512, hidden 2048, 256 experts, top-8, I=512, shared expert, 8-bit
    L, G = layer_pair(ctx, 1, 8, 256, 2048, 512)
    check_block(ctx, L, G, 512, 0)


@pytest.mark.parametrize("bits", [8, 5])
def test_full_geometry_decode_token(ctx, bits):
    L, G = layer_pair(ctx, 2, bits, 256, 2048, 512)
    check_block(ctx, L, G, 1, 0)


def test_paths_agree_and_are_batch_independent(ctx):
    # each token's result must not depend on which other tokens share the batch
    L, G = layer_pair(ctx, 36, 8, 64, 256, 128)
    T = 40
    x = O.gen_bf16(12, O.ACT_STREAM, T * L.D).reshape(T, L.D)
    y_all, ids_all, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    y_a, ids_a, _, _ = di.moe_block(G, x[:17], di.PATH_GROUPED)
    y_b, ids_b, _, _ = di.moe_block(G, x[17:], di.PATH_GROUPED)
    assert np.array_equal(np.concatenate([ids_a, ids_b]), ids_all)
    assert np.array_equal(np.concatenate([y_a, y_b]), y_all)


def test_non_finite_input_fails_and_leaves_output(ctx):
    L, G = layer_pair(ctx, 37, 8, 64, 256, 128)
    T = 8
    x = O.gen_bf16(13, O.ACT_STREAM, T * L.D).reshape(T, L.D)
    x[3, 5] = 0x7FC0  # NaN
    y = np.full_like(x, 0x1234)
    for flags in (di.PATH_GROUPED, di.PATH_GEMV):
        with pytest.raises(di.DeepInferError, match="Non-finite"):
            G.block(x, T, y, None, None, flags)
        assert np.all(y == 0x1234)


def test_invalid_block_calls_rejected_before_submission(ctx):
    L, G = layer_pair(ctx, 37, 8, 64, 256, 128)
    x = np.zeros((4, 256), np.uint16)
    y = np.full_like(x, 7)
    with pytest.raises(di.DeepInferError):
        G.block(x, 0, y)
    with pytest.raises(di.DeepInferError):
        G.block(x, 4, y, flags=di.PATH_GEMV | di.PATH_GROUPED)
    bad = np.full((4, 8), 64, np.int32)
    with pytest.raises(di.DeepInferError, match="out of bounds"):
        G.block(x, 4, y, bad, None, di.FORCE_ROUTES)
    assert np.all(y == 7)


def test_zipf_router_bias_shifts_load(ctx):
    E = 64
    b = (-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    L = O.Layer(38, bits=8, E=E, D=256, I=64, router_bias=b)
    G = di.MoeLayer.from_oracle(ctx, L)
    _, _, ids = check_block(ctx, L, G, 256, di.PATH_GROUPED)
    counts = np.bincount(ids.reshape(-1), minlength=E)
    assert counts[:8].sum() > counts[-8:].sum()
    G.close()


def test_stack_teacher_forced_layers(ctx):
    # x_{l+1} = x_l + block_l(bf16(RMSNorm(x_l) * w_l)); every layer is checked on the GPU's own
    # layer input h_l, so routing must match bit for bit at every depth
    n, D = 3, 256
    pairs = [layer_pair(ctx, 40, 8, 64, D, 128, layer=l) for l in range(n)]
    norms = (1.0 + 0.1 * np.sin(np.arange(n * D))).astype(np.float32).reshape(n, D)
    for flags, T in ((di.PATH_GROUPED, 24), (di.PATH_GEMV, 12), (di.PATH_GEMV, 1)):
        x0 = O.bf16_to_f32(O.gen_bf16(14, O.ACT_STREAM + T, T * D)).reshape(T, D)
        xg, ht, it, _ = di.moe_stack(ctx, [p[1] for p in pairs], norms, x0, 1e-6, flags, trace=True)
        x = x0.copy()
        for l, (L, _) in enumerate(pairs):
            rc, out, ids, _, _ = O.moe_block(L, ht[l], O.MODE_F32)
            assert rc == 0 and np.array_equal(ids, it[l])
            x = x + out
        ma, rl = O.tolerance_report(xg, x)
        assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


@pytest.mark.parametrize("bits", [8, 5])
def test_full_geometry_decode_stack(ctx, bits):
    # one token through two full-size layers in the persistent stack kernel (one launch for both),
    # checked layer by layer like the test above; a second call must give the same result
    n, D, T = 2, 2048, 1
    pairs = [layer_pair(ctx, 42, bits, 256, D, 512, layer=l) for l in range(n)]
    norms = (1.0 + 0.05 * np.cos(np.arange(n * D))).astype(np.float32).reshape(n, D)
    x0 = O.bf16_to_f32(O.gen_bf16(16, O.ACT_STREAM, T * D)).reshape(T, D)
    for _ in range(2):
        xg, ht, it, _ = di.moe_stack(ctx, [p[1] for p in pairs], norms, x0, 1e-6, di.PATH_GEMV, trace=True)
        x = x0.copy()
        for l, (L, _) in enumerate(pairs):
            rc, out, ids, _, _ = O.moe_block(L, ht[l], O.MODE_F32)
            assert rc == 0 and np.array_equal(ids, it[l])
            x = x + out
        ma, rl = O.tolerance_report(xg, x)
        assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


@pytest.mark.parametrize("bits", [8, 5])
def test_persistent_stack_small_geometry(ctx, bits):
    # D = I = 512 and E = 64: the one-token stack runs as one persistent kernel whose exchanges
    # carry 65 router words (the shared expert's gate logit after the last expert); layer 1 has a
    # router bias. Repeated calls must give the same bits (fresh exchange generations each call).
    n, D, E = 3, 512, 64
    bias = (-0.5 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    oracle_layers = [O.Layer(44, layer=l, bits=bits, E=E, D=D, I=512, router_bias=bias if l == 1 else None)
                     for l in range(n)]
    layers = [di.MoeLayer.from_oracle(ctx, L) for L in oracle_layers]
    norms = (1.0 + 0.1 * np.sin(np.arange(n * D))).astype(np.float32).reshape(n, D)
    x0 = O.bf16_to_f32(O.gen_bf16(17, O.ACT_STREAM, D)).reshape(1, D)
    first = None
    for _ in range(3):
        xg, ht, it, _ = di.moe_stack(ctx, layers, norms, x0, 1e-6, di.PATH_GEMV, trace=True)
        x = x0.copy()
        for l, L in enumerate(oracle_layers):
            rc, out, ids, _, _ = O.moe_block(L, ht[l], O.MODE_F32)
            assert rc == 0 and np.array_equal(ids, it[l])
            x = x + out
        ma, rl = O.tolerance_report(xg, x)
        assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)
        if first is None:
            first = xg
        assert np.array_equal(first, xg)
    for G in layers:
        G.close()


def test_stack_output_beyond_fixed_point_range_is_recomputed(ctx):
    # the one-token kernel adds the experts' outputs in a fixed-point accumulator that takes
    # contributions below 2^23; a shared expert whose down scales and biases are multiplied by 2^32
    # (exact in bf16) exceeds it, so the kernel leaves x unwritten and the host computes the token
    # with the per-layer kernels; an ordinary call afterwards runs in the persistent kernel again
    D = 512
    L = O.Layer(46, bits=8, E=64, D=D, I=512)
    m = L.m["shared_down"]
    for arr in (m.scales, m.biases):
        nz = (arr & 0x7F80) != 0
        arr[nz] += np.uint16(32 << 7)
    G = di.MoeLayer.from_oracle(ctx, L)
    x0 = O.bf16_to_f32(O.gen_bf16(18, O.ACT_STREAM, D)).reshape(1, D)
    xg, ht, it, _ = di.moe_stack(ctx, [G], np.ones((1, D), np.float32), x0, 1e-6, di.PATH_GEMV, trace=True)
    rc, out, ids, _, _ = O.moe_block(L, ht[0], O.MODE_F32)
    assert rc == 0 and np.array_equal(ids, it[0])
    ref = x0 + out
    assert np.abs(ref).max() > 2.0**26
    assert np.linalg.norm(xg - ref) / np.linalg.norm(ref) <= REL_L2
    G.close()
    L2, G2 = layer_pair(ctx, 47, 8, 64, D, 512)
    xg, ht, it, _ = di.moe_stack(ctx, [G2], np.ones((1, D), np.float32), x0, 1e-6, di.PATH_GEMV, trace=True)
    rc, out, ids, _, _ = O.moe_block(L2, ht[0], O.MODE_F32)
    assert rc == 0 and np.array_equal(ids, it[0])
    ma, rl = O.tolerance_report(xg, x0 + out)
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


def test_top8_exact_ties_go_to_the_lower_id(ctx):
    # router rows 3, 40, 77, 150 and 10, 11 are copies of one another with equal bias, so their
    # logits tie exactly; the selection order must be ascending id within each tie group in the
    # prefill top-8, the per-layer decode route kernel and the persistent stack kernel alike
    E, D = 256, 512
    L = O.Layer(45, bits=8, E=E, D=D, I=512)
    r = L.m["router"]
    bias = np.zeros(E, np.float32)
    for group, b in (((3, 40, 77, 150), 4.0), ((10, 11), 2.0)):
        for row in group[1:]:
            r.packed[0, row] = r.packed[0, group[0]]
            r.scales[0, row] = r.scales[0, group[0]]
            r.biases[0, row] = r.biases[0, group[0]]
        bias[list(group)] = b
    L.router_bias = bias
    G = di.MoeLayer.from_oracle(ctx, L)
    for T, flags in ((33, di.PATH_GROUPED), (1, di.PATH_GEMV)):
        _, _, ids = check_block(ctx, L, G, T, flags)
        assert list(ids[0, :4]) == [3, 40, 77, 150]
    x0 = O.bf16_to_f32(O.gen_bf16(18, O.ACT_STREAM, D)).reshape(1, D)
    norms = np.ones((1, D), np.float32)
    _, ht, it, _ = di.moe_stack(ctx, [G], norms, x0, 1e-6, di.PATH_GEMV, trace=True)
    _, _, oids, _, _ = O.moe_block(L, ht[0], O.MODE_F32)
    assert np.array_equal(it[0], oids) and list(it[0, 0, :4]) == [3, 40, 77, 150]
    G.close()


def test_router_many_tied_candidates_fall_back_to_all_exact(ctx):
    # 80 identical router rows with equal bias tie exactly and lead by a wide margin, so every token
    # has more candidates than the tensor-core router's exact check takes (64): the top-8 comes
    # from all 256 exact logits and must be the 8 lowest ids of the tied group
    E, D = 256, 512
    L = O.Layer(46, bits=8, E=E, D=D, I=512)
    r = L.m["router"]
    group = list(range(7, 247, 3))[:80]
    for row in group[1:]:
        r.packed[0, row] = r.packed[0, group[0]]
        r.scales[0, row] = r.scales[0, group[0]]
        r.biases[0, row] = r.biases[0, group[0]]
    bias = np.zeros(E, np.float32)
    bias[group] = 6.0
    L.router_bias = bias
    G = di.MoeLayer.from_oracle(ctx, L)
    for T, flags in ((40, di.PATH_GROUPED), (1, di.PATH_GEMV)):
        _, _, ids = check_block(ctx, L, G, T, flags)
        assert np.all(ids == np.array(group[:8], np.int32)[None, :])
    G.close()


def test_decode_stack_graph_replays_match(ctx):
    # the decode stack is captured as a CUDA graph on first use and replayed afterwards;
    # replays must give the same bits as the first (captured) run, and a changed input must flow
    n, D, T = 2, 256, 2
    pairs = [layer_pair(ctx, 41, 8, 64, D, 128, layer=l) for l in range(n)]
    norms = np.ones((n, D), np.float32)
    x0 = O.bf16_to_f32(O.gen_bf16(15, O.ACT_STREAM, T * D)).reshape(T, D)
    layers = [p[1] for p in pairs]
    a = di.moe_stack(ctx, layers, norms, x0, 1e-6, di.PATH_GEMV)[0]
    b = di.moe_stack(ctx, layers, norms, x0, 1e-6, di.PATH_GEMV)[0]
    c = di.moe_stack(ctx, layers, norms, x0 * 0.5, 1e-6, di.PATH_GEMV)[0]
    assert np.array_equal(a, b) and not np.array_equal(a, c)


def _oracle_rows(L, x, rows):
    # the oracle's block output and ids for a subset of rows (each token is independent)
    rc, out, ids, _, _ = O.moe_block(L, x[rows], O.MODE_F32)
    assert rc == 0
    return out, ids


def test_cfg3_zipf_32k_prefill_5bit(ctx):
    # BASELINE configs[3] on one GPU: one 5-bit full-geometry layer, 32K tokens, router logits
    # biased by -1.1 ln(e + 1) so a few experts take most routes (ragged, imbalanced grouped GEMMs).
    # Sampled rows against the oracle; the same rows alone give the same bits.
    E, D, T = 256, 2048, 32768
    bias = (-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    L = O.Layer(50, bits=5, E=E, D=D, I=512, router_bias=bias)
    G = di.MoeLayer.from_oracle(ctx, L)
    x = O.gen_bf16(19, O.ACT_STREAM, T * D).reshape(T, D)
    y, ids, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    counts = np.bincount(ids.reshape(-1), minlength=E)
    assert counts.max() > 8 * counts.mean() and counts[:8].sum() > 0.1 * ids.size
    rows = np.random.default_rng(3).choice(T, 48, replace=False)
    rows.sort()
    out, oids = _oracle_rows(L, x, rows)
    assert np.array_equal(ids[rows], oids)
    ma, rl = O.tolerance_report(O.bf16_to_f32(y[rows]), out)
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)
    y_s, ids_s, _, _ = di.moe_block(G, np.ascontiguousarray(x[rows]), di.PATH_GROUPED)
    assert np.array_equal(ids_s, ids[rows]) and np.array_equal(y_s, y[rows])
    G.close()


def test_cfg4_ragged_packed_batch_matches_unpacked_requests(ctx):
    # BASELINE configs[4] on one GPU: 16 requests of lengths drawn in [1, 4096] plus 48 single-token
    # rows packed into one batch through one 8-bit full-geometry layer; every request run on its own
    # gives the same bits row for row, and sampled rows match the oracle
    E, D = 256, 2048
    L, G = layer_pair(ctx, 1, 8, E, D, 512)
    rng = np.random.default_rng(4)
    lengths = list(rng.integers(1, 4097, 16)) + [1] * 48
    T = int(sum(lengths))
    x = O.gen_bf16(20, O.ACT_STREAM, T * D).reshape(T, D)
    y, ids, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    start = 0
    for n in lengths:
        y_r, ids_r, _, _ = di.moe_block(G, np.ascontiguousarray(x[start:start + n]), di.PATH_GROUPED)
        assert np.array_equal(ids_r, ids[start:start + n]) and np.array_equal(y_r, y[start:start + n]), (start, n)
        start += n
    rows = np.sort(rng.choice(T, 48, replace=False))
    out, oids = _oracle_rows(L, x, rows)
    assert np.array_equal(ids[rows], oids)
    ma, rl = O.tolerance_report(O.bf16_to_f32(y[rows]), out)
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


def test_router_weights_changed_after_a_call_are_used(ctx):
    # the tensor-core router keeps each layer's router-row norms and f32 rows between calls; new
    # router weights, uploaded or written through the host staging buffer, must reach the next call
    E, D = 256, 512
    L = O.Layer(48, bits=8, E=E, D=D, I=64)
    G = di.MoeLayer.from_oracle(ctx, L)
    check_block(ctx, L, G, 96, di.PATH_GROUPED)
    L.m["router"] = O.Layer(49, bits=8, E=E, D=D, I=64).m["router"]
    G.mats["router"].load(L.m["router"])
    check_block(ctx, L, G, 96, di.PATH_GROUPED)
    L.m["router"] = O.Layer(50, bits=8, E=E, D=D, I=64).m["router"]
    for i, a in enumerate((L.m["router"].packed, L.m["router"].scales, L.m["router"].biases)):
        G.mats["router"].write(i, a)
    check_block(ctx, L, G, 96, di.PATH_GROUPED)
    G.close()
