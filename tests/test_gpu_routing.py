"""Routing and permutation parity at the benchmark's own geometry (256 experts, hidden 2048).

Bar (north star): routing ids and the expert-grouped permutation bit-exact, ties to the lower
expert id.

- The prefill router computes approximate logits on the tensor cores and recomputes only the
  near-boundary candidates in the canonical f32 order. Its ids, probabilities and block outputs
  must equal, bit for bit and for every token, those of the router that evaluates every logit in
  the canonical order (DI_MOE_ROUTER_EXACT), which the oracle pins on sampled rows. Checked on
  the 8K-token 8-bit batch of the benchmark, the 32K-token 5-bit Zipf batch and the ragged packed
  batch ([3], [4]).
- The permutation read back from the GPU must equal the oracle's stable counting sort
  (native/DeepInfer.Metal/prefill_moe.mm:8-17; the coverage check of
  native/DeepInfer.Metal/prefill_expert_checks.mm:44-49) for routed and forced patterns.
- The benchmark's 40-layer 8K-token stack is checked teacher-forced: every layer's ids against
  the all-exact router on that layer's input rows, and sampled rows against the oracle.
"""
import numpy as np
import pytest

import deepinfer_cuda as di
import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 5e-3
BENCH_SEED = 20261201  # the seed bench.py generates its layers from


@pytest.fixture(scope="module")
def ctx():
    c = di.Context(resident=0)
    yield c
    c.close()


def _tc_vs_exact(G, x):
    y, ids, probs, _ = di.moe_block(G, x, di.PATH_GROUPED)
    ye, ide, pe, _ = di.moe_block(G, x, di.PATH_GROUPED | di.ROUTER_EXACT)
    assert np.array_equal(ids, ide), f"{int((ids != ide).any(axis=1).sum())} tokens route differently"
    assert np.array_equal(probs.view(np.uint32), pe.view(np.uint32))
    assert np.array_equal(y, ye)
    return y, ids


def _oracle_rows(L, x, y, ids, rows):
    rc, out, oids, _, _ = O.moe_block(L, x[rows], O.MODE_F32)
    assert rc == 0 and np.array_equal(ids[rows], oids)
    ma, rl = O.tolerance_report(O.bf16_to_f32(y[rows]), out)
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


def test_tensor_core_router_equals_all_exact_8k_8bit(ctx):
    # one 8-bit layer of the benchmark's weights, 8192 tokens
    G = di.MoeLayer.generated(ctx, BENCH_SEED, 0, bits=8)
    x = O.gen_bf16(BENCH_SEED, O.ACT_STREAM, 8192 * 2048).reshape(8192, 2048)
    y, ids = _tc_vs_exact(G, x)
    L = O.Layer(BENCH_SEED, layer=0, bits=8)
    _oracle_rows(L, x, y, ids, np.sort(np.random.default_rng(1).choice(8192, 32, replace=False)))
    G.close()


def test_tensor_core_router_equals_all_exact_32k_zipf_5bit(ctx):
    # 5-bit weights, 32K tokens, router logits biased toward Zipf(1.1) loads
    E, T = 256, 32768
    bias = (-1.1 * np.log(np.arange(E) + 1.0)).astype(np.float32)
    G = di.MoeLayer.generated(ctx, 51, 0, bits=5)
    G.set_router_bias(bias)
    x = O.gen_bf16(21, O.ACT_STREAM, T * 2048).reshape(T, 2048)
    _, ids = _tc_vs_exact(G, x)
    counts = np.bincount(ids.reshape(-1), minlength=E)
    assert counts.max() > 8 * counts.mean()
    G.close()


def test_tensor_core_router_equals_all_exact_ragged_batch(ctx):
    # 16 requests of lengths in [1, 4096] and 48 single tokens, packed
    rng = np.random.default_rng(4)
    T = int(sum(rng.integers(1, 4097, 16))) + 48
    G = di.MoeLayer.generated(ctx, 52, 0, bits=8)
    x = O.gen_bf16(22, O.ACT_STREAM, T * 2048).reshape(T, 2048)
    _tc_vs_exact(G, x)
    G.close()


@pytest.mark.parametrize("T", [64, 65, 512, 8192])
def test_permutation_matches_oracle_routed(ctx, T):
    L = O.Layer(60, bits=8, E=256, D=256, I=64)
    G = di.MoeLayer.from_oracle(ctx, L)
    x = O.gen_bf16(23, O.ACT_STREAM + T, T * 256).reshape(T, 256)
    _, ids, _, _ = di.moe_block(G, x, di.PATH_GROUPED)
    perm, off, cnt = ctx.last_routes(T, 256)
    counts, offsets, routes = O.permute(ids, 256)
    assert np.array_equal(cnt[:256], counts) and np.array_equal(off[:256], offsets)
    assert np.array_equal(perm, routes)
    assert off[256] == 8 * T and cnt[256] == T  # the shared expert's segment follows the routed ones
    # every route exactly once, under its own expert, in ascending route order
    # (prefill_expert_checks.mm:44-49)
    assert np.array_equal(np.sort(perm), np.arange(8 * T))
    for e in np.flatnonzero(cnt[:256]):
        seg = perm[off[e]:off[e] + cnt[e]]
        assert np.all(ids.reshape(-1)[seg] == e) and np.all(np.diff(seg) > 0)
    G.close()


@pytest.mark.parametrize("pattern", [0, 1, 2])
@pytest.mark.parametrize("T", [129, 8192])
def test_permutation_matches_oracle_forced(ctx, pattern, T):
    # the hot / scattered / skewed route patterns of prefill_expert_checks.mm:26-27
    L = O.Layer(61, bits=8, E=256, D=256, I=64)
    G = di.MoeLayer.from_oracle(ctx, L)
    t = np.arange(T)[:, None]
    s = np.arange(8)[None, :]
    forced = [s + 0 * t, (t * 7 + s * 13) % 256, (t // 5 * 11 + s * 19) % 256][pattern].astype(np.int32)
    x = O.gen_bf16(24, O.ACT_STREAM + T, T * 256).reshape(T, 256)
    di.moe_block(G, x, di.PATH_GROUPED, forced=forced)
    perm, off, cnt = ctx.last_routes(T, 256)
    counts, offsets, routes = O.permute(forced, 256)
    assert np.array_equal(cnt[:256], counts) and np.array_equal(off[:256], offsets)
    assert np.array_equal(perm, routes)
    G.close()


def test_bench_stack_teacher_forced_40_layers(ctx):
    # the benchmark's own workload: 40 layers of 256 experts (hidden 2048, 8-bit) over 8192 tokens.
    # Every layer's ids (all tokens) equal the all-exact router's on that layer's input rows;
    # sampled rows of three layers match the oracle.
    n, T, D = 40, 8192, 2048
    layers = [di.MoeLayer.generated(ctx, BENCH_SEED, l, bits=8) for l in range(n)]
    x0 = O.bf16_to_f32(O.gen_bf16(BENCH_SEED, O.ACT_STREAM + 7, T * D)).reshape(T, D)
    norms = np.ones((n, D), np.float32)
    xg, ht, it, _ = di.moe_stack(ctx, layers, norms, x0, 1e-6, di.PATH_GROUPED, trace=True)
    assert np.all(np.isfinite(xg))
    for l in range(n):
        y, ids, _, _ = di.moe_block(layers[l], ht[l], di.PATH_GROUPED | di.ROUTER_EXACT)
        assert np.array_equal(ids, it[l]), f"layer {l}"
        if l in (0, 19, 39):
            rows = np.sort(np.random.default_rng(l).choice(T, 12, replace=False))
            _oracle_rows(O.Layer(BENCH_SEED, layer=l, bits=8), ht[l], y, ids, rows)
    for G in layers:
        G.close()


def test_first_call_of_a_fresh_context_equals_later_calls():
    # A fresh context's first call runs on a freshly allocated workspace with cold caches; its
    # outputs must equal the next calls' bit for bit (a race that lets a later store overwrite an
    # expert-row chunk still being copied out would show up here first). Several fresh contexts,
    # the benchmark's 8K-token 8-bit layer.
    x = O.gen_bf16(BENCH_SEED, O.ACT_STREAM, 8192 * 2048).reshape(8192, 2048)
    ref = None
    for _ in range(4):
        c = di.Context(resident=0)
        G = di.MoeLayer.generated(c, BENCH_SEED, 0, bits=8)
        first = di.moe_block(G, x, di.PATH_GROUPED)[0]
        second = di.moe_block(G, x, di.PATH_GROUPED)[0]
        assert np.array_equal(first, second)
        if ref is None:
            ref = first
        assert np.array_equal(first, ref)
        G.close()
        c.close()
