// Router, top-8 selection and the stable expert-grouped permutation.
//
// Router logits follow one fixed f32 evaluation order so that expert ids are reproducible
// bit for bit by the CPU oracle: lane l of a 32-lane group owns columns 256*b + 8*l + j
// (j = 0..7), accumulated b-major with w = fma(q, scale, bias) and acc = fma(w, x, acc),
// then the xor butterfly 16,8,4,2,1 -- the lane partition and reduction of the reference
// CUDA gemv kernel (native/DeepInfer.Cuda/split_prefix.cu:63-67, :106-120).
#pragma once
#include "common.cuh"
#include "peer.cuh"

namespace di {

// ------------------------------------------------------------------ shared helpers

// fma over a pair of f32 lanes: d = a*b + c elementwise, one rounding each (sm_100 FFMA2).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Raw codes, scales and biases of one lane's columns of an 8-bit router row, up to 8 column
// blocks of 256 (D <= 2048), loaded ahead of the activation row they will meet.
struct RouterRaw {
    uint2 q[8];
    uint16_t s[8], b[8];
};
__device__ __forceinline__ void router_raw_load(const QView &m, int row, int D, RouterRaw &r) {
    const uint32_t lane = lane_id();
    const uint32_t *w = m.packed + (size_t)row * m.words_per_row();
    const uint16_t *sc = m.scales + (size_t)row * m.groups_per_row();
    const uint16_t *bi = m.biases + (size_t)row * m.groups_per_row();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int base = k * 256 + lane * 8;
        if (base < D) {
            r.q[k] = __ldg(reinterpret_cast<const uint2 *>(w + base / 4));
            r.s[k] = __ldg(sc + base / 64);
            r.b[k] = __ldg(bi + base / 64);
        }
    }
}
// The canonical dot product (below) of a preloaded row with x (shared or global memory).
__device__ __forceinline__ float router_raw_dot(const RouterRaw &r, const uint16_t *x, int D) {
    const uint32_t lane = lane_id();
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int base = k * 256 + lane * 8;
        if (base >= D) break;
        const uint4 xv = *reinterpret_cast<const uint4 *>(x + base);
        const float s = bf16_bits_to_f32(r.s[k]), bb = bf16_bits_to_f32(r.b[k]);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float wv = fmaf(byte_to_f32(j < 4 ? r.q[k].x : r.q[k].y, j & 3), s, bb);
            const float xf = (j & 1) ? bf16_hi(xw[j >> 1]) : bf16_lo(xw[j >> 1]);
            acc = fmaf(wv, xf, acc);
        }
    }
    return warp_sum_butterfly(acc);
}

// Canonical dot product of one 8-bit router row with one bf16 activation row (in global or
// shared memory), evaluated by a whole warp; returns the same value in every lane. The codes,
// scales and biases of up to 8 column blocks are requested before any of them is used (one
// memory round trip per 2048 columns instead of one per block); the arithmetic order is the
// canonical one.
__device__ __forceinline__ float canonical_dot_warp(const QView &m, int row, const uint16_t *x, int D) {
    const uint32_t lane = lane_id();
    const uint32_t *w = m.packed + (size_t)row * m.words_per_row();
    const uint16_t *sc = m.scales + (size_t)row * m.groups_per_row();
    const uint16_t *bi = m.biases + (size_t)row * m.groups_per_row();
    const int nb = D / 256;
    float acc = 0.0f;
    for (int b0 = 0; b0 < nb; b0 += 8) {
        uint2 q[8];
        uint16_t sv[8], bv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int base = (b0 + k) * 256 + lane * 8;
            if (b0 + k < nb) {
                q[k] = __ldg(reinterpret_cast<const uint2 *>(w + base / 4));
                sv[k] = __ldg(sc + base / 64);
                bv[k] = __ldg(bi + base / 64);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (b0 + k >= nb) break;
            const int base = (b0 + k) * 256 + lane * 8;
            const uint4 xv = *reinterpret_cast<const uint4 *>(x + base);  // x may be shared or global
            const float s = bf16_bits_to_f32(sv[k]), bb = bf16_bits_to_f32(bv[k]);
            const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float wv = fmaf(byte_to_f32(j < 4 ? q[k].x : q[k].y, j & 3), s, bb);
                const float xf = (j & 1) ? bf16_hi(xw[j >> 1]) : bf16_lo(xw[j >> 1]);
                acc = fmaf(wv, xf, acc);
            }
        }
    }
    return warp_sum_butterfly(acc);
}

// ------------------------------------------------------------------ router GEMM (SIMT)
//
// logits[t, e] for a tile of 64 tokens x 16 experts per CTA (16 warps: 8 token groups x 2
// expert groups, 8x8 outputs per warp). 256-column blocks of x and the 8-bit codes are staged
// with cp.async three deep; one barrier per block. After it, the CTA dequantises the next
// block's 16 x 256 weights once into f32 shared memory (w = fma(q, s, b), double buffered)
// while every lane accumulates its 64 outputs over its own 8 columns of the current block in
// the canonical order with paired f32 FMAs (pairs of tokens). The 32-lane reduction is a
// reduce-scatter whose every partial sum is the one the xor butterfly 16,8,4,2,1 forms
// (a + b == b + a exactly), so each logit is bit-identical to the butterfly's.
namespace router {
constexpr int TT = 64, TE = 16, KB = 256, THREADS = 512, XS = 3;
struct Smem {
    uint16_t x[XS][TT][KB];       // 32 KB per stage
    uint8_t q[XS][TE][KB];        // 4 KB per stage
    uint16_t s[XS][TE][KB / 64];
    uint16_t b[XS][TE][KB / 64];
    // dequantised weights of a block, laid out [expert][half][lane][4] so that lane l's
    // columns 8l..8l+3 (half 0) and 8l+4..8l+7 (half 1) are contiguous across lanes
    float w[2][TE][2][32][4];
};
}  // namespace router

__global__ void __launch_bounds__(router::THREADS, 1)
router_logits_kernel(const uint16_t *__restrict__ x, int T, int D, QView W, const float *__restrict__ bias,
                     float *__restrict__ logits) {
    using namespace router;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    const int E = W.rows;
    const int wt = (warp & 7) * 8, we = (warp >> 3) * 8;  // warp's token / expert offsets in the tile
    const int nkb = D / KB;
    const int wpr = W.words_per_row(), gpr = W.groups_per_row();

    auto stage = [&](int kb) {
        const int buf = kb % XS;
        // x: 64 rows x 512 B = 2048 chunks of 16 B, 4 per thread
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = tid + i * THREADS, r = c >> 5, ch = c & 31;
            const int t = t0 + r;
            const uint16_t *src = x + (size_t)min(t, T - 1) * D + kb * KB + ch * 8;
            cp_async_16(&sm.x[buf][r][ch * 8], src, t < T);
        }
        if (tid < 256) {  // codes: 16 rows x 256 B = 256 chunks
            const int r = tid >> 4, ch = tid & 15, e = e0 + r;
            const uint32_t *src = W.packed + (size_t)min(e, E - 1) * wpr + kb * (KB / 4) + ch * 4;
            cp_async_16(&sm.q[buf][r][ch * 16], src, e < E);
        } else if (tid < 256 + 2 * TE) {  // scales / biases: 4 groups (8 bytes) per expert row
            const int i = tid - 256, r = i >> 1, e = min(e0 + r, E - 1);
            const uint16_t *src = ((i & 1) ? W.biases : W.scales) + (size_t)e * gpr + kb * (KB / 64);
            cp_async_8((i & 1) ? (void *)sm.b[buf][r] : (void *)sm.s[buf][r], src);
        }
        cp_async_commit();
    };
    // thread -> (expert tid / 32, lane tid % 32's 8 columns) of a block
    auto dequant = [&](int kb) {
        const int buf = kb % XS, r = tid >> 5, l = tid & 31;
        const float sc = bf16_bits_to_f32(sm.s[buf][r][l >> 3]), bi = bf16_bits_to_f32(sm.b[buf][r][l >> 3]);
        const uint2 q = *reinterpret_cast<const uint2 *>(&sm.q[buf][r][l * 8]);
        float4 v0, v1;
        v0.x = fmaf(byte_to_f32(q.x, 0), sc, bi);
        v0.y = fmaf(byte_to_f32(q.x, 1), sc, bi);
        v0.z = fmaf(byte_to_f32(q.x, 2), sc, bi);
        v0.w = fmaf(byte_to_f32(q.x, 3), sc, bi);
        v1.x = fmaf(byte_to_f32(q.y, 0), sc, bi);
        v1.y = fmaf(byte_to_f32(q.y, 1), sc, bi);
        v1.z = fmaf(byte_to_f32(q.y, 2), sc, bi);
        v1.w = fmaf(byte_to_f32(q.y, 3), sc, bi);
        *reinterpret_cast<float4 *>(&sm.w[kb & 1][r][0][l][0]) = v0;
        *reinterpret_cast<float4 *>(&sm.w[kb & 1][r][1][l][0]) = v1;
    };

    float2 acc[4][8];  // [token pair][expert]: (token 2p, token 2p+1)
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[p][e] = make_float2(0.f, 0.f);

    stage(0);
    cp_async_wait<0>();
    __syncthreads();
    if (nkb > 1) stage(1);
    dequant(0);
    for (int kb = 0; kb < nkb; ++kb) {
        cp_async_wait<0>();  // block kb + 1 (this thread's copies)
        __syncthreads();     // every copy of kb + 1, w of kb, and the reads of block kb - 1 are done
        if (kb + 2 < nkb) stage(kb + 2);
        if (kb + 1 < nkb) dequant(kb + 1);
        const int xb = kb % XS, wb = kb & 1;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            // x of this lane's columns 8l + 4h .. +3 for the warp's 8 tokens, as f32 pairs (t, t+1)
            float2 xp[4][4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint2 a = *reinterpret_cast<const uint2 *>(&sm.x[xb][wt + 2 * p][lane * 8 + 4 * h]);
                const uint2 c = *reinterpret_cast<const uint2 *>(&sm.x[xb][wt + 2 * p + 1][lane * 8 + 4 * h]);
                xp[p][0] = make_float2(bf16_lo(a.x), bf16_lo(c.x));
                xp[p][1] = make_float2(bf16_hi(a.x), bf16_hi(c.x));
                xp[p][2] = make_float2(bf16_lo(a.y), bf16_lo(c.y));
                xp[p][3] = make_float2(bf16_hi(a.y), bf16_hi(c.y));
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 wv = *reinterpret_cast<const float4 *>(&sm.w[wb][we + e][h][lane][0]);
                const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 w2 = make_float2(w4[j], w4[j]);
#pragma unroll
                    for (int p = 0; p < 4; ++p) acc[p][e] = ffma2(xp[p][j], w2, acc[p][e]);
                }
            }
        }
    }
    // reduce-scatter over the 32 lanes: outputs o = p*16 + e*2 + k (token 2p+k, expert e);
    // at mask m the lane keeps the upper or lower half of its list and adds the partner's
    // partial of the same outputs; lane l ends with outputs 2l and 2l + 1
    float v[64];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            v[p * 16 + e * 2] = acc[p][e].x;
            v[p * 16 + e * 2 + 1] = acc[p][e].y;
        }
#pragma unroll
    for (int m = 16, n = 64; m >= 1; m >>= 1, n >>= 1) {
        const bool high = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = high ? v[i] : v[i + n / 2];
            const float keep = high ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(kFull, send, m);
        }
    }
    const int p = lane >> 3, ee = e0 + we + (lane & 7), ta = t0 + wt + 2 * p;
    if (ee < E) {
        const float bb = bias ? bias[ee] : 0.f;
        if (ta < T) logits[(size_t)ta * E + ee] = v[0] + bb;
        if (ta + 1 < T) logits[(size_t)(ta + 1) * E + ee] = v[1] + bb;
    }
}

// Decode-sized router: one warp per expert row, all T (<= 8) tokens per warp.
__global__ void router_logits_gemv_kernel(const uint16_t *__restrict__ x, int T, int D, QView W,
                                          const float *__restrict__ bias, float *__restrict__ logits) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp >= W.rows) return;
    const float bb = bias ? bias[warp] : 0.f;
    for (int t = 0; t < T; ++t) {
        float v = canonical_dot_warp(W, warp, x + (size_t)t * D, D);
        if (lane_id() == 0) logits[(size_t)t * W.rows + warp] = v + bb;
    }
}

// ------------------------------------------------------------------ top-8 + histogram
//
// One warp per token. Selection: 8 rounds of a warp arg-max over (value desc, index asc),
// i.e. the 8 largest logits in descending order with ties to the lower expert id
// (Qwen36Model.cs:246-258; graph_top8 in gpu_graph.mm:134-146). probs = softmax over the
// 8 chosen logits (Qwen36Model.cs:259-261, :293-298). Non-finite logits set kErrNonFinite.
// The warp also computes the shared-route gate logit (canonical order). Each CTA owns a
// contiguous token range and writes the per-expert route counts of that range.
// The 8 largest logits in descending order with ties to the lower expert id. v[j] is this
// lane's candidate lane + 32j; all lanes return the same sel/chosen. Non-finite candidates must
// already be replaced by -inf. Each lane first sorts its 8 candidates (a 19-comparator network
// on (value desc, id asc)); each of the 8 rounds is then a warp max of the lanes' heads as
// order-preserving integer keys and, among equal keys, a warp min of their ids (redux.sync),
// after which the winning lane drops its head. -0 ranks as +0 (they compare equal as floats).
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ void select_top8(const float *v, int E, int32_t *sel, float *chosen) {
    const int lane = lane_id();
    uint32_t key[8], id[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        id[j] = (uint32_t)(lane + 32 * j);
        key[j] = (int)id[j] < E ? order_key(v[j]) : 0u;  // every real key (even -inf's) is above 0
    }
    auto cmpswap = [&](int a, int b) {  // afterwards (key, id)[a] precedes (key, id)[b]
        const bool sw = key[b] > key[a] || (key[b] == key[a] && id[b] < id[a]);
        const uint32_t ka = key[a], ia = id[a];
        key[a] = sw ? key[b] : ka;
        id[a] = sw ? id[b] : ia;
        key[b] = sw ? ka : key[b];
        id[b] = sw ? ia : id[b];
    };
    cmpswap(0, 2); cmpswap(1, 3); cmpswap(4, 6); cmpswap(5, 7);
    cmpswap(0, 4); cmpswap(1, 5); cmpswap(2, 6); cmpswap(3, 7);
    cmpswap(0, 1); cmpswap(2, 3); cmpswap(4, 5); cmpswap(6, 7);
    cmpswap(2, 4); cmpswap(3, 5);
    cmpswap(1, 4); cmpswap(3, 6);
    cmpswap(1, 2); cmpswap(3, 4); cmpswap(5, 6);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        const uint32_t best = __reduce_max_sync(kFull, key[0]);
        const uint32_t win = __reduce_min_sync(kFull, key[0] == best ? id[0] : 0xffffffffu);
        sel[n] = (int32_t)win;
        chosen[n] = key_value(best);
        if (id[0] == win) {
#pragma unroll
            for (int j = 0; j < 7; ++j) {
                key[j] = key[j + 1];
                id[j] = id[j + 1];
            }
            key[7] = 0u;
            id[7] = 0xffffffffu;
        }
    }
}

namespace topk {
constexpr int WARPS = 16, TOK_PER_WARP = 4, TOK_PER_CTA = WARPS * TOK_PER_WARP;  // 64 tokens = 512 routes
}

__global__ void __launch_bounds__(topk::WARPS * 32)
topk_count_kernel(const float *__restrict__ logits, int T, int E, const uint16_t *__restrict__ x, int D,
                  QView gateW, const int32_t *__restrict__ forced_ids, int32_t *__restrict__ ids, float *__restrict__ probs,
                  float *__restrict__ gate_logit, int32_t *__restrict__ block_counts, uint32_t *__restrict__ err) {
    using namespace topk;
    __shared__ int32_t hist[256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int k = 0; k < TOK_PER_WARP; ++k) {
        const int t = blockIdx.x * TOK_PER_CTA + warp * TOK_PER_WARP + k;
        if (t >= T) break;
        const float *lg = logits + (size_t)t * E;
        int32_t sel[8];
        float chosen[8];
        if (forced_ids) {
            // graph_force_route (gpu_graph.mm:153-159): ids given, probs from their logits;
            // out-of-range ids are flagged and clamped so later kernels stay in bounds
            bool bad = false;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                int id = forced_ids[(size_t)t * 8 + n];
                bad |= (id < 0 || id >= E);
                sel[n] = min(max(id, 0), E - 1);
                chosen[n] = lg[sel[n]];
            }
            if (bad && lane == 0) atomicOr(err, kErrBadExpert);
        } else {
            float v[8];
            bool nonfinite = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int e = lane + 32 * j;
                v[j] = e < E ? lg[e] : 0.f;
                // a non-finite logit fails the call; it is ranked as -inf so that the
                // selection stays well defined (valid, distinct ids) for the later kernels
                if (e < E && !isfinite(v[j])) {
                    nonfinite = true;
                    v[j] = -INFINITY;
                }
            }
            if (__any_sync(kFull, nonfinite) && lane == 0) atomicOr(err, kErrNonFinite);
            select_top8(v, E, sel, chosen);
        }
        // softmax over the chosen logits
        float mx = chosen[0];
#pragma unroll
        for (int n = 1; n < 8; ++n) mx = fmaxf(mx, chosen[n]);
        float p[8], sum = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            p[n] = expf(chosen[n] - mx);
            sum += p[n];
        }
        float g = canonical_dot_warp(gateW, 0, x + (size_t)t * D, D);
        if (lane < 8) {
            int n = lane;
            float pv = 0.f;
            int32_t sv = 0;
#pragma unroll
            for (int m = 0; m < 8; ++m)
                if (m == n) {
                    pv = p[m];
                    sv = sel[m];
                }
            ids[(size_t)t * 8 + n] = sv;
            probs[(size_t)t * 8 + n] = pv / sum;
            atomicAdd(&hist[sv], 1);
        }
        if (lane == 0) gate_logit[t] = g;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) block_counts[(size_t)blockIdx.x * E + i] = hist[i];
}

// ------------------------------------------------------------------ scan + tile list
//
// Single CTA. Histogram buckets e < n_hist (routed experts, plus optionally a bucket for
// routes that belong to another GPU): block_base[blk][e] = routes of e in blocks before blk;
// counts; segment offsets (exclusive scan over buckets). The shared expert is segment n_hist
// with `shared_count` rows placed after all routed positions (offset 8*rows). Emits the work
// tiles of the grouped GEMMs for buckets e < n_tiled and the shared segment: (segment, first
// position, rows), at most `bn` rows each, balanced.
struct Tile {
    int32_t seg, p0, n;
};

constexpr int kMaxBuckets = 260;

__global__ void __launch_bounds__(1024)
scan_tiles_kernel(const int32_t *__restrict__ block_counts, int nblocks, int n_hist, int n_tiled, int rows,
                  int shared_count, int bn, int32_t *__restrict__ block_base, int32_t *__restrict__ seg_count,
                  int32_t *__restrict__ seg_off, Tile *__restrict__ tiles, int32_t *__restrict__ n_tiles, int max_tiles,
                  uint32_t *__restrict__ err) {
    pdl_enter();
    __shared__ int32_t cnt[kMaxBuckets], ntile[kMaxBuckets], toff[kMaxBuckets + 1], off[kMaxBuckets + 1];
    __shared__ int32_t wsum[32][2];
    const int tid = threadIdx.x, S = n_hist;  // segment S = shared expert
    const int lane = tid & 31, warp = tid >> 5;
    if (tid < n_hist) {
        // per-block exclusive prefix of this bucket, eight blocks' counts requested at a time
        int run = 0, b = 0;
        for (; b + 8 <= nblocks; b += 8) {
            int v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = block_counts[(size_t)(b + j) * n_hist + tid];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                block_base[(size_t)(b + j) * n_hist + tid] = run;
                run += v[j];
            }
        }
        for (; b < nblocks; ++b) {
            block_base[(size_t)b * n_hist + tid] = run;
            run += block_counts[(size_t)b * n_hist + tid];
        }
        cnt[tid] = run;
    }
    if (tid == 0) cnt[S] = shared_count;
    __syncthreads();
    // exclusive scans over the buckets e <= S of the routed counts (e < S) and of the tile counts,
    // by warp shuffles and a scan of the warp totals
    int cv = 0, nv = 0;
    if (tid <= S) {
        cv = tid < S ? cnt[tid] : 0;
        nv = (tid < n_tiled || tid == S) ? (cnt[tid] + bn - 1) / bn : 0;
        ntile[tid] = nv;
    }
    int ci = cv, ni = nv;  // inclusive within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int uc = __shfl_up_sync(kFull, ci, o), un = __shfl_up_sync(kFull, ni, o);
        if (lane >= o) {
            ci += uc;
            ni += un;
        }
    }
    if (lane == 31) {
        wsum[warp][0] = ci;
        wsum[warp][1] = ni;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = (S + 32) / 32;  // warps holding buckets 0..S
        int wc = lane < nw ? wsum[lane][0] : 0, wn = lane < nw ? wsum[lane][1] : 0;
        const int c0 = wc, n0 = wn;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int uc = __shfl_up_sync(kFull, wc, o), un = __shfl_up_sync(kFull, wn, o);
            if (lane >= o) {
                wc += uc;
                wn += un;
            }
        }
        if (lane < nw) {
            wsum[lane][0] = wc - c0;  // exclusive over warps
            wsum[lane][1] = wn - n0;
        }
        if (lane == nw - 1) {
            int tr = wn;
            toff[S + 1] = tr;
            if (tr > max_tiles) {
                atomicOr(err, kErrCapacity);
                tr = 0;
            }
            *n_tiles = tr;
        }
    }
    __syncthreads();
    if (tid <= S) {
        off[tid] = tid == S ? 8 * rows : wsum[warp][0] + ci - cv;
        toff[tid] = wsum[warp][1] + ni - nv;
    }
    __syncthreads();
    if (tid <= S) {
        seg_count[tid] = cnt[tid];
        seg_off[tid] = off[tid];
        if (toff[S + 1] <= max_tiles)
            for (int i = 0; i < ntile[tid]; ++i) {
                // balanced split: tile sizes differ by at most one row
                const int a = (int)((int64_t)i * cnt[tid] / ntile[tid]);
                const int b = (int)((int64_t)(i + 1) * cnt[tid] / ntile[tid]);
                tiles[toff[tid] + i] = Tile{tid, off[tid] + a, b - a};
            }
    }
}

// ------------------------------------------------------------------ stable scatter
//
// Each CTA re-reads the routes of its token range in ascending route order and places
// route r = t*8 + slot at seg_off[e] + block_base[blk][e] + (rank of r among earlier
// routes of e in this block): the stable counting sort (prefill_moe.mm:12-14 order).
constexpr int kScatterWarps = topk::TOK_PER_CTA * 8 / 32;  // one warp per 32 routes of a block
// The stable scatter fused with the copy of the block's token rows into expert order: after
// the positions are known, each warp copies its tokens' rows (read once) to their 8 positions
// each, so the permuted rows are written without a second pass over the permutation. SPLIT CTAs
// share a block of 64 tokens: each recomputes the block's positions (cheap), the first writes the
// permutation, and each copies the rows of every SPLIT-th token of its warps, so the copies spread
// over SPLIT times as many CTAs. D % 256 == 0 and D <= 8192.
template <int SPLIT>
__global__ void __launch_bounds__(kScatterWarps * 32)
scatter_permute_kernel(const int32_t *__restrict__ ids, int T, int E, const int32_t *__restrict__ block_base,
                       const int32_t *__restrict__ seg_off, int32_t *__restrict__ perm_route,
                       int32_t *__restrict__ route_pos, const uint16_t *__restrict__ x, int D,
                       uint16_t *__restrict__ xp, int copy_buckets) {
    pdl_enter();
    __shared__ int32_t cnt[kScatterWarps][kMaxBuckets];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kScatterWarps * kMaxBuckets; i += blockDim.x) (&cnt[0][0])[i] = 0;
    __syncthreads();
    const int blk = blockIdx.x / SPLIT, part = blockIdx.x % SPLIT;
    const int r = blk * topk::TOK_PER_CTA * 8 + warp * 32 + lane;
    const bool valid = r < T * 8;
    const int e = valid ? ids[r] : -1 - lane;
    const unsigned peers = __match_any_sync(kFull, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && lane == __ffs(peers) - 1) cnt[warp][e] = __popc(peers);
    __syncthreads();
    for (int c = threadIdx.x; c < E; c += blockDim.x) {
        int run = 0;
#pragma unroll
        for (int w = 0; w < kScatterWarps; ++w) {
            const int v = cnt[w][c];
            cnt[w][c] = run;
            run += v;
        }
    }
    __syncthreads();
    int pos = 0;
    if (valid) {
        pos = seg_off[e] + block_base[(size_t)blk * E + e] + cnt[warp][e] + rank;
        if (part == 0) {
            perm_route[pos] = r;
            route_pos[r] = pos;
        }
    }
    // rows: lane l's route is token (r >> 3), slot (l & 7); the warp's 4 tokens
    const int chunks = D / 8;  // 16-byte chunks per row
    for (int k = part; k < 4; k += SPLIT) {
        const int t = (blk * topk::TOK_PER_CTA * 8 + warp * 32) / 8 + k;
        if (t >= T) break;
        // the token's routes whose rows are copied: buckets below copy_buckets (the expert-parallel
        // path leaves out the routes of other GPUs' experts)
        const unsigned live = __ballot_sync(kFull, valid && e < copy_buckets);
        const unsigned mine = (live >> (k * 8)) & 0xffu;
        if (!mine) continue;
        const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t * D);
        for (int c0 = 0; c0 < chunks; c0 += 256) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + j * 32 + lane;
                if (c < chunks) v[j] = src[c];
            }
#pragma unroll
            for (int sl = 0; sl < 8; ++sl) {
                const int ps = __shfl_sync(kFull, pos, k * 8 + sl);
                if (!((mine >> sl) & 1u)) continue;
                uint4 *dst = reinterpret_cast<uint4 *>(xp + (size_t)ps * D);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = c0 + j * 32 + lane;
                    if (c < chunks) dst[c] = v[j];
                }
            }
        }
    }
}

// ------------------------------------------------------------------ combine + next RMSNorm
//
// Stacked layers: one CTA of NT threads per token (128: two 8-column chunks per thread for D = 2048
// measured 6% faster than 256). resid[t] += out[t] with out the combine
// above (same f32 expression and order per column), then -- when the next layer's norm weights
// are given -- h[t] = bf16(resid[t] * rsqrt(mean(resid[t]^2) + eps) * w) (gpu_graph.mm:48-61)
// from the updated row still in registers, so the next layer's RMSNorm costs no extra pass.
// D % 8 == 0 and D <= 8192.
template <int NT>
__global__ void __launch_bounds__(NT)
combine_norm_kernel(const uint16_t *__restrict__ yp, const int32_t *__restrict__ route_pos,
                    const uint16_t *__restrict__ ys, const float *__restrict__ gate_logit,
                    const float *__restrict__ probs, int D, float *__restrict__ resid,
                    const float *__restrict__ norm_w, float eps, uint16_t *__restrict__ h,
                    uint16_t *__restrict__ h_trace, const uint32_t *__restrict__ err) {
    pdl_enter();
    __shared__ float part[NT / 32];
    if (*err) return;  // a failed call leaves the residual untouched
    const int t = blockIdx.x, tid = threadIdx.x;
    const float g = sigmoid_ref(gate_logit[t]);
    float pr[8];
    int32_t pos[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        pr[s] = probs[(size_t)t * 8 + s];
        pos[s] = route_pos[(size_t)t * 8 + s];
    }
    constexpr int KC = 8192 / (NT * 8);  // chunks of 8 columns per thread
    float r[KC][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
        const int c = (tid + k * NT) * 8;
        if (c >= D) break;
        float o[8];
        {
            const uint4 v = *reinterpret_cast<const uint4 *>(ys + (size_t)t * D + c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = ((j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1])) * g;
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint4 v = *reinterpret_cast<const uint4 *>(yp + (size_t)pos[s] * D + c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float prod = pr[s] * ((j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1]));
                o[j] = o[j] + prod;
            }
        }
        float4 *rp = reinterpret_cast<float4 *>(resid + (size_t)t * D + c);
        float4 a = rp[0], b = rp[1];
        a.x += o[0]; a.y += o[1]; a.z += o[2]; a.w += o[3];
        b.x += o[4]; b.y += o[5]; b.z += o[6]; b.w += o[7];
        rp[0] = a;
        rp[1] = b;
        r[k][0] = a.x; r[k][1] = a.y; r[k][2] = a.z; r[k][3] = a.w;
        r[k][4] = b.x; r[k][5] = b.y; r[k][6] = b.z; r[k][7] = b.w;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(r[k][j], r[k][j], ss);
    }
    if (!norm_w) return;
#pragma unroll
    for (int n = 16; n; n >>= 1) ss += __shfl_xor_sync(kFull, ss, n);
    if ((tid & 31) == 0) part[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) tot += part[i];
    const float scale = 1.0f / sqrtf(tot / (float)D + eps);
#pragma unroll
    for (int k = 0; k < KC; ++k) {
        const int c = (tid + k * NT) * 8;
        if (c >= D) break;
        const float4 w0 = *reinterpret_cast<const float4 *>(norm_w + c), w1 = *reinterpret_cast<const float4 *>(norm_w + c + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint4 o;
        o.x = (uint32_t)f32_to_bf16_bits(r[k][0] * scale * wv[0]) | ((uint32_t)f32_to_bf16_bits(r[k][1] * scale * wv[1]) << 16);
        o.y = (uint32_t)f32_to_bf16_bits(r[k][2] * scale * wv[2]) | ((uint32_t)f32_to_bf16_bits(r[k][3] * scale * wv[3]) << 16);
        o.z = (uint32_t)f32_to_bf16_bits(r[k][4] * scale * wv[4]) | ((uint32_t)f32_to_bf16_bits(r[k][5] * scale * wv[5]) << 16);
        o.w = (uint32_t)f32_to_bf16_bits(r[k][6] * scale * wv[6]) | ((uint32_t)f32_to_bf16_bits(r[k][7] * scale * wv[7]) << 16);
        *reinterpret_cast<uint4 *>(h + (size_t)t * D + c) = o;
        if (h_trace) *reinterpret_cast<uint4 *>(h_trace + (size_t)t * D + c) = o;
    }
}

// ------------------------------------------------------------------ combine
//
// out[t] = sigmoid(gate_t) * shared[t] + sum_j p[t,j] * y[8t+j]   (Qwen36Model.cs:242-244),
// f32 arithmetic in that order, rounded once to bf16. 8 columns per thread. The expert rows are
// stored in expert order: route r's row is yp[route_pos[r]], the shared rows follow in ys.
__global__ void combine_kernel(const uint16_t *__restrict__ yp, const int32_t *__restrict__ route_pos,
                               const uint16_t *__restrict__ ys,
                               const float *__restrict__ gate_logit, const float *__restrict__ probs, int T, int D,
                               uint16_t *__restrict__ out, float *__restrict__ resid,
                               const uint32_t *__restrict__ err) {
    pdl_enter();
    const int per_tok = D / 8;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)T * per_tok) return;
    if (*err) return;  // a failed call leaves the output untouched
    const int t = idx / per_tok, c = (idx % per_tok) * 8;
    const float g = sigmoid_ref(gate_logit[t]);
    float o[8];
    {
        uint4 v = *reinterpret_cast<const uint4 *>(ys + (size_t)t * D + c);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = ((j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1])) * g;
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const float p = probs[(size_t)t * 8 + s];
        uint4 v = *reinterpret_cast<const uint4 *>(yp + (size_t)route_pos[(size_t)t * 8 + s] * D + c);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float prod = p * ((j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1]));
            o[j] = o[j] + prod;
        }
    }
    if (out) {
        uint4 r;
        r.x = pack_bf16x2(o[0], o[1]);
        r.y = pack_bf16x2(o[2], o[3]);
        r.z = pack_bf16x2(o[4], o[5]);
        r.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4 *>(out + (size_t)t * D + c) = r;
    }
    if (resid) {
        float4 *rp = reinterpret_cast<float4 *>(resid + (size_t)t * D + c);
        float4 a = rp[0], b = rp[1];
        a.x += o[0]; a.y += o[1]; a.z += o[2]; a.w += o[3];
        b.x += o[4]; b.y += o[5]; b.z += o[6]; b.w += o[7];
        rp[0] = a;
        rp[1] = b;
    }
}

// ------------------------------------------------------------------ router: tensor cores + exact check
//
// The routing ids must be those of the canonical f32 logits, which the tensor cores cannot
// produce. But they can bound them. Approximate logits a[t, e] come from the grouped GEMM (DOWN
// mode, one "expert" = the router matrix, bf16 output): its weights are W' = bf16(W), W = fma(q,
// s, b) as the canonical order computes them, and its bf16 x bf16 products are exact in f32. With
// r_e = W'_e - W_e (known from the weights),
//   |a[t,e] - logit[t,e]| <= ||r_e|| ||x_t|| + 2^-12 ||W_e|| ||x_t|| + 2^-8 |a[t,e]|  =: eps[t,e]
// (Cauchy-Schwarz for the weight rounding). 2^-12 = K * 2^-23 for K = 2048 is the worst case of
// adding the K products one at a time with truncation (an error below one f32 ulp, 2^-23
// relative, per addition) -- no rounding mode or internal order of the MMA accumulation is
// assumed. Any blocked order (K = 16 per instruction, 128 instruction results added into TMEM)
// errs far less, and the margin absorbs the canonical order's own f32 error (< 70 roundings to
// nearest per lane chain and butterfly, 2^-17.8 relative). The last term covers the bf16 output
// rounding, 2^-9 |A|, twice over. An expert can be among the true top-8 only if a + eps >= L8,
// the 8th largest a - eps. Those candidates (about 12 of 256) are recomputed in the canonical
// order and the top-8 is selected from the exact values, so ids, ties and probabilities equal
// the all-exact router's.
constexpr float kRouterAccumRel = 0x1p-12f;
constexpr float kRouterOutRel = 0x1p-8f;
constexpr float kNormMargin = 1.0f + 0x1p-10f;  // f32 rounding of the norms themselves
constexpr int kRouterMaxCand = 64;             // above this a token falls back to all experts

// ||r_e||, ||W_e|| of every router row (rows < E) into wn[e], wn[E + e], and the rows' f32 weights
// W = fma(q, s, b) -- the values the canonical order multiplies -- into wf [E][D]; one warp per row.
__global__ void __launch_bounds__(256) router_row_norms_kernel(QView R, int E, int D, float *__restrict__ wn,
                                                               float *__restrict__ wf) {
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (e >= E) return;
    const uint32_t *w = R.packed + (size_t)e * R.words_per_row();
    float rr = 0.f, ww = 0.f;
    for (int c = lane * 4; c < D; c += 128) {  // 4 codes (one word) per lane per step
        const uint32_t q4 = w[c / 4];
        const float s = bf16_bits_to_f32(R.scales[(size_t)e * R.groups_per_row() + c / 64]);
        const float b = bf16_bits_to_f32(R.biases[(size_t)e * R.groups_per_row() + c / 64]);
        float Wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float W = fmaf(byte_to_f32(q4, j), s, b);
            const float r = bf16_bits_to_f32(f32_to_bf16_bits(W)) - W;  // exact (Sterbenz)
            rr = fmaf(r, r, rr);
            ww = fmaf(W, W, ww);
            Wv[j] = W;
        }
        *reinterpret_cast<float4 *>(wf + (size_t)e * D + c) = make_float4(Wv[0], Wv[1], Wv[2], Wv[3]);
    }
    rr = warp_sum_butterfly(rr);
    ww = warp_sum_butterfly(ww);
    if (lane == 0) {
        wn[e] = sqrtf(rr) * kNormMargin;
        wn[E + e] = sqrtf(ww) * kNormMargin;
    }
}

// Work tiles of a one-segment grouped GEMM (the approximate-logit GEMM, dense projections): segment
// 0, `rows` tokens each (at most 256).
__global__ void router_tiles_kernel(int T, int rows, Tile *__restrict__ tiles, int32_t *__restrict__ n_tiles) {
    pdl_enter();
    const int n = (T + rows - 1) / rows;
    for (int i = threadIdx.x; i < n; i += blockDim.x) tiles[i] = Tile{0, i * rows, min(rows, T - i * rows)};
    if (threadIdx.x == 0) *n_tiles = n;
}

// The canonical dot product (canonical_dot_warp) with the activation row held in registers: xr[k]
// = x[256k + 8 lane .. +8] (bf16).
__device__ __forceinline__ float canonical_dot_xreg(const QView &m, int row, const uint4 (&xr)[8], int D) {
    const uint32_t lane = lane_id();
    const uint32_t *w = m.packed + (size_t)row * m.words_per_row();
    const uint16_t *sc = m.scales + (size_t)row * m.groups_per_row();
    const uint16_t *bi = m.biases + (size_t)row * m.groups_per_row();
    uint2 q[8];
    uint16_t sv[8], bv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (k * 256 < D) {
            const int base = k * 256 + lane * 8;
            q[k] = __ldg(reinterpret_cast<const uint2 *>(w + base / 4));
            sv[k] = __ldg(sc + base / 64);
            bv[k] = __ldg(bi + base / 64);
        }
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k * 256 >= D) break;
        const float s = bf16_bits_to_f32(sv[k]), bb = bf16_bits_to_f32(bv[k]);
        const uint32_t xw[4] = {xr[k].x, xr[k].y, xr[k].z, xr[k].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float wv = fmaf(byte_to_f32(j < 4 ? q[k].x : q[k].y, j & 3), s, bb);
            const float xf = (j & 1) ? bf16_hi(xw[j >> 1]) : bf16_lo(xw[j >> 1]);
            acc = fmaf(wv, xf, acc);
        }
    }
    return warp_sum_butterfly(acc);
}

// canonical_dot_xreg of two rows at once: both rows' loads are in flight together, the two rows'
// dequantisation and FMA chains run as packed pairs (fma.rn.f32x2 rounds each half exactly as fmaf)
// and the butterflies interleave; each result is bit-identical to the single-row one.
__device__ __forceinline__ void canonical_dot_xreg2(const QView &m, int row0, int row1, const uint4 (&xr)[8], int D,
                                                    float &out0, float &out1) {
    const uint32_t lane = lane_id();
    const uint32_t *w0 = m.packed + (size_t)row0 * m.words_per_row(), *w1 = m.packed + (size_t)row1 * m.words_per_row();
    const uint16_t *s0 = m.scales + (size_t)row0 * m.groups_per_row(), *s1 = m.scales + (size_t)row1 * m.groups_per_row();
    const uint16_t *b0 = m.biases + (size_t)row0 * m.groups_per_row(), *b1 = m.biases + (size_t)row1 * m.groups_per_row();
    uint2 qa[8], qb[8];
    uint32_t sa[8], sb[8];  // scale | bias << 16
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (k * 256 < D) {
            const int base = k * 256 + lane * 8;
            qa[k] = __ldg(reinterpret_cast<const uint2 *>(w0 + base / 4));
            qb[k] = __ldg(reinterpret_cast<const uint2 *>(w1 + base / 4));
            sa[k] = (uint32_t)__ldg(s0 + base / 64) | ((uint32_t)__ldg(b0 + base / 64) << 16);
            sb[k] = (uint32_t)__ldg(s1 + base / 64) | ((uint32_t)__ldg(b1 + base / 64) << 16);
        }
    float2 acc = make_float2(0.0f, 0.0f);  // (row0, row1)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k * 256 >= D) break;
        const float2 sc = make_float2(bf16_lo(sa[k]), bf16_lo(sb[k])), bi = make_float2(bf16_hi(sa[k]), bf16_hi(sb[k]));
        const uint32_t xw[4] = {xr[k].x, xr[k].y, xr[k].z, xr[k].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xf = (j & 1) ? bf16_hi(xw[j >> 1]) : bf16_lo(xw[j >> 1]);
            const float2 q = make_float2(byte_to_f32(j < 4 ? qa[k].x : qa[k].y, j & 3),
                                         byte_to_f32(j < 4 ? qb[k].x : qb[k].y, j & 3));
            acc = ffma2(ffma2(q, sc, bi), make_float2(xf, xf), acc);
        }
    }
    float acc0 = acc.x, acc1 = acc.y;
#pragma unroll
    for (int n = 16; n; n >>= 1) {
        acc0 += __shfl_xor_sync(kFull, acc0, n);
        acc1 += __shfl_xor_sync(kFull, acc1, n);
    }
    out0 = acc0;
    out1 = acc1;
}

// canonical_dot_xreg2 with the rows' f32 weights precomputed (wf [rows][D], the same W values):
// two 16-byte loads per 8 columns instead of code loads and conversions.
__device__ __forceinline__ void canonical_dot_wf2(const float *wf, int row0, int row1, const uint4 (&xr)[8], int D,
                                                  float &out0, float &out1) {
    const uint32_t lane = lane_id();
    const float *w0 = wf + (size_t)row0 * D, *w1 = wf + (size_t)row1 * D;
    float2 acc = make_float2(0.0f, 0.0f);  // (row0, row1)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        if (k * 256 >= D) break;
        const int base = k * 256 + lane * 8;
        const float4 a0 = __ldg(reinterpret_cast<const float4 *>(w0 + base)), a1 = __ldg(reinterpret_cast<const float4 *>(w0 + base + 4));
        const float4 b0 = __ldg(reinterpret_cast<const float4 *>(w1 + base)), b1 = __ldg(reinterpret_cast<const float4 *>(w1 + base + 4));
        const float wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const uint32_t xw[4] = {xr[k].x, xr[k].y, xr[k].z, xr[k].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xf = (j & 1) ? bf16_hi(xw[j >> 1]) : bf16_lo(xw[j >> 1]);
            acc = ffma2(make_float2(wa[j], wb[j]), make_float2(xf, xf), acc);
        }
    }
    float acc0 = acc.x, acc1 = acc.y;
#pragma unroll
    for (int n = 16; n; n >>= 1) {
        acc0 += __shfl_xor_sync(kFull, acc0, n);
        acc1 += __shfl_xor_sync(kFull, acc1, n);
    }
    out0 = acc0;
    out1 = acc1;
}

// The 8th largest of 256 values (8 per lane, v[j] of expert lane + 32 j < E; the others ignored),
// counting equal values separately; every lane returns it.
__device__ __forceinline__ float eighth_largest(const float *v, int E) {
    const int lane = lane_id();
    uint32_t key[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) key[j] = lane + 32 * j < E ? order_key(v[j]) : 0u;
    auto cs = [&](int a, int b) {  // descending
        const uint32_t hi = max(key[a], key[b]), lo = min(key[a], key[b]);
        key[a] = hi;
        key[b] = lo;
    };
    cs(0, 2); cs(1, 3); cs(4, 6); cs(5, 7);
    cs(0, 4); cs(1, 5); cs(2, 6); cs(3, 7);
    cs(0, 1); cs(2, 3); cs(4, 5); cs(6, 7);
    cs(2, 4); cs(3, 5);
    cs(1, 4); cs(3, 6);
    cs(1, 2); cs(3, 4); cs(5, 6);
    int need = 8;
    uint32_t res = 0u;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        const uint32_t best = __reduce_max_sync(kFull, key[0]);
        const int c = __popc(__ballot_sync(kFull, key[0] == best));
        if (c >= need) {
            res = best;
            break;
        }
        need -= c;
        if (key[0] == best) {
#pragma unroll
            for (int j = 0; j < 7; ++j) key[j] = key[j + 1];
            key[7] = 0u;
        }
    }
    return key_value(res);
}

// The 8 largest of up to 64 (value, id) entries, two per lane (slots 0 and 1; absent entries have
// key 0), descending with ties to the lower id; all lanes return the same sel/chosen.
__device__ __forceinline__ void select_top8_pairs(float v0, uint32_t id0, bool has0, float v1, uint32_t id1, bool has1,
                                                  int32_t *sel, float *chosen) {
    uint32_t k0 = has0 ? order_key(v0) : 0u, k1 = has1 ? order_key(v1) : 0u;
    if (k1 > k0 || (k1 == k0 && id1 < id0)) {  // slot 0 holds the lane's better entry
        uint32_t t = k0; k0 = k1; k1 = t;
        t = id0; id0 = id1; id1 = t;
    }
    if (!has0 && !has1) id0 = id1 = 0xffffffffu;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        const uint32_t best = __reduce_max_sync(kFull, k0);
        const uint32_t win = __reduce_min_sync(kFull, k0 == best ? id0 : 0xffffffffu);
        sel[n] = (int32_t)win;
        chosen[n] = key_value(best);
        if (id0 == win && k0 == best) {
            k0 = k1;
            id0 = id1;
            k1 = 0u;
            id1 = 0xffffffffu;
        }
    }
}

// Expert-parallel dispatch fused into the router (router_select_kernel<true>): token t of this
// rank goes to row slot rank * cap + t of every rank's meta and, where that rank owns one of its
// experts (E_l experts per rank), of its rx -- the rows already sit in the routing warp's registers.
struct RouterDispatch {
    EpPeers peers;
    int G, rank, cap, E_l;
    uint32_t *ticket;  // this rank's CTA ticket of the dispatch
};

// The token row (canonical lane partition in xr) into row slot rank * cap + t of the rx of every
// rank in `dests`, by plain stores over NVLink.
__device__ __forceinline__ void dispatch_row(const RouterDispatch &dsp, uint32_t dests, int t, int D,
                                             const uint4 (&xr)[8]) {
    const int lane = threadIdx.x & 31;
    for (int d = 0; d < dsp.G; ++d) {
        if (!((dests >> d) & 1u)) continue;
        uint16_t *dst = dsp.peers.rx[d] + ((size_t)dsp.rank * dsp.cap + t) * D;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k * 256 < D) *reinterpret_cast<uint4 *>(dst + k * 256 + lane * 8) = xr[k];
    }
}

template <bool DISPATCH>
__device__ __forceinline__ void router_select_token(
    const uint16_t *__restrict__ approx, const float *__restrict__ wn, const float *__restrict__ wf,
    const uint16_t *__restrict__ x, int t, int E, int D, QView R, QView SR, const float *__restrict__ bias,
    const int32_t *__restrict__ forced_ids, int32_t *__restrict__ ids, float *__restrict__ probs,
    float *__restrict__ gate_logit, int32_t *__restrict__ block_counts, uint32_t *__restrict__ err,
    const RouterDispatch &dsp) {
    __shared__ float all_lg[8][256];  // per warp: every exact logit, when a token has too many candidates
    __shared__ uint32_t cand_mask[8][8];  // per warp: candidate bits of experts 32 j + lane
    __shared__ int16_t cand_id[8][kRouterMaxCand];  // per warp: the candidates, ascending
    const int lane = threadIdx.x & 31;
    float *lg_all = all_lg[threadIdx.x >> 5];
    // the token's row in registers, canonical lane partition; its norm
    uint4 xr[8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        xr[k] = make_uint4(0, 0, 0, 0);
        if (k * 256 < D) {
            xr[k] = *reinterpret_cast<const uint4 *>(x + (size_t)t * D + k * 256 + lane * 8);
            const uint32_t w4[4] = {xr[k].x, xr[k].y, xr[k].z, xr[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float lo = bf16_lo(w4[j]), hi = bf16_hi(w4[j]);
                ss = fmaf(lo, lo, ss);
                ss = fmaf(hi, hi, ss);
            }
        }
    }
    const float nx = sqrtf(warp_sum_butterfly(ss)) * kNormMargin;
    int32_t sel[8];
    float chosen[8];
    bool bad = false;
    uint32_t sent_ranks = 0;  // DISPATCH: ranks the row has already gone to
    if (forced_ids) {
        int32_t id = 0;
        if (lane < 8) {
            id = forced_ids[(size_t)t * 8 + lane];
            bad = id < 0 || id >= E;
            id = min(max(id, 0), E - 1);
        }
        if (__any_sync(kFull, bad) && lane == 0) atomicOr(err, kErrBadExpert);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const int e = __shfl_sync(kFull, id, n);
            const float lg = canonical_dot_xreg(R, e, xr, D) + (bias ? bias[e] : 0.f);
            sel[n] = e;
            chosen[n] = lg;
        }
    } else {
        // approximate logits and their bounds; lane l holds experts l + 32 j
        float lo_[8], hi_[8];
        bool nonfinite = false;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane + 32 * j;
            lo_[j] = -INFINITY;
            hi_[j] = -INFINITY;
            if (e < E) {
                const float a = bf16_bits_to_f32(approx[(size_t)t * E + e]) + (bias ? bias[e] : 0.f);
                if (!isfinite(a)) {
                    nonfinite = true;
                } else {
                    const float eps = (wn[e] + kRouterAccumRel * wn[E + e]) * nx + kRouterOutRel * fabsf(a);
                    lo_[j] = a - eps;
                    hi_[j] = a + eps;
                }
            }
        }
        if (__any_sync(kFull, nonfinite) && lane == 0) atomicOr(err, kErrNonFinite);
        const float L8 = eighth_largest(lo_, E);
        uint32_t *mask = cand_mask[threadIdx.x >> 5];
        int ncand = 0;
        uint32_t cand_ranks = 0;  // ranks owning a candidate (DISPATCH)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const bool cj = lane + 32 * j < E && hi_[j] >= L8;
            const uint32_t mj = __ballot_sync(kFull, cj);
            if (lane == 0) mask[j] = mj;
            ncand += __popc(mj);
            if constexpr (DISPATCH)
                if (cj) cand_ranks |= 1u << ((lane + 32 * j) / dsp.E_l);
        }
        __syncwarp();
        if constexpr (DISPATCH) {
            // the row leaves now, to every rank that owns a candidate (a superset of the ranks of
            // the final 8), so the NVLink stores overlap the exact dots below; a rank that ends up
            // owning none of the 8 ignores the row (its metadata, written last, says so)
            const uint32_t dm = ncand > kRouterMaxCand ? (1u << dsp.G) - 1u : __reduce_or_sync(kFull, cand_ranks);
            dispatch_row(dsp, dm, t, D, xr);
            sent_ranks = dm;
        }
        // exact logits of the candidates (all experts if there are too many), ascending id; the
        // i-th goes to lane i % 32, slot i / 32
        const bool all = ncand > kRouterMaxCand;
        float v0 = 0.f, v1 = 0.f;
        uint32_t i0 = 0, i1 = 0;
        bool h0 = false, h1 = false;
        if (all) {
            for (int e = 0; e < E; e += 2) {
                float a0, a1;
                canonical_dot_wf2(wf, e, min(e + 1, E - 1), xr, D, a0, a1);
                a0 += bias ? bias[e] : 0.f;
                a1 += bias ? bias[min(e + 1, E - 1)] : 0.f;
                if (lane == 0) {
                    lg_all[e] = isfinite(a0) ? a0 : -INFINITY;
                    if (e + 1 < E) lg_all[e + 1] = isfinite(a1) ? a1 : -INFINITY;
                }
            }
        } else {
            int16_t *ci = cand_id[threadIdx.x >> 5];
            if (lane == 0) {
                int n = 0;
                for (int j = 0; j < 8; ++j)
                    for (uint32_t m = mask[j]; m; m &= m - 1) ci[n++] = (int16_t)(__ffs(m) - 1 + 32 * j);
            }
            __syncwarp();
            for (int i = 0; i < ncand; i += 2) {
                const int e0 = ci[i], e1 = ci[min(i + 1, ncand - 1)];
                float a0, a1;
                canonical_dot_wf2(wf, e0, e1, xr, D, a0, a1);
                a0 += bias ? bias[e0] : 0.f;
                a1 += bias ? bias[e1] : 0.f;
                if (!isfinite(a0)) a0 = -INFINITY;
                if (!isfinite(a1)) a1 = -INFINITY;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int ii = i + u;
                    if (ii >= ncand || lane != (ii & 31)) continue;
                    const float lg = u ? a1 : a0;
                    const uint32_t e = (uint32_t)(u ? e1 : e0);
                    if (ii < 32) { v0 = lg; i0 = e; h0 = true; }
                    else { v1 = lg; i1 = e; h1 = true; }
                }
            }
        }
        if (all) {
            __syncwarp();
            float vall[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vall[j] = lane + 32 * j < E ? lg_all[lane + 32 * j] : -INFINITY;
            select_top8(vall, E, sel, chosen);
        } else
            select_top8_pairs(v0, i0, h0, v1, i1, h1, sel, chosen);
    }
    // softmax over the chosen logits, the gate logit, outputs and the block's route counts
    float mx = chosen[0];
#pragma unroll
    for (int n = 1; n < 8; ++n) mx = fmaxf(mx, chosen[n]);
    float p[8], sum = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        p[n] = expf(chosen[n] - mx);
        sum += p[n];
    }
    const float g = canonical_dot_xreg(SR, 0, xr, D);
    if (lane < 8) {
        float pv = 0.f;
        int32_t sv = 0;
#pragma unroll
        for (int m = 0; m < 8; ++m)
            if (m == lane) {
                pv = p[m];
                sv = sel[m];
            }
        ids[(size_t)t * 8 + lane] = sv;
        probs[(size_t)t * 8 + lane] = pv / sum;
        if (block_counts) atomicAdd(&block_counts[(size_t)(t / topk::TOK_PER_CTA) * E + sv], 1);
        if constexpr (DISPATCH) {
            for (int d = 0; d < dsp.G; ++d) {
                RowMeta &m = dsp.peers.meta[d][(size_t)dsp.rank * dsp.cap + t];
                m.ids[lane] = sv;
                m.probs[lane] = pv / sum;
            }
        }
    }
    if (lane == 0) gate_logit[t] = g;
    if constexpr (DISPATCH) {
        uint32_t dests = 0;
#pragma unroll
        for (int n = 0; n < 8; ++n) dests |= 1u << (sel[n] / dsp.E_l);
        dispatch_row(dsp, dests & ~sent_ranks, t, D, xr);  // forced routes: nothing sent yet
    }
}

// One warp per token: approximate logits -> candidates -> exact logits -> top-8, softmax, the
// shared-route gate logit, and the route counts of the token's 64-token block (block_counts zeroed
// beforehand; null: not counted). forced: the token's 8 ids are given (their exact logits give the
// probabilities). DISPATCH: the token row and its routing also go out to the expert-parallel
// ranks, and the last CTA signals their arrival. Three CTAs per SM (80 registers) measured 7%
// faster than two; the dispatching variant keeps the token row live to the end and takes two
// (three would spill it).
template <bool DISPATCH>
__global__ void __launch_bounds__(256, DISPATCH ? 2 : 3)
router_select_kernel(const uint16_t *__restrict__ approx, const float *__restrict__ wn, const float *__restrict__ wf,
                     const uint16_t *__restrict__ x,
                     int T, int E, int D, QView R, QView SR, const float *__restrict__ bias,
                     const int32_t *__restrict__ forced_ids, int32_t *__restrict__ ids, float *__restrict__ probs,
                     float *__restrict__ gate_logit, int32_t *__restrict__ block_counts, uint32_t *__restrict__ err,
                     RouterDispatch dsp) {
    pdl_enter();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t < T) router_select_token<DISPATCH>(approx, wn, wf, x, t, E, D, R, SR, bias, forced_ids, ids, probs,
                                             gate_logit, block_counts, err, dsp);
    if constexpr (DISPATCH) ep_signal(dsp.ticket, dsp.peers, dsp.G, dsp.rank, 2 * dsp.G + dsp.rank, T);
}

}  // namespace di
