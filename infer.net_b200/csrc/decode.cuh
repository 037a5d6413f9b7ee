// Decode (small T) path of the MoE block: three kernels per layer, chained with programmatic
// dependent launch so that each kernel streams its weights into L2 while the previous one is
// still running.
//
//   decode_route_kernel    RMSNorm of the residual row (stacked layers) or the given bf16 input,
//                          router logits in the canonical f32 order (bit-exact with the oracle),
//                          then -- in the last CTA to finish -- top-8, softmax and the shared
//                          gate logit (Qwen36Model.cs:246-262; gpu_graph.mm:134-146)
//   decode_gate_up_kernel  act = silu(gate . h) * (up . h) for the 8 routed slots and the shared
//                          expert (quantized.mm:148-189)
//   decode_down_kernel     the 9 down rows of one output dim, then the combine
//                          sigmoid(g) * shared + sum_j p_j * expert_j (Qwen36Model.cs:242-244)
//                          and the residual update x += out
#pragma once
#include "common.cuh"
#include "gemv.cuh"
#include "route.cuh"

namespace di {

constexpr int kDecodeMaxTokens = 16;

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Asynchronous L2 prefetch of a contiguous range (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    const uint64_t g = (uint64_t)__cvta_generic_to_global(p);  // the .global form needs a global address
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(g), "r"(bytes) : "memory");
}

// Prefetch one row of a quantised matrix (codes, scales, biases).
__device__ __forceinline__ void prefetch_qrow(const QView &m, size_t row) {
    prefetch_l2(m.packed + row * m.words_per_row(), (uint32_t)m.words_per_row() * 4u);
    const uint32_t gb = (uint32_t)m.groups_per_row() * 2u;
    if ((gb & 15u) == 0) {
        prefetch_l2(m.scales + row * m.groups_per_row(), gb);
        prefetch_l2(m.biases + row * m.groups_per_row(), gb);
    }
}

// grid: ceil(E/8) CTAs x 256 threads (warp per router row); dynamic smem T*D*2 bytes.
// Stacked mode (x != null): h = bf16(x * rsqrt(mean(x^2) + eps) * norm_w), written by CTA 0
// to h_out (and h_trace). Block mode: h = h_in.
__global__ void __launch_bounds__(256)
decode_route_kernel(const float *__restrict__ x, const float *__restrict__ norm_w, float eps,
                    const uint16_t *__restrict__ h_in, int T, int D, QView R, QView SR,
                    const float *__restrict__ bias, uint16_t *__restrict__ h_out, uint16_t *__restrict__ h_trace,
                    float *__restrict__ logits, int32_t *__restrict__ ids, float *__restrict__ probs,
                    float *__restrict__ gate, uint32_t *__restrict__ counter, uint32_t *__restrict__ err) {
    extern __shared__ __align__(16) uint16_t hs[];
    __shared__ float part[8][kDecodeMaxTokens];
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = R.rows, row = blockIdx.x * 8 + warp;
    // weights do not depend on the previous kernel: load them before waiting for it
    const bool pre = D <= 2048;
    RouterRaw rr, sr;
    if (pre) {
        if (row < E) router_raw_load(R, row, D, rr);
        if (warp == 0) router_raw_load(SR, 0, D, sr);
    } else if (lane == 0 && row < E) {
        prefetch_qrow(R, (size_t)row);
    }
    grid_dep_wait();
    if (x) {
        for (int t = 0; t < T; ++t) {
            float ss = 0.f;
            for (int d = threadIdx.x; d < D; d += 256) ss = fmaf(x[(size_t)t * D + d], x[(size_t)t * D + d], ss);
#pragma unroll
            for (int n = 16; n; n >>= 1) ss += __shfl_xor_sync(kFull, ss, n);
            if (lane == 0) part[warp][t] = ss;
        }
        __syncthreads();
        for (int t = 0; t < T; ++t) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) tot += part[w][t];
            const float scale = 1.0f / sqrtf(tot / (float)D + eps);
            for (int d = threadIdx.x; d < D; d += 256) {
                const uint16_t v = f32_to_bf16_bits(x[(size_t)t * D + d] * scale * norm_w[d]);
                hs[t * D + d] = v;
                if (blockIdx.x == 0) {
                    h_out[(size_t)t * D + d] = v;
                    if (h_trace) h_trace[(size_t)t * D + d] = v;
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < T * D / 8; i += 256)
            reinterpret_cast<uint4 *>(hs)[i] = reinterpret_cast<const uint4 *>(h_in)[i];
    }
    __syncthreads();
    grid_dep_launch();
    if (row < E) {
        const float bb = bias ? bias[row] : 0.f;
        for (int t = 0; t < T; ++t) {
            const float v = pre ? router_raw_dot(rr, hs + t * D, D) : canonical_dot_warp(R, row, hs + t * D, D);
            if (lane == 0) logits[(size_t)t * E + row] = v + bb;
        }
    }
    // the last CTA to finish selects the experts of every token
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (pre && T > 1)  // the shared gate row preloaded by warp 0 goes to every warp
        for (int k = 0; k < 8; ++k) {
            sr.q[k].x = __shfl_sync(kFull, sr.q[k].x, lane);
            sr.q[k].y = __shfl_sync(kFull, sr.q[k].y, lane);
        }
    for (int t = warp; t < T; t += 8) {
        float v[8];
        bool nonfinite = false;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane + 32 * j;
            v[j] = e < E ? __ldcg(logits + (size_t)t * E + e) : 0.f;
            if (e < E && !isfinite(v[j])) {
                nonfinite = true;
                v[j] = -INFINITY;
            }
        }
        if (__any_sync(kFull, nonfinite) && lane == 0) atomicOr(err, kErrNonFinite);
        int32_t sel[8];
        float chosen[8];
        select_top8(v, E, sel, chosen);
        float mx = chosen[0], p[8], sum = 0.f;
#pragma unroll
        for (int n = 1; n < 8; ++n) mx = fmaxf(mx, chosen[n]);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            p[n] = expf(chosen[n] - mx);
            sum += p[n];
        }
        const float g = (pre && warp == 0) ? router_raw_dot(sr, hs + t * D, D) : canonical_dot_warp(SR, 0, hs + t * D, D);
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
        }
        if (lane == 0) gate[t] = g;
    }
    if (threadIdx.x == 0) *counter = 0;  // ready for the next launch
}

// act[t, j, i] = silu(gate_j[i] . h_t) * (up_j[i] . h_t); one warp per (t, j, i), j = 8 is the
// shared expert. grid: T*9*I/8 CTAs x 256 threads; dynamic smem D*2 bytes.
template <int BITS>
__global__ void __launch_bounds__(256)
decode_gate_up_kernel(const uint16_t *__restrict__ h, int T, int D, int I, QView g, QView u, QView sg, QView su,
                      const int32_t *__restrict__ ids, float *__restrict__ act) {
    extern __shared__ __align__(16) uint16_t xs[];
    const int per_tok = 9 * I;
    const int warp0 = blockIdx.x * 8;
    const int t = warp0 / per_tok;  // one token per CTA (per_tok is a multiple of 8)
    const int w = warp0 + (threadIdx.x >> 5) - t * per_tok;
    const int j = w / I, i = w % I;
    const bool shared = j == 8;
    if (shared && lane_id() < 2) prefetch_qrow(lane_id() ? su : sg, (size_t)i);
    grid_dep_wait();
    grid_dep_launch();
    for (int k = threadIdx.x; k < D / 8; k += blockDim.x)
        reinterpret_cast<uint4 *>(xs)[k] = reinterpret_cast<const uint4 *>(h + (size_t)t * D)[k];
    __syncthreads();
    const QView G = shared ? sg : g, U = shared ? su : u;
    const size_t row = (size_t)(shared ? 0 : ids[(size_t)t * 8 + j]) * I + i;
    float ga = 0.f, ua = 0.f;
    // the raw chunks of up to 4 x 32 columns-of-16 per pass are all requested before use
    constexpr int MAXC = 4;
    const int nc = D / 16;
    for (int c0 = lane_id(); c0 < nc; c0 += 32 * MAXC) {
        RawChunk<BITS> rg[MAXC], ru[MAXC];
#pragma unroll
        for (int k = 0; k < MAXC; ++k) {
            const int c = c0 + 32 * k;
            if (c < nc) {
                rg[k] = load_chunk<BITS>(G, row, c);
                ru[k] = load_chunk<BITS>(U, row, c);
            }
        }
#pragma unroll
        for (int k = 0; k < MAXC; ++k) {
            const int c = c0 + 32 * k;
            if (c >= nc) break;
            float wg[16], wu[16], xv[16];
            chunk_weights<BITS>(rg[k], c, wg);
            chunk_weights<BITS>(ru[k], c, wu);
            load_x16_bf16(xs, c, xv);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                ga = fmaf(wg[e], xv[e], ga);
                ua = fmaf(wu[e], xv[e], ua);
            }
        }
    }
    ga = warp_sum_butterfly(ga);
    ua = warp_sum_butterfly(ua);
    if (lane_id() == 0) act[((size_t)t * 9 + j) * I + i] = silu_ref(ga) * ua;
}

// out[t, d] = sigmoid(gate_t) * (shared_down[d] . act_s) + sum_j p[t,j] * (down_j[d] . act_j);
// one warp per (t, d). The prologue prefetches the 9 rows (expert ids from the route kernel,
// which has completed once the gate/up kernel released this launch; a stale id only costs a
// wasted prefetch). resid (f32 [T, D]) += out when given; out (bf16) written when given.
template <int BITS>
__global__ void __launch_bounds__(256)
decode_down_kernel(const float *__restrict__ act, int T, int D, int I, QView dn, QView sd,
                   const int32_t *__restrict__ ids, const float *__restrict__ probs,
                   const float *__restrict__ gate_logit, uint16_t *__restrict__ out, float *__restrict__ resid,
                   const uint32_t *__restrict__ err) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = lane_id();
    const bool live = warp < T * D;
    const int t = live ? warp / D : 0, d = live ? warp % D : 0;
    float y[9], acc[9];
    int row[9];  // expert * D + d (< 2^31)
#pragma unroll
    for (int j = 0; j < 9; ++j) {
        acc[j] = 0.f;
        row[j] = (j == 8 ? 0 : min(max(ids[(size_t)t * 8 + j], 0), dn.experts - 1)) * D + d;
    }
    // The weights do not depend on the gate/up kernel: the first chunk of each of the 9 rows is
    // loaded before waiting for it (the ids are final: the route kernel completed before the
    // gate/up kernel released this launch).
    const int nc = I / 16;
    RawChunk<BITS> raw[9];
    if (live && lane < nc)
#pragma unroll
        for (int j = 0; j < 9; ++j) raw[j] = load_chunk<BITS>(j == 8 ? sd : dn, row[j], lane);
    grid_dep_wait();
    grid_dep_launch();
    if (!live) return;
    for (int c = lane; c < nc; c += 32) {
        if (c != lane)
#pragma unroll
            for (int j = 0; j < 9; ++j) raw[j] = load_chunk<BITS>(j == 8 ? sd : dn, row[j], c);
#pragma unroll
        for (int j = 0; j < 9; ++j) {
            float w[16];
            chunk_weights<BITS>(raw[j], c, w);
            const float4 *ap = reinterpret_cast<const float4 *>(act + ((size_t)t * 9 + j) * I + c * 16);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 av = ap[k];
                acc[j] = fmaf(w[4 * k], av.x, acc[j]);
                acc[j] = fmaf(w[4 * k + 1], av.y, acc[j]);
                acc[j] = fmaf(w[4 * k + 2], av.z, acc[j]);
                acc[j] = fmaf(w[4 * k + 3], av.w, acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 9; ++j) y[j] = warp_sum_butterfly(acc[j]);
    if (lane == 0) {
        if (*err) return;
        float o = y[8] * sigmoid_ref(gate_logit[t]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float prod = probs[(size_t)t * 8 + j] * y[j];
            o = o + prod;
        }
        if (out) out[(size_t)t * D + d] = f32_to_bf16_bits(o);
        if (resid) resid[(size_t)t * D + d] += o;
    }
}

}  // namespace di

namespace di {

// ------------------------------------------------------------------ fused decode FFN (T = 1)
//
// gate/up + SwiGLU + down + combine of one token in one kernel of one CTA per SM (16 warps).
// Phase 1: the CTA bulk-copies its share of the 9 experts' weight rows -- (gate, up) row pairs p in
// [c*9I/G, (c+1)*9I/G) and the 9 down rows of the outputs d in [c*D/G, (c+1)*D/G) -- into shared
// memory, so the layer's whole weight stream is in flight at once (the shared expert's rows before
// the route kernel has finished, the routed rows once its ids are known). The rows of one expert
// in a CTA's share are consecutive in HBM, so each field (codes, scales, biases) of each expert is
// one copy. One warp issues them, gate/up before down, so the gate/up rows land first and phase 2
// runs while the down rows stream in. Phase 2: act = silu(gate . h) * (up . h) of its pairs
// (quantized.mm:148-189). A grid barrier (all CTAs are resident: one CTA per SM). Phase 3: act is
// staged once in the gate/up region; out[d] = sigmoid(gate_logit) * (shared_down[d] . act_s) +
// sum_j p_j * (down_j[d] . act_j) (Qwen36Model.cs:242-244), one warp per output with the combine
// weights folded into the lanes' partial sums, resid += out. Needs D % 512 == 0 and I % 512 == 0
// (16-byte rows of scales) and the layout below to fit in shared memory.
// Shared memory, field-major: gate/up region = gate codes [pairs][gu_row], up codes, gate scales
// [pairs][gu_grp], gate biases, up scales, up biases; down region = codes [9][outs][dn_row], scales
// [9][outs][dn_grp], biases.
constexpr int kFfnThreads = 512;
struct FfnLayout {
    int pairs, outs;                     // per CTA (upper bounds)
    int gu_row, gu_grp, dn_row, dn_grp;  // bytes of a code row / of a scale or bias row
    int gu_off, dn_off, bar_off, total;
    __host__ __device__ int gu_code(int m) const { return gu_off + m * pairs * gu_row; }             // m: 0 gate, 1 up
    __host__ __device__ int gu_sb(int m, int k) const { return gu_off + 2 * pairs * gu_row + (2 * m + k) * pairs * gu_grp; }
    __host__ __device__ int dn_code() const { return dn_off; }
    __host__ __device__ int dn_sb(int k) const { return dn_off + 9 * outs * dn_row + k * 9 * outs * dn_grp; }
};
__host__ __device__ inline FfnLayout ffn_layout(int D, int I, int bits, int grid) {
    FfnLayout f;
    f.pairs = (9 * I + grid - 1) / grid;
    f.outs = (D + grid - 1) / grid;
    f.gu_row = D * bits / 8;
    f.gu_grp = D / 64 * 2;
    f.dn_row = I * bits / 8;
    f.dn_grp = I / 64 * 2;
    f.gu_off = (D * 2 + 127) & ~127;
    // the gate/up region also holds act [9][I] f32 and the 9 combine weights in phase 3
    const int gu_bytes = max(2 * f.pairs * (f.gu_row + 2 * f.gu_grp), 9 * I * 4 + 64);
    f.dn_off = f.gu_off + ((gu_bytes + 127) & ~127);
    f.bar_off = f.dn_off + ((9 * f.outs * (f.dn_row + 2 * f.dn_grp) + 127) & ~127);
    f.total = f.bar_off + 64;
    return f;
}

// mbarrier.expect_tx without an arrival (registers bytes of copies issued before the arrival)
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 16 weights of chunk c of a code row held in shared memory (scale / bias rows beside it).
template <int BITS>
__device__ __forceinline__ void smem_chunk_weights(const uint8_t *codes, const uint16_t *sc, const uint16_t *bi, int c,
                                                   float *w) {
    RawChunk<BITS> r;
    r.s = sc[c >> 2];
    r.b = bi[c >> 2];
    if constexpr (BITS == 8) {
        const uint4 q = *reinterpret_cast<const uint4 *>(codes + c * 16);
        r.q[0] = q.x; r.q[1] = q.y; r.q[2] = q.z; r.q[3] = q.w;
    } else {
        const uint32_t *wd = reinterpret_cast<const uint32_t *>(codes) + ((5 * c) >> 1);
        r.q[0] = wd[0]; r.q[1] = wd[1]; r.q[2] = wd[2];
    }
    chunk_weights<BITS>(r, c, w);
}

template <int BITS>
__global__ void __launch_bounds__(kFfnThreads, 1)
decode_ffn_kernel(const uint16_t *__restrict__ h, int D, int I, QView g, QView u, QView sg, QView su, QView dn, QView sd,
                  const int32_t *__restrict__ ids, const float *__restrict__ probs, const float *__restrict__ gate_logit,
                  float *__restrict__ act, uint16_t *__restrict__ out, float *__restrict__ resid,
                  uint32_t *__restrict__ grid_ctr, uint32_t gen, uint32_t *__restrict__ err) {
    extern __shared__ __align__(128) uint8_t sm[];
    const FfnLayout f = ffn_layout(D, I, BITS, gridDim.x);
    uint16_t *xs = reinterpret_cast<uint16_t *>(sm);
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + f.bar_off);  // [0] gate/up rows, [1] down rows
    int32_t *ids_s = reinterpret_cast<int32_t *>(sm + f.bar_off + 16);  // the 8 routed expert ids
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int P = 9 * I, p_lo = (int)((long long)blockIdx.x * P / gridDim.x),
              p_hi = (int)((long long)(blockIdx.x + 1) * P / gridDim.x);
    const int d_lo = (int)((long long)blockIdx.x * D / gridDim.x), d_hi = (int)((long long)(blockIdx.x + 1) * D / gridDim.x);
    const int np = p_hi - p_lo, nd = d_hi - d_lo;
    const int j_lo = p_lo / I, j_hi = (p_hi - 1) / I, nseg = np > 0 ? j_hi - j_lo + 1 : 0;
    // Copies of the CTA's share, one per field of each expert segment: gate/up segments are the
    // pairs of one expert slot j (rows e_j*I + i0 .. i1), down segments are one expert's rows
    // e_j*D + d_lo .. d_hi. Copy k < nseg*6 is a gate/up field, the rest down fields; `routed`
    // selects the copies of routed experts (their ids come from ids_s).
    auto issue_copy = [&](int k, bool routed) {
        if (k < nseg * 6) {
            const int sg_ = k / 6, field = k % 6, j = j_lo + sg_;
            if ((j < 8) != routed) return;
            const int i0 = j == j_lo ? p_lo % I : 0, i1 = j == j_hi ? (p_hi - 1) % I + 1 : I;
            const int q0 = j * I + i0 - p_lo, cnt = i1 - i0;
            const int e = j < 8 ? ids_s[j] : 0;
            const int m = field & 1, kind = field >> 1;  // m: gate / up; kind: codes, scales, biases
            const QView &W = m ? (j < 8 ? u : su) : (j < 8 ? g : sg);
            const size_t row = (size_t)e * I + i0;
            if (kind == 0)
                bulk_load(sm + f.gu_code(m) + q0 * f.gu_row, reinterpret_cast<const uint8_t *>(W.packed) + row * f.gu_row,
                          (uint32_t)cnt * f.gu_row, &bar[0]);
            else
                bulk_load(sm + f.gu_sb(m, kind - 1) + q0 * f.gu_grp, (kind == 1 ? W.scales : W.biases) + row * (f.gu_grp / 2),
                          (uint32_t)cnt * f.gu_grp, &bar[0]);
        } else {
            const int kk = k - nseg * 6, j = kk / 3, kind = kk % 3;
            if ((j < 8) != routed || nd == 0) return;
            const int e = j < 8 ? ids_s[j] : 0;
            const QView &W = j < 8 ? dn : sd;
            const size_t row = (size_t)e * D + d_lo;
            if (kind == 0)
                bulk_load(sm + f.dn_code() + j * f.outs * f.dn_row, reinterpret_cast<const uint8_t *>(W.packed) + row * f.dn_row,
                          (uint32_t)nd * f.dn_row, &bar[1]);
            else
                bulk_load(sm + f.dn_sb(kind - 1) + j * f.outs * f.dn_grp, (kind == 1 ? W.scales : W.biases) + row * (f.dn_grp / 2),
                          (uint32_t)nd * f.dn_grp, &bar[1]);
        }
    };
    const int ncopies = nseg * 6 + 27;
    // the barriers expect the whole share's bytes up front; the shared expert's rows do not depend
    // on the route kernel and are requested before waiting for it
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbarrier_init();
        mbar_arrive_expect_tx(&bar[0], (uint32_t)np * 2 * (f.gu_row + 2 * f.gu_grp));
        mbar_arrive_expect_tx(&bar[1], (uint32_t)(9 * nd * (f.dn_row + 2 * f.dn_grp)));
    }
    __syncthreads();
    if (warp == 0)
        for (int k = lane; k < ncopies; k += 32) issue_copy(k, false);
    grid_dep_wait();  // the route kernel has written h, ids, probs and the gate logit
    if (tid < 8) ids_s[tid] = min(max(ids[tid], 0), g.experts - 1);
    for (int k = tid; k < D / 8; k += blockDim.x) reinterpret_cast<uint4 *>(xs)[k] = reinterpret_cast<const uint4 *>(h)[k];
    __syncthreads();
    if (warp == 0)  // in lane order: gate/up copies (k < nseg*6) are requested before the down copies
        for (int k = lane; k < ncopies; k += 32) issue_copy(k, true);
    bool ok = mbar_wait(&bar[0], 0, err, kErrTimeout);
    // ---- phase 2: the CTA's (gate, up) pairs
    if (ok)
        for (int q = warp; q < np; q += nw) {
            const int p = p_lo + q, j = p / I, i = p % I;
            const uint8_t *gc = sm + f.gu_code(0) + q * f.gu_row, *uc = sm + f.gu_code(1) + q * f.gu_row;
            const uint16_t *gs = reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 0) + q * f.gu_grp);
            const uint16_t *gb = reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 1) + q * f.gu_grp);
            const uint16_t *us = reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 0) + q * f.gu_grp);
            const uint16_t *ub = reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 1) + q * f.gu_grp);
            float ga[2] = {0.f, 0.f}, ua[2] = {0.f, 0.f};
            for (int c = lane; c < D / 16; c += 32) {
                float wg[16], wu[16], xv[16];
                smem_chunk_weights<BITS>(gc, gs, gb, c, wg);
                smem_chunk_weights<BITS>(uc, us, ub, c, wu);
                load_x16_bf16(xs, c, xv);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    ga[e & 1] = fmaf(wg[e], xv[e], ga[e & 1]);
                    ua[e & 1] = fmaf(wu[e], xv[e], ua[e & 1]);
                }
            }
            const float gsum = warp_sum_butterfly(ga[0] + ga[1]);
            const float usum = warp_sum_butterfly(ua[0] + ua[1]);
            if (lane == 0) act[(size_t)j * I + i] = silu_ref(gsum) * usum;
        }
    // ---- grid barrier: every CTA's act values are written
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(grid_ctr, 1u);
        const uint32_t target = gen * gridDim.x;
        const uint64_t t0 = global_ns();
        for (uint32_t n = 0;; ++n) {
            if (*reinterpret_cast<volatile uint32_t *>(grid_ctr) >= target) break;
            if ((n & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
                atomicOr(err, kErrTimeout);
                break;
            }
        }
        __threadfence();
    }
    __syncthreads();
    grid_dep_launch();
    // act of all 9 experts into the (now free) gate/up region, with the combine weights after it
    float *acts = reinterpret_cast<float *>(sm + f.gu_off);
    float *coef = acts + 9 * I;
    const int cpr = I / 16;  // chunks per down row
    // float4 q of chunk c of expert j goes to [j][q][c]: the lanes of phase 3 (consecutive c) then
    // read consecutive float4s
    for (int k = tid; k < 9 * I / 4; k += blockDim.x) {
        const int j = k / (4 * cpr), rem = k - j * 4 * cpr;
        reinterpret_cast<float4 *>(acts)[j * 4 * cpr + (rem & 3) * cpr + (rem >> 2)] =
            __ldcg(reinterpret_cast<const float4 *>(act) + k);
    }
    if (tid < 9) coef[tid] = tid < 8 ? probs[tid] : sigmoid_ref(gate_logit[0]);
    ok = mbar_wait(&bar[1], 0, err, kErrTimeout) && ok;
    __syncthreads();
    if (!ok || *reinterpret_cast<volatile uint32_t *>(err)) return;
    // ---- phase 3: the CTA's outputs; lane tasks k = (expert j, chunk c) over the 9 down rows
    for (int o = warp; o < nd; o += nw) {
        const int d = d_lo + o;
        float a = 0.f;
        for (int k = lane; k < 9 * cpr; k += 32) {
            const int j = k / cpr, c = k - j * cpr, r = j * f.outs + o;
            float w[16];
            smem_chunk_weights<BITS>(sm + f.dn_code() + r * f.dn_row,
                                     reinterpret_cast<const uint16_t *>(sm + f.dn_sb(0) + r * f.dn_grp),
                                     reinterpret_cast<const uint16_t *>(sm + f.dn_sb(1) + r * f.dn_grp), c, w);
            const float4 *ap = reinterpret_cast<const float4 *>(acts) + j * 4 * cpr + c;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 av = ap[q * cpr];
                s0 = fmaf(w[4 * q], av.x, s0);
                s1 = fmaf(w[4 * q + 1], av.y, s1);
                s0 = fmaf(w[4 * q + 2], av.z, s0);
                s1 = fmaf(w[4 * q + 3], av.w, s1);
            }
            a = fmaf(coef[j], s0 + s1, a);
        }
        const float r = warp_sum_butterfly(a);
        if (lane == 0) {
            if (out) out[d] = f32_to_bf16_bits(r);
            if (resid) resid[d] += r;
        }
    }
}

}  // namespace di
