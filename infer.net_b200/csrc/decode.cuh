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
