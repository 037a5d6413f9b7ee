// Quantised GEMV kernels: the di_quant_* operators and the decode (small T) path of the
// MoE block. One warp per output row; codes are read with 16-byte coalesced loads, the
// per-64 scale/bias once per group, and the lane partials reduced with a shuffle tree.
#pragma once
#include "common.cuh"
#include "route.cuh"

namespace di {

// ------------------------------------------------------------------ generic operator GEMV
//
// di_quant_batch / matvec semantics (quantized.mm:35-59, :321-349): y[slot*rows + row] =
// W[experts[slot]][row] . x_slot with f32 input/output, any cols % 64 == 0, 5 or 8 bits.
// Evaluated in the canonical lane order (lane l owns columns 256b + 8l + j).
__device__ __forceinline__ float canonical_dot_f32(const QView &m, size_t row, const float *x) {
    const int lane = lane_id();
    const uint32_t *w = m.packed + row * m.words_per_row();
    const uint16_t *sc = m.scales + row * m.groups_per_row();
    const uint16_t *bi = m.biases + row * m.groups_per_row();
    float acc = 0.f;
    for (int base = lane * 8; base < m.cols; base += 256) {
        const float s = bf16_bits_to_f32(__ldg(sc + base / 64)), b = bf16_bits_to_f32(__ldg(bi + base / 64));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float wv = fmaf(code_to_f32(load_code(w, base + j, m.bits)), s, b);
            acc = fmaf(wv, __ldg(x + base + j), acc);
        }
    }
    return warp_sum_butterfly(acc);
}

struct GemvJob {
    QView m;
    const float *x;
    float *y;
    const uint32_t *experts;  // device copy of the job's expert ids
    int count, batched;
};

// blockIdx.y selects the job; warps of the grid cover (slot, row).
__global__ void quant_gemv_kernel(const GemvJob *__restrict__ jobs) {
    const GemvJob J = jobs[blockIdx.y];
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp >= J.count * J.m.rows) return;
    const int slot = warp / J.m.rows, row = warp % J.m.rows;
    const size_t r = (size_t)J.experts[slot] * J.m.rows + row;
    const float v = canonical_dot_f32(J.m, r, J.x + (J.batched ? (size_t)slot * J.m.cols : 0));
    if (lane_id() == 0) J.y[(size_t)slot * J.m.rows + row] = v;
}

// di_quant_experts first stage (quantized.mm:148-189): act[slot*rows + row] =
// silu(gate . x) * (up . x) for the selected experts, shared input x.
__global__ void quant_gate_up_kernel(QView g, QView u, const float *__restrict__ x, const uint32_t *__restrict__ experts,
                                     int count, float *__restrict__ act) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (warp >= count * g.rows) return;
    const int slot = warp / g.rows, row = warp % g.rows;
    const size_t r = (size_t)experts[slot] * g.rows + row;
    const float gv = canonical_dot_f32(g, r, x), uv = canonical_dot_f32(u, r, x);
    if (lane_id() == 0) act[(size_t)slot * g.rows + row] = silu_ref(gv) * uv;
}

// ------------------------------------------------------------------ decode block path
//
// 16 codes of row chunk c (columns 16c .. 16c+15): the raw words (loaded first, so that many
// chunks are in flight) and their f32 weights w = fma(q, scale, bias).
template <int BITS>
struct RawChunk {
    uint32_t q[BITS == 8 ? 4 : 3];
    uint16_t s, b;
};
template <int BITS>
__device__ __forceinline__ RawChunk<BITS> load_chunk(const QView &m, size_t row, int c) {
    RawChunk<BITS> r;
    const uint32_t *rw = m.packed + row * m.words_per_row();
    r.s = __ldg(m.scales + row * m.groups_per_row() + (c >> 2));
    r.b = __ldg(m.biases + row * m.groups_per_row() + (c >> 2));
    if constexpr (BITS == 8) {
        const uint4 q = ldg_nc_v4(rw + c * 4);
        r.q[0] = q.x; r.q[1] = q.y; r.q[2] = q.z; r.q[3] = q.w;
    } else {
        // 80 bits starting at bit 80c: words 5c/2 .. +2, offset 0 or 16
        const int w0 = (5 * c) >> 1;
        r.q[0] = ldg_nc_u32(rw + w0);
        r.q[1] = ldg_nc_u32(rw + w0 + 1);
        r.q[2] = ldg_nc_u32(rw + w0 + 2);
    }
    return r;
}
template <int BITS>
__device__ __forceinline__ void chunk_weights(const RawChunk<BITS> &r, int c, float *w) {
    const float s = bf16_bits_to_f32(r.s), b = bf16_bits_to_f32(r.b);
    if constexpr (BITS == 8) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = fmaf(byte_to_f32(r.q[i >> 2], i & 3), s, b);
    } else {
        uint32_t a = r.q[0], bb = r.q[1], cc = r.q[2];
        if (c & 1) {
            a = __funnelshift_r(a, bb, 16);
            bb = __funnelshift_r(bb, cc, 16);
            cc = cc >> 16;
        }
        const uint32_t q3[3] = {a, bb, cc};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int bit = 5 * i, k = bit >> 5, sh = bit & 31;
            uint32_t q = (sh + 5 <= 32) ? (q3[k] >> sh) : __funnelshift_r(q3[k], q3[k + 1], sh);
            w[i] = fmaf(code_to_f32(q & 31u), s, b);
        }
    }
}
template <int BITS>
__device__ __forceinline__ void load_weights16(const QView &m, size_t row, int c, float *w) {
    chunk_weights<BITS>(load_chunk<BITS>(m, row, c), c, w);
}

__device__ __forceinline__ void load_x16_bf16(const uint16_t *x, int c, float *v) {
    const uint4 *p = reinterpret_cast<const uint4 *>(x + c * 16);
    uint4 a = p[0], b = p[1];
    uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
}

// h[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * w) (gpu_graph.mm:48-61), one CTA per token.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, int D,
                                                      float eps, uint16_t *__restrict__ h, uint16_t *__restrict__ trace) {
    pdl_enter();
    __shared__ float part[8];
    const int t = blockIdx.x;
    const float *xr = x + (size_t)t * D;
    float ss = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) ss = fmaf(xr[d], xr[d], ss);
#pragma unroll
    for (int n = 16; n; n >>= 1) ss += __shfl_xor_sync(kFull, ss, n);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += part[i];
    const float scale = 1.0f / sqrtf(tot / (float)D + eps);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        uint16_t v = f32_to_bf16_bits(xr[d] * scale * w[d]);
        h[(size_t)t * D + d] = v;
        if (trace) trace[(size_t)t * D + d] = v;
    }
}

// ------------------------------------------------------------------ embedding row
__global__ void embedding_kernel(QView m, int token, float *__restrict__ out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= m.cols) return;
    const uint32_t *rw = m.packed + (size_t)token * m.words_per_row();
    const float s = bf16_bits_to_f32(m.scales[(size_t)token * m.groups_per_row() + c / 64]);
    const float b = bf16_bits_to_f32(m.biases[(size_t)token * m.groups_per_row() + c / 64]);
    out[c] = fmaf(code_to_f32(load_code(rw, c, m.bits)), s, b);
}

}  // namespace di
