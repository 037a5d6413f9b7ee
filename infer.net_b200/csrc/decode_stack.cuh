// Persistent one-token decode of a whole MoE stack: every layer of Qwen36Model.cs:218-262 for one
// token in ONE cooperative kernel of one CTA per SM, so no layer pays a kernel boundary.
//
// Per layer l (gpu_graph.mm:48-61 RMSNorm, :134-146 router/top-8, quantized.mm:148-189 expert
// GEMVs, Qwen36Model.cs:242-244 combine):
//   S0  the CTA requests its share of the shared expert's rows (bulk copies into shared memory)
//       and loads its router rows into registers -- neither depends on the token;
//   S1  the residual row x_l (exchanged, below) -> h = bf16(x * rsqrt(mean(x^2) + eps) * w),
//       computed redundantly, identically, in every CTA;
//   S2  its router rows' logits in the canonical f32 order (bit-exact with the oracle) ->
//       exchanged; the row after the last expert is the shared expert's gate logit;
//   S3  every CTA reads all logits and selects the same top-8 (ties to the lower id), softmax;
//   S4  it requests the routed experts' rows of its first group of (gate, up) pairs;
//   S5  act = silu(gate . h) * (up . h) of its pairs -> exchanged: the second group is requested
//       when the first has landed and computed while it streams in, the down rows when the
//       second has landed. Split-K: warp w owns chunks [w*D/256, (w+1)*D/256) of h (in
//       registers), its lanes (pair, chunk); the 16 warp partials of a pair are summed in a
//       fixed order;
//   S6  warp j < 9 reads act of expert slot j, one 16-element chunk per lane, from the exchange
//       words (laid out so that these reads coalesce);
//   S7  ...and dots it with the down rows of slot j for all of the CTA's outputs d; then
//       x_{l+1}[d] = x_l[d] + sum_j c_j * part_j[d] (c = p_0..p_7, sigmoid(gate logit)) ->
//       exchanged (the last layer writes x instead).
//
// Exchanges use flag-in-data words: {f32 value, generation} in one 64-bit store, so a reader
// polls the data itself and no fence orders data before a flag. Generations grow monotonically
// across calls (a device counter), so stale words never match. Each CTA also bumps an arrival
// counter of the exchange (relaxed, no fence) once its words are stored; readers wait for the
// count first and then read the words about once, instead of every CTA re-polling the same
// lines. The count is only a hint: the words' generations decide. A slow reader can never see a
// value overwritten by the next layer: every write of layer l+1 happens after every CTA finished
// reading the same exchange of layer l (each step depends on the previous exchange of all CTAs).
// All waits are bounded; a timeout sets kErrTimeout and every CTA leaves.
//
// Dot products: a code q becomes the exact f32 denormal q * 2^-149 (its bits), the activation is
// pre-scaled by 2^64, so sum_i w_i x_i = 2^85 * sum_i (q_i 2^-149)(x_i 2^64) and
// (q s + b) . x = s * (q . x) + b * sum(x) per 16-element chunk: one byte permute and half a
// packed FMA (fma.rn.f32x2) per weight. The scaled operands stay normal for |x| in [2^-40, 2^64].
#pragma once
#include "decode.cuh"

namespace di {
namespace ds {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kI = 512;            // intermediate size of the stack kernel: one chunk per lane in S7
constexpr int kGroupPairs = 16;    // (gate, up) pairs of a copy group; a CTA has at most two groups
constexpr int kMaxOuts = 16;       // outputs per CTA (rows of the S7 partial sums)
constexpr int kDescBytes = 384;    // one StackLayer in shared memory

struct StackLayer {
    QView R, SR, G, U, Dn, SG, SU, SD;
    const float *bias;  // router bias [E] or null
    const float *norm;  // RMSNorm weights [D]
};
static_assert(sizeof(StackLayer) % 4 == 0 && sizeof(StackLayer) <= kDescBytes, "descriptor slot");

struct StackParams {
    const StackLayer *layers;
    int n_layers, E;
    float eps;
    float *x;                       // residual row [D], in/out
    uint16_t *h_trace;              // [n_layers][D] or null
    int32_t *ids_trace;             // [n_layers][8] or null
    unsigned long long *ll_logit;   // [E + 1] exchange words
    unsigned long long *ll_act;     // [9][16][I/16]: act[j][c*16 + e] at j*I + e*(I/16) + c
    unsigned long long *ll_x;       // [D]
    uint32_t *gen_base;             // generations used by earlier calls
    uint32_t *ctr_x, *ctr_act, *ctr_logit;  // exchange arrivals (G per layer step)
    uint32_t *err;
};

// Shared memory of one CTA: h (bf16) [D]; h * 2^64 (f32) [4][D/16] float4 (float4 q of chunk c
// at [q][c]) and its chunk sums [D/16]; two layer descriptors; partial sums [16][16][2]; its
// router rows (codes [D], scales [D/64], biases [D/64] each); the
// gate/up region: gate codes [pairs][gu_row], up codes, gate scales, gate biases, up scales, up
// biases; the down region: codes [9][outs][dn_row], scales, biases; misc.
struct Layout {
    int pairs, outs, gu_row, gu_grp, dn_row, dn_grp;
    int xq_off, xc_off, desc_off, part_off, rr_off, gu_off, dn_off, misc_off, total;
    __host__ __device__ int rr_row_bytes(int D) const { return D + D / 16; }  // codes, scales, biases
    __host__ __device__ int gu_code(int m) const { return gu_off + m * pairs * gu_row; }
    __host__ __device__ int gu_sb(int m, int k) const { return gu_off + 2 * pairs * gu_row + (2 * m + k) * pairs * gu_grp; }
    __host__ __device__ int dn_code() const { return dn_off; }
    __host__ __device__ int dn_sb(int k) const { return dn_off + 9 * outs * dn_row + k * 9 * outs * dn_grp; }
    // misc: 3 mbarriers (gate/up group 0, group 1, down), ids[8], coef[9], red[16], abort flag,
    // own residual values [outs]
    __host__ __device__ int bar() const { return misc_off; }
    __host__ __device__ int ids() const { return misc_off + 32; }
    __host__ __device__ int coef() const { return misc_off + 64; }
    __host__ __device__ int red() const { return misc_off + 112; }
    __host__ __device__ int abort_flag() const { return misc_off + 176; }
    __host__ __device__ int xown() const { return misc_off + 192; }
};
__host__ __device__ inline Layout layout(int D, int I, int bits, int grid) {
    Layout f;
    f.pairs = (9 * I + grid - 1) / grid;
    f.outs = (D + grid - 1) / grid;
    f.gu_row = D * bits / 8;
    f.gu_grp = D / 64 * 2;
    f.dn_row = I * bits / 8;
    f.dn_grp = I / 64 * 2;
    f.xq_off = (D * 2 + 127) & ~127;
    f.xc_off = f.xq_off + D * 4;
    f.desc_off = f.xc_off + ((D / 16 * 4 + 127) & ~127);
    f.part_off = f.desc_off + 2 * kDescBytes;
    f.rr_off = f.part_off + kWarps * kGroupPairs * 2 * 4;
    f.gu_off = f.rr_off + 2 * (D + D / 16);  // the CTA's (at most two) router rows
    f.dn_off = f.gu_off + ((2 * f.pairs * (f.gu_row + 2 * f.gu_grp) + 127) & ~127);
    f.misc_off = f.dn_off + ((9 * f.outs * (f.dn_row + 2 * f.dn_grp) + 127) & ~127);
    f.total = f.misc_off + 192 + ((f.outs * 4 + 15) & ~15);
    return f;
}

__device__ __forceinline__ unsigned long long ll_pack(float v, uint32_t gen) {
    return ((unsigned long long)gen << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void ll_store(unsigned long long *p, float v, uint32_t gen) {
    *reinterpret_cast<volatile unsigned long long *>(p) = ll_pack(v, gen);
}
__device__ __forceinline__ bool timed_out(uint64_t t0, const uint32_t *err) {
    return global_ns() - t0 > kWaitLimitNs || (*reinterpret_cast<const volatile uint32_t *>(err) & kErrTimeout);
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long *p) {
    return *reinterpret_cast<const volatile unsigned long long *>(p);
}
// Wait until an arrival counter reaches `target` (wrap-safe); false after the time limit or once
// another CTA has timed out.
__device__ __forceinline__ bool wait_count(const uint32_t *ctr, uint32_t target, const uint32_t *err) {
    const volatile uint32_t *c = reinterpret_cast<const volatile uint32_t *>(ctr);
    if ((int)(*c - target) >= 0) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t n = 1;; ++n) {
        if ((int)(*c - target) >= 0) return true;
        if ((n & 255u) == 0 && timed_out(t0, err)) return false;
    }
}

// Words p[idx[a]] (idx[a] < 0: none) until all carry `gen`: every pass issues its loads back to
// back, so a thread waits about one L2 round trip, not one per word. False after the time limit or
// once another CTA has timed out.
template <int N>
__device__ __forceinline__ bool ll_gather(const unsigned long long *p, const int (&idx)[N], uint32_t gen, float (&v)[N],
                                          const uint32_t *err) {
    unsigned long long w[N];
#pragma unroll
    for (int a = 0; a < N; ++a) w[a] = idx[a] >= 0 ? ll_load(p + idx[a]) : ((unsigned long long)gen << 32);
    uint64_t t0 = 0;
    for (uint32_t n = 0;; ++n) {
        bool all = true;
#pragma unroll
        for (int a = 0; a < N; ++a)
            if ((uint32_t)(w[a] >> 32) != gen) {
                all = false;
                w[a] = ll_load(p + idx[a]);
            }
        if (all) break;
        if (n == 0)
            t0 = global_ns();
        else if ((n & 255u) == 0 && timed_out(t0, err))
            return false;
    }
#pragma unroll
    for (int a = 0; a < N; ++a) v[a] = __uint_as_float((uint32_t)w[a]);
    return true;
}
// Words p[a * stride] for a < N (all present), as ll_gather.
template <int N>
__device__ __forceinline__ bool ll_gather_strided(const unsigned long long *p, int stride, uint32_t gen, float (&v)[N],
                                                  const uint32_t *err) {
    unsigned long long w[N];
#pragma unroll
    for (int a = 0; a < N; ++a) w[a] = ll_load(p + a * stride);
    uint64_t t0 = 0;
    for (uint32_t n = 0;; ++n) {
        bool all = true;
#pragma unroll
        for (int a = 0; a < N; ++a)
            if ((uint32_t)(w[a] >> 32) != gen) {
                all = false;
                w[a] = ll_load(p + a * stride);
            }
        if (all) break;
        if (n == 0)
            t0 = global_ns();
        else if ((n & 255u) == 0 && timed_out(t0, err))
            return false;
    }
#pragma unroll
    for (int a = 0; a < N; ++a) v[a] = __uint_as_float((uint32_t)w[a]);
    return true;
}
// idx[a] = first + a * stride where below count, else -1
template <int N>
__device__ __forceinline__ void strided_idx(int (&idx)[N], int first, int stride, int count) {
#pragma unroll
    for (int a = 0; a < N; ++a) idx[a] = first + a * stride < count ? first + a * stride : -1;
}

// The 16 codes of chunk c of a code row in shared memory, as f32 denormals q * 2^-149.
template <int BITS>
__device__ __forceinline__ void chunk_denormals(const uint8_t *row, int c, float *w) {
    if constexpr (BITS == 8) {
        const uint4 q = *reinterpret_cast<const uint4 *>(row + c * 16);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = __uint_as_float(__byte_perm(qw[i >> 2], 0u, 0x4440u + (i & 3)));
    } else {
        const uint32_t *wd = reinterpret_cast<const uint32_t *>(row) + ((5 * c) >> 1);
        uint32_t a = wd[0], b = wd[1], cc = wd[2];
        if (c & 1) {  // odd chunks start 16 bits into their first word
            a = __funnelshift_r(a, b, 16);
            b = __funnelshift_r(b, cc, 16);
            cc = cc >> 16;
        }
        const uint32_t q3[3] = {a, b, cc};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int bit = 5 * i, k = bit >> 5, sh = bit & 31;
            const uint32_t q = (sh + 5 <= 32) ? (q3[k] >> sh) : __funnelshift_r(q3[k], q3[k + 1], sh);
            w[i] = __uint_as_float(q & 31u);
        }
    }
}

constexpr float kXScale = 0x1p64f;      // activation pre-scale
constexpr float kDotScale = 0x1p85f;    // 2^149 / 2^64

// packed f32 pairs for fma.rn.f32x2
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float hsum2(unsigned long long v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return a + b;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// sum_i w[i] * x[i] over a chunk of 16: w the denormal codes, x4 its four float4s (scaled)
__device__ __forceinline__ float chunk_dot(const float *w, const float4 *x4) {
    unsigned long long a0 = 0ull, a1 = 0ull;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        a0 = fma2(pk2(w[4 * q], w[4 * q + 1]), pk2(x4[q].x, x4[q].y), a0);
        a1 = fma2(pk2(w[4 * q + 2], w[4 * q + 3]), pk2(x4[q].z, x4[q].w), a1);
    }
    return hsum2(a0) + hsum2(a1);
}

// A router row staged in shared memory (codes [D], scales, biases) into the registers of the
// canonical dot product (the layout router_raw_load reads from global memory).
__device__ __forceinline__ void router_row_from_smem(const uint8_t *row, int D, RouterRaw &r) {
    const uint32_t lane = lane_id();
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(row + D), *bi = sc + D / 64;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int base = k * 256 + lane * 8;
        if (base < D) {
            r.q[k] = *reinterpret_cast<const uint2 *>(row + base);
            r.s[k] = sc[base / 64];
            r.b[k] = bi[base / 64];
        }
    }
}

// The hidden size is a template parameter (512, 1024 or 2048) and I = kI: with the geometry known
// to the compiler, the loop-invariant state fits in registers (a spill would go to L2 here: the
// shared-memory carve-out leaves almost no L1).
template <int BITS, int D>
__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(const StackParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int I = kI;
    const int E = p.E, G = gridDim.x, cta = blockIdx.x;
    const Layout f = layout(D, I, BITS, G);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint16_t *xs = reinterpret_cast<uint16_t *>(sm);
    float4 *xq = reinterpret_cast<float4 *>(sm + f.xq_off);      // h * 2^64, [4][D/16]
    float *xcs = reinterpret_cast<float *>(sm + f.xc_off);       // chunk sums of h
    float *part = reinterpret_cast<float *>(sm + f.part_off);    // S5 [warp][pair][gate/up], S7 [slot][out]
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + f.bar());  // gate/up group 0, group 1, down
    int32_t *ids_s = reinterpret_cast<int32_t *>(sm + f.ids());
    float *coef = reinterpret_cast<float *>(sm + f.coef());
    float *red = reinterpret_cast<float *>(sm + f.red());
    volatile int *abort_s = reinterpret_cast<volatile int *>(sm + f.abort_flag());
    float *xown = reinterpret_cast<float *>(sm + f.xown());
    constexpr int cpd = D / 16, cpw = cpd / kWarps;  // chunks of h; S5: chunks per warp
    const int cl = lane & (cpw - 1), slot = lane / cpw, my_c = warp * cpw + cl;

    // this CTA's shares: (gate, up) pairs [p_lo, p_hi) of the 9*I, outputs [d_lo, d_hi), router rows [r_lo, r_hi) of E+1
    const int P = 9 * I;
    const int p_lo = (int)((long long)cta * P / G), p_hi = (int)((long long)(cta + 1) * P / G), np = p_hi - p_lo;
    const int d_lo = (int)((long long)cta * D / G), d_hi = (int)((long long)(cta + 1) * D / G), nd = d_hi - d_lo;
    const int r_lo = (int)((long long)cta * (E + 1) / G), r_hi = (int)((long long)(cta + 1) * (E + 1) / G);
    const int j_lo = p_lo / I;
    // local pairs [0, np): segment 0 is expert slot j_lo up to seg_end, segment 1 slot j_lo + 1;
    // copy group 0 is pairs [0, g_end), group 1 the rest
    const int seg_end = np > 0 ? min(np, (j_lo + 1) * I - p_lo) : 0;
    const int g_end = min(np, kGroupPairs);
    const uint32_t pair_bytes = 2u * (f.gu_row + 2 * f.gu_grp), slot_dn_bytes = (uint32_t)nd * (f.dn_row + 2 * f.dn_grp);
    const int q_shared = max(0, min(np, 8 * I - p_lo));  // local pairs from here on are the shared expert's
    const uint32_t shared0 = (uint32_t)max(0, g_end - q_shared) * pair_bytes;
    const uint32_t shared1 = (uint32_t)max(0, np - max(g_end, q_shared)) * pair_bytes;
    const uint32_t routed0 = (uint32_t)g_end * pair_bytes - shared0;
    const uint32_t routed1 = (uint32_t)(np - g_end) * pair_bytes - shared1;
    constexpr int kGroupCopies = 12;  // per group: 2 segments x 6 fields
    constexpr int kGuCopies = 2 * kGroupCopies;
    constexpr int kCopies = kGuCopies + 27;
    constexpr int kDescWords = (int)sizeof(StackLayer) / 4;

    if (tid == 0) {
        for (int b = 0; b < 3; ++b) mbar_init(&bar[b], 1);
        fence_mbarrier_init();
        *abort_s = 0;
    }
    if (tid < kDescWords)
        reinterpret_cast<uint32_t *>(sm + f.desc_off)[tid] = reinterpret_cast<const uint32_t *>(p.layers)[tid];
    // every CTA reads the generation base before its first exchange write; CTA 0 advances it at
    // its end, which is after the first exchange (so after every CTA has read it)
    const uint32_t base = *reinterpret_cast<const volatile uint32_t *>(p.gen_base);
    __syncthreads();

    bool armed = false;  // thread 0: this layer's arrivals (with the routed bytes) are done
    uint32_t ph = 0;
    for (int l = 0; l < p.n_layers; ++l) {
        const StackLayer &Ly = *reinterpret_cast<const StackLayer *>(sm + f.desc_off + (l & 1) * kDescBytes);
        const uint32_t gen = base + (uint32_t)l + 1;
        ph = (uint32_t)l & 1u;
        // copy k: k < 24 field k%6 of gate/up piece (group k/12, segment (k%12)/6), else down
        // field (k-24)%3 of expert slot (k-24)/3; `routed` selects slots 0..7 or slot 8
        auto issue_copy = [&](int k, bool routed) {
            if (k < kGuCopies) {
                const int gr = k / kGroupCopies, sg = (k % kGroupCopies) / 6, field = k % 6;
                const int q0 = max(sg ? seg_end : 0, gr ? g_end : 0), q1 = min(sg ? np : seg_end, gr ? np : g_end);
                const int j = j_lo + sg;
                if (q0 >= q1 || (j < 8) != routed) return;
                const int e = j < 8 ? ids_s[j] : 0;
                const int m = field & 1, kind = field >> 1;  // m: gate / up; kind: codes, scales, biases
                const QView &W = m ? (j < 8 ? Ly.U : Ly.SU) : (j < 8 ? Ly.G : Ly.SG);
                const size_t row = (size_t)e * I + (p_lo + q0 - j * I);
                uint64_t *b = &bar[gr];
                if (kind == 0)
                    bulk_load(sm + f.gu_code(m) + q0 * f.gu_row,
                              reinterpret_cast<const uint8_t *>(W.packed) + row * f.gu_row, (uint32_t)(q1 - q0) * f.gu_row, b);
                else
                    bulk_load(sm + f.gu_sb(m, kind - 1) + q0 * f.gu_grp,
                              (kind == 1 ? W.scales : W.biases) + row * (f.gu_grp / 2), (uint32_t)(q1 - q0) * f.gu_grp, b);
            } else {
                const int kk = k - kGuCopies, j = kk / 3, kind = kk % 3;
                if ((j < 8) != routed || nd == 0) return;
                const int e = j < 8 ? ids_s[j] : 0;
                const QView &W = j < 8 ? Ly.Dn : Ly.SD;
                const size_t row = (size_t)e * D + d_lo;
                if (kind == 0)
                    bulk_load(sm + f.dn_code() + j * f.outs * f.dn_row,
                              reinterpret_cast<const uint8_t *>(W.packed) + row * f.dn_row, (uint32_t)nd * f.dn_row, &bar[2]);
                else
                    bulk_load(sm + f.dn_sb(kind - 1) + j * f.outs * f.dn_grp,
                              (kind == 1 ? W.scales : W.biases) + row * (f.dn_grp / 2), (uint32_t)nd * f.dn_grp, &bar[2]);
            }
        };
        const int my_k = lane * kWarps + warp;  // the copy this thread issues, if below kCopies
        // ---- S0: the shared expert's rows and the router rows (token independent). The bytes of
        // the shared copies are expected now, the routed ones with the arrivals in S3.
        fence_proxy_async_smem();  // this layer's copies overwrite what the last one read
        if (tid == 0) {
            armed = false;
            mbar_expect_tx(&bar[0], shared0);
            mbar_expect_tx(&bar[1], shared1);
            mbar_expect_tx(&bar[2], slot_dn_bytes);
        }
        __syncthreads();
        if (my_k < kCopies) issue_copy(my_k, false);
        // the CTA's router rows into shared memory: piece k of D/16 code pieces, D/512 scale
        // pieces and D/512 bias pieces of 16 bytes per row
        {
            const int per_row = D / 16 + D / 256;
            if (tid < (r_hi - r_lo) * per_row) {
                const int rr_i = tid / per_row, k = tid - rr_i * per_row, row = r_lo + rr_i;
                const QView &R = row < E ? Ly.R : Ly.SR;
                const size_t rrow = row < E ? (size_t)row : 0;
                const void *src;
                if (k < D / 16)
                    src = reinterpret_cast<const uint8_t *>(R.packed) + rrow * D + k * 16;
                else if (k < D / 16 + D / 512)
                    src = reinterpret_cast<const uint8_t *>(R.scales + rrow * (D / 64)) + (k - D / 16) * 16;
                else
                    src = reinterpret_cast<const uint8_t *>(R.biases + rrow * (D / 64)) + (k - D / 16 - D / 512) * 16;
                cp_async_16(sm + f.rr_off + rr_i * f.rr_row_bytes(D) + k * 16, src, true);
            }
            cp_async_commit();
        }
        const int my_row = r_lo + warp;
        const float row_bias = my_row < E && Ly.bias ? Ly.bias[my_row] : 0.f;
        float nw[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) nw[a] = tid + a * kThreads < D ? Ly.norm[tid + a * kThreads] : 0.f;
        // the next layer's descriptor into the other slot (read from S0 of the next layer on)
        if (l + 1 < p.n_layers && tid >= kThreads - kDescWords)
            reinterpret_cast<uint32_t *>(sm + f.desc_off + ((l + 1) & 1) * kDescBytes)[tid - (kThreads - kDescWords)] =
                reinterpret_cast<const uint32_t *>(p.layers + l + 1)[tid - (kThreads - kDescWords)];

        // ---- S1: residual row -> h; thread t holds x[t + 512 a]
        float xv[4];
        bool ok = true;
        if (l == 0) {
#pragma unroll
            for (int a = 0; a < 4; ++a) xv[a] = tid + a * kThreads < D ? p.x[tid + a * kThreads] : 0.f;
        } else {
            if (tid == 0 && !wait_count(p.ctr_x, (gen - 1) * (uint32_t)G, p.err)) *abort_s = 1;
            __syncthreads();
            int idx[4];
            strided_idx(idx, tid, kThreads, D);
            ok = !*abort_s && ll_gather<4>(p.ll_x, idx, gen - 1, xv, p.err);
#pragma unroll
            for (int a = 0; a < 4; ++a)
                if (tid + a * kThreads >= D) xv[a] = 0.f;
        }
        if (!ok) {
            atomicOr(p.err, kErrTimeout);
            *abort_s = 1;
        }
        float ss = 0.f;
#pragma unroll
        for (int a = 0; a < 4; ++a) ss = fmaf(xv[a], xv[a], ss);
        ss = warp_sum_butterfly(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (*abort_s) break;
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += red[w];
        const float scale = 1.0f / sqrtf(tot / (float)D + p.eps);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int d = tid + a * kThreads;  // a warp holds 32 consecutive d: two chunks of 16
            float hf = 0.f;
            if (d < D) {
                const uint16_t h = f32_to_bf16_bits(xv[a] * scale * nw[a]);
                hf = bf16_bits_to_f32(h);
                xs[d] = h;
                reinterpret_cast<float *>(xq)[((d & 15) >> 2) * cpd * 4 + (d >> 4) * 4 + (d & 3)] = hf * kXScale;
                if (cta == 0 && p.h_trace) p.h_trace[(size_t)l * D + d] = h;
                if (d >= d_lo && d < d_hi) xown[d - d_lo] = xv[a];
            }
            // chunk sums: the 16 lanes of a chunk (D is a multiple of 512, so d < D for all or none)
#pragma unroll
            for (int n = 8; n; n >>= 1) hf += __shfl_xor_sync(kFull, hf, n);
            if (d < D && (d & 15) == 0) xcs[d >> 4] = hf;
        }
        cp_async_wait<0>();  // the router rows
        __syncthreads();

        // ---- S2: router logits of this CTA's rows (row E: the shared expert's gate logit)
        if (my_row < r_hi) {
            RouterRaw rr;
            router_row_from_smem(sm + f.rr_off + warp * f.rr_row_bytes(D), D, rr);
            float v = router_raw_dot(rr, xs, D);
            if (my_row < E) v = v + row_bias;
            if (lane == 0) ll_store(p.ll_logit + my_row, v, gen);
        }
        __syncthreads();
        if (tid == 0) atomicAdd(p.ctr_logit, 1u);

        // ---- S3: all logits -> the same top-8 in every CTA; word 8 of every lane is the gate logit
        if (warp == 0) {
            if (lane == 0 && !wait_count(p.ctr_logit, gen * (uint32_t)G, p.err)) *abort_s = 1;
            __syncwarp();
            float v[9];
            int idx[9];
            strided_idx(idx, lane, 32, E);
            idx[8] = E;
            ok = !*abort_s && ll_gather<9>(p.ll_logit, idx, gen, v, p.err);
            if (!__all_sync(kFull, ok)) {
                if (lane == 0) {
                    atomicOr(p.err, kErrTimeout);
                    *abort_s = 1;
                }
            } else {
                const float g = v[8];
                bool nonfinite = false;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (lane + 32 * j < E && !isfinite(v[j])) {
                        nonfinite = true;
                        v[j] = -INFINITY;
                    }
                if (__any_sync(kFull, nonfinite) && lane == 0 && cta == 0) atomicOr(p.err, kErrNonFinite);
                int32_t sel[8];
                float chosen[8];
                select_top8(v, E, sel, chosen);
                float mx = chosen[0], pr[8], sum = 0.f;
#pragma unroll
                for (int n = 1; n < 8; ++n) mx = fmaxf(mx, chosen[n]);
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    pr[n] = expf(chosen[n] - mx);
                    sum += pr[n];
                }
                if (lane < 8) {
                    float pv = 0.f;
                    int32_t sv = 0;
#pragma unroll
                    for (int m = 0; m < 8; ++m)
                        if (m == lane) {
                            pv = pr[m];
                            sv = sel[m];
                        }
                    ids_s[lane] = min(max(sv, 0), E - 1);
                    coef[lane] = pv / sum;
                    if (cta == 0 && p.ids_trace) p.ids_trace[(size_t)l * 8 + lane] = sv;
                }
                if (lane == 0) {
                    coef[8] = sigmoid_ref(g);
                    mbar_arrive_expect_tx(&bar[0], routed0);
                    mbar_arrive_expect_tx(&bar[1], routed1);
                    mbar_arrive_expect_tx(&bar[2], 8u * slot_dn_bytes);
                    armed = true;
                }
            }
        }
        __syncthreads();
        if (*abort_s) break;

        // ---- S4: the routed rows of gate/up group 0
        if (my_k < kGroupCopies) issue_copy(my_k, true);

        // ---- S5: act of the CTA's pairs, group by group
        float4 x4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x4[i] = xq[i * cpd + my_c];
        const float xcv = xcs[my_c];
        // partial (gate, up) dots of chunk my_c for the group's pairs slot + slots*k; summed over
        // the warp's chunks (butterfly within the slot's lanes) into part[warp][pair][gate/up]
        auto group_partials = [&](int qb, int qe) {
            constexpr int kSlots = 32 / cpw, kRounds = kGroupPairs / kSlots;
            float gp[kRounds], up[kRounds];
#pragma unroll
            for (int k = 0; k < kRounds; ++k) {
                const int q = qb + slot + kSlots * k;
                gp[k] = up[k] = 0.f;
                if (q < qe) {
                    float wg[16], wu[16];
                    chunk_denormals<BITS>(sm + f.gu_code(0) + q * f.gu_row, my_c, wg);
                    chunk_denormals<BITS>(sm + f.gu_code(1) + q * f.gu_row, my_c, wu);
                    const int so = q * f.gu_grp + (my_c >> 2) * 2;  // byte offset of this chunk's group
                    const float gs = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 0) + so));
                    const float gb = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 1) + so));
                    const float us = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 0) + so));
                    const float ub = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 1) + so));
                    gp[k] = fmaf(gs, chunk_dot(wg, x4) * kDotScale, gb * xcv);
                    up[k] = fmaf(us, chunk_dot(wu, x4) * kDotScale, ub * xcv);
                }
            }
            // sum over the warp's chunks: butterflies within each slot's lanes, rounds interleaved
#pragma unroll
            for (int n = 1; n < cpw; n <<= 1)
#pragma unroll
                for (int k = 0; k < kRounds; ++k) {
                    gp[k] += __shfl_xor_sync(kFull, gp[k], n);
                    up[k] += __shfl_xor_sync(kFull, up[k], n);
                }
            if (cl == 0)
#pragma unroll
                for (int k = 0; k < kRounds; ++k) {
                    const int ql = slot + kSlots * k;
                    if (qb + ql < qe) {
                        part[(warp * kGroupPairs + ql) * 2] = gp[k];
                        part[(warp * kGroupPairs + ql) * 2 + 1] = up[k];
                    }
                }
        };
        // warp 0: pair (lane >> 1) of the group, lane & 1 gate / up: the 16 warp partials in order
        auto group_act = [&](int qb, int qe) {
            if (warp != 0) return;
            const int ql = lane >> 1, q = qb + ql;
            float s = 0.f;
            if (q < qe)
#pragma unroll
                for (int w = 0; w < kWarps; ++w) s += part[(w * kGroupPairs + ql) * 2 + (lane & 1)];
            const float u = __shfl_down_sync(kFull, s, 1);
            if (q < qe && !(lane & 1)) {
                const int pp = p_lo + q, j = pp / I, i = pp - j * I;
                ll_store(p.ll_act + (size_t)j * I + (i & 15) * (I / 16) + (i >> 4), silu_ref(s) * u, gen);
            }
        };
        ok = mbar_wait(&bar[0], ph, p.err, kErrTimeout);
        // group 1 streams while group 0 is computed (issued whatever the wait gave, so that every
        // requested byte lands before this CTA can leave)
        if (my_k >= kGroupCopies && my_k < kGuCopies) issue_copy(my_k, true);
        if (ok) group_partials(0, g_end);
        __syncthreads();
        if (ok) group_act(0, g_end);
        ok = mbar_wait(&bar[1], ph, p.err, kErrTimeout) && ok;
        if (my_k >= kGuCopies && my_k < kCopies) issue_copy(my_k, true);  // down rows, behind group 1
        __syncthreads();  // group 0's partials are consumed
        if (ok) group_partials(g_end, np);
        if (!ok) *abort_s = 1;
        __syncthreads();
        if (*abort_s) break;
        group_act(g_end, np);
        __syncthreads();
        if (tid == 0) {
            atomicAdd(p.ctr_act, 1u);
            if (!wait_count(p.ctr_act, gen * (uint32_t)G, p.err)) {
                atomicOr(p.err, kErrTimeout);
                *abort_s = 1;
            }
        }
        __syncthreads();
        if (*abort_s) break;

        // ---- S6 + S7: warp 7 + j: act of slot j, chunk `lane`, against the down rows of slot j
        // (warp 0, which ran the top-8 and the act sums, stays out)
        if (warp >= kWarps - 9) {
            const int j = warp - (kWarps - 9);
            float av[16];
            ok = ll_gather_strided<16>(p.ll_act + j * I + lane, I / 16, gen, av, p.err);
            float asum = 0.f;
            float4 a4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                asum += (av[4 * q] + av[4 * q + 1]) + (av[4 * q + 2] + av[4 * q + 3]);
                a4[q] = make_float4(av[4 * q] * kXScale, av[4 * q + 1] * kXScale, av[4 * q + 2] * kXScale,
                                    av[4 * q + 3] * kXScale);
            }
            ok = ok && mbar_wait(&bar[2], ph, p.err, kErrTimeout);
            if (!ok) {
                atomicOr(p.err, kErrTimeout);
                *abort_s = 1;
            } else {
                // four outputs at a time: their loads, dots and butterflies interleave
                for (int o0 = 0; o0 < nd; o0 += 4) {
                    float v[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int o = o0 + u;
                        v[u] = 0.f;
                        if (o < nd) {
                            const int r = j * f.outs + o;
                            float w[16];
                            chunk_denormals<BITS>(sm + f.dn_code() + r * f.dn_row, lane, w);
                            const int so = r * f.dn_grp + (lane >> 2) * 2;
                            const float sc = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.dn_sb(0) + so));
                            const float bi = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.dn_sb(1) + so));
                            v[u] = fmaf(sc, chunk_dot(w, a4) * kDotScale, bi * asum);
                        }
                    }
#pragma unroll
                    for (int n = 16; n; n >>= 1)
#pragma unroll
                        for (int u = 0; u < 4; ++u) v[u] += __shfl_xor_sync(kFull, v[u], n);
                    if (lane == 0)
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            if (o0 + u < nd) part[j * kMaxOuts + o0 + u] = v[u];
                }
            }
        }
        __syncthreads();
        if (*abort_s) break;
        const bool last = l + 1 == p.n_layers;
        if (tid < nd) {
            float out = 0.f;
#pragma unroll
            for (int j = 0; j < 9; ++j) out = fmaf(coef[j], part[j * kMaxOuts + tid], out);
            const int d = d_lo + tid;
            const float xn = xown[tid] + out;
            if (last)
                p.x[d] = xn;
            else
                ll_store(p.ll_x + d, xn, gen);
        }
        __syncthreads();  // the regions are reused by the next layer's copies
        if (tid == 0) atomicAdd(p.ctr_x, 1u);
    }
    if (tid == 0) {
        if (*abort_s) {
            // leave no copy in flight into this CTA's shared memory: complete the barriers' phases
            // (arriving without the routed bytes if they were never requested) and wait for them
            if (!armed)
                for (int b = 0; b < 3; ++b) mbar_arrive_expect_tx(&bar[b], 0);
            for (int b = 0; b < 3; ++b) mbar_wait(&bar[b], ph, p.err, kErrTimeout);
        }
        if (cta == 0) *reinterpret_cast<volatile uint32_t *>(p.gen_base) = base + (uint32_t)p.n_layers;
    }
}

}  // namespace ds
}  // namespace di
