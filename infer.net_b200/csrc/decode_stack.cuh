// Persistent one-token decode of a whole MoE stack: every layer of Qwen36Model.cs:218-262 for one
// token in ONE cooperative kernel of one CTA per SM, so no layer pays a kernel boundary.
//
// Work split. The 9 expert slots (8 routed + the shared expert) x I = 512 intermediate columns are
// 144 units of 32 columns; CTA u < 144 owns unit (slot u / 16, columns [32 (u % 16), +32)): the 32
// (gate, up) row pairs of those columns and the same 32 columns of every down row. Its act values
// therefore stay in the CTA, and its share of the layer output is a partial sum over 32 columns
// for every one of the D outputs. The partial sums of all units are added in a fixed-point
// accumulator by 64-bit integer atomics (exact, so the result does not depend on their order).
//
// Per layer l (gpu_graph.mm:48-61 RMSNorm, :134-146 router/top-8, quantized.mm:148-189 expert
// GEMVs, Qwen36Model.cs:242-244 combine):
//   S0  token-independent copies: the CTA's router rows, and -- for a shared-expert unit -- all of
//       its weights, requested before the token arrives;
//   S1  x_l = x_{l-1} + y_{l-1} once every CTA has added into y_{l-1}; h = bf16(RMSNorm(x_l) * w),
//       computed redundantly, identically, in every CTA (every CTA holds all of x);
//   S2  its router rows' logits in the canonical f32 order (bit-exact with the oracle) ->
//       exchanged; the row after the last expert is the shared expert's gate logit;
//   S3  every CTA reads all logits and selects the same top-8 (ties to the lower id), softmax;
//       a routed unit requests its expert's rows (four gate/up groups, then the down columns);
//   S4  act = silu(gate . h) * (up . h) of its 32 pairs, group by group as they land. Split-K:
//       warp w owns chunks [w*D/256, (w+1)*D/256) of h (in registers), its lanes (pair, chunk);
//       the 16 warp partials of a pair are summed in a fixed order;
//   S5  for every output d: c_slot * sum over its 32 columns of down[d][i] * act[i] (a lane pair
//       per row, 16 columns each), rounded to a multiple of 2^-32; one bulk reduction of the copy
//       engine adds the CTA's D values into y_l at L2; then the CTA's arrival on the layer's
//       counter (after a device-scope fence).
// The last layer's sum is added to x by CTA 0, which writes the output row.
//
// The logits travel in flag-in-data words: {f32 value, generation} in one 64-bit store, so a
// reader polls the data itself and no fence orders data before a flag. Generations grow
// monotonically across calls (a device counter), so stale words never match. Each CTA also bumps
// an arrival counter once its words are stored; readers wait for the count first and then read
// the words about once. The accumulator y alternates between two buffers by layer parity; a CTA
// clears its slice of the buffer of layer l + 1 after the logits exchange of layer l, when every
// CTA has read it (as y_{l-1}) and before any CTA can add into it (after the exchange of l + 1).
// All waits are bounded; a timeout sets kErrTimeout and every CTA leaves.
//
// Dot products: a code q becomes the exact f32 denormal q * 2^-149 (its bits), the activation is
// pre-scaled by 2^64, so sum_i w_i x_i = 2^85 * sum_i (q_i 2^-149)(x_i 2^64) and
// (q s + b) . x = s * (q . x) + b * sum(x) per 16-element chunk: one byte permute and half a
// packed FMA (fma.rn.f32x2) per weight. The scaled operands stay normal for |x| in [2^-40, 2^64].
#pragma once
#include <cuda.h>

#include "decode.cuh"

namespace di {
namespace ds {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kI = 512;                       // intermediate size of the stack kernel
constexpr int kSlice = 32;                    // intermediate columns of one unit
constexpr int kSlicesPerSlot = kI / kSlice;   // 16
constexpr int kUnits = 9 * kSlicesPerSlot;    // 144: the kernel needs at least this many CTAs
constexpr int kGroupPairs = 8;                // (gate, up) pairs of a copy group
constexpr int kGroups = kSlice / kGroupPairs; // 4
constexpr int kDnBox = 256;                   // rows of one down-column tensor copy
constexpr int kDnRowBytes = 32;               // bytes of a row in the down-column copies
constexpr int kDescBytes = 384;               // one StackLayer in shared memory
// The fixed-point accumulator: a contribution c adds round(c * 2^32); |c| < 2^23, so the 144
// contributions of an output stay below 2^62.2 (no overflow). A larger or non-finite one sets
// kErrRange and the host recomputes the token with the per-layer kernels.
constexpr float kAccScale = 0x1p32f;
constexpr int kAccCopies = 4;  // CTA c adds into copy c % 4: 36 contributions per address, not 144
constexpr float kAccInv = 0x1p-32f;
constexpr float kAccLimit = 0x1p23f;

struct StackLayer {
    QView R, SR, G, U, Dn, SG, SU, SD;
    const float *bias;  // router bias [E] or null
    const float *norm;  // RMSNorm weights [D]
};
static_assert(sizeof(StackLayer) % 4 == 0 && sizeof(StackLayer) <= kDescBytes, "descriptor slot");

struct StackParams {
    const StackLayer *layers;
    const CUtensorMap *dn_maps;     // [n_layers][2]: routed, shared down codes (box 32 B x 256 rows)
    int n_layers, E;
    float eps;
    float *x;                       // residual row [D], in/out
    uint16_t *h_trace;              // [n_layers][D] or null
    int32_t *ids_trace;             // [n_layers][8] or null
    unsigned long long *ll_logit;   // [E + 1] exchange words
    unsigned long long *acc;        // [2][kAccCopies][D] fixed-point layer outputs: layer l adds into acc[l & 1]
    uint32_t *gen_base;             // generations used by earlier calls
    uint32_t *ctr_y, *ctr_logit;    // arrivals (G per layer step)
    uint32_t *err;
};

// Shared memory of one CTA: h (f32) [4][D/16] float4 (float4 q of chunk c at [q][c]) and its chunk
// sums [D/16]; two layer descriptors; gate/up partial sums [16 warps][32 pairs][2]; its router
// rows (codes [D], scales [D/64], biases [D/64] each); the gate/up region of the unit: gate codes
// [32][gu_row], up codes, gate scales, gate biases, up scales, up biases (once consumed, it holds the
// unit's fixed-point output vector [D]); the down columns [D][32 B]; misc.
struct Layout {
    int gu_row, gu_grp;
    int xc_off, desc_off, part_off, rr_off, gu_off, dn_off, misc_off, total;
    __host__ __device__ int rr_row_bytes(int D) const { return D + D / 16; }  // codes, scales, biases
    __host__ __device__ int gu_code(int m) const { return gu_off + m * kSlice * gu_row; }
    __host__ __device__ int gu_sb(int m, int k) const { return gu_off + 2 * kSlice * gu_row + (2 * m + k) * kSlice * gu_grp; }
    // misc: 5 mbarriers (gate/up groups 0-3, down), ids[8], coef[9], red[16], abort flag, act[32]
    __host__ __device__ int bar() const { return misc_off; }
    __host__ __device__ int ids() const { return misc_off + 64; }
    __host__ __device__ int coef() const { return misc_off + 96; }
    __host__ __device__ int red() const { return misc_off + 144; }
    __host__ __device__ int abort_flag() const { return misc_off + 208; }
    __host__ __device__ int act() const { return misc_off + 224; }
};
__host__ __device__ inline Layout layout(int D, int bits) {
    Layout f;
    f.gu_row = D * bits / 8;
    f.gu_grp = D / 64 * 2;
    f.xc_off = D * 4;
    f.desc_off = f.xc_off + ((D / 16 * 4 + 127) & ~127);
    f.part_off = f.desc_off + 2 * kDescBytes;
    f.rr_off = f.part_off + kWarps * kSlice * 2 * 4;
    f.gu_off = (f.rr_off + 2 * (D + D / 16) + 127) & ~127;  // the CTA's (at most two) router rows
    f.dn_off = (f.gu_off + 2 * kSlice * (f.gu_row + 2 * f.gu_grp) + 127) & ~127;
    f.misc_off = (f.dn_off + D * kDnRowBytes + 127) & ~127;
    f.total = f.misc_off + 224 + kSlice * 4;
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
// idx[a] = first + a * stride where below count, else -1
template <int N>
__device__ __forceinline__ void strided_idx(int (&idx)[N], int first, int stride, int count) {
#pragma unroll
    for (int a = 0; a < N; ++a) idx[a] = first + a * stride < count ? first + a * stride : -1;
}

// The 16 codes of chunk c of a code row in shared memory, as f32 denormals q * 2^-149 (row
// 16-byte aligned for 8-bit codes, 4-byte aligned for 5-bit ones).
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
// The canonical router dot product (router_raw_dot's order: lane l owns columns 256k + 8l + j,
// one fma chain per lane, then the xor butterfly) with h read from the CTA's f32 chunk layout.
template <int D>
__device__ __forceinline__ float router_dot_h(const RouterRaw &r, const float4 *hq) {
    constexpr int cpd = D / 16;
    const uint32_t lane = lane_id();
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < D / 256; ++k) {
        const int base = k * 256 + (int)lane * 8, c = base >> 4, q0 = (base & 15) >> 2;
        const float4 lo = hq[q0 * cpd + c], hi = hq[(q0 + 1) * cpd + c];
        const float xf[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        const float s = bf16_bits_to_f32(r.s[k]), bb = bf16_bits_to_f32(r.b[k]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float wv = fmaf(byte_to_f32(j < 4 ? r.q[k].x : r.q[k].y, j & 3), s, bb);
            acc = fmaf(wv, xf[j], acc);
        }
    }
    return warp_sum_butterfly(acc);
}

__device__ __forceinline__ float acc_value(unsigned long long v) { return __ll2float_rn((long long)v) * kAccInv; }

// Per-layer timeline of two CTAs (CTA 0, a routed unit, and CTA 143, a shared-expert unit),
// compiled in only with -DDI_DECODE_TIMELINE (a profiling build; read by di_debug_decode_timeline):
// %globaltimer at the layer's start (0), after the previous layer's output is complete (1), h
// ready (2), this CTA's logits published (3), the top-8 known (4), the copies requested (5), the
// first gate/up group landed (6), every copy landed (7), act complete (8), the output vector
// complete (9), and the reduction and arrival done (10).
constexpr int kTlEvents = 11, kTlLayers = 64;
#ifdef DI_DECODE_TIMELINE
__device__ unsigned long long g_ds_tl[2][kTlLayers][kTlEvents];
__device__ __forceinline__ void ds_mark(int ev, int l) {
    const int c = blockIdx.x == 0 ? 0 : blockIdx.x == kUnits - 1 ? 1 : -1;
    if (c >= 0 && threadIdx.x == 0 && l < kTlLayers) g_ds_tl[c][l][ev] = global_ns();
}
#else
__device__ __forceinline__ void ds_mark(int, int) {}
#endif

// The hidden size is a template parameter (512, 1024 or 2048) and I = kI: with the geometry known
// to the compiler, the loop-invariant state fits in registers (a spill would go to L2 here: the
// shared-memory carve-out leaves almost no L1).
template <int BITS, int D>
__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(const StackParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int I = kI;
    const int E = p.E, G = gridDim.x, cta = blockIdx.x;
    const Layout f = layout(D, BITS);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4 *hq = reinterpret_cast<float4 *>(sm);                  // h (f32), [4][D/16]
    float *xcs = reinterpret_cast<float *>(sm + f.xc_off);       // chunk sums of h
    float *part = reinterpret_cast<float *>(sm + f.part_off);    // [warp][pair][gate/up]
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + f.bar());  // gate/up groups 0-3, down
    int32_t *ids_s = reinterpret_cast<int32_t *>(sm + f.ids());
    float *coef = reinterpret_cast<float *>(sm + f.coef());
    float *red = reinterpret_cast<float *>(sm + f.red());
    volatile int *abort_s = reinterpret_cast<volatile int *>(sm + f.abort_flag());
    float *act_s = reinterpret_cast<float *>(sm + f.act());
    constexpr int cpd = D / 16, cpw = cpd / kWarps;  // chunks of h; S4: chunks per warp
    const int cl = lane & (cpw - 1), slot = lane / cpw, my_c = warp * cpw + cl;

    // this CTA's unit (slot uj, columns [uk * 32, +32)), its slice of the outputs (cleared in the
    // accumulator) and its router rows [r_lo, r_hi) of E + 1
    const bool has_unit = cta < kUnits;
    const int uj = has_unit ? cta / kSlicesPerSlot : 0, uk = cta % kSlicesPerSlot;
    const bool shared_unit = has_unit && uj == 8, routed_unit = has_unit && uj < 8;
    const int d_lo = (int)((long long)cta * D / G), d_hi = (int)((long long)(cta + 1) * D / G), nd = d_hi - d_lo;
    const int r_lo = (int)((long long)cta * (E + 1) / G), r_hi = (int)((long long)(cta + 1) * (E + 1) / G);
    // the unit's bytes of a down row: [x_lo, x_lo + 32 * BITS / 8); its copies start at the 16-byte
    // boundary x_box below (32 bytes from there always cover them)
    const int x_lo = uk * kSlice * BITS / 8, x_box = x_lo & ~15, dn_delta = x_lo - x_box;
    const uint32_t group_bytes = (uint32_t)kGroupPairs * 2u * (uint32_t)(f.gu_row + 2 * f.gu_grp);
    constexpr uint32_t kDnBytes = (uint32_t)D * kDnRowBytes;
    constexpr int kGuCopies = kGroups * 6;  // per group: gate and up codes, scales, biases
    constexpr int kCopies = kGuCopies + D / kDnBox;
    static_assert(kCopies <= 32, "one warp issues the copies");
    constexpr int kDescWords = (int)sizeof(StackLayer) / 4;

    if (tid == 0) {
        for (int b = 0; b <= kGroups; ++b) mbar_init(&bar[b], 1);
        fence_mbarrier_init();
        *abort_s = 0;
    }
    if (tid < kDescWords)
        reinterpret_cast<uint32_t *>(sm + f.desc_off)[tid] = reinterpret_cast<const uint32_t *>(p.layers)[tid];
    // layer 0 adds into acc[0]: clear this CTA's slice of its copies before its first arrival (the
    // fence below orders the stores before it); acc[1] is cleared during layer 0
    if (tid < kAccCopies * nd) p.acc[(size_t)(tid / nd) * D + d_lo + tid % nd] = 0ull;
    // every CTA reads the generation base before its first exchange write; CTA 0 advances it at
    // its end, which is after the first exchange (so after every CTA has read it)
    const uint32_t base = *reinterpret_cast<const volatile uint32_t *>(p.gen_base);
    __syncthreads();
    if (tid == 0) __threadfence();

    bool armed = false;  // thread 0: this layer's copies are requested (they must land before leaving)
    uint32_t ph = 0;
    float xv[D / kThreads];  // x[tid + 512 a]: every CTA holds the whole residual row
    for (int l = 0; l < p.n_layers; ++l) {
        const StackLayer &Ly = *reinterpret_cast<const StackLayer *>(sm + f.desc_off + (l & 1) * kDescBytes);
        const uint32_t gen = base + (uint32_t)l + 1;
        ds_mark(0, l);
        ph = (uint32_t)l & 1u;
        // copy k of the unit: k < 24 field k%6 of gate/up group k/6, else down-column box k-24
        auto issue_copy = [&](int k, int e) {
            if (k < kGuCopies) {
                const int g = k / 6, field = k % 6, m = field & 1, kind = field >> 1;  // m: gate / up
                const QView &W = m ? (shared_unit ? Ly.SU : Ly.U) : (shared_unit ? Ly.SG : Ly.G);
                const int q0 = g * kGroupPairs;
                const size_t row = (size_t)e * I + uk * kSlice + q0;
                if (kind == 0)
                    bulk_load(sm + f.gu_code(m) + q0 * f.gu_row,
                              reinterpret_cast<const uint8_t *>(W.packed) + row * f.gu_row,
                              (uint32_t)kGroupPairs * f.gu_row, &bar[g]);
                else
                    bulk_load(sm + f.gu_sb(m, kind - 1) + q0 * f.gu_grp,
                              (kind == 1 ? W.scales : W.biases) + row * (f.gu_grp / 2), (uint32_t)kGroupPairs * f.gu_grp,
                              &bar[g]);
            } else {
                const int b = k - kGuCopies;
                tma_load_2d(sm + f.dn_off + b * kDnBox * kDnRowBytes, p.dn_maps + 2 * l + (shared_unit ? 1 : 0), x_box,
                            e * D + b * kDnBox, &bar[kGroups]);
            }
        };
        // lane k of the last warp issues copy k: one warp issues them all, in order (gate/up group 0
        // first, the down columns last)
        const int my_k = warp == kWarps - 1 ? lane : kCopies;
        // ---- S0: token-independent copies (the shared expert's unit, the router rows)
        fence_proxy_async_smem();  // this layer's copies overwrite what the last one read
        if (shared_unit && tid == 0) {
            for (int g = 0; g < kGroups; ++g) mbar_arrive_expect_tx(&bar[g], group_bytes);
            mbar_arrive_expect_tx(&bar[kGroups], kDnBytes);
            armed = true;
        }
        __syncthreads();
        if (shared_unit && my_k < kCopies) issue_copy(my_k, 0);
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
        float nw[D / kThreads];
#pragma unroll
        for (int a = 0; a < D / kThreads; ++a) nw[a] = Ly.norm[tid + a * kThreads];
        // the next layer's descriptor into the other slot (read from S0 of the next layer on)
        if (l + 1 < p.n_layers && tid >= kThreads - kDescWords)
            reinterpret_cast<uint32_t *>(sm + f.desc_off + ((l + 1) & 1) * kDescBytes)[tid - (kThreads - kDescWords)] =
                reinterpret_cast<const uint32_t *>(p.layers + l + 1)[tid - (kThreads - kDescWords)];

        // ---- S1: x_l = x_{l-1} + y_{l-1} -> h
        if (l == 0) {
#pragma unroll
            for (int a = 0; a < D / kThreads; ++a) xv[a] = p.x[tid + a * kThreads];
        } else {
            if (tid == 0) {
                if (!wait_count(p.ctr_y, (gen - 1) * (uint32_t)G, p.err)) {
                    atomicOr(p.err, kErrTimeout);
                    *abort_s = 1;
                } else {
                    ld_acquire_gpu(p.ctr_y);  // every CTA's additions into y_{l-1} precede its (release) arrival
                    if (*reinterpret_cast<const volatile uint32_t *>(p.err) & kErrRange) *abort_s = 1;
                }
            }
            __syncthreads();
            if (*abort_s) break;
            ds_mark(1, l);
            const unsigned long long *y = p.acc + (size_t)((l - 1) & 1) * kAccCopies * D;
            unsigned long long yv[D / kThreads][kAccCopies];
#pragma unroll
            for (int a = 0; a < D / kThreads; ++a)
#pragma unroll
                for (int k = 0; k < kAccCopies; ++k) yv[a][k] = __ldcg(y + k * D + tid + a * kThreads);
#pragma unroll
            for (int a = 0; a < D / kThreads; ++a) {
                unsigned long long t = 0ull;
#pragma unroll
                for (int k = 0; k < kAccCopies; ++k) t += yv[a][k];
                xv[a] += acc_value(t);
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int a = 0; a < D / kThreads; ++a) ss = fmaf(xv[a], xv[a], ss);
        ss = warp_sum_butterfly(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += red[w];
        const float scale = 1.0f / sqrtf(tot / (float)D + p.eps);
#pragma unroll
        for (int a = 0; a < D / kThreads; ++a) {
            const int d = tid + a * kThreads;  // a warp holds 32 consecutive d: two chunks of 16
            const uint16_t h = f32_to_bf16_bits(xv[a] * scale * nw[a]);
            float hf = bf16_bits_to_f32(h);
            reinterpret_cast<float *>(hq)[((d & 15) >> 2) * cpd * 4 + (d >> 4) * 4 + (d & 3)] = hf;
            if (cta == 0 && p.h_trace) p.h_trace[(size_t)l * D + d] = h;
            // chunk sums: the 16 lanes of a chunk
#pragma unroll
            for (int n = 8; n; n >>= 1) hf += __shfl_xor_sync(kFull, hf, n);
            if ((d & 15) == 0) xcs[d >> 4] = hf;
        }
        cp_async_wait<0>();  // the router rows
        __syncthreads();
        ds_mark(2, l);

        // ---- S2: router logits of this CTA's rows (row E: the shared expert's gate logit)
        if (my_row < r_hi) {
            RouterRaw rr;
            router_row_from_smem(sm + f.rr_off + warp * f.rr_row_bytes(D), D, rr);
            float v = router_dot_h<D>(rr, hq);
            if (my_row < E) v = v + row_bias;
            if (lane == 0) ll_store(p.ll_logit + my_row, v, gen);
        }
        __syncthreads();
        if (tid == 0) atomicAdd(p.ctr_logit, 1u);
        ds_mark(3, l);

        // ---- S3: all logits -> the same top-8 in every CTA; word 8 of every lane is the gate logit
        if (warp == 0) {
            bool ok = true;
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
                    if (routed_unit) {
                        for (int b = 0; b < kGroups; ++b) mbar_arrive_expect_tx(&bar[b], group_bytes);
                        mbar_arrive_expect_tx(&bar[kGroups], kDnBytes);
                        armed = true;
                    }
                }
            }
        }
        __syncthreads();
        if (*abort_s) break;
        ds_mark(4, l);
        // every CTA has read y_{l-1} (before its logits): clear this CTA's slice of the buffer that
        // layer l + 1 adds into
        if (tid < kAccCopies * nd) p.acc[(size_t)(((l + 1) & 1) * kAccCopies + tid / nd) * D + d_lo + tid % nd] = 0ull;
        if (has_unit) {
            const int e = routed_unit ? ids_s[uj] : 0;
            if (routed_unit && my_k < kCopies) issue_copy(my_k, e);
            ds_mark(5, l);
            // the scale (even lane) or bias (odd lane) of the unit's group of down rows
            // (tid >> 1) + 256 a, requested now and used in S5 (they stream behind the copies)
            uint32_t dsb[D / 256];
            {
                const QView &W = shared_unit ? Ly.SD : Ly.Dn;
                const uint16_t *src = ((lane & 1) ? W.biases : W.scales) + (size_t)e * D * (I / 64) + uk * kSlice / 64;
#pragma unroll
                for (int a = 0; a < D / 256; ++a) dsb[a] = ld_nc_u16(src + (size_t)((tid >> 1) + 256 * a) * (I / 64));
            }

            // ---- S4: act of the unit's 32 pairs, group by group
            float4 x4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 hv = hq[i * cpd + my_c];
                x4[i] = make_float4(hv.x * kXScale, hv.y * kXScale, hv.z * kXScale, hv.w * kXScale);
            }
            const float xcv = xcs[my_c];
            // partial (gate, up) dots of chunk my_c for the group's pairs slot + slots*k; summed over
            // the warp's chunks (butterfly within the slot's lanes) into part[warp][pair][gate/up]
            auto group_partials = [&](int g) {
                constexpr int kSlots = 32 / cpw, kRounds = (kGroupPairs + kSlots - 1) / kSlots;
                float gp[kRounds], up[kRounds];
#pragma unroll
                for (int k = 0; k < kRounds; ++k) {
                    const int ql = slot + kSlots * k, q = g * kGroupPairs + ql;
                    gp[k] = up[k] = 0.f;
                    if (ql < kGroupPairs) {
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
                        if (ql < kGroupPairs) {
                            float *pp = part + (warp * kSlice + g * kGroupPairs + ql) * 2;
                            pp[0] = gp[k];
                            pp[1] = up[k];
                        }
                    }
            };
            bool ok = true;
#pragma unroll 1
            for (int g = 0; g < kGroups; ++g) {
                ok = mbar_wait(&bar[g], ph, p.err, kErrTimeout) && ok;
                if (g == 0) ds_mark(6, l);
                if (ok) group_partials(g);
            }
            ok = mbar_wait(&bar[kGroups], ph, p.err, kErrTimeout) && ok;
            ds_mark(7, l);
            if (!ok) *abort_s = 1;
            __syncthreads();
            if (*abort_s) break;
            // thread 2q + m (q < 32): pair q's 16 warp partials of gate (m = 0) or up (m = 1) in order
            if (tid < 2 * kSlice) {
                float sv = 0.f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) sv += part[(w * kSlice + (tid >> 1)) * 2 + (tid & 1)];
                const float u = __shfl_down_sync(kFull, sv, 1);
                if (!(tid & 1)) act_s[tid >> 1] = silu_ref(sv) * u;
            }
            __syncthreads();  // the unit's act values are complete
            ds_mark(8, l);

            // ---- S5: lane pair (row r, half hf): 16 columns of down row r against act, pairs summed;
            // c_slot * sum rounded to the accumulator's grid into the unit's output vector, which one
            // bulk reduction adds into y_l
            const int hf = lane & 1;
            float4 a4[4];
            float asum = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 av = reinterpret_cast<const float4 *>(act_s)[4 * hf + q];
                asum += (av.x + av.y) + (av.z + av.w);
                a4[q] = make_float4(av.x * kXScale, av.y * kXScale, av.z * kXScale, av.w * kXScale);
            }
            const float cj = coef[uj];
            unsigned long long *vec = reinterpret_cast<unsigned long long *>(sm + f.gu_off);  // gate/up consumed
            bool range = false;
#pragma unroll
            for (int a = 0; a < D / 256; ++a) {
                const int r = (tid >> 1) + 256 * a;
                float w[16];
                chunk_denormals<BITS>(sm + f.dn_off + r * kDnRowBytes + dn_delta, hf, w);
                const float sc = bf16_bits_to_f32(__shfl_sync(kFull, dsb[a], lane & ~1));
                const float bi = bf16_bits_to_f32(__shfl_sync(kFull, dsb[a], lane | 1));
                float v = fmaf(sc, chunk_dot(w, a4) * kDotScale, bi * asum);
                v += __shfl_xor_sync(kFull, v, 1);
                const float c = cj * v;
                if (!hf) {
                    long long qv = 0;
                    if (fabsf(c) < kAccLimit)
                        qv = __float2ll_rn(c * kAccScale);
                    else
                        range = true;  // also NaN
                    vec[r] = (unsigned long long)qv;
                }
            }
            fence_proxy_async_smem();  // the vector, for the copy engine
            if (range) atomicOr(p.err, kErrRange);
            ds_mark(9, l);
            armed = false;  // every copy of the layer has landed
        }
        __syncthreads();  // the regions are reused by the next layer's copies; the vector is complete
        if (tid == 0) {
            if (has_unit) {
                bulk_reduce_add_u64(p.acc + (size_t)((l & 1) * kAccCopies + cta % kAccCopies) * D, sm + f.gu_off,
                                    (uint32_t)D * 8u);
                bulk_commit();
                bulk_wait<0>();  // added at L2 (and the vector read: the next copies may overwrite it)
                fence_proxy_async_global();
            }
            red_release_gpu_add(p.ctr_y, 1u);  // after this CTA's additions and accumulator clears
        }
        ds_mark(10, l);
    }
    cp_async_wait<0>();  // an abandoned layer may still be copying its router rows
    __syncthreads();
    if (cta == 0 && !*abort_s) {
        // the output row: x = x_{L-1} + y_{L-1}
        if (tid == 0) {
            if (!wait_count(p.ctr_y, (base + (uint32_t)p.n_layers) * (uint32_t)G, p.err)) {
                atomicOr(p.err, kErrTimeout);
                *abort_s = 1;
            } else {
                ld_acquire_gpu(p.ctr_y);
                if (*reinterpret_cast<const volatile uint32_t *>(p.err) & kErrRange) *abort_s = 1;
            }
        }
        __syncthreads();
        if (!*abort_s) {
            const unsigned long long *y = p.acc + (size_t)((p.n_layers - 1) & 1) * kAccCopies * D;
#pragma unroll
            for (int a = 0; a < D / kThreads; ++a) {
                unsigned long long t = 0ull;
#pragma unroll
                for (int k = 0; k < kAccCopies; ++k) t += __ldcg(y + k * D + tid + a * kThreads);
                p.x[tid + a * kThreads] = xv[a] + acc_value(t);
            }
        }
    }
    if (tid == 0) {
        // leave no copy in flight into this CTA's shared memory
        if (*abort_s && armed)
            for (int b = 0; b <= kGroups; ++b) mbar_wait(&bar[b], ph, p.err, kErrTimeout);
        if (cta == 0) *reinterpret_cast<volatile uint32_t *>(p.gen_base) = base + (uint32_t)p.n_layers;
    }
}

}  // namespace ds
}  // namespace di
