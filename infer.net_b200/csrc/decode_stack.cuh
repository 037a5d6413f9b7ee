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
//   S4  it requests its share of the 8 routed experts' gate/up and down rows;
//   S5  (gate, up) pairs of its share -> act = silu(gate . h) * (up . h) -> exchanged;
//   S6  all act values into shared memory;
//   S7  the down rows of its outputs d: x_{l+1}[d] = x_l[d] + sigmoid(g) * shared_d + sum_j p_j
//       * expert_j[d] -> exchanged (the last layer writes x instead).
//
// Exchanges use flag-in-data words: {f32 value, generation} in one 64-bit store, so a reader
// polls the data itself and no fence orders data before a flag. Generations grow monotonically
// across calls (a device counter), so stale words never match. For the two wide exchanges (x:
// D words, act: 9 I words, read by every thread of every CTA) each CTA also bumps an arrival
// counter (relaxed, no fence) once its words are stored; readers wait for the count first and
// then read the words about once, instead of 148 x 512 threads re-polling the same lines. The
// count is only a hint: the words' generations decide. A slow reader can
// never see a value overwritten by the next layer: every write of layer l+1 happens after every
// CTA finished reading the same exchange of layer l (each step depends on the previous exchange
// of all CTAs). All waits are bounded; a timeout sets kErrTimeout and every CTA leaves.
//
// Dot products: a code q becomes the exact f32 denormal q * 2^-149 (its bits), the activation is
// pre-scaled by 2^64, so sum_i w_i x_i = 2^85 * sum_i (q_i 2^-149)(x_i 2^64) and
// (q s + b) . x = s * (q . x) + b * sum(x) per 16-element chunk: one byte permute and one FMA per
// weight. The scaled operands stay normal for |x| in [2^-40, 2^64].
#pragma once
#include "decode.cuh"

namespace di {
namespace ds {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCpl = 4;  // chunks of 16 per lane in phase 2: D <= 2048
constexpr int kPairsPerWarp = 2;  // (gate, up) pairs per warp: 9 I / grid <= 32
constexpr int kMaxActWords = 9;   // act words per thread: 9 I <= 9 * kThreads (I <= 512)

struct StackLayer {
    QView R, SR, G, U, Dn, SG, SU, SD;
    const float *bias;  // router bias [E] or null
    const float *norm;  // RMSNorm weights [D]
};

struct StackParams {
    const StackLayer *layers;
    int n_layers, D, I, E;
    float eps;
    float *x;                       // residual row [D], in/out
    uint16_t *h_trace;              // [n_layers][D] or null
    int32_t *ids_trace;             // [n_layers][8] or null
    unsigned long long *ll_logit;   // [E + 1] exchange words
    unsigned long long *ll_act;     // [9 I]
    unsigned long long *ll_x;       // [D]
    uint32_t *gen_base;             // generations used by earlier calls
    uint32_t *ctr_x, *ctr_act;      // arrivals at the x and act exchanges (G per layer step)
    uint32_t *err;
};

// Shared memory of one CTA. gate/up region: gate codes [pairs][gu_row], up codes, gate scales,
// gate biases, up scales, up biases; in S6/S7 it holds act [9][4][I/16] float4 (scaled by 2^64)
// and the chunk sums [9][I/16]. down region: codes [9][outs][dn_row], scales, biases.
struct Layout {
    int pairs, outs, gu_row, gu_grp, dn_row, dn_grp;
    int gu_off, dn_off, misc_off, total;
    __host__ __device__ int gu_code(int m) const { return gu_off + m * pairs * gu_row; }
    __host__ __device__ int gu_sb(int m, int k) const { return gu_off + 2 * pairs * gu_row + (2 * m + k) * pairs * gu_grp; }
    __host__ __device__ int dn_code() const { return dn_off; }
    __host__ __device__ int dn_sb(int k) const { return dn_off + 9 * outs * dn_row + k * 9 * outs * dn_grp; }
    // misc: 2 mbarriers, ids[8], coef[9] (+pad), red[32], abort flag, own residual values [outs]
    __host__ __device__ int bar() const { return misc_off; }
    __host__ __device__ int ids() const { return misc_off + 16; }
    __host__ __device__ int coef() const { return misc_off + 48; }
    __host__ __device__ int red() const { return misc_off + 96; }
    __host__ __device__ int abort_flag() const { return misc_off + 224; }
    __host__ __device__ int xown() const { return misc_off + 240; }
};
__host__ __device__ inline Layout layout(int D, int I, int bits, int grid) {
    Layout f;
    f.pairs = (9 * I + grid - 1) / grid;
    f.outs = (D + grid - 1) / grid;
    f.gu_row = D * bits / 8;
    f.gu_grp = D / 64 * 2;
    f.dn_row = I * bits / 8;
    f.dn_grp = I / 64 * 2;
    f.gu_off = (D * 2 + 127) & ~127;  // h (bf16) first
    const int gu_bytes = 2 * f.pairs * (f.gu_row + 2 * f.gu_grp);
    const int act_bytes = 9 * I * 4 + 9 * (I / 16) * 4;
    f.dn_off = f.gu_off + (((gu_bytes > act_bytes ? gu_bytes : act_bytes) + 127) & ~127);
    f.misc_off = f.dn_off + ((9 * f.outs * (f.dn_row + 2 * f.dn_grp) + 127) & ~127);
    f.total = f.misc_off + 240 + ((f.outs * 4 + 15) & ~15);
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
constexpr float kXUnscale = 0x1p-64f;

template <int BITS>
__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(const StackParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int D = p.D, I = p.I, E = p.E, G = gridDim.x, cta = blockIdx.x;
    const Layout f = layout(D, I, BITS, G);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint16_t *xs = reinterpret_cast<uint16_t *>(sm);
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + f.bar());  // [0] gate/up rows, [1] down rows
    int32_t *ids_s = reinterpret_cast<int32_t *>(sm + f.ids());
    float *coef = reinterpret_cast<float *>(sm + f.coef());
    float *red = reinterpret_cast<float *>(sm + f.red());
    volatile int *abort_s = reinterpret_cast<volatile int *>(sm + f.abort_flag());
    float *xown = reinterpret_cast<float *>(sm + f.xown());
    float *acts = reinterpret_cast<float *>(sm + f.gu_off);  // S6/S7
    const int cpr = I / 16, cpl = D / 512;
    float *asum = acts + 9 * I;

    // this CTA's shares: (gate, up) pairs [p_lo, p_hi) of the 9*I, outputs [d_lo, d_hi), router rows [r_lo, r_hi) of E+1
    const int P = 9 * I;
    const int p_lo = (int)((long long)cta * P / G), p_hi = (int)((long long)(cta + 1) * P / G), np = p_hi - p_lo;
    const int d_lo = (int)((long long)cta * D / G), d_hi = (int)((long long)(cta + 1) * D / G), nd = d_hi - d_lo;
    const int r_lo = (int)((long long)cta * (E + 1) / G), r_hi = (int)((long long)(cta + 1) * (E + 1) / G);
    const int j_lo = p_lo / I, j_hi = (p_hi - 1) / I, nseg = np > 0 ? j_hi - j_lo + 1 : 0;
    const int ncopies = nseg * 6 + 27;
    const uint32_t pair_bytes = 2u * (f.gu_row + 2 * f.gu_grp), slot_dn_bytes = (uint32_t)nd * (f.dn_row + 2 * f.dn_grp);
    const int shared_pairs = np > 0 && j_hi == 8 ? p_hi - max(p_lo, 8 * I) : 0;
    const uint32_t gu_shared = (uint32_t)shared_pairs * pair_bytes, gu_routed = (uint32_t)(np - shared_pairs) * pair_bytes;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbarrier_init();
        *abort_s = 0;
    }
    // every CTA reads the generation base before its first exchange write; CTA 0 advances it at
    // its end, which is after the first exchange (so after every CTA has read it)
    const uint32_t base = *reinterpret_cast<const volatile uint32_t *>(p.gen_base);
    __syncthreads();

    bool armed = false;  // thread 0: this layer's barrier arrivals (with the routed bytes) are done
    uint32_t ph = 0;
    for (int l = 0; l < p.n_layers; ++l) {
        const StackLayer &Ly = p.layers[l];
        const uint32_t gen = base + (uint32_t)l + 1;
        ph = (uint32_t)l & 1u;
        // copy k of this CTA's share: k < nseg*6 a gate/up field of one expert segment, else a down
        // field of expert slot (k - nseg*6)/3; `routed` selects slots 0..7 (ids known) or slot 8
        auto issue_copy = [&](int k, bool routed) {
            if (k < nseg * 6) {
                const int sg_ = k / 6, field = k % 6, j = j_lo + sg_;
                if ((j < 8) != routed) return;
                const int i0 = j == j_lo ? p_lo % I : 0, i1 = j == j_hi ? (p_hi - 1) % I + 1 : I;
                const int q0 = j * I + i0 - p_lo, cnt = i1 - i0;
                const int e = j < 8 ? ids_s[j] : 0;
                const int m = field & 1, kind = field >> 1;
                const QView &W = m ? (j < 8 ? Ly.U : Ly.SU) : (j < 8 ? Ly.G : Ly.SG);
                const size_t row = (size_t)e * I + i0;
                if (kind == 0)
                    bulk_load(sm + f.gu_code(m) + q0 * f.gu_row,
                              reinterpret_cast<const uint8_t *>(W.packed) + row * f.gu_row, (uint32_t)cnt * f.gu_row,
                              &bar[0]);
                else
                    bulk_load(sm + f.gu_sb(m, kind - 1) + q0 * f.gu_grp,
                              (kind == 1 ? W.scales : W.biases) + row * (f.gu_grp / 2), (uint32_t)cnt * f.gu_grp,
                              &bar[0]);
            } else {
                const int kk = k - nseg * 6, j = kk / 3, kind = kk % 3;
                if ((j < 8) != routed || nd == 0) return;
                const int e = j < 8 ? ids_s[j] : 0;
                const QView &W = j < 8 ? Ly.Dn : Ly.SD;
                const size_t row = (size_t)e * D + d_lo;
                if (kind == 0)
                    bulk_load(sm + f.dn_code() + j * f.outs * f.dn_row,
                              reinterpret_cast<const uint8_t *>(W.packed) + row * f.dn_row, (uint32_t)nd * f.dn_row,
                              &bar[1]);
                else
                    bulk_load(sm + f.dn_sb(kind - 1) + j * f.outs * f.dn_grp,
                              (kind == 1 ? W.scales : W.biases) + row * (f.dn_grp / 2), (uint32_t)nd * f.dn_grp,
                              &bar[1]);
            }
        };
        // ---- S0: the shared expert's rows and the router rows (token independent). The bytes of
        // the shared copies are expected now, the routed ones with the arrival in S3.
        fence_proxy_async_smem();  // this layer's copies overwrite what the last one read and wrote
        if (tid == 0) {
            armed = false;
            mbar_expect_tx(&bar[0], gu_shared);
            mbar_expect_tx(&bar[1], slot_dn_bytes);
        }
        __syncthreads();
        // copy k by lane k / kWarps of warp k % kWarps: few serial issues per warp
        if (lane * kWarps + warp < ncopies) issue_copy(lane * kWarps + warp, false);
        RouterRaw rr;
        const int my_row = r_lo + warp;
        if (my_row < r_hi) router_raw_load(my_row < E ? Ly.R : Ly.SR, my_row < E ? my_row : 0, D, rr);
        const float row_bias = my_row < E && Ly.bias ? Ly.bias[my_row] : 0.f;
        float nw[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) nw[a] = tid + a * kThreads < D ? Ly.norm[tid + a * kThreads] : 0.f;

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
            const int d = tid + a * kThreads;
            if (d < D) {
                const uint16_t h = f32_to_bf16_bits(xv[a] * scale * nw[a]);
                xs[d] = h;
                if (cta == 0 && p.h_trace) p.h_trace[(size_t)l * D + d] = h;
                if (d >= d_lo && d < d_hi) xown[d - d_lo] = xv[a];
            }
        }
        __syncthreads();

        // ---- S2: router logits of this CTA's rows (row E: the shared expert's gate logit)
        if (my_row < r_hi) {
            float v = router_raw_dot(rr, xs, D);
            if (my_row < E) v = v + row_bias;
            if (lane == 0) ll_store(p.ll_logit + my_row, v, gen);
        }

        // ---- S3: all logits -> the same top-8 in every CTA; word 8 of every lane is the gate logit
        if (warp == 0) {
            float v[9];
            int idx[9];
            strided_idx(idx, lane, 32, E);
            idx[8] = E;
            ok = ll_gather<9>(p.ll_logit, idx, gen, v, p.err);
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
                    mbar_arrive_expect_tx(&bar[0], gu_routed);
                    mbar_arrive_expect_tx(&bar[1], 8u * slot_dn_bytes);
                    armed = true;
                }
            }
        }
        __syncthreads();
        if (*abort_s) break;

        // ---- S4: the routed experts' rows
        if (lane * kWarps + warp < ncopies) issue_copy(lane * kWarps + warp, true);

        // ---- S5: (gate, up) pairs -> act; warp w takes pairs w, w + 16, ... (at most kPairsPerWarp),
        // chunk by chunk so that only one chunk of h is held in registers
        ok = mbar_wait(&bar[0], ph, p.err, kErrTimeout);
        if (ok) {
            float ga[kPairsPerWarp], ua[kPairsPerWarp];
#pragma unroll
            for (int t = 0; t < kPairsPerWarp; ++t) ga[t] = ua[t] = 0.f;
#pragma unroll 1
            for (int m = 0; m < kMaxCpl; ++m) {
                if (m < cpl) {
                    const int c = lane + 32 * m;
                    float xr[16], xc = 0.f;
                    load_x16_bf16(xs, c, xr);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        xc += xr[i];
                        xr[i] *= kXScale;
                    }
#pragma unroll
                    for (int t = 0; t < kPairsPerWarp; ++t) {
                        const int q = warp + kWarps * t;
                        if (q < np) {
                            float wg[16], wu[16];
                            chunk_denormals<BITS>(sm + f.gu_code(0) + q * f.gu_row, c, wg);
                            chunk_denormals<BITS>(sm + f.gu_code(1) + q * f.gu_row, c, wu);
                            float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll
                            for (int e = 0; e < 16; e += 2) {
                                g0 = fmaf(wg[e], xr[e], g0);
                                g1 = fmaf(wg[e + 1], xr[e + 1], g1);
                                u0 = fmaf(wu[e], xr[e], u0);
                                u1 = fmaf(wu[e + 1], xr[e + 1], u1);
                            }
                            const int so = q * f.gu_grp + (c >> 2) * 2;  // byte offset of this chunk's group
                            const float gs = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 0) + so));
                            const float gb = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(0, 1) + so));
                            const float us = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 0) + so));
                            const float ub = bf16_bits_to_f32(*reinterpret_cast<const uint16_t *>(sm + f.gu_sb(1, 1) + so));
                            ga[t] = fmaf(gs, (g0 + g1) * kDotScale, fmaf(gb, xc, ga[t]));
                            ua[t] = fmaf(us, (u0 + u1) * kDotScale, fmaf(ub, xc, ua[t]));
                        }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kPairsPerWarp; ++t) {
                const int q = warp + kWarps * t;
                if (q < np) {
                    const float gsum = warp_sum_butterfly(ga[t]), usum = warp_sum_butterfly(ua[t]);
                    const int pp = p_lo + q, j = pp / I, i = pp - j * I;
                    if (lane == 0) ll_store(p.ll_act + (size_t)j * I + i, silu_ref(gsum) * usum, gen);
                }
            }
        }
        if (!ok) *abort_s = 1;
        __syncthreads();  // the gate/up region is free from here on
        if (*abort_s) break;
        if (tid == 0) {
            atomicAdd(p.ctr_act, 1u);
            if (!wait_count(p.ctr_act, gen * (uint32_t)G, p.err)) {
                atomicOr(p.err, kErrTimeout);
                *abort_s = 1;
            }
        }
        __syncthreads();
        if (*abort_s) break;

        // ---- S6: all act values -> shared memory, float4 q of chunk c of expert j at [j][q][c]
        {
            float av[kMaxActWords];
            int idx[kMaxActWords];
            strided_idx(idx, tid, kThreads, 9 * I);
            ok = ll_gather<kMaxActWords>(p.ll_act, idx, gen, av, p.err);
            if (ok) {
#pragma unroll
                for (int a = 0; a < kMaxActWords; ++a) {
                    const int e = tid + a * kThreads;
                    if (e < 9 * I) {
                        const int j = e / I, i = e - j * I, c = i >> 4, q = (i >> 2) & 3, r = i & 3;
                        acts[((size_t)(j * 4 + q) * cpr + c) * 4 + r] = av[a] * kXScale;
                    }
                }
            } else {
                atomicOr(p.err, kErrTimeout);
                *abort_s = 1;
            }
        }
        __syncthreads();
        if (*abort_s) break;
        for (int k = tid; k < 9 * cpr; k += kThreads) {
            const int j = k / cpr, c = k - j * cpr;
            const float4 *ap = reinterpret_cast<const float4 *>(acts) + (size_t)j * 4 * cpr + c;
            float s = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 a = ap[q * cpr];
                s += (a.x + a.y) + (a.z + a.w);
            }
            asum[k] = s * kXUnscale;
        }
        ok = mbar_wait(&bar[1], ph, p.err, kErrTimeout);
        if (!ok) *abort_s = 1;
        __syncthreads();
        if (*abort_s) break;

        // ---- S7: this CTA's outputs; lane tasks (expert slot j, chunk c) over the 9 down rows
        const bool last = l + 1 == p.n_layers;
        for (int o = warp; o < nd; o += kWarps) {
            float a = 0.f;
            for (int k = lane; k < 9 * cpr; k += 32) {
                const int j = k / cpr, c = k - j * cpr, r = j * f.outs + o;
                float w[16];
                chunk_denormals<BITS>(sm + f.dn_code() + r * f.dn_row, c, w);
                const float4 *ap = reinterpret_cast<const float4 *>(acts) + (size_t)j * 4 * cpr + c;
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 av = ap[q * cpr];
                    s0 = fmaf(w[4 * q], av.x, s0);
                    s1 = fmaf(w[4 * q + 1], av.y, s1);
                    s0 = fmaf(w[4 * q + 2], av.z, s0);
                    s1 = fmaf(w[4 * q + 3], av.w, s1);
                }
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(sm + f.dn_sb(0) + r * f.dn_grp);
                const uint16_t *bi = reinterpret_cast<const uint16_t *>(sm + f.dn_sb(1) + r * f.dn_grp);
                const float dot = fmaf(bf16_bits_to_f32(sc[c >> 2]), (s0 + s1) * kDotScale,
                                       bf16_bits_to_f32(bi[c >> 2]) * asum[k]);
                a = fmaf(coef[j], dot, a);
            }
            a = warp_sum_butterfly(a);
            if (lane == 0) {
                const int d = d_lo + o;
                const float xn = xown[o] + a;
                if (last)
                    p.x[d] = xn;
                else
                    ll_store(p.ll_x + d, xn, gen);
            }
        }
        __syncthreads();  // the regions are reused by the next layer's copies
        if (tid == 0) atomicAdd(p.ctr_x, 1u);
    }
    if (tid == 0) {
        if (*abort_s) {
            // leave no copy in flight into this CTA's shared memory: complete the barriers' phases
            // (arriving without the routed bytes if they were never requested) and wait for them
            if (!armed) {
                mbar_arrive_expect_tx(&bar[0], 0);
                mbar_arrive_expect_tx(&bar[1], 0);
            }
            mbar_wait(&bar[0], ph, p.err, kErrTimeout);
            mbar_wait(&bar[1], ph, p.err, kErrTimeout);
        }
        if (cta == 0) *reinterpret_cast<volatile uint32_t *>(p.gen_base) = base + (uint32_t)p.n_layers;
    }
}

}  // namespace ds
}  // namespace di
