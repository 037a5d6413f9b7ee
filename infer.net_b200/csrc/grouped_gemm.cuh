// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// D[f, n] = sum_k W[e][f, k] * B[n, k] for every work unit (expert segment tile, 128-row
// block of W). W is an affine-quantised MLX stack dequantised in shared memory; B rows are
// the tokens routed to the expert (gathered from x for gate/up, contiguous activation rows
// for down). Both operands are K-major bf16 tiles with the 128-byte swizzle; the f32
// accumulator lives in tensor memory.
//
//   MODE_GATE_UP: two accumulators (gate rows, up rows of the same 128 intermediate
//                 indices), epilogue act = silu(gate) * up -> bf16 act[p, i]
//                 (quantized.mm:148-189; prefill_moe.mm:23-53 semantics)
//   MODE_DOWN:    one accumulator, double buffered; epilogue writes the bf16 expert row
//                 to its route slot y[r, d] (r = t*8 + slot) or the shared row ys[t, d]
//                 (prefill_moe.mm:54-78 semantics)
//
// Warp roles (512 threads): 0-3 epilogue (TMEM lane quadrants), 4 MMA issue + TMEM owner,
// 5-7 B loaders (cp.async), 8-15 W dequantisers.
#pragma once
#include "common.cuh"
#include "route.cuh"

namespace di {
namespace gg {

constexpr int MODE_GATE_UP = 0, MODE_DOWN = 1;
constexpr int BM = 128, BN = 256, BK = 64;
constexpr int THREADS = 512;
constexpr int kA = BM * 128;        // bytes of one 128 x 64 bf16 A tile
constexpr int kB = BN * 128;        // bytes of one <=256 x 64 bf16 B tile

template <int MODE>
struct Cfg {
    static constexpr int NA = MODE == MODE_GATE_UP ? 2 : 1;
    static constexpr int STAGES = MODE == MODE_GATE_UP ? 3 : 4;
    static constexpr int STAGE_BYTES = NA * kA + kB;
    static constexpr int ACC_SLOTS = MODE == MODE_GATE_UP ? 1 : 2;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
};

struct Params {
    QView w1, w2;              // routed experts: gate, up (GATE_UP) or down (DOWN)
    QView s1, s2;              // shared expert:  gate, up (GATE_UP) or down (DOWN)
    const uint16_t *src;       // GATE_UP: x [T, K]; DOWN: act [P, K]
    const int32_t *perm_route; // [8T] route id of each permuted position
    const Tile *tiles;
    const int32_t *n_tiles;
    int T, K, rows, E;
    uint16_t *out;             // GATE_UP: act [P, rows]; DOWN: y [8T, rows]
    uint16_t *out_shared;      // DOWN: ys [T, rows]
    uint32_t *err;
};

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

// 16 codes of an 8-bit row chunk -> 8 packed bf16x2 words.
__device__ __forceinline__ void dequant16_8bit(uint4 q, float s, float b, uint32_t *o) {
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float v0 = fmaf(byte_to_f32(w[i], 0), s, b), v1 = fmaf(byte_to_f32(w[i], 1), s, b);
        float v2 = fmaf(byte_to_f32(w[i], 2), s, b), v3 = fmaf(byte_to_f32(w[i], 3), s, b);
        o[2 * i] = pack_bf16x2(v0, v1);
        o[2 * i + 1] = pack_bf16x2(v2, v3);
    }
}

// 32 codes of a 5-bit half group (5 words, bit 0 aligned) -> 16 packed bf16x2 words.
__device__ __forceinline__ void dequant32_5bit(const uint32_t *w, float s, float b, uint32_t *o) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float v[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int bit = 5 * (i + h), a = bit >> 5, sh = bit & 31;
            uint32_t q = (sh + 5 <= 32) ? (w[a] >> sh) : __funnelshift_r(w[a], w[a + 1], sh);
            v[h] = fmaf(code_to_f32(q & 31u), s, b);
        }
        o[i >> 1] = pack_bf16x2(v[0], v[1]);
    }
}

template <int MODE, int BITS>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm_kernel(Params p) {
    using C = Cfg<MODE>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
    uint8_t *smem = smem_raw + pad;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full = bars, *empty = bars + C::STAGES;
    uint64_t *accf = bars + 2 * C::STAGES, *acce = accf + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    auto a_tile = [&](int s, int m) { return smem + s * C::STAGE_BYTES + m * kA; };
    auto b_tile = [&](int s) { return smem + s * C::STAGE_BYTES + C::NA * kA; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int RB = (p.rows + BM - 1) / BM;
    const int nk = p.K / BK;
    const int n_units = (*p.n_tiles) * RB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 8 + 3);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&accf[a], 1);
            mbar_init(&acce[a], 4);
        }
        fence_mbarrier_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp >= 8) {
        // ---------------------------------------------------------------- W dequantisers
        const int tid = threadIdx.x - 256;
        constexpr int JOBS = MODE == MODE_GATE_UP ? (BITS == 8 ? 4 : 2) : (BITS == 8 ? 2 : 1);
        int it = 0;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const bool shared = tl.seg >= p.E;
            const int expert = shared ? 0 : tl.seg;
            for (int kb = 0; kb < nk && ok; ++kb, ++it) {
                // issue this k-block's global loads before waiting for the stage
                uint32_t qw[JOBS][BITS == 8 ? 4 : 5];
                float sc[JOBS], bi[JOBS];
                bool live[JOBS];
#pragma unroll
                for (int j = 0; j < JOBS; ++j) {
                    const int job = j * 256 + tid;
                    int mat, r, part;
                    if constexpr (BITS == 8) { mat = job >> 9; r = (job & 511) >> 2; part = job & 3; }
                    else { mat = job >> 8; r = (job & 255) >> 1; part = job & 1; }
                    const QView W = mat ? (shared ? p.s2 : p.w2) : (shared ? p.s1 : p.w1);
                    const int row = rb * BM + r;
                    live[j] = row < p.rows;
                    const size_t ridx = (size_t)expert * W.rows + min(row, p.rows - 1);
                    const uint32_t *src = W.packed + ridx * W.words_per_row();
                    if constexpr (BITS == 8) {
                        uint4 q = ldg_nc_v4(src + kb * 16 + part * 4);
                        qw[j][0] = q.x; qw[j][1] = q.y; qw[j][2] = q.z; qw[j][3] = q.w;
                    } else {
#pragma unroll
                        for (int w = 0; w < 5; ++w) qw[j][w] = ldg_nc_u32(src + kb * 10 + part * 5 + w);
                    }
                    sc[j] = bf16_bits_to_f32(__ldg(W.scales + ridx * W.groups_per_row() + kb));
                    bi[j] = bf16_bits_to_f32(__ldg(W.biases + ridx * W.groups_per_row() + kb));
                }
                const int s = it % C::STAGES;
                const uint32_t ph = (it / C::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrTimeout)) { ok = false; break; }
#pragma unroll
                for (int j = 0; j < JOBS; ++j) {
                    const int job = j * 256 + tid;
                    if constexpr (BITS == 8) {
                        const int mat = job >> 9, r = (job & 511) >> 2, part = job & 3;
                        uint32_t o[8];
                        if (live[j]) dequant16_8bit(make_uint4(qw[j][0], qw[j][1], qw[j][2], qw[j][3]), sc[j], bi[j], o);
                        else
#pragma unroll
                            for (int i = 0; i < 8; ++i) o[i] = 0;
                        uint8_t *t = a_tile(s, mat);
                        *reinterpret_cast<uint4 *>(t + sw128_offset(r, 2 * part)) = make_uint4(o[0], o[1], o[2], o[3]);
                        *reinterpret_cast<uint4 *>(t + sw128_offset(r, 2 * part + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                    } else {
                        const int mat = job >> 8, r = (job & 255) >> 1, part = job & 1;
                        uint32_t o[16];
                        if (live[j]) dequant32_5bit(qw[j], sc[j], bi[j], o);
                        else
#pragma unroll
                            for (int i = 0; i < 16; ++i) o[i] = 0;
                        uint8_t *t = a_tile(s, mat);
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            *reinterpret_cast<uint4 *>(t + sw128_offset(r, 4 * part + c)) =
                                make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
        }
    } else if (warp >= 5) {
        // ---------------------------------------------------------------- B loaders
        const int tid = threadIdx.x - 160;  // 0..95
        int it = 0, pending = -1;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n);
            for (int kb = 0; kb < nk && ok; ++kb, ++it) {
                const int s = it % C::STAGES;
                const uint32_t ph = (it / C::STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                uint8_t *bt = b_tile(s);
                for (int c = tid; c < N * 8; c += 96) {
                    const int n = c >> 3, ch = c & 7;
                    const bool valid = n < tl.n;
                    const int pos = tl.p0 + min(n, tl.n - 1);
                    size_t row;
                    if constexpr (MODE == MODE_GATE_UP) row = shared ? (size_t)(pos - 8 * p.T) : (size_t)(p.perm_route[pos] >> 3);
                    else row = (size_t)pos;
                    cp_async_16(bt + sw128_offset(n, ch), p.src + row * p.K + kb * BK + ch * 8, valid);
                }
                cp_async_commit();
                if (pending >= 0) {
                    cp_async_wait<1>();
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[pending]);
                }
                pending = s;
            }
        }
        if (pending >= 0) {
            cp_async_wait<0>();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive(&full[pending]);
        }
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issue
        if (lane == 0) {
            int it = 0, uc = 0;
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++uc) {
                const Tile tl = p.tiles[u / RB];
                const int N = round16(tl.n);
                const uint32_t idesc = idesc_bf16_f32(BM, N);
                const int slot = C::ACC_SLOTS == 2 ? (uc & 1) : 0;
                const uint32_t use = C::ACC_SLOTS == 2 ? (uc >> 1) : uc;
                if (!mbar_wait(&acce[slot], (use & 1) ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d0 = tmem + slot * 256;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, p.err, kErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(b_tile(s)));
                    const uint64_t a1 = smem_desc_sw128(smem_u32(a_tile(s, 0)));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint32_t acc = (kb | k) != 0;
                        tc_mma_bf16(d0, a1 + 2 * k, bdesc + 2 * k, idesc, acc);
                        if constexpr (MODE == MODE_GATE_UP) {
                            const uint64_t a2 = smem_desc_sw128(smem_u32(a_tile(s, 1)));
                            tc_mma_bf16(tmem + 256, a2 + 2 * k, bdesc + 2 * k, idesc, acc);
                        }
                    }
                    tc_commit(&empty[s]);
                }
                if (!ok) break;
                tc_commit(&accf[slot]);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp;  // TMEM lanes 32q .. 32q+31
        int uc = 0;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++uc) {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n);
            const int slot = C::ACC_SLOTS == 2 ? (uc & 1) : 0;
            const uint32_t use = C::ACC_SLOTS == 2 ? (uc >> 1) : uc;
            if (!mbar_wait(&accf[slot], use & 1, p.err, kErrTimeout)) { ok = false; break; }
            tc_fence_after();
            const int row = rb * BM + 32 * q + lane;
            const bool rv = row < p.rows;
            const uint32_t tl_addr = tmem + ((uint32_t)(32 * q) << 16) + slot * 256;
            for (int c = 0; c < N; c += 16) {
                float v[16];
                tmem_ld16(tl_addr + c, v);
                if constexpr (MODE == MODE_GATE_UP) {
                    float w[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + 256 + c, w);
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c + j;
                        if (rv && n < tl.n)
                            p.out[(size_t)(tl.p0 + n) * p.rows + row] = f32_to_bf16_bits(silu_ref(v[j]) * w[j]);
                    }
                } else {
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c + j;
                        if (rv && n < tl.n) {
                            const int pos = tl.p0 + n;
                            if (shared) p.out_shared[(size_t)(pos - 8 * p.T) * p.rows + row] = f32_to_bf16_bits(v[j]);
                            else p.out[(size_t)p.perm_route[pos] * p.rows + row] = f32_to_bf16_bits(v[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[slot]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace gg
}  // namespace di
