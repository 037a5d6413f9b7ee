// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// D[m, n] = sum_k A[m, k] * B[n, k] for every work unit (a token tile of one expert segment
// x a block of weight rows). A is dequantised in shared memory from the affine-quantised MLX
// codes; B rows are the tokens routed to the expert (gathered from x for gate/up, contiguous
// activation rows for down). Both operands are K-major bf16 tiles with the 128-byte swizzle;
// the f32 accumulators live in tensor memory.
//
//   MODE_GATE_UP: the 128 A rows of a unit interleave 16 gate rows and the 16 up rows of the
//                 same intermediate indices in every 32-lane TMEM quadrant, so the SwiGLU
//                 epilogue pairs them with one warp shuffle; a unit covers 64 intermediate
//                 indices and up to 256 tokens. act = silu(gate) * up -> bf16 act[p, i]
//                 (quantized.mm:148-189; prefill_moe.mm:23-53 semantics)
//   MODE_DOWN:    128 rows of the down matrix; the epilogue writes the bf16 expert rows in
//                 expert order, yp[position, d] (the combine finds route r's row through the
//                 inverse permutation), as 16-token x 32-dim tensor stores
//                 (prefill_moe.mm:54-78 semantics)
//
// Data movement is asynchronous and issued by two producer warps: per pipeline stage (64
// K-columns, one quantisation group) a tensor copy of the stage's code bytes (into a code ring
// of its own, released as soon as the dequantisers hold the codes in registers, so code
// fetches run ahead of the MMA) and of its B rows, which
// are contiguous for every unit (gate/up reads the token rows already permuted into expert
// order, down the activation rows), as at most five boxes of 16 << i rows issued by as many
// lanes at once; per unit one bulk copy each of the scales and biases of the unit's rows.
// (Row gathers at 64-byte granularity -- cp.async or tile::gather4 -- run at a fraction of the
// L2 bandwidth that large tiled boxes reach, and gate/up re-reads its B rows once per block
// of 64 intermediates.) The dequantiser warps only read shared memory, convert and write the
// swizzled bf16 A tile.
//
// Warp roles (512 threads): 0-3 epilogue (one TMEM lane quadrant each), 4 MMA issue + TMEM
// owner, 5 code and scale producer, 6 B producer, 7 idle, 8-15 A dequantisers in two groups
// of 4 warps that take alternate pipeline stages.
//
// Stage size: every stage costs a fixed round trip (MMA commit -> producer -> tensor copy ->
// dequantiser -> MMA issue, several hundred cycles on B200) and fixed issue work, so stages
// carry 64 K-columns (four K=16 MMAs per commit) rather than 32.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "route.cuh"

namespace di {
namespace gg {

constexpr int MODE_GATE_UP = 0, MODE_DOWN = 1;
constexpr int BM = 128;          // A rows per unit (one MMA M)
constexpr int BN = 256;          // max tokens per unit (one 256-column accumulator slot)
constexpr int BK = 64;           // K per pipeline stage: 128-byte bf16 rows, one group of 64 codes
// Pipeline depths. The two dequantiser groups take alternate stages, so a code slot must belong
// to one group: an odd number of code slots would let a group's parity wait on a slot match the
// fill before the one it waits for, while the other group's fill is still in flight. Four code
// slots and three A/B stages fit 227 KB (four A/B stages would leave room for two code slots
// only, measured slower).
template <int MODE>
__host__ __device__ constexpr int stages() { return 3; }
template <int MODE>
__host__ __device__ constexpr int cstages() { return 4; }
static_assert(cstages<0>() % 2 == 0 && cstages<1>() % 2 == 0, "each code slot belongs to one dequantiser group");
constexpr int THREADS = 512;
constexpr int kA = BM * 128;     // bytes of one A stage tile (bf16)
constexpr int kB = BN * 128;     // bytes of one B stage tile (bf16)
constexpr int kCode = BM * 64;   // bytes of one stage's code window (64 bytes per A row)
constexpr int STAGE_BYTES = kA + kB;
constexpr int CSTAGES = 4;       // code ring slots of the pair kernel
constexpr int kScaleBuf = 16384; // pair kernel: scales + biases of one unit's rows (<= 32 groups per row)
constexpr int kStageOut = 4 * 2 * 16 * 64;  // epilogue staging: 4 warps x 2 buffers x 16 tokens x 64 bytes
constexpr int kBoxes = 5;               // down B boxes of 16 << i rows, i < kBoxes
template <int MODE>
__host__ __device__ constexpr int smem_bytes() {
    return 1024 + stages<MODE>() * STAGE_BYTES + cstages<MODE>() * kCode + kStageOut + 512;
}
static_assert(smem_bytes<0>() <= 227 * 1024 && smem_bytes<1>() <= 227 * 1024, "grouped GEMM shared memory");
constexpr uint32_t TMEM_COLS = 512;

template <int MODE>
__host__ __device__ constexpr int rows_per_unit() { return MODE == MODE_GATE_UP ? 64 : 128; }

// Tensor maps: index = matrix (0 gate / down, 1 up) + 2 * shared-expert.
struct Params {
    CUtensorMap code[4];       // uint8 [experts*rows, row bytes], box 64 bytes x rows_per_unit, 64B swizzle
    CUtensorMap bmap[kBoxes];  // B rows by position: GATE_UP xp [8T, K], DOWN act [P, K]; box 64 x (16 << i), 128B swizzle
    CUtensorMap smap[kBoxes];  // GATE_UP shared-expert B rows: x [rows, K]; same boxes
    CUtensorMap ymap;          // DOWN output yp [P, rows] bf16, box 32 x 16, no swizzle
    QView w[4];                // the same matrices: scales / biases (bulk copies), geometry
    const int32_t *perm_route; // [8T] route id of each permuted position
    const Tile *tiles;
    const int32_t *n_tiles;
    int shared_pos0;           // first permuted position of the shared-expert segment
    int shared_src0;           // GATE_UP: source row of that first shared position
    int K, rows, E;            // rows: I (GATE_UP) or D (DOWN); segments >= E are the shared expert
    uint16_t *out;             // GATE_UP: act [P, rows]; DOWN: yp [P, rows] (written through ymap)
    uint32_t *err;
};

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

// Byte offset of 16-byte chunk c (0..3) of row r in a 64B-swizzled K-major tile
// (address bits [7,9) XOR-ed into bits [4,6)).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t r, uint32_t c) {
    return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Two codes (integer-valued f32 magics 2^23 + q) -> bf16x2 of q*s + b.
__device__ __forceinline__ uint32_t dq_pair(uint32_t m0, uint32_t m1, float2 s2, float2 b2) {
    const float2 magic = make_float2(-8388608.0f, -8388608.0f);
    float2 q = fadd2(make_float2(__uint_as_float(m0), __uint_as_float(m1)), magic);
    float2 w = ffma2(q, s2, b2);
    return pack_bf16x2(w.x, w.y);
}

// 16 codes of an 8-bit chunk -> 8 packed bf16x2 words.
__device__ __forceinline__ void dequant16_8bit(uint4 q, float s, float b, uint32_t *o) {
    const float2 s2 = make_float2(s, s), b2 = make_float2(b, b);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o[2 * i] = dq_pair(__byte_perm(w[i], 0x4B000000u, 0x7540u), __byte_perm(w[i], 0x4B000000u, 0x7541u), s2, b2);
        o[2 * i + 1] =
            dq_pair(__byte_perm(w[i], 0x4B000000u, 0x7542u), __byte_perm(w[i], 0x4B000000u, 0x7543u), s2, b2);
    }
}

// 32 codes of a 5-bit half group (5 words, bit 0 aligned) -> 16 packed bf16x2 words.
__device__ __forceinline__ void dequant32_5bit(const uint32_t *w, float s, float b, uint32_t *o) {
    const float2 s2 = make_float2(s, s), b2 = make_float2(b, b);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        uint32_t m[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int bit = 5 * (i + h), a = bit >> 5, sh = bit & 31;
            const uint32_t q = (sh + 5 <= 32) ? (w[a] >> sh) : __funnelshift_r(w[a], w[a + 1], sh);
            m[h] = 0x4B000000u | (q & 31u);
        }
        o[i >> 1] = dq_pair(m[0], m[1], s2, b2);
    }
}

// A-tile row m of a unit -> (matrix, row within the unit's block of that matrix). GATE_UP: in
// quadrant q = m/32, lanes 0-15 are gate rows and lanes 16-31 the up rows of intermediates
// rb*64 + 16q + (m & 15).
template <int MODE>
__device__ __forceinline__ void a_row(int m, int &mat, int &r) {
    if constexpr (MODE == MODE_GATE_UP) {
        mat = (m >> 4) & 1;
        r = (m >> 5) * 16 + (m & 15);
    } else {
        mat = 0;
        r = m;
    }
}

// Byte offset of the stage's code window for K-block kb: 8-bit rows hold 64 code bytes per
// block (aligned); 5-bit blocks are 40 bytes, fetched as the 16-byte-aligned 64-byte window
// that contains them (the tensor copy's x coordinate must be 16-byte aligned).
template <int BITS>
__device__ __forceinline__ int code_x(int kb) { return BITS == 8 ? kb * 64 : ((kb * 40) & ~15); }

// Per-role cycle counters, compiled in only with -DDI_GG_TIMING (a profiling build; read by
// di_debug_gg_timing): for each kernel kind (0 gate_up, 1 down, 3 the router's approximate
// logits) and CTA, the SM cycles lane 0 of one warp of each role spends in each barrier wait and
// in its whole loop.
enum GgTimer : int {
    T_KERNEL = 0,
    T_DQ_CODES, T_DQ_EMPTY, T_DQ_SCALES, T_DQ_LOOP,  // dequantiser warp 8
    T_CP_EMPTY, T_CP_SCALE_EMPTY, T_CP_LOOP,         // code + scale producer
    T_BP_EMPTY, T_BP_LOOP,                           // B producer
    T_MMA_B, T_MMA_A, T_MMA_ACC, T_MMA_LOOP,         // MMA issue
    T_EPI_WAIT, T_EPI_LOOP,                          // epilogue warp 0
    T_MMA_ISSUE, T_MMA_COMMIT,                       // MMA issue: the MMA instructions, the stage commit
    T_COUNT = 18
};
#ifdef DI_GG_TIMING
__device__ unsigned long long g_gg_timing[4][256][T_COUNT];
__device__ __forceinline__ void gg_time(int kind, int slot, long long t0) {
    if (lane_id() == 0 && blockIdx.x < 256)
        atomicAdd(&g_gg_timing[kind][blockIdx.x][slot], (unsigned long long)(clock64() - t0));
}
__device__ __forceinline__ long long gg_now() { return clock64(); }
#else
__device__ __forceinline__ void gg_time(int, int, long long) {}
__device__ __forceinline__ long long gg_now() { return 0; }
#endif

// Accumulator slots alternate between units; every role derives the same assignment.
struct SlotPlan {
    int next = 0;
    uint32_t uses[2] = {0, 0};
    // returns the slot; phase = completed fills of that slot before this unit
    __device__ __forceinline__ int take(uint32_t &phase) {
        const int s = next;
        next ^= 1;
        phase = uses[s]++;
        return s;
    }
};

template <int MODE, int BITS>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm_kernel(const __grid_constant__ Params p) {
    constexpr int STAGES = stages<MODE>(), CSTAGES = cstages<MODE>();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
    uint8_t *smem = smem_raw + pad;
    uint8_t *code_ring = smem + STAGES * STAGE_BYTES;
    uint8_t *stage_out = code_ring + CSTAGES * kCode;
    uint64_t *bars = reinterpret_cast<uint64_t *>(stage_out + kStageOut);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *cfull = bars + 2 * STAGES, *cempty = cfull + CSTAGES;
    uint64_t *accf = cempty + CSTAGES, *acce = accf + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    auto a_tile = [&](int s) { return smem + s * STAGE_BYTES; };
    auto b_tile = [&](int s) { return smem + s * STAGE_BYTES + kA; };
    auto c_tile = [&](int cs) { return code_ring + cs * kCode; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RPU = rows_per_unit<MODE>();
    constexpr int NMAT = MODE == MODE_GATE_UP ? 2 : 1;
    const int RB = (p.rows + RPU - 1) / RPU;
    const int nk = p.K / BK;  // K is a multiple of 64
    const int gpr = p.K / 64;
    const int tkind = MODE + (p.E == 1 ? 2 : 0);  // timing build: gate_up, down, router logits
    const long long t_kernel = gg_now();
    pdl_trigger();  // the set-up below (barriers, TMEM, tensor maps) touches no global memory

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 5);   // the dequantiser warps of the stage's group + B producer arrive (+ B bytes)
            mbar_init(&empty[s], 1);  // MMA commit
        }
        for (int c = 0; c < CSTAGES; ++c) {
            mbar_init(&cfull[c], 1);   // code producer arrive + code bytes
            mbar_init(&cempty[c], 4);  // the dequantiser warps holding the codes in registers
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&accf[a], 1);
            mbar_init(&acce[a], 4);
        }
        fence_mbarrier_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 6 && lane == 0) {
        for (int i = 0; i < kBoxes; ++i) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.bmap[i]) : "memory");
            if constexpr (MODE == MODE_GATE_UP) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.smap[i]) : "memory");
        }
    }
    if (warp == 5 && lane == 0)
        for (int i = 0; i < 4; ++i) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.code[i]) : "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    pdl_wait();  // the predecessor's tile list, rows and counts
    const int n_units = (*p.n_tiles) * RB;

    // Flat pipeline index `it` = ul * nk + kb over this CTA's units ul (unit u = blockIdx.x +
    // ul * gridDim.x) and K-blocks kb. Stage s = it % STAGES, phase (it / STAGES) & 1.
    if (warp >= 8) {
        // ---------------------------------------------------------------- A dequantisers
        // group g takes the stages of the flat index with it % 2 == g (each stage is one
        // quantisation group); thread m of the group converts A row m. Its row's scales and biases
        // come from global memory in windows of 8 groups (16 bytes each), one window ahead of use:
        // the next unit's first window is requested during the current unit's last.
        const int g = (warp - 8) >> 2, m = threadIdx.x - 256 - 128 * g;  // 0..127
        const bool timed = warp == 8;
        const long long t_loop = gg_now();
        int mat, r;
        a_row<MODE>(m, mat, r);
        const bool vec_scales = (gpr & 7) == 0;  // rows of scales are 16-byte aligned
        // this thread's scale and bias rows in unit u's matrix (live: the row lies inside it)
        struct RowRef {
            const uint16_t *s, *b;
            bool live;
        };
        struct Win {
            uint4 s, b;
        };
        auto row_of = [&](int u) -> RowRef {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const bool shared = tl.seg >= p.E;
            const QView &W = p.w[mat + 2 * shared];
            if (rb * RPU + r >= p.rows) return RowRef{nullptr, nullptr, false};
            const size_t row = (size_t)(shared ? 0 : tl.seg) * W.rows + rb * RPU + r;
            return RowRef{W.scales + row * gpr, W.biases + row * gpr, true};
        };
        auto load_win = [&](const RowRef &rr, int w) -> Win {
            Win v{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
            if (!rr.live) return v;
            if (vec_scales) {
                v.s = __ldg(reinterpret_cast<const uint4 *>(rr.s) + w);
                v.b = __ldg(reinterpret_cast<const uint4 *>(rr.b) + w);
            } else {
                auto pair = [&](const uint16_t *q, int g0) {
                    return (g0 < gpr ? (uint32_t)__ldg(q + g0) : 0u) | (g0 + 1 < gpr ? (uint32_t)__ldg(q + g0 + 1) << 16 : 0u);
                };
                v.s = make_uint4(pair(rr.s, 8 * w), pair(rr.s, 8 * w + 2), pair(rr.s, 8 * w + 4), pair(rr.s, 8 * w + 6));
                v.b = make_uint4(pair(rr.b, 8 * w), pair(rr.b, 8 * w + 2), pair(rr.b, 8 * w + 4), pair(rr.b, 8 * w + 6));
            }
            return v;
        };
        RowRef cur = blockIdx.x < n_units ? row_of(blockIdx.x) : RowRef{nullptr, nullptr, false};
        Win pf = load_win(cur, 0);  // the prefetched window
        int it0 = 0;  // flat index of the unit's first stage
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, it0 += nk) {
            const int un = u + gridDim.x;  // this CTA's next unit
            const bool live = cur.live;
            RowRef nxt{nullptr, nullptr, false};
            bool nready = false;
            Win w{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
            int win = -1;
            for (int kb = (g - it0) & 1; kb < nk; kb += 2) {
                if ((kb >> 3) != win) {
                    win = kb >> 3;
                    w = pf;
                    if (8 * (win + 1) < gpr) {
                        pf = load_win(cur, win + 1);
                    } else if (un < n_units) {
                        nxt = row_of(un);
                        pf = load_win(nxt, 0);
                        nready = true;
                    }
                }
                const int e = kb & 7;
                const uint32_t sw = e < 2 ? w.s.x : e < 4 ? w.s.y : e < 6 ? w.s.z : w.s.w;
                const uint32_t bw = e < 2 ? w.b.x : e < 4 ? w.b.y : e < 6 ? w.b.z : w.b.w;
                const float sc = (e & 1) ? bf16_hi(sw) : bf16_lo(sw);
                const float bi = (e & 1) ? bf16_hi(bw) : bf16_lo(bw);
                const int it = it0 + kb, s = it % STAGES, cs = it % CSTAGES;
                const long long t_c = gg_now();
                if (!mbar_wait(&cfull[cs], (it / CSTAGES) & 1, p.err, kErrTimeout)) { ok = false; break; }
                if (timed) gg_time(tkind, T_DQ_CODES, t_c);
                const uint8_t *crow = c_tile(cs) + mat * (RPU * 64);
                uint4 cw[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) cw[c] = *reinterpret_cast<const uint4 *>(crow + sw64_offset(r, c));
                __syncwarp();
                if (lane == 0) mbar_arrive(&cempty[cs]);  // the code slot may be refilled
                uint32_t o[32];
                if constexpr (BITS == 8) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) dequant16_8bit(cw[c], sc, bi, o + 8 * c);
                } else {
                    const uint32_t w16[16] = {cw[0].x, cw[0].y, cw[0].z, cw[0].w, cw[1].x, cw[1].y, cw[1].z, cw[1].w,
                                              cw[2].x, cw[2].y, cw[2].z, cw[2].w, cw[3].x, cw[3].y, cw[3].z, cw[3].w};
                    const bool odd = ((kb * 40) & 15) != 0;  // the block starts 8 bytes into the window
                    uint32_t w10[10];
#pragma unroll
                    for (int i = 0; i < 10; ++i) w10[i] = odd ? w16[i + 2] : w16[i];
                    dequant32_5bit(w10, sc, bi, o);
                    dequant32_5bit(w10 + 5, sc, bi, o + 16);
                }
                if (!live)
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = 0;
                // the A tile is free once the MMA of the stage's previous use has completed
                const long long t_e = gg_now();
                if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                if (timed) gg_time(tkind, T_DQ_EMPTY, t_e);
                uint8_t *t = a_tile(s);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4 *>(t + sw128_offset(m, c)) =
                        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
            if (!ok) break;
            if (!nready && un < n_units) {  // a unit with no stage of this group's parity
                nxt = row_of(un);
                pf = load_win(nxt, 0);
            }
            cur = nxt;
        }
        if (timed) gg_time(tkind, T_DQ_LOOP, t_loop);
    } else if (warp == 5) {
        // ---------------------------------------------------------------- code and scale producer
        int it = 0;
        const long long t_loop = gg_now();
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const bool shared = tl.seg >= p.E;
            const int expert = shared ? 0 : tl.seg;
            const int row0 = expert * p.w[(lane & 1) + 2 * shared].rows + rb * RPU;
            for (int kb = 0; kb < nk; ++kb, ++it) {
                const int cs = it % CSTAGES;
                if (lane == 0) {
                    const long long t_c = gg_now();
                    ok = mbar_wait(&cempty[cs], ((it / CSTAGES) & 1) ^ 1, p.err, kErrTimeout);
                    gg_time(tkind, T_CP_EMPTY, t_c);
                    if (ok) mbar_arrive_expect_tx(&cfull[cs], kCode);
                }
                ok = __shfl_sync(kFull, ok, 0);
                if (!ok) break;
                if (lane < NMAT)
                    tma_load_2d(c_tile(cs) + lane * (RPU * 64), &p.code[lane + 2 * shared], code_x<BITS>(kb), row0,
                                &cfull[cs]);
            }
        }
        gg_time(tkind, T_CP_LOOP, t_loop);
        if (!ok && lane == 0) {
            // copies still in flight must land before the CTA's shared memory is released
            for (int k = max(0, it - CSTAGES); k < it; ++k)
                mbar_wait(&cfull[k % CSTAGES], (k / CSTAGES) & 1, p.err, kErrTimeout);
        }
    } else if (warp == 6) {
        // ---------------------------------------------------------------- B producer
        int it = 0;
        const long long t_loop = gg_now();
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n);
            // lane i < kBoxes copies 16 << i rows when bit i of N/16 is set, larger boxes first
            const int nb16 = N >> 4;
            const bool box_mine = lane < kBoxes && ((nb16 >> lane) & 1);
            const int box_off = box_mine ? 16 * ((nb16 >> (lane + 1)) << (lane + 1)) : 0;
            const bool shared_src = MODE == MODE_GATE_UP && shared;
            const int row0 = (shared_src ? p.shared_src0 + (tl.p0 - p.shared_pos0) : tl.p0) + box_off;
            const CUtensorMap *bm = shared_src ? &p.smap[box_mine ? lane : 0] : &p.bmap[box_mine ? lane : 0];
            for (int kb = 0; kb < nk; ++kb, ++it) {
                const int s = it % STAGES;
                if (lane == 0) {
                    const long long t_e = gg_now();
                    ok = mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, p.err, kErrTimeout);
                    gg_time(tkind, T_BP_EMPTY, t_e);
                    if (ok) mbar_arrive_expect_tx(&full[s], (uint32_t)N * 128u);
                }
                ok = __shfl_sync(kFull, ok, 0);
                if (!ok) break;
                if (box_mine) tma_load_2d(b_tile(s) + box_off * 128, bm, kb * BK, row0, &full[s]);
            }
        }
        gg_time(tkind, T_BP_LOOP, t_loop);
        if (!ok && lane == 0)
            for (int k = max(0, it - STAGES); k < it; ++k)
                mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.err, kErrTimeout);
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issue
        // A shared-memory access by this thread (an mbarrier wait included) waits until the MMAs
        // it issued before have read their operands, so each stage's wait costs the pipe that
        // latency. With three stages, waiting for two stages at a time measured slower (the
        // producers lose a stage of lead), so the loop waits stage by stage (WG = 1).
        if (lane == 0) {
            int it = 0, ul = 0;
            const long long t_loop = gg_now();
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ul) {
                const Tile tl = p.tiles[u / RB];
                const int N = round16(tl.n);
                const int slot = ul & 1;  // accumulator slots alternate between units
                const uint32_t phase = (uint32_t)(ul >> 1);
                const long long t_a = gg_now();
                if (!mbar_wait(&acce[slot], (phase & 1) ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                gg_time(tkind, T_MMA_ACC, t_a);
                tc_fence_after();
                const uint32_t d = tmem + slot * 256;
                const uint32_t id = idesc_bf16_f32(BM, N);
                constexpr int WG = 1;  // stages per wait
                for (int kb = 0; kb < nk; kb += WG) {
                    const int n2 = WG == 2 && kb + 1 < nk ? 2 : 1;
                    const long long t_f = gg_now();
                    for (int j = 0; j < n2 && ok; ++j)
                        ok = mbar_wait(&full[(it + j) % STAGES], ((it + j) / STAGES) & 1, p.err, kErrTimeout);
                    if (!ok) break;
                    gg_time(tkind, T_MMA_A, t_f);
                    tc_fence_after();
                    const long long t_i = gg_now();
                    for (int j = 0; j < n2; ++j, ++it) {
                        const int s = it % STAGES;
                        const uint64_t adesc = smem_desc_sw128(smem_u32(a_tile(s)));
                        const uint64_t bdesc = smem_desc_sw128(smem_u32(b_tile(s)));
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            tc_mma_bf16(d, adesc + 2 * k, bdesc + 2 * k, id, (kb + j) > 0 || k > 0);
                        tc_commit(&empty[s]);
                    }
                    gg_time(tkind, T_MMA_ISSUE, t_i);
                }
                if (!ok) break;
                tc_commit(&accf[slot]);
            }
            gg_time(tkind, T_MMA_LOOP, t_loop);
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---------------------------------------------------------------- epilogue
        const int q = warp;  // TMEM lanes 32q .. 32q+31
        uint8_t *so = stage_out + q * 2 * 16 * 64;
        int chunk_no = 0;  // DOWN: staging buffer of a chunk = chunk_no & 1
        SlotPlan plan;
        const long long t_loop = gg_now();
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const int N = round16(tl.n);
            uint32_t phase;
            const int slot = plan.take(phase);
            const long long t_w = gg_now();
            if (!mbar_wait(&accf[slot], phase & 1, p.err, kErrTimeout)) { ok = false; break; }
            if (q == 0) gg_time(tkind, T_EPI_WAIT, t_w);
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + slot * 256;
            // software pipeline: the TMEM columns of chunk c + 16 are requested while chunk c is
            // processed
            float v[16], vn[16];
            tmem_ld16(lane_base, vn);
            for (int c = 0; c < N; c += 16) {
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = vn[j];
                if (c + 16 < N) tmem_ld16(lane_base + c + 16, vn);
                if constexpr (MODE == MODE_GATE_UP) {
                    // lanes 0-15 hold the gate rows of intermediates rb*64 + 16q + (lane & 15), lanes
                    // 16-31 their up rows; branch-free: lanes 0-15 finish tokens 0-7 of the chunk,
                    // lanes 16-31 tokens 8-15
                    const bool lo = lane < 16;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const float a = v[jj], b = v[jj + 8];
                        const float oa = __shfl_xor_sync(kFull, a, 16), ob = __shfl_xor_sync(kFull, b, 16);
                        const float gt = lo ? a : ob, up = lo ? oa : b;
                        const float act = __fdividef(gt, 1.0f + __expf(-gt)) * up;
                        reinterpret_cast<uint16_t *>(so)[(jj + (lo ? 0 : 8)) * 16 + (lane & 15)] = f32_to_bf16_bits(act);
                    }
                    __syncwarp();
                    // 16 tokens x 16 intermediates (32 bytes): lane -> (token lane/2, half lane%2)
                    const int tk = lane >> 1, half = lane & 1, n = c + tk;
                    const int i = rb * 64 + 16 * q + half * 8;
                    if (n < tl.n && i < p.rows) {
                        const uint4 val = *reinterpret_cast<const uint4 *>(so + tk * 32 + half * 16);
                        *reinterpret_cast<uint4 *>(p.out + (size_t)(tl.p0 + n) * p.rows + i) = val;
                    }
                    __syncwarp();
                } else {
                    // lane holds output dim rb*128 + 32q + lane for 16 tokens: stage [token][dim]
                    // and store the 16 x 32 tile with one tensor store (the tail rows of a tile,
                    // which must not spill into the next tile's positions, with plain stores)
                    uint8_t *sb = so + (chunk_no & 1) * 1024;
                    ++chunk_no;
                    if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 16; ++j) reinterpret_cast<uint16_t *>(sb)[j * 32 + lane] = f32_to_bf16_bits(v[j]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    const int d0 = rb * 128 + 32 * q;
                    // every chunk commits one bulk group (an empty one for plain stores), so that
                    // bulk_wait_read<1> above always frees the buffer of the chunk before last
                    if (tl.n - c >= 16) {
                        if (lane == 0) {
                            tma_store_2d(&p.ymap, sb, d0, tl.p0 + c);
                            bulk_commit();
                        }
                    } else {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int ck = lane + 32 * h, tk = ck >> 2, part = ck & 3, n = c + tk;
                            const int d = d0 + part * 8;
                            if (n < tl.n && d < p.rows)
                                *reinterpret_cast<uint4 *>(p.out + (size_t)(tl.p0 + n) * p.rows + d) =
                                    *reinterpret_cast<const uint4 *>(sb + tk * 64 + part * 16);
                        }
                        if (lane == 0) bulk_commit();
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[slot]);
        }
        if (q == 0) gg_time(tkind, T_EPI_LOOP, t_loop);
        if constexpr (MODE == MODE_DOWN)
            if (lane == 0) bulk_wait<0>();  // tensor stores complete before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) gg_time(tkind, T_KERNEL, t_kernel);
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ------------------------------------------------------------------ CTA-pair kernel
//
// The same grouped GEMM on CTA pairs (2-CTA clusters): one pair unit is a token tile (<= 256
// tokens) x 256 A rows, the even CTA's 128 rows and the odd CTA's 128 rows (two consecutive row
// blocks of the single-CTA kernel), and one pair MMA (cta_group::2, M = 256) issued by the even
// CTA computes both CTAs' accumulators. Each CTA dequantises its own A rows and loads its half of
// the unit's B rows, so per SM the B operand -- copied into and read from shared memory -- is half
// as large, and one MMA-issuing thread drives two tensor cores.
//
// Synchronisation across the pair (the even CTA, rank 0, owns the stage and accumulator
// barriers the MMA waits on):
//   - A ready: the even CTA's dequantiser warps arrive on its full[s]; the odd CTA's, after their
//     fence.proxy.async and a named barrier among the group, signal through the async proxy: one
//     thread copies 16 bytes into the even CTA's shared memory with a bulk copy that completes its
//     bytes on the even CTA's bfull[s] (a per-stage release of four warps' writes at cluster scope
//     that costs the writers no wait);
//   - B ready: the even CTA's B producer arms bfull[s] with both halves' bytes and those 16; both
//     CTAs' tensor copies complete on it (cta_group::2 copies, no multicast);
//   - stage and accumulator free: the MMA thread's commits arrive on empty[s] / accf[slot] in both
//     CTAs (a multicast commit);
//   - accumulator drained: both CTAs' epilogue warps arrive on the even CTA's acce[slot] (8).
// Barrier initialisation and the kernel's end are cluster-wide barriers, so no CTA signals a
// barrier its partner has not initialised or has already left.
constexpr int P_STAGES = 4;
constexpr int kBh = 128 * 128;   // bytes of one CTA's half of a B stage tile (<= 128 token rows)
constexpr int P_STAGE_BYTES = kA + kBh;
constexpr int P_SMEM = 1024 + P_STAGES * P_STAGE_BYTES + CSTAGES * kCode + 2 * kScaleBuf + kStageOut + 512;
static_assert(P_SMEM <= 227 * 1024, "pair grouped GEMM shared memory");

template <int MODE, int BITS>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm_pair_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
    uint8_t *smem = smem_raw + pad;
    uint8_t *code_ring = smem + P_STAGES * P_STAGE_BYTES;
    uint8_t *scale_buf = code_ring + CSTAGES * kCode;
    uint8_t *stage_out = scale_buf + 2 * kScaleBuf;
    uint64_t *bars = reinterpret_cast<uint64_t *>(stage_out + kStageOut);
    uint64_t *full = bars, *bfull = bars + P_STAGES, *empty = bars + 2 * P_STAGES;
    uint64_t *cfull = bars + 3 * P_STAGES, *cempty = cfull + CSTAGES;
    uint64_t *sfull = cempty + CSTAGES, *sempty = sfull + 2;
    uint64_t *accf = sempty + 2, *acce = accf + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    uint64_t *aready = reinterpret_cast<uint64_t *>(tmem_slot + 2);  // odd CTA: its group's A rows written
    uint8_t *sig_src = reinterpret_cast<uint8_t *>(bars) + 320;  // 16 bytes the odd CTA sends per stage
    uint8_t *sig_dst = sig_src + 16;                              // where they land in the even CTA
    auto a_tile = [&](int s) { return smem + s * P_STAGE_BYTES; };
    auto b_tile = [&](int s) { return smem + s * P_STAGE_BYTES + kA; };
    auto c_tile = [&](int cs) { return code_ring + cs * kCode; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = (int)cluster_id_x(), npairs = (int)nclusters_x();
    constexpr int RPU = rows_per_unit<MODE>();
    constexpr int NMAT = MODE == MODE_GATE_UP ? 2 : 1;
    const int RB = (p.rows + RPU - 1) / RPU;  // row blocks of one CTA
    const int PRB = (RB + 1) / 2;             // pair row blocks
    const int nk = p.K / BK;
    const int gpr = p.K / 64;
    const int n_units = (*p.n_tiles) * PRB;
    // CTA row block of pair unit u
    auto cta_rb = [&](int u) { return 2 * (u % PRB) + (int)rank; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 4);   // the even CTA's dequantiser warps of the stage's group
            mbar_init(&bfull[s], 1);  // the even CTA's B producer arrive + both CTAs' B bytes + 16 signal bytes
            mbar_init(&empty[s], 1);  // the pair MMA's commit
        }
        for (int c = 0; c < CSTAGES; ++c) {
            mbar_init(&cfull[c], 1);
            mbar_init(&cempty[c], 4);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sfull[a], 1);
            mbar_init(&sempty[a], 8);
            mbar_init(&accf[a], 1);
            mbar_init(&acce[a], 8);  // the epilogue warps of both CTAs
        }
        for (int s = 0; s < P_STAGES; ++s) mbar_init(&aready[s], 4);
        fence_mbarrier_init();
    }
    if (warp == 4) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);  // the same warp in both CTAs
        tmem_relinquish_pair();
    }
    if (warp == 6 && lane == 0)
        for (int i = 0; i < kBoxes; ++i) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&p.bmap[i]) : "memory");
            if constexpr (MODE == MODE_GATE_UP) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.smap[i]) : "memory");
        }
    if (warp == 5 && lane == 0)
        for (int i = 0; i < 4; ++i) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.code[i]) : "memory");
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised and the tensor memory is allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp >= 8) {
        // ---------------------------------------------------------------- A dequantisers
        const int g = (warp - 8) >> 2, m = threadIdx.x - 256 - 128 * g;  // 0..127
        int mat, r;
        a_row<MODE>(m, mat, r);
        const bool fast_scales = (gpr & 7) == 0;
        const uint32_t bfull_leader = mapa_shared(bfull, 0), sig_leader = mapa_shared(sig_dst, 0);
        int it0 = 0;
        for (int ul = 0, u = pair; u < n_units && ok; ++ul, u += npairs, it0 += nk) {
            const int rb = cta_rb(u), sb = ul & 1;
            const bool live = rb * RPU + r < p.rows;
            if (!mbar_wait(&sfull[sb], (ul >> 1) & 1, p.err, kErrTimeout)) { ok = false; break; }
            const uint16_t *s_row =
                reinterpret_cast<const uint16_t *>(scale_buf + sb * kScaleBuf) + ((mat * 2) * RPU + r) * gpr;
            const uint16_t *b_row = s_row + RPU * gpr;
            uint4 swin = make_uint4(0, 0, 0, 0), bwin = swin;
            int win = -1;
            for (int kb = (g - it0) & 1; kb < nk; kb += 2) {
                float sc, bi;
                if (fast_scales) {
                    if ((kb >> 3) != win) {
                        win = kb >> 3;
                        swin = *reinterpret_cast<const uint4 *>(s_row + 8 * win);
                        bwin = *reinterpret_cast<const uint4 *>(b_row + 8 * win);
                    }
                    const int e = kb & 7;
                    const uint32_t sw = e < 2 ? swin.x : e < 4 ? swin.y : e < 6 ? swin.z : swin.w;
                    const uint32_t bw = e < 2 ? bwin.x : e < 4 ? bwin.y : e < 6 ? bwin.z : bwin.w;
                    sc = (e & 1) ? bf16_hi(sw) : bf16_lo(sw);
                    bi = (e & 1) ? bf16_hi(bw) : bf16_lo(bw);
                } else {
                    sc = bf16_bits_to_f32(s_row[kb]);
                    bi = bf16_bits_to_f32(b_row[kb]);
                }
                const int it = it0 + kb, s = it % P_STAGES, cs = it % CSTAGES;
                if (!mbar_wait(&cfull[cs], (it / CSTAGES) & 1, p.err, kErrTimeout)) { ok = false; break; }
                const uint8_t *crow = c_tile(cs) + mat * (RPU * 64);
                uint4 cw[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) cw[c] = *reinterpret_cast<const uint4 *>(crow + sw64_offset(r, c));
                __syncwarp();
                if (lane == 0) mbar_arrive(&cempty[cs]);
                uint32_t o[32];
                if constexpr (BITS == 8) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) dequant16_8bit(cw[c], sc, bi, o + 8 * c);
                } else {
                    const uint32_t w16[16] = {cw[0].x, cw[0].y, cw[0].z, cw[0].w, cw[1].x, cw[1].y, cw[1].z, cw[1].w,
                                              cw[2].x, cw[2].y, cw[2].z, cw[2].w, cw[3].x, cw[3].y, cw[3].z, cw[3].w};
                    const bool odd = ((kb * 40) & 15) != 0;
                    uint32_t w10[10];
#pragma unroll
                    for (int i = 0; i < 10; ++i) w10[i] = odd ? w16[i + 2] : w16[i];
                    dequant32_5bit(w10, sc, bi, o);
                    dequant32_5bit(w10 + 5, sc, bi, o + 16);
                }
                if (!live)
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = 0;
                // the A tile is free once the pair MMA of the stage's previous use has completed
                if (!mbar_wait(&empty[s], ((it / P_STAGES) & 1) ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                uint8_t *t = a_tile(s);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4 *>(t + sw128_offset(m, c)) =
                        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (leader) {
                    if (lane == 0) mbar_arrive(&full[s]);
                } else {
                    if (lane == 0) mbar_arrive(&aready[s]);
                    // the group's first warp: once all 128 rows are written and fenced, signal the even CTA
                    if (m == 0) {
                        if (mbar_wait(&aready[s], (it / P_STAGES) & 1, p.err, kErrTimeout))
                            bulk_copy_to_cluster(sig_leader, sig_src, 16, bfull_leader + s * 8u);
                        else
                            ok = false;
                    }
                    ok = __shfl_sync(kFull, ok, 0);
                    if (!ok) break;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[sb]);
        }
    } else if (warp == 5) {
        // ---------------------------------------------------------------- code and scale producer
        int it = 0, ul = 0;
        for (int u = pair; u < n_units && ok; u += npairs, ++ul) {
            const Tile tl = p.tiles[u / PRB];
            const int rb = cta_rb(u), sb = ul & 1;
            const bool shared = tl.seg >= p.E;
            const int expert = shared ? 0 : tl.seg;
            const bool rows_live = rb * RPU < p.rows;  // the odd CTA's rows may lie past the matrix
            if (lane == 0) {
                ok = mbar_wait(&sempty[sb], ((ul >> 1) & 1) ^ 1, p.err, kErrTimeout);
                if (ok) {
                    const int nrows = rows_live ? min(RPU, p.rows - rb * RPU) : 0;
                    const uint32_t bytes = (uint32_t)(nrows * gpr * 2);
                    mbar_arrive_expect_tx(&sfull[sb], bytes * 2 * NMAT);
                    if (nrows > 0)
                        for (int mt = 0; mt < NMAT; ++mt) {
                            const QView &W = p.w[mt + 2 * shared];
                            const size_t r0 = (size_t)expert * W.rows + rb * RPU;
                            uint8_t *dst = scale_buf + sb * kScaleBuf + (size_t)(mt * 2) * RPU * gpr * 2;
                            bulk_load(dst, W.scales + r0 * gpr, bytes, &sfull[sb]);
                            bulk_load(dst + RPU * gpr * 2, W.biases + r0 * gpr, bytes, &sfull[sb]);
                        }
                }
            }
            ok = __shfl_sync(kFull, ok, 0);
            if (!ok) break;
            // rows past the matrix read the last valid block's codes (their A rows are zeroed)
            const int crb = rows_live ? rb : rb - 1;
            const int row0 = expert * p.w[(lane & 1) + 2 * shared].rows + crb * RPU;
            for (int kb = 0; kb < nk; ++kb, ++it) {
                const int cs = it % CSTAGES;
                if (lane == 0) {
                    ok = mbar_wait(&cempty[cs], ((it / CSTAGES) & 1) ^ 1, p.err, kErrTimeout);
                    if (ok) mbar_arrive_expect_tx(&cfull[cs], kCode);
                }
                ok = __shfl_sync(kFull, ok, 0);
                if (!ok) break;
                if (lane < NMAT)
                    tma_load_2d(c_tile(cs) + lane * (RPU * 64), &p.code[lane + 2 * shared], code_x<BITS>(kb), row0,
                                &cfull[cs]);
            }
        }
        if (!ok && lane == 0) {
            for (int k = max(0, it - CSTAGES); k < it; ++k)
                mbar_wait(&cfull[k % CSTAGES], (k / CSTAGES) & 1, p.err, kErrTimeout);
            for (int k = max(0, ul - 1); k <= ul; ++k) mbar_wait(&sfull[k & 1], (k >> 1) & 1, p.err, kErrTimeout);
        }
    } else if (warp == 6) {
        // ---------------------------------------------------------------- B producer (this CTA's half)
        const uint32_t bfull_leader = mapa_shared(bfull, 0);
        int it = 0;
        for (int u = pair; u < n_units && ok; u += npairs) {
            const Tile tl = p.tiles[u / PRB];
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n), Nh = N >> 1;  // Nh is a multiple of 8
            // lane i < kBoxes copies 8 << i rows when bit i of Nh/8 is set, larger boxes first
            const int nb8 = Nh >> 3;
            const bool box_mine = lane < kBoxes && ((nb8 >> lane) & 1);
            const int box_off = box_mine ? 8 * ((nb8 >> (lane + 1)) << (lane + 1)) : 0;
            const bool shared_src = MODE == MODE_GATE_UP && shared;
            const int row0 = (shared_src ? p.shared_src0 + (tl.p0 - p.shared_pos0) : tl.p0) + (int)rank * Nh + box_off;
            const CUtensorMap *bm = shared_src ? &p.smap[box_mine ? lane : 0] : &p.bmap[box_mine ? lane : 0];
            for (int kb = 0; kb < nk; ++kb, ++it) {
                const int s = it % P_STAGES;
                if (lane == 0) {
                    ok = mbar_wait(&empty[s], ((it / P_STAGES) & 1) ^ 1, p.err, kErrTimeout);
                    if (ok && leader) mbar_arrive_expect_tx(&bfull[s], (uint32_t)N * 128u + 16u);  // both halves
                }
                ok = __shfl_sync(kFull, ok, 0);
                if (!ok) break;
                if (box_mine)
                    tma_load_2d_pair(b_tile(s) + box_off * 128, bm, kb * BK, row0, bfull_leader + s * 8u);
            }
        }
        // copies in flight complete on the even CTA's barriers, which the MMA waits for; the final
        // cluster barrier keeps both CTAs alive until then
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issue (even CTA)
        if (leader && lane == 0) {
            int it = 0;
            SlotPlan plan;
            for (int u = pair; u < n_units && ok; u += npairs) {
                const Tile tl = p.tiles[u / PRB];
                const int N = round16(tl.n);
                uint32_t phase;
                const int slot = plan.take(phase);
                if (!mbar_wait_cluster(&acce[slot], (phase & 1) ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + slot * 256;
                const uint32_t id = idesc_bf16_f32(2 * BM, N);
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % P_STAGES;
                    const uint32_t ph = (it / P_STAGES) & 1;
                    if (!mbar_wait_cluster(&bfull[s], ph, p.err, kErrTimeout) ||
                        !mbar_wait_cluster(&full[s], ph, p.err, kErrTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(smem_u32(a_tile(s)));
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(b_tile(s)));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        tc_mma_bf16_pair(d, adesc + 2 * k, bdesc + 2 * k, id, (kb | k) != 0);
                    tc_commit_pair(&empty[s], 0x3);
                }
                if (!ok) break;
                tc_commit_pair(&accf[slot], 0x3);
            }
            if (!ok) {
                // copies still in flight land on this CTA's bfull barriers: wait for the last stages'
                for (int k = max(0, it - P_STAGES); k < it; ++k)
                    mbar_wait(&bfull[k % P_STAGES], (k / P_STAGES) & 1, p.err, kErrTimeout);
            }
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---------------------------------------------------------------- epilogue (this CTA's rows)
        const int q = warp;
        uint8_t *so = stage_out + q * 2 * 16 * 64;
        int chunk_no = 0;
        SlotPlan plan;
        const uint32_t acce_leader = mapa_shared(acce, 0);
        for (int u = pair; u < n_units && ok; u += npairs) {
            const Tile tl = p.tiles[u / PRB];
            const int rb = cta_rb(u);
            const int N = round16(tl.n);
            uint32_t phase;
            const int slot = plan.take(phase);
            if (!mbar_wait(&accf[slot], phase & 1, p.err, kErrTimeout)) { ok = false; break; }
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + slot * 256;
            float v[16], vn[16];
            tmem_ld16(lane_base, vn);
            for (int c = 0; c < N; c += 16) {
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = vn[j];
                if (c + 16 < N) tmem_ld16(lane_base + c + 16, vn);
                if constexpr (MODE == MODE_GATE_UP) {
                    const bool lo = lane < 16;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const float a = v[jj], b = v[jj + 8];
                        const float oa = __shfl_xor_sync(kFull, a, 16), ob = __shfl_xor_sync(kFull, b, 16);
                        const float gt = lo ? a : ob, up = lo ? oa : b;
                        const float act = __fdividef(gt, 1.0f + __expf(-gt)) * up;
                        reinterpret_cast<uint16_t *>(so)[(jj + (lo ? 0 : 8)) * 16 + (lane & 15)] = f32_to_bf16_bits(act);
                    }
                    __syncwarp();
                    const int tk = lane >> 1, half = lane & 1, n = c + tk;
                    const int i = rb * 64 + 16 * q + half * 8;
                    if (n < tl.n && i < p.rows) {
                        const uint4 val = *reinterpret_cast<const uint4 *>(so + tk * 32 + half * 16);
                        *reinterpret_cast<uint4 *>(p.out + (size_t)(tl.p0 + n) * p.rows + i) = val;
                    }
                    __syncwarp();
                } else {
                    uint8_t *sb = so + (chunk_no & 1) * 1024;
                    ++chunk_no;
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 16; ++j) reinterpret_cast<uint16_t *>(sb)[j * 32 + lane] = f32_to_bf16_bits(v[j]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    const int d0 = rb * 128 + 32 * q;
                    // one bulk group per chunk (empty for plain stores or dead rows), as above
                    if (d0 < p.rows && tl.n - c >= 16) {
                        if (lane == 0) {
                            tma_store_2d(&p.ymap, sb, d0, tl.p0 + c);
                            bulk_commit();
                        }
                    } else {
                        if (d0 < p.rows) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int ck = lane + 32 * h, tk = ck >> 2, part = ck & 3, n = c + tk;
                                const int d = d0 + part * 8;
                                if (n < tl.n && d < p.rows)
                                    *reinterpret_cast<uint4 *>(p.out + (size_t)(tl.p0 + n) * p.rows + d) =
                                        *reinterpret_cast<const uint4 *>(sb + tk * 64 + part * 16);
                            }
                        }
                        if (lane == 0) bulk_commit();
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) mbar_arrive(&acce[slot]);
                else mbar_arrive_cluster(acce_leader + slot * 8u);
            }
        }
        if constexpr (MODE == MODE_DOWN)
            if (lane == 0) bulk_wait<0>();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while its partner may still signal it or read its memory
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
}

}  // namespace gg
}  // namespace di
