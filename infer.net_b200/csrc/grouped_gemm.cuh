// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// D[m, n] = sum_k A[m, k] * B[n, k] for every work unit (a token tile of one expert segment
// x a block of weight rows). A is dequantised in shared memory from the affine-quantised MLX
// codes; B rows are the tokens routed to the expert (gathered from x for gate/up, contiguous
// activation rows for down). Both operands are K-major bf16 tiles with the 64-byte swizzle;
// the f32 accumulators live in tensor memory.
//
//   MODE_GATE_UP: the 128 A rows of a unit interleave 16 gate rows and the 16 up rows of the
//                 same intermediate indices in every 32-lane TMEM quadrant, so the SwiGLU
//                 epilogue pairs them with one warp shuffle; a unit covers 64 intermediate
//                 indices and up to 512 tokens (two 256-column accumulators), so at 8K tokens
//                 every expert's weights are dequantised once. act = silu(gate) * up -> bf16
//                 act[p, i] (quantized.mm:148-189; prefill_moe.mm:23-53 semantics)
//   MODE_DOWN:    128 rows of the down matrix; the epilogue writes each bf16 expert row to its
//                 route slot y[r, d] (r = t*8 + slot) or the shared row ys[t, d]
//                 (prefill_moe.mm:54-78 semantics)
//
// Warp roles (512 threads): 0-3 epilogue (one TMEM lane quadrant each), 4 MMA issue + TMEM
// owner, 5-7 B loaders (cp.async), 8-15 A dequantisers in two groups of 4 warps that take
// alternate pipeline stages.
#pragma once
#include "common.cuh"
#include "route.cuh"

namespace di {
namespace gg {

constexpr int MODE_GATE_UP = 0, MODE_DOWN = 1;
constexpr int BM = 128;          // A rows per unit (one MMA M)
constexpr int BN = 256;          // max tokens per unit (one 256-column accumulator slot)
constexpr int BK = 32;           // K per pipeline stage: 64-byte rows
constexpr int STAGES = 7;
constexpr int RING = 4;         // dequantiser code ring: own stages in flight per thread
constexpr int kRingSlot = 48;   // bytes per thread per slot: 32 code bytes + 2 scale words + 2 bias words
constexpr int THREADS = 512;
constexpr int kA = BM * 64;      // bytes of one A stage tile
constexpr int kB = BN * 64;      // bytes of one B stage tile
constexpr int STAGE_BYTES = kA + kB;
constexpr int kTable = BN * 4;   // token row table of the B loaders
constexpr int kStageOut = 4 * 16 * 64;  // epilogue staging: 4 warps x 16 tokens x 64 bytes
constexpr int kRing = 256 * RING * kRingSlot;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + kTable + kStageOut + kRing + 256;
constexpr uint32_t TMEM_COLS = 512;

template <int MODE>
__host__ __device__ constexpr int rows_per_unit() { return MODE == MODE_GATE_UP ? 64 : 128; }

struct Params {
    QView w1, w2;              // routed experts: gate, up (GATE_UP) or down (DOWN)
    QView s1, s2;              // shared expert:  gate, up (GATE_UP) or down (DOWN)
    const uint16_t *src;       // GATE_UP: x [T, K]; DOWN: act [P, K]
    const int32_t *perm_route; // [8T] route id of each permuted position
    const Tile *tiles;
    const int32_t *n_tiles;
    int shared_pos0;           // first permuted position of the shared-expert segment
    int shared_src0;           // GATE_UP: source row of that first shared position
    int K, rows, E;            // rows: I (GATE_UP) or D (DOWN); segments >= E are the shared expert
    uint16_t *out;             // GATE_UP: act [P, rows]; DOWN: y [8T, rows]
    uint16_t *out_shared;      // DOWN: ys [T, rows]
    uint32_t *err;
};

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

// Byte offset of 16-byte chunk c (0..3) of row r in a 64B-swizzled K-major tile
// (address bits [7,9) XOR-ed into bits [4,6)).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t r, uint32_t c) {
    return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}

// Shared-memory descriptor: K-major, 64-byte swizzle, 8-row atoms 512 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512u >> 4) << 32;    // stride byte offset between 8-row groups
    d |= (uint64_t)1u << 46;             // descriptor version for tcgen05
    d |= (uint64_t)4u << 61;             // SWIZZLE_64B
    return d;
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

// A-tile row m of a unit -> weight row. GATE_UP: in quadrant q = m/32, lanes 0-15 are gate rows
// and lanes 16-31 the up rows of intermediates rb*64 + 16q + (m & 15).
template <int MODE>
__device__ __forceinline__ void a_row(int m, int rb, int &mat, int &row) {
    if constexpr (MODE == MODE_GATE_UP) {
        mat = (m >> 4) & 1;
        row = rb * 64 + (m >> 5) * 16 + (m & 15);
    } else {
        mat = 0;
        row = rb * 128 + m;
    }
}

// Accumulator slots: a unit with N <= 256 takes one 256-column slot (alternating), a larger
// unit takes both. Every role derives the same assignment from the unit sequence.
struct SlotPlan {
    int next = 0;
    uint32_t uses[2] = {0, 0};
    // returns a bitmask of slots; phase[s] = completed fills of slot s before this unit
    __device__ __forceinline__ int take(int N, uint32_t *phase) {
        const int mask = N <= 256 ? (1 << next) : 3;
        if (N <= 256) next ^= 1;
        for (int s = 0; s < 2; ++s) {
            phase[s] = uses[s];
            if (mask >> s & 1) uses[s]++;
        }
        return mask;
    }
};

// Codes, scale and bias of one dequantiser thread's share of one stage (2 jobs of 16 codes
// for 8-bit, 1 job of 32 codes for 5-bit), loaded ahead of use.
template <int BITS>
struct Fetch {
    static constexpr int JOBS = BITS == 8 ? 2 : 1, WORDS = BITS == 8 ? 4 : 5;
    uint32_t q[JOBS][WORDS];
    float s[JOBS], b[JOBS];
    bool live[JOBS];
    bool valid;

    template <int MODE>
    __device__ __forceinline__ void load(const Params &p, const Tile &tl, int rb, int kb, int tid) {
        const bool shared = tl.seg >= p.E;
        const int expert = shared ? 0 : tl.seg;
#pragma unroll
        for (int j = 0; j < JOBS; ++j) {
            const int job = j * 128 + tid;
            // 8-bit: job = (m, part), 2 parts of 16 codes per 32-wide row; 5-bit: job = m
            const int m = BITS == 8 ? (job >> 1) : job, part = BITS == 8 ? (job & 1) : 0;
            int mat, row;
            a_row<MODE>(m, rb, mat, row);
            const QView W = mat ? (shared ? p.s2 : p.w2) : (shared ? p.s1 : p.w1);
            live[j] = row < p.rows;
            const size_t ridx = (size_t)expert * W.rows + min(row, p.rows - 1);
            const uint32_t *src = W.packed + ridx * W.words_per_row();
            if constexpr (BITS == 8) {
                const uint4 v = ldg_nc_v4(src + kb * 8 + part * 4);
                q[j][0] = v.x; q[j][1] = v.y; q[j][2] = v.z; q[j][3] = v.w;
            } else {
#pragma unroll
                for (int w = 0; w < 5; ++w) q[j][w] = ldg_nc_u32(src + kb * 5 + w);
            }
            s[j] = bf16_bits_to_f32(__ldg(W.scales + ridx * W.groups_per_row() + (kb >> 1)));
            b[j] = bf16_bits_to_f32(__ldg(W.biases + ridx * W.groups_per_row() + (kb >> 1)));
        }
    }

    template <int MODE>
    __device__ __forceinline__ void store(uint8_t *t, int tid) const {
#pragma unroll
        for (int j = 0; j < JOBS; ++j) {
            const int job = j * 128 + tid;
            if constexpr (BITS == 8) {
                const int m = job >> 1, part = job & 1;
                uint32_t o[8];
                if (live[j]) dequant16_8bit(make_uint4(q[j][0], q[j][1], q[j][2], q[j][3]), s[j], b[j], o);
                else
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] = 0;
                *reinterpret_cast<uint4 *>(t + sw64_offset(m, 2 * part)) = make_uint4(o[0], o[1], o[2], o[3]);
                *reinterpret_cast<uint4 *>(t + sw64_offset(m, 2 * part + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
            } else {
                const int m = job;
                uint32_t o[16];
                if (live[j]) dequant32_5bit(q[j], s[j], b[j], o);
                else
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = 0;
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    *reinterpret_cast<uint4 *>(t + sw64_offset(m, c)) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
            }
        }
    }
};

template <int MODE, int BITS>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm_kernel(Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t pad = ((raw_base + 1023u) & ~1023u) - raw_base;
    uint8_t *smem = smem_raw + pad;
    int32_t *tok_table = reinterpret_cast<int32_t *>(smem + STAGES * STAGE_BYTES);
    uint8_t *stage_out = reinterpret_cast<uint8_t *>(tok_table + BN);
    uint8_t *ring = stage_out + kStageOut;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kRing);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *accf = bars + 2 * STAGES, *acce = accf + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    auto a_tile = [&](int s) { return smem + s * STAGE_BYTES; };
    auto b_tile = [&](int s) { return smem + s * STAGE_BYTES + kA; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RPU = rows_per_unit<MODE>();
    const int RB = (p.rows + RPU - 1) / RPU;
    const int nk = p.K / BK;
    const int n_units = (*p.n_tiles) * RB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 4 + 96);  // one dequant group (4 warp arrivals) + 96 loader threads' copies
            mbar_init(&empty[s], 1);
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
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    // Flat pipeline index `it`: unit u = blockIdx.x + (it / nk) * gridDim.x, k-block it % nk.
    if (warp >= 8) {
        // ---------------------------------------------------------------- A dequantisers
        // group g (warps 8-11 or 12-15) fills the stages it with it % 2 == g. Each thread streams
        // its own codes, scale and bias words with cp.async into a private RING-deep slot ring
        // (layout [slot][field][thread], conflict-free), RING own stages ahead of their use.
        const int g = (warp - 8) >> 2, tid = threadIdx.x - 256 - 128 * g;  // 0..127
        const int rt = threadIdx.x - 256;                                    // ring column 0..255
        const int total = (int)blockIdx.x < n_units ? ((n_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1) * nk : 0;
        constexpr int JOBS = BITS == 8 ? 2 : 1;
        auto slot_codes = [&](int sl, int j) { return ring + (size_t)sl * 256 * kRingSlot + ((size_t)j * 256 + rt) * 16; };
        auto slot_word = [&](int sl, int f) {  // f: 0,1 scale words of jobs 0,1; 2,3 bias words
            return ring + (size_t)sl * 256 * kRingSlot + 2 * 256 * 16 + ((size_t)f * 256 + rt) * 4;
        };
        int cached_tile = -1, cached_expert = 0;
        bool cached_shared = false;
        uint32_t parity = 0;  // bit (slot*2 + job): the group's bf16 is the high half of its copied word
        auto issue = [&](int it, int sl) {
            if (it < total) {
                const int u = blockIdx.x + (it / nk) * gridDim.x, kb = it % nk, rb = u % RB;
                if (u / RB != cached_tile) {
                    cached_tile = u / RB;
                    const int seg = p.tiles[cached_tile].seg;
                    cached_shared = seg >= p.E;
                    cached_expert = cached_shared ? 0 : seg;
                }
#pragma unroll
                for (int j = 0; j < JOBS; ++j) {
                    const int job = j * 128 + tid;
                    const int m = BITS == 8 ? (job >> 1) : job, part = BITS == 8 ? (job & 1) : 0;
                    int mat, row;
                    a_row<MODE>(m, rb, mat, row);
                    const QView W = mat ? (cached_shared ? p.s2 : p.w2) : (cached_shared ? p.s1 : p.w1);
                    const size_t ridx = (size_t)cached_expert * W.rows + min(row, p.rows - 1);
                    const uint32_t *src = W.packed + ridx * W.words_per_row();
                    if constexpr (BITS == 8) {
                        cp_async_16(slot_codes(sl, j), src + kb * 8 + part * 4, true);
                    } else {
                        // words 0-3 in this thread's first 16-byte field, word 4 in its second
#pragma unroll
                        for (int w = 0; w < 4; ++w) cp_async_4(slot_codes(sl, 0) + 4 * w, src + kb * 5 + w);
                        cp_async_4(slot_codes(sl, 1), src + kb * 5 + 4);
                    }
                    const size_t gi = ridx * W.groups_per_row() + (kb >> 1);
                    cp_async_4(slot_word(sl, j), W.scales + (gi & ~(size_t)1));
                    cp_async_4(slot_word(sl, 2 + j), W.biases + (gi & ~(size_t)1));
                    const uint32_t bit = 1u << (sl * 2 + j);
                    parity = (gi & 1) ? (parity | bit) : (parity & ~bit);
                }
            }
            cp_async_commit();  // one group per own stage, empty at the end of the sequence
        };
        // prologue: own stages 0 .. RING-1
#pragma unroll
        for (int k = 0; k < RING; ++k) issue(g + 2 * k, k);
        for (int k = 0;; ++k) {
            const int cur = g + 2 * k;
            if (cur >= total || !ok) break;
            const int sl = k % RING;
            cp_async_wait<RING - 1>();  // own stage k has landed in slot sl
            Fetch<BITS> f;
            {
                const int u = blockIdx.x + (cur / nk) * gridDim.x, rb = u % RB;
#pragma unroll
                for (int j = 0; j < JOBS; ++j) {
                    const int job = j * 128 + tid;
                    const int m = BITS == 8 ? (job >> 1) : job;
                    int mat, row;
                    a_row<MODE>(m, rb, mat, row);
                    f.live[j] = row < p.rows;
                    if constexpr (BITS == 8) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(slot_codes(sl, j));
                        f.q[j][0] = v.x; f.q[j][1] = v.y; f.q[j][2] = v.z; f.q[j][3] = v.w;
                    } else {
#pragma unroll
                        for (int w = 0; w < 4; ++w) f.q[j][w] = *reinterpret_cast<const uint32_t *>(slot_codes(sl, 0) + 4 * w);
                        f.q[j][4] = *reinterpret_cast<const uint32_t *>(slot_codes(sl, 1));
                    }
                    // the group's bf16 sits in the low or high half of the copied word
                    const uint32_t odd = (parity >> (sl * 2 + j)) & 1u;
                    const uint32_t sw = *reinterpret_cast<const uint32_t *>(slot_word(sl, j));
                    const uint32_t bw = *reinterpret_cast<const uint32_t *>(slot_word(sl, 2 + j));
                    f.s[j] = bf16_bits_to_f32(odd ? (sw >> 16) : (sw & 0xffffu));
                    f.b[j] = bf16_bits_to_f32(odd ? (bw >> 16) : (bw & 0xffffu));
                }
            }
            issue(cur + 2 * RING, sl);  // the slot is free again: fetch own stage k + RING into it
            const int s = cur % STAGES;
            const uint32_t ph = (cur / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrTimeout)) { ok = false; break; }
            f.template store<MODE>(a_tile(s), tid);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
        cp_async_wait<0>();
    } else if (warp >= 5) {
        // ---------------------------------------------------------------- B loaders
        // loader warp w owns the 8-row groups g with g % 3 == w: it alone writes and reads
        // their table entries, so only __syncwarp is needed. Per group, lane l copies 16-byte
        // chunk l % 4 of row 8g + l / 4.
        const int w = warp - 5;
        int it = 0;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n);
            __syncwarp();
            for (int g8 = w; g8 < N / 8; g8 += 3) {
                if (lane < 8) {
                    const int n = g8 * 8 + lane;
                    const int pos = tl.p0 + min(n, tl.n - 1);
                    int row;
                    if constexpr (MODE == MODE_GATE_UP) row = shared ? p.shared_src0 + (pos - p.shared_pos0) : (p.perm_route[pos] >> 3);
                    else row = pos;
                    tok_table[n] = row;
                }
            }
            __syncwarp();
            for (int kb = 0; kb < nk && ok; ++kb, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrTimeout)) { ok = false; break; }
                uint8_t *bt = b_tile(s);
                const uint16_t *base = p.src + kb * BK;
                for (int g8 = w; g8 < N / 8; g8 += 3) {
                    const int n = g8 * 8 + (lane >> 2), ch = lane & 3;
                    cp_async_16(bt + sw64_offset(n, ch), base + (size_t)tok_table[n] * p.K + ch * 8, n < tl.n);
                }
                // the stage is published when this thread's copies land (no wait here)
                cp_async_arrive_noinc(&full[s]);
            }
        }
        cp_async_wait<0>();
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issue
        if (lane == 0) {
            int it = 0;
            SlotPlan plan;
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const Tile tl = p.tiles[u / RB];
                const int N = round16(tl.n);
                uint32_t phase[2];
                const int mask = plan.take(N, phase);
                for (int s2 = 0; s2 < 2 && ok; ++s2)
                    if (mask >> s2 & 1)
                        if (!mbar_wait(&acce[s2], (phase[s2] & 1) ^ 1, p.err, kErrTimeout)) ok = false;
                if (!ok) break;
                tc_fence_after();
                // tokens [0, n0) accumulate in the first slot of the mask, [256, N) in slot 1
                const int first = (mask == 2) ? 1 : 0;
                const int n0 = N < 256 ? N : 256, n1 = N - n0;
                const uint32_t d0 = tmem + first * 256, d1 = tmem + 256;
                const uint32_t id0 = idesc_bf16_f32(BM, n0), id1 = n1 > 0 ? idesc_bf16_f32(BM, n1) : 0;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, p.err, kErrTimeout)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw64(smem_u32(a_tile(s)));
                    const uint64_t bdesc = smem_desc_sw64(smem_u32(b_tile(s)));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint32_t acc = (kb | k) != 0;
                        tc_mma_bf16(d0, adesc + 2 * k, bdesc + 2 * k, id0, acc);
                        // second accumulator: B rows from 256 on start 256 x 64 bytes further
                        if (n1 > 0) tc_mma_bf16(d1, adesc + 2 * k, bdesc + ((256 * 64) >> 4) + 2 * k, id1, acc);
                    }
                    tc_commit(&empty[s]);
                }
                if (!ok) break;
                for (int s2 = 0; s2 < 2; ++s2)
                    if (mask >> s2 & 1) tc_commit(&accf[s2]);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp;  // TMEM lanes 32q .. 32q+31
        uint8_t *so = stage_out + q * 16 * 64;
        SlotPlan plan;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const Tile tl = p.tiles[u / RB];
            const int rb = u % RB;
            const bool shared = tl.seg >= p.E;
            const int N = round16(tl.n);
            uint32_t phase[2];
            const int mask = plan.take(N, phase);
            for (int s2 = 0; s2 < 2 && ok; ++s2)
                if (mask >> s2 & 1)
                    if (!mbar_wait(&accf[s2], phase[s2] & 1, p.err, kErrTimeout)) ok = false;
            if (!ok) break;
            tc_fence_after();
            const int first = (mask == 2) ? 1 : 0;
            auto col_of = [&](int c) -> uint32_t { return (c < 256) ? first * 256 + c : 256 + (c - 256); };
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
            // software pipeline: the TMEM columns (and, for down, the output rows) of chunk c + 16
            // are requested while chunk c is processed
            float v[16], vn[16];
            int rid = 0, rid_next = 0;  // DOWN: output row of token (c + lane) for lanes < 16
            auto route_of = [&](int c) -> int {
                const int n = c + (lane & 15);
                if (n >= tl.n) return 0;
                const int pos = tl.p0 + n;
                return shared ? -1 - (pos - p.shared_pos0) : p.perm_route[pos];
            };
            tmem_ld16(lane_base + col_of(0), vn);
            if constexpr (MODE == MODE_DOWN) rid_next = route_of(0);
            for (int c = 0; c < N; c += 16) {
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = vn[j];
                rid = rid_next;
                if (c + 16 < N) {
                    tmem_ld16(lane_base + col_of(c + 16), vn);
                    if constexpr (MODE == MODE_DOWN) rid_next = route_of(c + 16);
                }
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
                    // lane holds output dim rb*128 + 32q + lane for 16 tokens
#pragma unroll
                    for (int j = 0; j < 16; ++j) reinterpret_cast<uint16_t *>(so)[j * 32 + lane] = f32_to_bf16_bits(v[j]);
                    __syncwarp();
                    // 16 tokens x 64 bytes = 64 chunks of 16 bytes, two per lane
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int ck = lane + 32 * h, tk = ck >> 2, part = ck & 3, n = c + tk;
                        const int d = rb * 128 + 32 * q + part * 8;
                        const int r = __shfl_sync(kFull, rid, tk);
                        if (n < tl.n && d < p.rows) {
                            const uint4 val = *reinterpret_cast<const uint4 *>(so + tk * 64 + part * 16);
                            uint16_t *dst = r >= 0 ? p.out + (size_t)r * p.rows : p.out_shared + (size_t)(-1 - r) * p.rows;
                            *reinterpret_cast<uint4 *>(dst + d) = val;
                        }
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                for (int s2 = 0; s2 < 2; ++s2)
                    if (mask >> s2 & 1) mbar_arrive(&acce[s2]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace gg
}  // namespace di
