// Expert-parallel dispatch / combine (one process per GPU; the kernels write each other's
// buffers directly over NVLink, NCCL only bootstraps the group).
//
// GPU r of G owns experts [r*E_l, (r+1)*E_l) of every layer and a contiguous shard of the
// tokens. A token is sent once to every GPU that owns at least one of its 8 experts, with its
// 8 expert ids and probabilities; the receiver runs its experts on the received rows, reduces
// each row's local slots to one partial row sum_j p_j * y_j (slot order), and sends it back;
// the owner adds the partial rows of all GPUs (ascending GPU order) to the shared expert's
// sigmoid-gated output (Qwen36Model.cs:242-244) and to the residual stream.
//
// The permutation stays the single-GPU one: a receiver orders the routes of each of its
// experts by (source GPU, source row, slot), and because tokens are sharded contiguously in
// GPU order this is the ascending route order r = t*8 + slot of the whole batch.
#pragma once
#include "common.cuh"
#include "peer.cuh"
#include "route.cuh"

namespace di {

// Dispatch: one warp per (local token t, destination d) pair writes t's routing metadata into
// region `rank` of d's meta (row t) and, when one of t's experts lives on d, t's row into d's rx
// (row t), by direct stores over NVLink. The warp's token row is requested before the metadata
// test, so the pair costs one round trip to local memory.
__global__ void __launch_bounds__(256)
ep_dispatch_kernel(const uint16_t *__restrict__ h, const int32_t *__restrict__ ids, const float *__restrict__ probs,
                   int T, int D, int G, int rank, int cap, int E_l, EpPeers peers, uint32_t *ticket) {
    pdl_enter();
    const int lane = threadIdx.x & 31, warps = gridDim.x * (blockDim.x >> 5);
    for (int td = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); td < T * G; td += warps) {
        const int t = td / G, d = td - t * G;
        const uint4 *src = reinterpret_cast<const uint4 *>(h + (size_t)t * D);
        uint4 v[8];  // D <= 2048: 8 chunks of 16 bytes per lane
#pragma unroll
        for (int c = 0; c < 8; ++c)
            if (lane + 32 * c < D / 8) v[c] = __ldg(src + lane + 32 * c);
        int e = 0;
        float p = 0.f;
        if (lane < 8) {
            e = __ldg(ids + (size_t)t * 8 + lane);
            p = __ldg(probs + (size_t)t * 8 + lane);
        }
        const size_t row = (size_t)rank * cap + t;
        if (lane < 8) {
            peers.meta[d][row].ids[lane] = e;
            peers.meta[d][row].probs[lane] = p;
        }
        if (!__any_sync(kFull, lane < 8 && e / E_l == d)) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(peers.rx[d] + row * D);
#pragma unroll
        for (int c = 0; c < 8; ++c)
            if (lane + 32 * c < D / 8) dst[lane + 32 * c] = v[c];
    }
    ep_signal(ticket, peers, G, rank, 2 * G + rank, T);
}

// Receiver: waits for every rank's dispatch, then the local expert of every (row, slot) of the
// G*cap row slots -- E_l for a slot owned by another rank or a row slot nobody filled -- and the
// per-block histogram over E_l + 1 buckets (blocks of topk::TOK_PER_CTA rows).
__global__ void __launch_bounds__(256)
ep_recv_routes_kernel(const RowMeta *__restrict__ meta, const uint32_t *__restrict__ sync, uint32_t target, int G,
                      int cap, int E_off, int E_l, EpPeers peers, int32_t *__restrict__ ids_local,
                      int32_t *__restrict__ block_counts, uint32_t *__restrict__ err) {
    pdl_enter();
    __shared__ int32_t hist[kMaxBuckets];
    __shared__ int32_t cnt[kMaxRanks];
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = ep_wait_counters(sync, G, target, sync + 3 * G, peers, err);
        for (int s = 0; s < G; ++s) cnt[s] = (int)*reinterpret_cast<const volatile uint32_t *>(sync + 2 * G + s);
    }
    for (int i = threadIdx.x; i <= E_l; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int R = G * cap;
    const int r0 = blockIdx.x * topk::TOK_PER_CTA * 8;
    for (int r = r0 + threadIdx.x; r < min(r0 + topk::TOK_PER_CTA * 8, R * 8); r += blockDim.x) {
        const int i = r >> 3, s = i / cap;
        int b = E_l;
        if (ok && i - s * cap < cnt[s]) {
            const int e = __ldcg(&meta[i].ids[r & 7]) - E_off;
            if (e >= 0 && e < E_l) b = e;
        }
        ids_local[r] = b;
        atomicAdd(&hist[b], 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i <= E_l; i += blockDim.x) block_counts[(size_t)blockIdx.x * (E_l + 1) + i] = hist[i];
}

// Receiver: one warp per row (s, k) with at least one local slot: partial row z = sum over its
// local slots j (slot order) of p_j * y_j (f32, then bf16), stored straight into region `rank` of
// rank s's back buffer (row k). y_j = yp[route_pos[8i + j]] (expert rows in expert order).
// The local slots' rows are requested together (kSendSlots at a time) by cp.async into the warp's
// own shared-memory staging, so a row costs one round trip to memory instead of one per chunk,
// and the row accumulator (8 chunks x 8 floats per lane) lives in registers. Each lane reads back
// only the chunks it copied itself, so completion of its own copies is the only wait.
constexpr int kSendWarps = 8, kSendSlots = 6;
inline size_t ep_send_smem(int D) { return (size_t)kSendWarps * kSendSlots * D * 2; }

__global__ void __launch_bounds__(kSendWarps * 32, 1)
ep_reduce_send_kernel(const uint16_t *__restrict__ yp, const int32_t *__restrict__ route_pos,
                      const int32_t *__restrict__ ids_local, const RowMeta *__restrict__ meta,
                      const uint32_t *__restrict__ sync, int G, int rank, int cap, int D, int E_l, EpPeers peers,
                      uint32_t *ticket, const uint32_t *__restrict__ err) {
    pdl_enter();
    extern __shared__ uint4 send_stage[];
    __shared__ int32_t cnt[kMaxRanks];
    if (threadIdx.x < G) cnt[threadIdx.x] = (int)__ldcg(sync + 2 * G + threadIdx.x);
    __syncthreads();
    const bool live = !(*reinterpret_cast<const volatile uint32_t *>(err) & kErrTimeout);
    const int lane = threadIdx.x & 31, warps = gridDim.x * kSendWarps, nch = D / 8;
    uint4 *stage = send_stage + (size_t)(threadIdx.x >> 5) * kSendSlots * nch;
    // a row's slot metadata (lane j < 8: local expert, position of its output row, weight); the
    // next row's is requested before the current row is processed, so the row's own chain is one
    // round trip (its output rows)
    const int rows = G * cap;
    auto fetch = [&](int r, int &id, int &ps, float &pr) {
        id = E_l;
        ps = 0;
        pr = 0.f;
        if (r < rows && lane < 8) {
            id = ids_local[(size_t)r * 8 + lane];
            ps = route_pos[(size_t)r * 8 + lane];
            pr = __ldcg(&meta[r].probs[lane]);
        }
    };
    int c_id, c_pos;
    float c_p;
    fetch(blockIdx.x * kSendWarps + (threadIdx.x >> 5), c_id, c_pos, c_p);
    for (int i = blockIdx.x * kSendWarps + (threadIdx.x >> 5); live && i < rows; i += warps) {
        int n_id, n_pos;
        float n_p;
        fetch(i + warps, n_id, n_pos, n_p);
        const int s = i / cap, k = i - s * cap;
        const bool mine = k < cnt[s] && lane < 8 && c_id < E_l;
        const int pos = mine ? c_pos : 0;
        const float p = mine ? c_p : 0.f;
        c_id = n_id;
        c_pos = n_pos;
        c_p = n_p;
        const uint32_t slots = __ballot_sync(kFull, mine);
        if (!slots) continue;  // no expert of this rank: the row was not sent here
        float o[8][8];
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
#pragma unroll
            for (int m = 0; m < 8; ++m) o[cc][m] = 0.f;
        uint32_t left = slots;
        while (left) {
            // the next (up to) kSendSlots local slots, ascending
            int js[kSendSlots];
            int ng = 0;
#pragma unroll
            for (int q = 0; q < kSendSlots; ++q) {
                js[q] = left ? __ffs(left) - 1 : 0;
                if (left) {
                    left &= left - 1;
                    ++ng;
                }
            }
#pragma unroll
            for (int q = 0; q < kSendSlots; ++q) {
                const int r = __shfl_sync(kFull, pos, js[q]);
                if (q < ng) {
                    const uint16_t *src = yp + (size_t)r * D;
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        const int c = lane + 32 * cc;
                        if (c < nch) cp_async_16(stage + q * nch + c, src + c * 8, true);
                    }
                }
            }
            cp_async_commit();
            cp_async_wait<0>();
#pragma unroll
            for (int q = 0; q < kSendSlots; ++q) {
                const float pj = __shfl_sync(kFull, p, js[q]);
                if (q >= ng) continue;
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    const int c = lane + 32 * cc;
                    if (c >= nch) continue;
                    const uint4 v = stage[q * nch + c];
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int m = 0; m < 8; ++m) {
                        const float prod = pj * ((m & 1) ? bf16_hi(w[m >> 1]) : bf16_lo(w[m >> 1]));
                        o[cc][m] = o[cc][m] + prod;
                    }
                }
            }
        }
        uint4 *dst = reinterpret_cast<uint4 *>(peers.back[s] + ((size_t)rank * cap + k) * D);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const int c = lane + 32 * cc;
            if (c >= nch) continue;
            uint4 r;
            r.x = pack_bf16x2(o[cc][0], o[cc][1]);
            r.y = pack_bf16x2(o[cc][2], o[cc][3]);
            r.z = pack_bf16x2(o[cc][4], o[cc][5]);
            r.w = pack_bf16x2(o[cc][6], o[cc][7]);
            dst[c] = r;
        }
    }
    ep_signal(ticket, peers, G, G + rank, 0, -1);
}

// Owner, one CTA of 256 threads per local token: waits for every rank's partial rows, then
// out[t] = sigmoid(gate_t) * ys[t] + sum over the ranks d (ascending) that own one of t's experts
// of back[d][t];
// resid[t] += out; and, when norm_w is given, the next layer's input row h[t] = bf16(resid[t] *
// rsqrt(mean(resid[t]^2) + eps) * norm_w) (gpu_graph.mm:48-61).
__global__ void __launch_bounds__(256)
ep_combine_kernel(const uint16_t *__restrict__ back, const int32_t *__restrict__ ids, int E_l, int G, int cap,
                  const uint32_t *__restrict__ sync, uint32_t target, EpPeers peers, const uint16_t *__restrict__ ys,
                  const float *__restrict__ gate_logit, int D, float *__restrict__ resid,
                  const float *__restrict__ norm_w, float eps, uint16_t *__restrict__ h, uint32_t *__restrict__ err) {
    pdl_enter();
    __shared__ int ok;
    __shared__ float part[8];
    if (threadIdx.x == 0) ok = ep_wait_counters(sync + G, G, target, sync + 3 * G, peers, err);
    __syncthreads();
    if (!ok) return;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float g = sigmoid_ref(gate_logit[t]);
    uint32_t dests = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) dests |= 1u << (__ldg(ids + (size_t)t * 8 + j) / E_l);
    int32_t row[kMaxRanks];
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d) row[d] = (d < G && ((dests >> d) & 1u)) ? t : -1;
    float r[1][8];  // D <= 2048: one chunk of 8 per thread
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 1; ++k) {
        const int c = (tid + k * 256) * 8;
        if (c >= D) break;
        float o[8];
        {
            const uint4 v = *reinterpret_cast<const uint4 *>(ys + (size_t)t * D + c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = ((j & 1) ? bf16_hi(w[j >> 1]) : bf16_lo(w[j >> 1])) * g;
        }
#pragma unroll
        for (int d = 0; d < kMaxRanks; ++d) {
            if (row[d] < 0) continue;
            const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(back + ((size_t)d * cap + row[d]) * D + c));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int m = 0; m < 8; ++m) o[m] = o[m] + ((m & 1) ? bf16_hi(w[m >> 1]) : bf16_lo(w[m >> 1]));
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
    for (int i = 0; i < 8; ++i) tot += part[i];
    const float scale = 1.0f / sqrtf(tot / (float)D + eps);
#pragma unroll
    for (int k = 0; k < 1; ++k) {
        const int c = (tid + k * 256) * 8;
        if (c >= D) break;
        const float4 w0 = *reinterpret_cast<const float4 *>(norm_w + c), w1 = *reinterpret_cast<const float4 *>(norm_w + c + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint4 o;
        o.x = pack_bf16x2(r[k][0] * scale * wv[0], r[k][1] * scale * wv[1]);
        o.y = pack_bf16x2(r[k][2] * scale * wv[2], r[k][3] * scale * wv[3]);
        o.z = pack_bf16x2(r[k][4] * scale * wv[4], r[k][5] * scale * wv[5]);
        o.w = pack_bf16x2(r[k][6] * scale * wv[6], r[k][7] * scale * wv[7]);
        *reinterpret_cast<uint4 *>(h + (size_t)t * D + c) = o;
    }
}

}  // namespace di
