// Expert-parallel dispatch / combine helpers (one process per GPU, NCCL between them).
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
#include "route.cuh"

namespace di {

constexpr int kMaxRanks = 8;

struct RowMeta {
    int32_t ids[8];
    float probs[8];
};

// Single CTA of 1024 threads: for every local token t and GPU d, send_idx[t*G + d] = position
// of t among the tokens sent to d (or -1), send_count[d], send_off[d] (exclusive scan).
__global__ void __launch_bounds__(1024)
ep_layout_kernel(const int32_t *__restrict__ ids, int T, int E_l, int G, int32_t *__restrict__ send_idx,
                 int32_t *__restrict__ send_count, int32_t *__restrict__ send_off) {
    __shared__ int32_t part[1024][kMaxRanks + 1];
    const int tid = threadIdx.x;
    const int per = (T + 1023) / 1024, t0 = tid * per, t1 = min(t0 + per, T);
    int cnt[kMaxRanks] = {};
    for (int t = t0; t < t1; ++t) {
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) mask |= 1u << (ids[(size_t)t * 8 + j] / E_l);
        for (int d = 0; d < G; ++d) cnt[d] += (mask >> d) & 1u;
    }
    for (int d = 0; d < G; ++d) part[tid][d] = cnt[d];
    __syncthreads();
    if (tid < G) {  // exclusive scan over threads, per destination
        int run = 0;
        for (int i = 0; i < 1024; ++i) {
            const int v = part[i][tid];
            part[i][tid] = run;
            run += v;
        }
        send_count[tid] = run;
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int d = 0; d < G; ++d) {
            send_off[d] = run;
            run += send_count[d];
        }
    }
    int pos[kMaxRanks];
    for (int d = 0; d < G; ++d) pos[d] = part[tid][d];
    for (int t = t0; t < t1; ++t) {
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) mask |= 1u << (ids[(size_t)t * 8 + j] / E_l);
        for (int d = 0; d < G; ++d) send_idx[(size_t)t * G + d] = ((mask >> d) & 1u) ? pos[d]++ : -1;
    }
}

// One CTA per local token: copies h[t] and its routing metadata into each destination's block
// of the send buffers (row send_off[d] + send_idx[t, d]).
__global__ void __launch_bounds__(256)
ep_pack_kernel(const uint16_t *__restrict__ h, const int32_t *__restrict__ ids, const float *__restrict__ probs, int D,
               int G, const int32_t *__restrict__ send_idx, const int32_t *__restrict__ send_off,
               uint16_t *__restrict__ send_x, RowMeta *__restrict__ send_meta) {
    const int t = blockIdx.x;
    for (int d = 0; d < G; ++d) {
        const int k = send_idx[(size_t)t * G + d];
        if (k < 0) continue;
        const size_t row = (size_t)send_off[d] + k;
        const uint4 *src = reinterpret_cast<const uint4 *>(h + (size_t)t * D);
        uint4 *dst = reinterpret_cast<uint4 *>(send_x + row * D);
        for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = src[i];
        if (threadIdx.x < 8) {
            send_meta[row].ids[threadIdx.x] = ids[(size_t)t * 8 + threadIdx.x];
            send_meta[row].probs[threadIdx.x] = probs[(size_t)t * 8 + threadIdx.x];
        }
    }
}

// Receiver: local expert of every (row, slot) -- or E_l for a slot owned by another GPU -- and
// the per-block histogram over E_l + 1 buckets (blocks of topk::TOK_PER_CTA rows).
__global__ void __launch_bounds__(256)
ep_recv_count_kernel(const RowMeta *__restrict__ meta, int R, int E_off, int E_l, int32_t *__restrict__ ids_local,
                     int32_t *__restrict__ block_counts) {
    __shared__ int32_t hist[kMaxBuckets];
    for (int i = threadIdx.x; i <= E_l; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int r0 = blockIdx.x * topk::TOK_PER_CTA * 8;
    for (int r = r0 + threadIdx.x; r < min(r0 + topk::TOK_PER_CTA * 8, R * 8); r += blockDim.x) {
        const int e = meta[r >> 3].ids[r & 7] - E_off;
        const int b = (e >= 0 && e < E_l) ? e : E_l;
        ids_local[r] = b;
        atomicAdd(&hist[b], 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i <= E_l; i += blockDim.x) block_counts[(size_t)blockIdx.x * (E_l + 1) + i] = hist[i];
}

// Receiver: z[i] = sum over local slots j (slot order) of p[i,j] * y[8i+j], f32 then bf16; the
// expert rows are stored in expert order, y[8i+j] = yp[route_pos[8i+j]].
__global__ void ep_reduce_kernel(const uint16_t *__restrict__ yp, const int32_t *__restrict__ route_pos,
                                 const int32_t *__restrict__ ids_local,
                                 const RowMeta *__restrict__ meta, int R, int D, int E_l, uint16_t *__restrict__ z) {
    const int per_row = D / 8;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)R * per_row) return;
    const int i = idx / per_row, c = (idx % per_row) * 8;
    float o[8] = {};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (ids_local[(size_t)i * 8 + j] >= E_l) continue;
        const float p = meta[i].probs[j];
        const uint4 v = *reinterpret_cast<const uint4 *>(yp + (size_t)route_pos[(size_t)i * 8 + j] * D + c);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float prod = p * ((k & 1) ? bf16_hi(w[k >> 1]) : bf16_lo(w[k >> 1]));
            o[k] = o[k] + prod;
        }
    }
    uint4 r;
    r.x = pack_bf16x2(o[0], o[1]);
    r.y = pack_bf16x2(o[2], o[3]);
    r.z = pack_bf16x2(o[4], o[5]);
    r.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4 *>(z + (size_t)i * D + c) = r;
}

// Owner: out[t] = sigmoid(gate_t) * ys[t] + sum_d back[send_off[d] + send_idx[t, d]] (ascending
// d); resid[t] += out.
__global__ void ep_combine_kernel(const uint16_t *__restrict__ back, const int32_t *__restrict__ send_idx,
                                  const int32_t *__restrict__ send_off, int G, const uint16_t *__restrict__ ys,
                                  const float *__restrict__ gate_logit, int T, int D, float *__restrict__ resid,
                                  const uint32_t *__restrict__ err) {
    const int per_tok = D / 8;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)T * per_tok) return;
    if (*err) return;
    const int t = idx / per_tok, c = (idx % per_tok) * 8;
    const float g = sigmoid_ref(gate_logit[t]);
    float o[8];
    {
        const uint4 v = *reinterpret_cast<const uint4 *>(ys + (size_t)t * D + c);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = ((k & 1) ? bf16_hi(w[k >> 1]) : bf16_lo(w[k >> 1])) * g;
    }
    for (int d = 0; d < G; ++d) {
        const int k = send_idx[(size_t)t * G + d];
        if (k < 0) continue;
        const uint4 v = *reinterpret_cast<const uint4 *>(back + ((size_t)send_off[d] + k) * D + c);
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
}

}  // namespace di
