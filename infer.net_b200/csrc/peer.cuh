// Peer-memory plumbing of the expert-parallel path: the symmetric buffers every rank maps from
// every other rank (CUDA IPC over NVLink), the routing metadata that travels with a token row, and
// the bounded arrival counters by which writing kernels signal the readers of a layer step.
#pragma once
#include "common.cuh"

namespace di {

constexpr int kMaxRanks = 8;

struct RowMeta {
    int32_t ids[8];
    float probs[8];
};

// Symmetric buffers of one rank, mapped into every rank of the group (CUDA IPC over NVLink).
// Region s of a buffer holds what rank s wrote into it, row k = rank s's local token k (rows are
// not compacted: a token's row slot is the same in every destination, so no send layout is built):
//   rx   [G][cap][D] bf16   token rows dispatched to this rank (written only where the token has
//                           an expert here)
//   meta [G][cap]           expert ids and probabilities of every token of rank s (written for
//                           every token, so that rows without a local expert read as such)
//   back [G][cap][D] bf16   partial rows returned to this rank (for the tokens it sent out)
//   sync [4G+2] u32         [0,G) dispatch arrivals from rank s, [G,2G) combine arrivals,
//                           [2G,3G) token counts of rank s, [3G] abort word, [3G+1], [3G+2]
//                           this rank's CTA tickets of its dispatch and of its partial-row send
// A writing kernel signals every rank once per layer step: after a CTA barrier one thread fences
// at system scope (cumulative over the CTA's stores, which the barrier orders before it) and takes
// a ticket; the last CTA writes the token count (dispatch), fences, and bumps the arrival counter of
// every rank, so after step n it reads n. The last CTA also resets its ticket.
struct EpPeers {
    uint16_t *rx[kMaxRanks];
    RowMeta *meta[kMaxRanks];
    uint16_t *back[kMaxRanks];
    uint32_t *sync[kMaxRanks];
};

// Thread 0 of a CTA: wait until counters ctr[0..G) all reach `target`. Fails fast on an earlier
// timeout of this rank or an abort written by another rank; on its own timeout it sets the error
// word and writes the abort word of every rank.
__device__ inline bool ep_wait_counters(const uint32_t *ctr, int G, uint32_t target, const uint32_t *abort_word,
                                        const EpPeers &peers, uint32_t *err) {
    const uint64_t t0 = global_ns();
    for (int s = 0; s < G; ++s) {
        const volatile uint32_t *c = ctr + s;
        for (uint32_t n = 0;; ++n) {
            if ((int)(*c - target) >= 0) break;
            if ((n & 63u) == 0) {
                if ((*reinterpret_cast<const volatile uint32_t *>(err) & kErrTimeout) ||
                    *reinterpret_cast<const volatile uint32_t *>(abort_word)) {
                    atomicOr(err, kErrTimeout);
                    return false;
                }
                if (global_ns() - t0 > kWaitLimitNs) {
                    atomicOr(err, kErrTimeout);
                    for (int q = 0; q < G; ++q) atomicExch_system(peers.sync[q] + 3 * G, 1u);
                    return false;
                }
            }
        }
    }
    __threadfence();
    return true;
}

// Last-CTA signal of a writing kernel (all threads call it after their stores): arrival counter
// `slot` of every rank + 1; the dispatch also publishes its token count (count >= 0).
__device__ inline void ep_signal(uint32_t *ticket, const EpPeers &peers, int G, int slot, int count_slot,
                                 int count) {
    __shared__ uint32_t last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) {
        *ticket = 0;  // the next launch counts from zero (launches on one stream do not overlap)
        __threadfence_system();
        if (count >= 0)
            for (int q = 0; q < G; ++q) peers.sync[q][count_slot] = (uint32_t)count;
        __threadfence_system();
        for (int q = 0; q < G; ++q) atomicAdd_system(peers.sync[q] + slot, 1u);
    }
}

}  // namespace di
