// Shared device helpers for the MoE block kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "deepinfer_cuda targets sm_100a (B200) only"
#endif

namespace di {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// Device-side error word bits, copied back by the host after each call.
enum : uint32_t {
    kErrNonFinite = 1u,     // a router logit was NaN/Inf (Qwen36Model.cs:252)
    kErrBadExpert = 2u,     // forced route id out of range
    kErrCapacity = 4u,      // internal work list overflow (host sizing bug)
    kErrTimeout = 8u,       // a bounded device-side wait ran out
    kErrRange = 16u,        // a one-token stack output outside its fixed-point accumulator's range
};

// Geometry of one quantised matrix as the kernels see it.
struct QView {
    const uint32_t *packed;
    const uint16_t *scales;
    const uint16_t *biases;
    int experts, rows, cols, bits;
    __host__ __device__ int words_per_row() const { return cols * bits / 32; }
    __host__ __device__ int groups_per_row() const { return cols / 64; }
};

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xffff0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// Integer code 0..255 -> exact float: 0x4B0000qq is 2^23 + q, subtracting 2^23 is exact.
__device__ __forceinline__ float byte_to_f32(uint32_t word, int i) {
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u + i)) - 8388608.0f;
}
__device__ __forceinline__ float code_to_f32(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

// Code `col` of a packed row, LSB-first across 32-bit words (quantized.mm:62-67).
__device__ __forceinline__ uint32_t load_code(const uint32_t *row_words, int col, int bits) {
    int bit = col * bits, at = bit >> 5, shift = bit & 31;
    uint32_t q = __ldg(row_words + at) >> shift;
    if (shift + bits > 32) q |= __ldg(row_words + at + 1) << (32 - shift);
    return q & ((1u << bits) - 1u);
}

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_ref(float x) { return x * sigmoid_ref(x); }

__device__ __forceinline__ float warp_sum_butterfly(float v) {
    // xor butterfly 16,8,4,2,1 (split_prefix.cu:63-67); every lane ends with the same bits
#pragma unroll
    for (int n = 16; n; n >>= 1) v += __shfl_xor_sync(kFull, v, n);
    return v;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

// ------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization may be
// scheduled before its predecessor on the stream has finished; pdl_enter(), executed by every
// thread before it touches global memory, waits until the predecessor grid has completed with its
// memory visible (which covers every earlier kernel of the stream), and lets this grid's successor
// be scheduled once every CTA of this grid has started. Both are no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
    pdl_wait();
    pdl_trigger();
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: every spin ends after ~2 s of wall time (checked on %globaltimer every 256
// polls). On timeout the thread records an error bit and reports failure; callers then skip
// their remaining work and exit cleanly, so a broken pipeline can never hang the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's global accesses of the async proxy (bulk copies, reductions) with its
// later generic ones.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bulk reduction: dst[i] += src[i] for `bytes` / 8 unsigned 64-bit words, performed at L2 by the
// copy engine (both addresses 16-byte aligned, bytes a multiple of 16); tracked by this thread's
// bulk async-groups.
__device__ __forceinline__ void bulk_reduce_add_u64(void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.u64 [%0], [%1], %2;" ::"l"(
                     __cvta_generic_to_global(dst)),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}
// Acquire load at device scope: later loads of this thread (and, through a CTA barrier, of the
// CTA) see every write that preceded the release it reads from.
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Release reduction at device scope: every write ordered before it (this thread's, and the CTA's
// through a preceding barrier) is visible to a reader that acquires the new value.
__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// A 16-bit load (zero-extended into a 32-bit register, so no instruction touches the value until
// it is used) through the read-only path that the compiler may not move or merge: its latency
// overlaps whatever runs until then.
__device__ __forceinline__ uint32_t ld_nc_u16(const uint16_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ void cp_async_16(void *smem_dst, const void *gmem_src, bool valid) {
    uint32_t n = valid ? 16u : 0u;  // src-size 0 zero-fills the 16 bytes
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_8(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_4(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
// Arrive on an mbarrier once every cp.async this thread issued so far has completed; the
// arrival counts toward the barrier's expected count (no pending-count increment).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------ bulk / tensor copies (TMA)

// Arrive on `bar` and raise its expected transaction bytes by `bytes`.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Contiguous global -> shared copy; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(__cvta_generic_to_global(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Asynchronous L2 prefetch of a contiguous global range (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(__cvta_generic_to_global(p)), "r"(bytes)
                 : "memory");
}
// 2-D tiled tensor store of the map's box at (x, y) from shared memory (128-byte aligned),
// tracked by this thread's bulk async-groups.
__device__ __forceinline__ void tma_store_2d(const void *map, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
                 "r"(y), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// 2-D tiled tensor copy of the map's box at (x, y); x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Four rows r0..r3 of a 2-D map with a one-row box, columns [x, x + box width), stored back to
// back at dst.
__device__ __forceinline__ void tma_gather4(void *dst, const void *map, int x, int r0, int r1, int r2, int r3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_nc_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_nc_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t *p) { return __ldg(p); }

// ------------------------------------------------------------------ tcgen05 wrappers

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, f32 accumulate, issued by one thread.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once all prior tcgen05 ops of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns starting at taddr (warp w reads lanes 32*(w%4)..).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------------ CTA pairs (cluster of 2)
//
// The pair forms of the tcgen05 operations: one MMA issued by the even CTA of a 2-CTA cluster
// computes a 256-row tile whose A rows and B columns are split between the two CTAs' shared memory
// and whose accumulator rows are split between their tensor memories (cta_group::2). Every tcgen05
// operation of a kernel that uses them must use the pair form.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// The shared::cluster address of the variable at this CTA's shared address `p` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrive on an mbarrier of a CTA of the cluster, releasing at cluster scope: every write of this
// thread (and, through a preceding warp or CTA barrier, of its warp or CTA) is visible to a thread
// of the cluster that acquires the phase.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// mbar_wait with acquire at cluster scope (phases completed by the other CTA of a pair).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, code);
            return false;
        }
    }
}
// Bulk copy of `bytes` from this CTA's shared memory into another CTA's (shared::cluster addresses
// of the destination and of an mbarrier there, whose transaction count it completes).
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, const void *src, uint32_t bytes,
                                                     uint32_t bar_cluster) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst_cluster),
                 "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
                 : "memory");
}
// Named barrier among `count` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Every thread of both CTAs: a cluster-wide barrier (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[both CTAs' smem] * B[both CTAs' smem]^T; issued by the even CTA only.
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the mbarrier at the same shared offset in each CTA of `mask` once all prior pair MMAs
// of this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}
// 2-D tensor copy into this CTA's shared memory whose completion is counted on an mbarrier of either
// CTA of the pair (its shared::cluster address); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 128 bytes,
// 8-row atoms 1024 bytes apart (SBO), tile base 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;              // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset
    d |= (uint64_t)1u << 46;              // descriptor version for tcgen05
    d |= (uint64_t)2u << 61;              // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
    return r * 128u + ((c ^ (r & 7u)) << 4);
}

}  // namespace di
