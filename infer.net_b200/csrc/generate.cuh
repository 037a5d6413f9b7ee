// Seeded synthetic inputs generated on the device, bit-identical to the test oracle's host
// generator: splitmix64 counter hash -> Irwin-Hall of four 16-bit uniforms (integer sum,
// exact int->f32, one f32 multiply), then the min/max affine group-64 quantiser with bf16
// scale = (max-min)/(2^b-1), bias = min and q = clamp(rint((w-bias)/scale)).
#pragma once
#include "common.cuh"

namespace di {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return mix64(seed ^ mix64(stream * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull));
}
__device__ __forceinline__ float normal_sample(uint64_t base, uint64_t index, float scale) {
    const uint64_t h = mix64(base + index);
    const int32_t s = (int32_t)(h & 0xffff) + (int32_t)((h >> 16) & 0xffff) + (int32_t)((h >> 32) & 0xffff) +
                      (int32_t)(h >> 48);
    return __fmul_rn((float)(s - 131070), scale);
}

// One thread per 64-value group of one row.
// row_offset: stream row of the matrix's first row (expert shards start at first_expert * rows).
__global__ void gen_quant_kernel(uint64_t base, float scale, int64_t total_rows, int64_t row_offset, int cols, int bits,
                                 uint32_t *__restrict__ packed, uint16_t *__restrict__ scales,
                                 uint16_t *__restrict__ biases) {
    const int groups = cols / 64;
    const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gi >= total_rows * groups) return;
    const int64_t r = gi / groups;
    const int g = gi % groups;
    float w[64];
    float lo, hi;
#pragma unroll
    for (int i = 0; i < 64; ++i) w[i] = normal_sample(base, (uint64_t)((r + row_offset) * cols + g * 64 + i), scale);
    lo = hi = w[0];
#pragma unroll
    for (int i = 1; i < 64; ++i) {
        lo = w[i] < lo ? w[i] : lo;
        hi = w[i] > hi ? w[i] : hi;
    }
    const float levels = (float)((1 << bits) - 1);
    const uint16_t sb = f32_to_bf16_bits(__fdiv_rn(__fsub_rn(hi, lo), levels));
    const uint16_t bb = f32_to_bf16_bits(lo);
    const float s = bf16_bits_to_f32(sb), b = bf16_bits_to_f32(bb);
    scales[r * groups + g] = sb;
    biases[r * groups + g] = bb;
    // codes of this group: 64*bits bits = 16 (8-bit) or 10 (5-bit) whole words
    uint32_t words[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) words[i] = 0;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        float q = s > 0.0f ? rintf(__fdiv_rn(__fsub_rn(w[i], b), s)) : 0.0f;
        q = q < 0.0f ? 0.0f : (q > levels ? levels : q);
        const uint32_t qi = (uint32_t)q;
        const int bit = i * bits, at = bit >> 5, sh = bit & 31;
        words[at] |= qi << sh;
        if (sh + bits > 32) words[at + 1] |= qi >> (32 - sh);
    }
    const int wpg = 2 * bits;  // words per group
    uint32_t *dst = packed + r * (cols * bits / 32) + g * wpg;
    for (int i = 0; i < wpg; ++i) dst[i] = words[i];
}

}  // namespace di
