/*
 * CPU oracle for the Qwen3.6-35B-A3B MoE feed-forward block (TEST INFRASTRUCTURE).
 *
 * This library is the parity checker and the timed CPU baseline ("port") only.
 * Nothing in the product path (infer.net_b200/) links, loads or calls it; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs do.
 *
 * It restates the reference's arithmetic for the block:
 *   - affine g64 dequant w = q*scale + bias, bf16 -> f32 by <<16
 *       (native/DeepInfer.Metal/quantized.mm:62-82, :384-397;
 *        native/DeepInfer.Cuda/split_prefix.cu:60, :84-87)
 *   - MLX LSB-first packing with codes crossing 32-bit words
 *       (tests/DeepInfer.Tests/QuantizedTests.cs:155-161)
 *   - the GEMV lane partition and xor-butterfly reduction of the reference CUDA
 *     gemv kernel (native/DeepInfer.Cuda/split_prefix.cu:63-67, :106-120), with
 *     nvcc's multiply-add contraction written out as fmaf
 *   - SelectExperts: top-8 by strict '>' insertion (ties -> lower expert id),
 *     non-finite logits rejected, softmax over the 8 chosen logits
 *       (src/DeepInfer.Backends/Models/Qwen36Model.cs:246-262, :293-298)
 *   - Moe: shared SwiGLU, sigmoid-gated shared output, p-weighted expert sum
 *       (src/DeepInfer.Backends/Models/Qwen36Model.cs:218-245, :272-287)
 *   - stable expert-grouped permutation of routes r = t*8+slot
 *       (native/DeepInfer.Metal/prefill_moe.mm:8-17)
 *   - residual + RMSNorm between stacked layers
 *       (native/DeepInfer.Metal/gpu_graph.mm:48-61; Qwen36Model.cs:142-144, :288-292)
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const uint32_t *packed;   /* [experts, rows, cols*bits/32] */
    const uint16_t *scales;   /* [experts, rows, cols/64] bf16 */
    const uint16_t *biases;   /* [experts, rows, cols/64] bf16 */
    int32_t experts, rows, cols, bits;
} oc_qmatrix;

typedef struct {
    oc_qmatrix router;        /* [1, E, D] 8-bit */
    oc_qmatrix gate, up;      /* [E, I, D] */
    oc_qmatrix down;          /* [E, D, I] */
    oc_qmatrix shared_gate;   /* [1, I, D] */
    oc_qmatrix shared_up;     /* [1, I, D] */
    oc_qmatrix shared_down;   /* [1, D, I] */
    oc_qmatrix shared_route;  /* [1, 1, D] 8-bit */
    const float *router_bias; /* optional [E] added to the logits (Zipf config), may be NULL */
} oc_layer;

/* arithmetic modes of oc_moe_block */
enum {
    OC_MODE_F32 = 0,      /* reference semantics: f32 weights/activations, canonical f32 GEMV order */
    OC_MODE_F64 = 1,      /* same dataflow with every dot product in double (tolerance anchor) */
    OC_MODE_BF16OPS = 2   /* tensor-core data path: bf16-rounded weights, bf16 act and bf16 expert rows,
                             double accumulation (tight check of the grouped GEMM kernels) */
};

int oc_abi_version(void);

/* bf16 helpers */
float oc_bf16_to_f32(uint16_t h);
uint16_t oc_f32_to_bf16(float f);

/* seeded synthetic generator (identical bits on host and device) */
uint64_t oc_mix64(uint64_t z);
uint64_t oc_stream_base(uint64_t seed, uint64_t stream);
float oc_normal_scale(float stddev);
float oc_normal(uint64_t base, uint64_t index, float scale);
void oc_gen_bf16(uint64_t seed, uint64_t stream, int64_t n, float stddev, uint16_t *out);
void oc_gen_quant_matrix(uint64_t seed, uint64_t stream, int experts, int rows, int cols, int bits,
                         float stddev, uint32_t *packed, uint16_t *scales, uint16_t *biases);
void oc_quantize_rows(const float *w, int64_t rows, int cols, int bits,
                      uint32_t *packed, uint16_t *scales, uint16_t *biases);

/* dequant and GEMV */
uint32_t oc_code(const oc_qmatrix *m, int expert, int row, int col);
float oc_weight(const oc_qmatrix *m, int expert, int row, int col);
float oc_dot_canonical(const oc_qmatrix *m, int expert, int row, const float *x);
double oc_dot_f64(const oc_qmatrix *m, int expert, int row, const float *x, int bf16_weights);
void oc_gemv(const oc_qmatrix *m, const float *x, float *y, const int32_t *experts, int count,
             int batched, int mode);

/* routing */
int oc_select_experts(const float *logits, int n_experts, int32_t *ids, float *probs);
int oc_force_route(const float *logits, const int32_t *forced, int32_t *ids, float *probs);
void oc_permute(const int32_t *ids, int tokens, int n_experts, int32_t *counts, int32_t *offsets,
                int32_t *routes);

/* the block: x bf16 [T, D] -> out f32 [T, D]; ids [T,8]; probs [T,8]; logits optional [T, E+1]
   (column E holds the shared-route gate logit). forced_ids optional [T,8]. Returns 0, or -1 on
   non-finite router logits (outputs then unspecified). */
int oc_moe_block(const oc_layer *L, const uint16_t *x, int T, int mode, const int32_t *forced_ids,
                 float *out, int32_t *ids, float *probs, float *logits, int threads);

/* residual stack: x f32 [T, D] updated in place through n layers:
   h = RMSNorm(x)*norm_w[l] rounded to bf16; x += moe_l(h).  norms: [n, D] f32. */
int oc_moe_stack(const oc_layer *layers, const float *norms, int n_layers, float eps, float *x, int T,
                 int mode, int32_t *ids_out, int threads);

/* RMSNorm of one row rounded to bf16 (gpu_graph.mm:48-61 arithmetic, single accumulator) */
void oc_rmsnorm_bf16(const float *x, const float *w, int D, float eps, uint16_t *out);

/* CPU baseline in the reference's CPU loop shape (cpu_block.c): one Vector<float> accumulator per
   GEMV row (CpuMatrix.Multiply, MatVec.cs:44-54) with the weights dequantised per 64-group, the
   router in the canonical order (ids equal oc_moe_block's), SIMD width chosen at run time. */
typedef struct oc_cpu_layer oc_cpu_layer;
oc_cpu_layer *oc_cpu_prepare(const oc_layer *L);  /* keeps pointers into L's matrices */
void oc_cpu_release(oc_cpu_layer *P);
const char *oc_cpu_isa(void);                     /* "avx512", "avx2" or "scalar" */
int oc_cpu_block(const oc_cpu_layer *P, const uint16_t *x, int T, float *out, int32_t *ids, float *probs,
                 int threads);
int oc_cpu_stack(const oc_cpu_layer *const *P, const float *norms, int n_layers, float eps, float *x, int T,
                 int32_t *ids_out, int threads);

#ifdef __cplusplus
}
#endif
#endif
