/*
 * deepinfer_cuda -- B200 (sm_100a) backend for the Qwen3.6-35B-A3B MoE feed-forward block.
 *
 * Plain C ABI: opaque handles, plain pointers and sizes, UTF-8 error text written into a
 * caller buffer (error, capacity). Every call validates all of its arguments before any
 * GPU work; an invalid call returns NULL / a nonzero status, submits nothing and leaves
 * every output untouched (native/DeepInfer.Metal/quantized.mm:323-331, :354-361).
 * Calls are synchronous: outputs are visible on return, and `ms` receives the GPU time
 * of the call's work measured with CUDA events (quantized.mm:215-229).
 * One context owns one CUDA stream on the device that was current at creation; a
 * context is not thread-safe (callers serialise per model, Qwen36Model.cs:18, :47-53).
 *
 * Part 1 replaces the managed QuantNative table (src/DeepInfer.Backends/Compute/
 * QuantizedMetal.cs:242-274, bound to native/DeepInfer.Metal/quantized.mm:241-397).
 * Part 2 adds batched entries for the whole block (router -> top-8 -> permute -> grouped
 * expert GEMMs -> shared expert -> combine); they replace the MoE part of
 * di_graph_forward / di_graph_prefill (gpu_graph.mm:307-320, gpu_prefill.mm:700-706).
 */
#ifndef DEEPINFER_CUDA_H
#define DEEPINFER_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DI_ABI_VERSION 1

/* ABI version probe; the C# loader checks it like di_cuda_prefix_abi_version
   (native/DeepInfer.Cuda/split_prefix.cu:14, src/DeepInfer.Backends/Split/SplitSessions.cs:66). */
int di_abi_version(void);

/* ------------------------------------------------------------------------------------
 * Part 1. Quantised GEMV operators (drop-in for QuantNative / deepinfer_metal).
 * Matrices are [experts, rows, columns] affine group-64 stacks in MLX layout:
 *   index 0 packed  uint32 [experts, rows, columns*bits/32], codes LSB-first, crossing words
 *   index 1 scales  bf16   [experts, rows, columns/64]
 *   index 2 biases  bf16   [experts, rows, columns/64]
 * and dequantise as w = q*scale + bias (quantized.mm:62-82).
 * ---------------------------------------------------------------------------------- */

/* QuantNative.Job (QuantizedMetal.cs:250-258; quantized.mm:24-30). Host float arrays. */
typedef struct di_quant_job {
    void *matrix;
    const float *input;       /* columns floats, or count*columns when batched */
    float *output;            /* count*rows floats */
    const uint32_t *experts;  /* count expert ids */
    int32_t count, batched;
} di_quant_job;

/* di_quant_create (quantized.mm:282-286; QuantizedMetal.cs:264). Reads DEEPINFER_CUDA_RESIDENCY
   and DEEPINFER_CUDA_RESIDENCY_REFRESH_MS like the Metal variant reads its residency variables. */
void *di_quant_create(char *error, int capacity);
/* di_quant_create_configured (quantized.mm:242-280; QuantizedMetal.cs:244-245). resident must be
   0 or 1 and refresh_ms in [0, 60000]. Weights are always device-resident on CUDA; resident=1
   additionally accounts them in di_quant_residency_bytes. */
void *di_quant_create_configured(int resident, int refresh_ms, char *error, int capacity);
void di_quant_destroy(void *ctx);                               /* quantized.mm:293 */
uint64_t di_quant_residency_bytes(void *ctx);                   /* quantized.mm:287-289 */
/* Uploads every host-staged weight buffer and waits (quantized.mm:290-292). */
void di_quant_residency_prepare(void *ctx);

/* quantized.mm:294-315: experts 1..256, rows >= 1, columns % 64 == 0, bits 5 or 8, group 64. */
void *di_quant_matrix_create(void *ctx, int experts, int rows, int columns, int bits, int group,
                             char *error, int capacity);
/* quantized.mm:316-319. Returns a HOST-writable staging buffer (pinned) for index 0/1/2 that the
   caller fills (QuantizedMetal.cs:162-177); its contents are uploaded to the device before the
   next compute call or at di_quant_residency_prepare. NULL for a bad index. */
void *di_quant_matrix_buffer(void *matrix, int index);
void di_quant_matrix_destroy(void *matrix);                     /* quantized.mm:320 */

/* quantized.mm:321-345: 1..8 independent GEMV jobs on distinct matrices, one submission. */
int di_quant_batch(void *ctx, const di_quant_job *jobs, int count, double *ms, char *error, int capacity);
/* quantized.mm:346-349 */
int di_quant_matvec(void *ctx, void *matrix, const float *x, float *y, const uint32_t *experts, int count,
                    int batched, double *ms, char *error, int capacity);
/* quantized.mm:350-383: gate/up -> SwiGLU -> down for `count` selected experts sharing `input`,
   plus the independent shared-expert down projection of `shared_input`. */
int di_quant_experts(void *ctx, void *gate, void *up, void *down, void *shared, const float *input,
                     const float *shared_input, const uint32_t *experts, int count, float *expert_output,
                     float *shared_output, double *ms, char *error, int capacity);
/* quantized.mm:384-397: dequantised row `token` of a one-expert matrix into out[columns]. */
int di_quant_embedding(void *matrix, int token, float *out);

/* Dense quantised projection of a token batch on the tensor cores: y[t, r] = sum_c x[t, c] *
   W[expert, r, c] for t < tokens, with bf16 operands (W dequantised as q*scale + bias and rounded
   to bf16) and f32 accumulation -- the arithmetic of the reference's batched prefill projections
   (native/DeepInfer.Metal/gpu_prefill.mm:603-614 with prefill_bf16.mm:47-53;
   native/DeepInfer.Cuda/prefill_batch.cuh:16-52), which serve every non-expert weight of a layer.
   x: bf16 [tokens, columns]; y: bf16 [tokens, rows]; host pointers, or device pointers with
   DI_MOE_DEVICE_IO (the only flag). Needs columns <= 2048 (a multiple of 128 for 5-bit) and rows
   a multiple of 8; expert in [0, experts). tokens in [1, 1048576]. */
int di_quant_gemm(void *ctx, void *matrix, int expert, const uint16_t *x, int tokens, uint16_t *y, int flags,
                  double *ms, char *error, int capacity);

/* Device-side access (no reference counterpart: Metal buffers are host-visible, CUDA device
   memory is not). The library does not see writes through this pointer: once it has been handed
   out for a router matrix, the tensor-core router recomputes that matrix's row norms on every call
   instead of keeping them per layer. */
void *di_quant_matrix_device_buffer(void *matrix, int index);
/* Copies `bytes` from host memory into buffer `index` (bytes must equal the buffer size). */
int di_quant_matrix_upload(void *matrix, int index, const void *src, uint64_t bytes, char *error, int capacity);
/* Fills the matrix with synthetic weights ~N(0, stddev) quantised by the min/max affine group-64
   rule, generated on the device bit-identically to the test oracle (seed, stream). Expert e of
   the matrix receives expert first_expert + e of the stream, so a GPU's expert shard equals the
   same experts of the full matrix. */
int di_quant_matrix_generate(void *matrix, uint64_t seed, uint64_t stream, float stddev, int first_expert,
                             char *error, int capacity);

/* ------------------------------------------------------------------------------------
 * Part 2. The MoE block.
 * A layer binds the eight matrices of one block (Qwen36Weights.cs:93-100):
 *   router [1,E,D] 8-bit, gate/up [E,I,D], down [E,D,I], shared_gate/shared_up [1,I,D],
 *   shared_down [1,D,I], shared_route [1,1,D] 8-bit; E in [8,256], D % 256 == 0, I % 64 == 0.
 * ---------------------------------------------------------------------------------- */

void *di_moe_layer_create(void *ctx, void *router, void *gate, void *up, void *down, void *shared_gate,
                          void *shared_up, void *shared_down, void *shared_route, char *error, int capacity);
void di_moe_layer_destroy(void *layer);
/* Optional per-expert logit bias (host f32[E]); NULL clears it. Used by the Zipf load config. */
int di_moe_layer_set_router_bias(void *layer, const float *bias, char *error, int capacity);

/* MLX checkpoints (Qwen36Weights.cs:55-100 over SafeTensors.cs:13-46): `directory` holds config.json
   (text_config: hidden_size, num_experts, moe_intermediate_size, num_experts_per_tok = 8,
   num_hidden_layers, norm_topk_prob; quantization: affine, group 64, 5 or 8 bits, per-matrix
   overrides), model.safetensors.index.json and the shards its weight_map names. Layer l's block
   is read from language_model.model.layers.{l}.mlp.gate (router, 8-bit), mlp.switch_mlp.{gate,up,
   down}_proj, mlp.shared_expert.{gate,up,down}_proj and mlp.shared_expert_gate (8-bit), each as
   .weight (U32 packed), .scales and .biases (BF16), and its RMSNorm weights from
   post_attention_layernorm.weight (BF16 or F32). Every header, dtype, shape, byte range and shard
   name is validated before anything is allocated or uploaded; a shard name must be a plain file
   name inside the directory. */
/* Validates layer `layer` of a checkpoint without a GPU; geometry receives {E, D, I, bits}. */
int di_moe_checkpoint_probe(const char *directory, int layer, int32_t *geometry, char *error, int capacity);
/* Loads and binds layer `layer`'s MoE block on ctx (the layer owns its eight matrices: destroy it
   with di_moe_layer_destroy); norm (optional, f32 [D]) receives the layer's RMSNorm weights. */
void *di_moe_layer_load(void *ctx, const char *directory, int layer, float *norm, char *error, int capacity);

/* flags for di_moe_block / di_moe_stack */
#define DI_MOE_DEVICE_IO 1      /* x, y, ids, probs (and norms/traces) are device pointers */
#define DI_MOE_FORCE_ROUTES 2   /* ids is an INPUT [T,8]: forced expert ids (gpu_graph.mm:153-159) */
#define DI_MOE_PATH_GEMV 4      /* force the decode GEMV path */
#define DI_MOE_PATH_GROUPED 8   /* force the grouped tensor-core path */
#define DI_MOE_PROFILE 16       /* di_moe_stack: record per-stage CUDA events (read by di_moe_last_profile) */
#define DI_MOE_ROUTER_EXACT 32  /* grouped path: every router logit in the canonical f32 order instead of
                                   tensor-core logits with an exact check of the near-boundary candidates
                                   (the same ids and probabilities; a checking aid, slower) */

/* y[t] = sigmoid(x_t . w_sr) * shared(x_t) + sum_j p[t,j] * expert_{ids[t,j]}(x_t)
   (Qwen36Model.cs:218-245). x: bf16 [T, D] (the normalised layer input); y: bf16 [T, D].
   ids (int32 [T,8]) and probs (f32 [T,8]) may be NULL unless DI_MOE_FORCE_ROUTES.
   Routing: 8 largest router logits in descending order, ties to the lower expert id,
   probs = softmax over the 8 (Qwen36Model.cs:246-262); a non-finite logit fails the call
   with "Non-finite router logits" and y is left untouched. T in [1, 65536]. */
int di_moe_block(void *ctx, void *layer, const uint16_t *x, int tokens, uint16_t *y, int32_t *ids, float *probs,
                 int flags, double *ms, char *error, int capacity);

/* n_layers stacked blocks over an f32 residual stream x [T, D] (in/out):
     h = bf16(RMSNorm(x) * norms[l]);  x += block_l(h)      (gpu_graph.mm:48-61)
   norms: f32 [n_layers, D]. h_trace (bf16 [n_layers, T, D]) and ids_trace (int32 [n_layers, T, 8])
   are optional per-layer dumps for teacher-forced checks. One token on the GEMV path runs the whole
   stack as one persistent kernel when the layers share D in {512, 1024, 2048}, I = 512 and E <= 256
   (its output is exact to 2^-32 per contribution; an output beyond its fixed-point range is
   recomputed by the per-layer kernels); other decode-sized T run as a CUDA graph of per-layer
   kernels. */
int di_moe_stack(void *ctx, void *const *layers, const float *norms, int n_layers, float eps, float *x, int tokens,
                 uint16_t *h_trace, int32_t *ids_trace, int flags, double *ms, char *error, int capacity);

/* Per-stage GPU milliseconds of the last di_moe_block (or profiled di_moe_stack, summed over its
   layers) on this context: [router, top8+count, scan, scatter, gate_up, down, combine, rmsnorm];
   returns the number written. */
int di_moe_last_profile(void *ctx, double *stage_ms, int n);

/* The expert-grouped permutation built by the last grouped-path di_moe_block on this context (for a
   stack: by its last layer), as prefill_build_groups orders it (native/DeepInfer.Metal/
   prefill_moe.mm:8-17): route r = t*8 + slot of expert e sits at position seg_offsets[e] + i, routes
   of one expert in ascending r. perm_route receives 8T route ids (max_routes >= 8T), seg_offsets and
   seg_counts E + 1 entries (entry E is the shared expert's segment: offset 8T, T rows). Returns 8T,
   or -1 when the last call built no permutation (decode path, failed call). */
int di_moe_last_routes(void *ctx, int32_t *perm_route, int32_t *seg_offsets, int32_t *seg_counts, int max_routes,
                       char *error, int capacity);

/* ------------------------------------------------------------------------------------
 * Part 3. Expert parallelism across the GPUs of one node (no reference counterpart: the
 * reference has no expert, tensor or collective parallelism, docs/ARCHITECTURE.md:63).
 * One process per GPU. GPU r of G owns experts [r*E/G, (r+1)*E/G) of every layer and a
 * contiguous shard of the tokens (shards in rank order); the router, shared expert and its
 * gate are replicated. Token rows travel to the GPUs that own their experts, and partial
 * expert sums travel back, as stores of the library's own kernels into the other GPUs' memory
 * over NVLink / NVSwitch (CUDA IPC mappings; NCCL only bootstraps the group and exchanges the
 * mapping handles). Results equal di_moe_stack on the concatenated tokens up to f32 summation
 * order; routing ids are identical.
 * ---------------------------------------------------------------------------------- */
#define DI_EP_ID_BYTES 128
/* Fills a 128-byte NCCL unique id on rank 0; the caller broadcasts it to every rank. */
int di_moe_ep_unique_id(uint8_t *id, char *error, int capacity);
/* Collective over all ranks (blocks until every rank joins). world in [1, 8]. */
void *di_moe_ep_create(void *ctx, const uint8_t *id, int rank, int world, char *error, int capacity);
void di_moe_ep_destroy(void *ep);
/* Binds one layer's shard: gate/up [E/G, I, D] and down [E/G, D, I] hold this rank's experts;
   router [1, E, D] and the shared matrices are full. Destroy with di_moe_layer_destroy. */
void *di_moe_ep_layer_create(void *ep, void *router, void *gate, void *up, void *down, void *shared_gate,
                             void *shared_up, void *shared_down, void *shared_route, char *error, int capacity);
/* di_moe_stack semantics on this rank's tokens x [tokens, D] (f32 residual, in/out); every rank
   calls it with the same layers. h_trace (bf16 [n_layers, tokens, D]) and ids_trace (int32
   [n_layers, tokens, 8]) are optional per-layer dumps of this rank's tokens, as in di_moe_stack.
   Flags: DI_MOE_DEVICE_IO, DI_MOE_PROFILE (di_moe_last_profile of the ep's context then returns this
   rank's milliseconds summed over the layers for [router logits, top-8 + dispatch, receive + scan,
   scatter, gate_up, down, partial-row send, combine]). */
int di_moe_ep_stack(void *ep, void *const *layers, const float *norms, int n_layers, float eps, float *x, int tokens,
                    uint16_t *h_trace, int32_t *ids_trace, int flags, double *ms, char *error, int capacity);

/* Allocation-free small-batch block. No counterpart in the reference. Some callers cannot call
   cudaMalloc once they are running: serving loops that forbid device allocation after start-up
   (cudaMalloc synchronises the device and its latency is unbounded), and processes whose device
   memory is already reserved by another allocator (a framework's caching pool), where a late
   cudaMalloc fails. di_moe_block's per-context workspace grows on demand, so it may allocate;
   this entry never does. It computes what di_moe_block computes on the decode (GEMV) path, with
   device pointers only: x bf16 [T,D] in, y bf16 [T,D] out, ids int32 [T,8] and probs f32 [T,8]
   optional outputs, T in [1, 16], T*D <= 49152. All of them must be device memory of the
   context's GPU; anything else is refused before any GPU work.
   Its scratch is one fixed device array of DI_MOE_STATIC_SCRATCH_BYTES on every GPU that loads
   the library (held until the process exits); a call that would need more (T*E*4 + T*9*I*4 + a
   few KB) is refused with an error before any GPU work. The first call on a device looks up that
   array's device address (a driver call, once per device). Every call on a device shares the
   array and it keeps the last call's contents: calls that overlap on the GPU (other threads,
   other contexts on the same device) race on it and must be serialised by the caller. */
#define DI_MOE_STATIC_MAX_TOKENS 16
#define DI_MOE_STATIC_SCRATCH_BYTES (512u * 1024u)
int di_moe_block_static(void *ctx, void *layer, const uint16_t *x, int tokens, uint16_t *y, int32_t *ids,
                        float *probs, double *ms, char *error, int capacity);

#ifdef __cplusplus
}
#endif
#endif
