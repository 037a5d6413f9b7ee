/*
 * CPU oracle for the Qwen3.6-35B-A3B MoE block -- TEST INFRASTRUCTURE ONLY.
 * Checker and timed CPU baseline; never part of the product path.
 * Every function names the reference file:line whose arithmetic it restates
 * (paths relative to the Infer.NET project root). Built with -ffp-contract=off so
 * that every fused multiply-add below is an explicit fmaf().
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int oc_abi_version(void) { return 1; }

/* ---------------------------------------------------------------- bf16 */

/* bf16 -> f32 by placing the 16 bits in the high half (quantized.mm:50-51, split_prefix.cu:60) */
float oc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* f32 -> bf16 round-to-nearest-even; NaN stays NaN (same rule as __float2bfloat16_rn). */
uint16_t oc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float round_bf16(float f) { return oc_bf16_to_f32(oc_f32_to_bf16(f)); }

/* ------------------------------------------------------ synthetic inputs
 * Counter-based generator shared bit-for-bit with the device generator
 * (infer.net_b200/csrc/generate.cuh). A normal sample is Irwin-Hall of four 16-bit
 * uniforms from one splitmix64 output: integer sum, exact int->f32, one f32 multiply.
 * No transcendental function is involved, so host and device agree exactly.
 */
uint64_t oc_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t oc_stream_base(uint64_t seed, uint64_t stream) {
    return oc_mix64(seed ^ oc_mix64(stream * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull));
}

/* scale so that oc_normal has standard deviation `stddev`: sqrt(3)/65536 * stddev in f32 */
float oc_normal_scale(float stddev) {
    const float k = 1.7320508075688772f / 65536.0f;
    return k * stddev;
}

float oc_normal(uint64_t base, uint64_t index, float scale) {
    uint64_t h = oc_mix64(base + index);
    int32_t s = (int32_t)(h & 0xffff) + (int32_t)((h >> 16) & 0xffff) + (int32_t)((h >> 32) & 0xffff) +
                (int32_t)(h >> 48);
    return (float)(s - 131070) * scale;
}

void oc_gen_bf16(uint64_t seed, uint64_t stream, int64_t n, float stddev, uint16_t *out) {
    uint64_t base = oc_stream_base(seed, stream);
    float scale = oc_normal_scale(stddev);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = oc_f32_to_bf16(oc_normal(base, (uint64_t)i, scale));
}

/* Pack one code LSB-first into the row's word stream, crossing a word boundary when
   needed (QuantizedTests.cs:155-161). */
static void pack_code(uint32_t *row_words, int col, int bits, uint32_t q) {
    int bit = col * bits, at = bit / 32, shift = bit % 32;
    row_words[at] |= q << shift;
    if (shift + bits > 32) row_words[at + 1] |= q >> (32 - shift);
}

/* Our min/max affine group-64 quantiser (the reference ships none; weights arrive
   pre-quantised, Qwen36Weights.cs:65-80): scale=(max-min)/(2^b-1) and bias=min, both
   rounded to bf16; q = clamp(rint((w-bias)/scale)). */
static void quantize_group(const float *w, int bits, uint32_t *row_words, int col0, uint16_t *scale_out,
                           uint16_t *bias_out) {
    float lo = w[0], hi = w[0];
    for (int i = 1; i < 64; i++) {
        lo = w[i] < lo ? w[i] : lo;
        hi = w[i] > hi ? w[i] : hi;
    }
    float levels = (float)((1 << bits) - 1);
    uint16_t sb = oc_f32_to_bf16((hi - lo) / levels), bb = oc_f32_to_bf16(lo);
    float s = oc_bf16_to_f32(sb), b = oc_bf16_to_f32(bb);
    *scale_out = sb;
    *bias_out = bb;
    for (int i = 0; i < 64; i++) {
        float q = s > 0.0f ? rintf((w[i] - b) / s) : 0.0f;
        q = q < 0.0f ? 0.0f : (q > levels ? levels : q);
        pack_code(row_words, col0 + i, bits, (uint32_t)q);
    }
}

void oc_quantize_rows(const float *w, int64_t rows, int cols, int bits, uint32_t *packed, uint16_t *scales,
                      uint16_t *biases) {
    int words = cols * bits / 32, groups = cols / 64;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        uint32_t *rw = packed + r * words;
        memset(rw, 0, (size_t)words * 4);
        for (int g = 0; g < groups; g++)
            quantize_group(w + r * cols + g * 64, bits, rw, g * 64, scales + r * groups + g, biases + r * groups + g);
    }
}

/* Weights of [experts, rows, cols] ~ N(0, stddev), quantised group by group. Sample
   index of element (e, r, c) is (e*rows + r)*cols + c within the stream. */
void oc_gen_quant_matrix(uint64_t seed, uint64_t stream, int experts, int rows, int cols, int bits, float stddev,
                         uint32_t *packed, uint16_t *scales, uint16_t *biases) {
    uint64_t base = oc_stream_base(seed, stream);
    float scale = oc_normal_scale(stddev);
    int64_t total_rows = (int64_t)experts * rows;
    int words = cols * bits / 32, groups = cols / 64;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < total_rows; r++) {
        float w[64];
        uint32_t *rw = packed + r * words;
        memset(rw, 0, (size_t)words * 4);
        for (int g = 0; g < groups; g++) {
            for (int i = 0; i < 64; i++) w[i] = oc_normal(base, (uint64_t)(r * cols + g * 64 + i), scale);
            quantize_group(w, bits, rw, g * 64, scales + r * groups + g, biases + r * groups + g);
        }
    }
}

/* ------------------------------------------------------------- dequant */

/* Code extraction, LSB-first across words (quantized.mm:62-67, :391-392). */
uint32_t oc_code(const oc_qmatrix *m, int expert, int row, int col) {
    const uint32_t *w = m->packed + ((int64_t)expert * m->rows + row) * (m->cols * m->bits / 32);
    int bit = col * m->bits, at = bit / 32, shift = bit % 32;
    uint32_t q = w[at] >> shift;
    if (shift + m->bits > 32) q |= w[at + 1] << (32 - shift);
    return q & ((1u << m->bits) - 1u);
}

/* w = q*scale + bias with one rounding: nvcc contracts split_prefix.cu:86 to this fma. */
float oc_weight(const oc_qmatrix *m, int expert, int row, int col) {
    int64_t p = ((int64_t)expert * m->rows + row) * (m->cols / 64) + col / 64;
    return fmaf((float)oc_code(m, expert, row, col), oc_bf16_to_f32(m->scales[p]), oc_bf16_to_f32(m->biases[p]));
}

/* Canonical f32 dot product: the lane partition of split_prefix.cu:113-117 (lane l owns
   columns base+j, base = 8l + 256i, j<8, summed in that order with fma) followed by the
   xor butterfly of split_prefix.cu:63-67 (offsets 16,8,4,2,1). The device router
   kernels reproduce exactly this sequence, so router logits match bit for bit. */
float oc_dot_canonical(const oc_qmatrix *m, int expert, int row, const float *x) {
    float lane[32], next[32];
    for (int l = 0; l < 32; l++) {
        float v = 0.0f;
        for (int base = l * 8; base < m->cols; base += 256)
            for (int j = 0; j < 8; j++) v = fmaf(oc_weight(m, expert, row, base + j), x[base + j], v);
        lane[l] = v;
    }
    for (int n = 16; n; n >>= 1) {
        for (int l = 0; l < 32; l++) next[l] = lane[l] + lane[l ^ n];
        memcpy(lane, next, sizeof lane);
    }
    return lane[0];
}

double oc_dot_f64(const oc_qmatrix *m, int expert, int row, const float *x, int bf16_weights) {
    double s = 0.0;
    for (int c = 0; c < m->cols; c++) {
        float w = oc_weight(m, expert, row, c);
        if (bf16_weights) w = round_bf16(w);
        s += (double)w * (double)x[c];
    }
    return s;
}

/* di_quant_matvec semantics: y[slot*rows + row] = W[experts[slot]] . x_slot, where
   x_slot = x + slot*cols when batched (quantized.mm:41-58, :346-349). mode 0 = canonical f32,
   mode 1 = double. */
void oc_gemv(const oc_qmatrix *m, const float *x, float *y, const int32_t *experts, int count, int batched,
             int mode) {
    for (int s = 0; s < count; s++) {
        const float *xs = x + (batched ? (int64_t)s * m->cols : 0);
#pragma omp parallel for schedule(static)
        for (int r = 0; r < m->rows; r++)
            y[(int64_t)s * m->rows + r] = mode == OC_MODE_F64 ? (float)oc_dot_f64(m, experts[s], r, xs, 0)
                                                               : oc_dot_canonical(m, experts[s], r, xs);
    }
}

/* ------------------------------------------------------------- routing */

static float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }  /* Qwen36Model.cs:272 */
static float siluf_ref(float x) { return x * sigmoidf_ref(x); }          /* Qwen36Model.cs:273 */

/* Softmax in place (Qwen36Model.cs:293-298). */
static void softmax8(float *x, int n) {
    float mx = -INFINITY, sum = 0.0f;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* SelectExperts (Qwen36Model.cs:246-262): insertion with strict '>' so equal logits keep the
   lower expert id first; any non-finite logit is an error. */
int oc_select_experts(const float *logits, int n_experts, int32_t *ids, float *probs) {
    for (int j = 0; j < 8; j++) ids[j] = -1;
    for (int e = 0; e < n_experts; e++) {
        if (!isfinite(logits[e])) return -1;
        for (int j = 0; j < 8; j++)
            if (ids[j] < 0 || logits[e] > logits[ids[j]]) {
                for (int k = 7; k > j; k--) ids[k] = ids[k - 1];
                ids[j] = e;
                break;
            }
    }
    for (int i = 0; i < 8; i++) probs[i] = logits[ids[i]];
    softmax8(probs, 8);
    return 0;
}

/* Forced routes (gpu_graph.mm:153-159): ids given, probs = softmax of their logits. */
int oc_force_route(const float *logits, const int32_t *forced, int32_t *ids, float *probs) {
    for (int i = 0; i < 8; i++) {
        ids[i] = forced[i];
        probs[i] = logits[forced[i]];
    }
    softmax8(probs, 8);
    return 0;
}

/* Stable expert-grouped permutation: for each expert e, the routes r = t*8+slot with
   ids[r] == e in ascending r (prefill_moe.mm:12-14), compacted at offsets[e]. */
void oc_permute(const int32_t *ids, int tokens, int n_experts, int32_t *counts, int32_t *offsets, int32_t *routes) {
    int total = tokens * 8;
    for (int e = 0; e < n_experts; e++) counts[e] = 0;
    for (int r = 0; r < total; r++) counts[ids[r]]++;
    int run = 0;
    for (int e = 0; e < n_experts; e++) {
        offsets[e] = run;
        run += counts[e];
    }
    int32_t *fill = (int32_t *)calloc((size_t)n_experts, sizeof(int32_t));
    for (int r = 0; r < total; r++) {
        int e = ids[r];
        routes[offsets[e] + fill[e]++] = r;
    }
    free(fill);
}

/* --------------------------------------------------------------- block */

static float dot_mode(const oc_qmatrix *m, int expert, int row, const float *x, int mode) {
    if (mode == OC_MODE_F32) return oc_dot_canonical(m, expert, row, x);
    return (float)oc_dot_f64(m, expert, row, x, mode == OC_MODE_BF16OPS);
}

/* One token through the block (Qwen36Model.cs:218-245):
     router + shared gate/up + shared route GEMVs, SelectExperts, shared SwiGLU,
     expert gate/up -> SwiGLU -> down (quantized.mm:148-189, :375), shared down,
     Output = shared*sigmoid(route) then += p_i * expert_i in slot order (AddScaled, no fma).
   The router logits always use the canonical f32 order so that ids are defined by it. */
static int block_token(const oc_layer *L, const float *x, int mode, const int32_t *forced, float *out, int32_t *ids,
                       float *probs, float *logits, float *scratch) {
    const int E = L->router.rows, D = L->gate.cols, I = L->gate.rows;
    float *lg = scratch, *sg = lg + E + 1, *act = sg + I, *y = act + I;
    for (int e = 0; e < E; e++) {
        lg[e] = oc_dot_canonical(&L->router, 0, e, x);
        if (L->router_bias) lg[e] += L->router_bias[e];
    }
    lg[E] = oc_dot_canonical(&L->shared_route, 0, 0, x);
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)(E + 1));
    int rc = forced ? oc_force_route(lg, forced, ids, probs) : oc_select_experts(lg, E, ids, probs);
    if (rc) return rc;
    int bf = mode == OC_MODE_BF16OPS;
    for (int i = 0; i < I; i++) {
        float g = dot_mode(&L->shared_gate, 0, i, x, mode), u = dot_mode(&L->shared_up, 0, i, x, mode);
        sg[i] = bf ? round_bf16(siluf_ref(g) * u) : siluf_ref(g) * u;
    }
    float gate = sigmoidf_ref(lg[E]);
    for (int d = 0; d < D; d++) {
        float s = dot_mode(&L->shared_down, 0, d, sg, mode);
        out[d] = (bf ? round_bf16(s) : s) * gate;
    }
    for (int slot = 0; slot < 8; slot++) {
        int e = ids[slot];
        for (int i = 0; i < I; i++) {
            float g = dot_mode(&L->gate, e, i, x, mode), u = dot_mode(&L->up, e, i, x, mode);
            act[i] = bf ? round_bf16(siluf_ref(g) * u) : siluf_ref(g) * u;
        }
        for (int d = 0; d < D; d++) {
            float v = dot_mode(&L->down, e, d, act, mode);
            y[d] = bf ? round_bf16(v) : v;
        }
        float p = probs[slot];
        for (int d = 0; d < D; d++) {
            float t = p * y[d];
            out[d] = out[d] + t;
        }
    }
    return 0;
}

int oc_moe_block(const oc_layer *L, const uint16_t *x, int T, int mode, const int32_t *forced_ids, float *out,
                 int32_t *ids, float *probs, float *logits, int threads) {
    const int E = L->router.rows, D = L->gate.cols, I = L->gate.rows;
    int status = 0;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#pragma omp parallel
    {
        float *xf = (float *)malloc(sizeof(float) * (size_t)D);
        float *scratch = (float *)malloc(sizeof(float) * (size_t)(E + 1 + 2 * I + D));
#pragma omp for schedule(dynamic, 1)
        for (int t = 0; t < T; t++) {
            for (int d = 0; d < D; d++) xf[d] = oc_bf16_to_f32(x[(int64_t)t * D + d]);
            int rc = block_token(L, xf, mode, forced_ids ? forced_ids + (int64_t)t * 8 : NULL, out + (int64_t)t * D,
                                 ids + (int64_t)t * 8, probs + (int64_t)t * 8,
                                 logits ? logits + (int64_t)t * (E + 1) : NULL, scratch);
            if (rc) {
#pragma omp atomic write
                status = rc;
            }
        }
        free(scratch);
        free(xf);
    }
    return status;
}

/* RMSNorm then round to bf16: scale = 1/sqrt(sum(x^2)/D + eps), h = x*scale*w
   (gpu_graph.mm:48-61 arithmetic; Qwen36Model.cs:288-292). */
void oc_rmsnorm_bf16(const float *x, const float *w, int D, float eps, uint16_t *out) {
    float ss = 0.0f;
    for (int d = 0; d < D; d++) ss = fmaf(x[d], x[d], ss);
    float scale = 1.0f / sqrtf(ss / (float)D + eps);
    for (int d = 0; d < D; d++) out[d] = oc_f32_to_bf16(x[d] * scale * w[d]);
}

int oc_moe_stack(const oc_layer *layers, const float *norms, int n_layers, float eps, float *x, int T, int mode,
                 int32_t *ids_out, int threads) {
    const int D = layers[0].gate.cols;
    uint16_t *h = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)T * D);
    float *y = (float *)malloc(sizeof(float) * (size_t)T * D);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * 8);
    float *probs = (float *)malloc(sizeof(float) * (size_t)T * 8);
    int rc = 0;
    for (int l = 0; l < n_layers && !rc; l++) {
        for (int t = 0; t < T; t++) oc_rmsnorm_bf16(x + (int64_t)t * D, norms + (int64_t)l * D, D, eps, h + (int64_t)t * D);
        rc = oc_moe_block(&layers[l], h, T, mode, NULL, y, ids, probs, NULL, threads);
        for (int64_t i = 0; i < (int64_t)T * D; i++) x[i] = x[i] + y[i];
        if (ids_out) memcpy(ids_out + (int64_t)l * T * 8, ids, sizeof(int32_t) * (size_t)T * 8);
    }
    free(h);
    free(y);
    free(ids);
    free(probs);
    return rc;
}
