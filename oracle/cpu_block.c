/*
 * CPU baseline of the MoE block in the reference's own CPU loop shape -- TEST INFRASTRUCTURE
 * (the timed CPU leg of bench.py and its parity test; never part of the product path).
 *
 * The reference's CPU arithmetic for this block is C#: Qwen36Model.Moe/SelectExperts
 * (src/DeepInfer.Backends/Models/Qwen36Model.cs:218-262) over CpuMatrix.Multiply
 * (src/DeepInfer.Backends/Compute/MatVec.cs:44-54), one token at a time. .NET is not on this
 * machine, so this file restates that loop shape in C with the vector width of the host:
 *   - every GEMV row is one Vector<float> accumulator, sum += w * x over the row in SIMD chunks
 *     (a multiply then an add, as Vector<float> arithmetic does), then Vector.Sum (MatVec.cs:48-53);
 *     the weights are dequantised in the loop, w = fma(q, scale, bias), with the group's scale and
 *     bias hoisted per 64 columns (the affine g64 rule of quantized.mm:62-82);
 *   - the router keeps the canonical f32 order (the lane partition and butterfly of
 *     native/DeepInfer.Cuda/split_prefix.cu:63-67, :106-120, as oc_dot_canonical), vectorised
 *     across the 32 lanes from router rows dequantised once when the layer is prepared (as
 *     CpuMatVecDevice.Upload converts a matrix to floats, MatVec.cs:23-34), so its expert ids
 *     equal the oracle's bit for bit;
 *   - SelectExperts, the shared SwiGLU and sigmoid gate and the p-weighted AddScaled sum follow
 *     Qwen36Model.cs:221-262, :272-298 (oc_select_experts in moe_oracle.c).
 * Tokens are independent (OpenMP over tokens); a single token splits each GEMV's rows over the
 * threads. The instruction set is chosen at run time (AVX-512, AVX2+FMA, or scalar).
 */
#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "moe_oracle.h"

struct oc_cpu_layer {
    oc_layer L;
    float *router_t;   /* [E][D/256][8][32]: W[e][256 i + 8 l + j] at [e][i][j][l] */
    float *route_t;    /* the shared-route gate row, same layout */
};

/* ---------------------------------------------------------------- instruction set */

enum { ISA_SCALAR = 0, ISA_AVX2 = 1, ISA_AVX512 = 2 };
static int g_isa = -1;

static int isa(void) {
    if (g_isa < 0) {
        __builtin_cpu_init();
        if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw")) g_isa = ISA_AVX512;
        else if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) g_isa = ISA_AVX2;
        else g_isa = ISA_SCALAR;
        const char *force = getenv("OC_CPU_ISA");  /* test aid: run a narrower path */
        if (force && strcmp(force, "avx2") == 0 && g_isa > ISA_AVX2) g_isa = ISA_AVX2;
        if (force && strcmp(force, "scalar") == 0) g_isa = ISA_SCALAR;
    }
    return g_isa;
}

const char *oc_cpu_isa(void) {
    static const char *names[] = {"scalar", "avx2", "avx512"};
    return names[isa()];
}

/* ---------------------------------------------------------------- codes of one 64-group */

/* The 64 codes of group g of a packed row as bytes (LSB-first, crossing words,
   QuantizedTests.cs:155-161). 8-bit rows are already bytes; 5-bit groups are 40 bytes. */
static const uint8_t *group_codes(const uint32_t *row, int g, int bits, uint8_t *tmp) {
    if (bits == 8) return (const uint8_t *)row + (size_t)g * 64;
    const uint8_t *b = (const uint8_t *)row + (size_t)g * 40;
    for (int k = 0; k < 8; k++) {
        uint64_t v = 0;
        memcpy(&v, b + 5 * k, 5);
        for (int j = 0; j < 8; j++) tmp[8 * k + j] = (uint8_t)((v >> (5 * j)) & 31u);
    }
    return tmp;
}

/* ---------------------------------------------------------------- Vector<float> row dots */

static float dot_row_scalar(const uint32_t *row, const uint16_t *sc, const uint16_t *bi, int bits, const float *x,
                            int cols) {
    float sum = 0.0f;
    uint8_t tmp[64];
    for (int g = 0; g < cols / 64; g++) {
        const uint8_t *q = group_codes(row, g, bits, tmp);
        const float s = oc_bf16_to_f32(sc[g]), b = oc_bf16_to_f32(bi[g]);
        for (int c = 0; c < 64; c++) {
            const float w = fmaf((float)q[c], s, b);
            const float p = w * x[g * 64 + c];
            sum = sum + p;
        }
    }
    return sum;
}

__attribute__((target("avx2,fma"))) static float dot_row_avx2(const uint32_t *row, const uint16_t *sc,
                                                               const uint16_t *bi, int bits, const float *x, int cols) {
    __m256 sum = _mm256_setzero_ps();
    uint8_t tmp[64];
    for (int g = 0; g < cols / 64; g++) {
        const uint8_t *q = group_codes(row, g, bits, tmp);
        const __m256 s = _mm256_set1_ps(oc_bf16_to_f32(sc[g])), b = _mm256_set1_ps(oc_bf16_to_f32(bi[g]));
        for (int k = 0; k < 8; k++) {
            const __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(q + 8 * k))));
            const __m256 w = _mm256_fmadd_ps(qf, s, b);
            sum = _mm256_add_ps(sum, _mm256_mul_ps(w, _mm256_loadu_ps(x + g * 64 + 8 * k)));
        }
    }
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(sum), _mm256_extractf128_ps(sum, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    h = _mm_add_ss(h, _mm_movehdup_ps(h));
    return _mm_cvtss_f32(h);
}

__attribute__((target("avx512f,avx512bw"))) static float dot_row_avx512(const uint32_t *row, const uint16_t *sc,
                                                                         const uint16_t *bi, int bits, const float *x,
                                                                         int cols) {
    __m512 sum = _mm512_setzero_ps();
    uint8_t tmp[64];
    for (int g = 0; g < cols / 64; g++) {
        const uint8_t *q = group_codes(row, g, bits, tmp);
        const __m512 s = _mm512_set1_ps(oc_bf16_to_f32(sc[g])), b = _mm512_set1_ps(oc_bf16_to_f32(bi[g]));
        for (int k = 0; k < 4; k++) {
            const __m512 qf = _mm512_cvtepi32_ps(_mm512_cvtepu8_epi32(_mm_loadu_si128((const __m128i *)(q + 16 * k))));
            const __m512 w = _mm512_fmadd_ps(qf, s, b);
            sum = _mm512_add_ps(sum, _mm512_mul_ps(w, _mm512_loadu_ps(x + g * 64 + 16 * k)));
        }
    }
    return _mm512_reduce_add_ps(sum);
}

/* One row of expert `e` of m times x (CpuMatrix.Multiply's row loop, MatVec.cs:46-53). */
static float dot_row(const oc_qmatrix *m, int e, int r, const float *x) {
    const int64_t row = (int64_t)e * m->rows + r, gpr = m->cols / 64;
    const uint32_t *w = m->packed + row * (m->cols * m->bits / 32);
    const uint16_t *sc = m->scales + row * gpr, *bi = m->biases + row * gpr;
    switch (isa()) {
    case ISA_AVX512: return dot_row_avx512(w, sc, bi, m->bits, x, m->cols);
    case ISA_AVX2: return dot_row_avx2(w, sc, bi, m->bits, x, m->cols);
    default: return dot_row_scalar(w, sc, bi, m->bits, x, m->cols);
    }
}

/* ---------------------------------------------------------------- canonical router rows */

/* Lane-transposed f32 rows of a router matrix: W[e][256 i + 8 l + j] -> t[e][i][j][l]. */
static float *transpose_router(const oc_qmatrix *m) {
    const int E = m->rows, D = m->cols, nb = D / 256;
    float *t = (float *)malloc(sizeof(float) * (size_t)E * D);
    if (!t) return NULL;
#pragma omp parallel for schedule(static)
    for (int e = 0; e < E; e++)
        for (int i = 0; i < nb; i++)
            for (int j = 0; j < 8; j++)
                for (int l = 0; l < 32; l++)
                    t[(((size_t)e * nb + i) * 8 + j) * 32 + l] = oc_weight(m, 0, e, 256 * i + 8 * l + j);
    return t;
}

/* The same transposition of one activation row. */
static void transpose_x(const float *x, int D, float *xt) {
    for (int i = 0; i < D / 256; i++)
        for (int j = 0; j < 8; j++)
            for (int l = 0; l < 32; l++) xt[(i * 8 + j) * 32 + l] = x[256 * i + 8 * l + j];
}

/* 32 lane sums of the canonical order, then the xor butterfly 16, 8, 4, 2, 1 (oc_dot_canonical). */
static float butterfly32(float *lane) {
    float next[32];
    for (int n = 16; n; n >>= 1) {
        for (int l = 0; l < 32; l++) next[l] = lane[l] + lane[l ^ n];
        memcpy(lane, next, sizeof next);
    }
    return lane[0];
}

static float canonical_scalar(const float *wt, const float *xt, int nb) {
    float lane[32] = {0};
    for (int k = 0; k < nb * 8; k++)
        for (int l = 0; l < 32; l++) lane[l] = fmaf(wt[k * 32 + l], xt[k * 32 + l], lane[l]);
    return butterfly32(lane);
}

__attribute__((target("avx2,fma"))) static float canonical_avx2(const float *wt, const float *xt, int nb) {
    __m256 a[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (int k = 0; k < nb * 8; k++)
        for (int v = 0; v < 4; v++)
            a[v] = _mm256_fmadd_ps(_mm256_loadu_ps(wt + k * 32 + 8 * v), _mm256_loadu_ps(xt + k * 32 + 8 * v), a[v]);
    float lane[32];
    for (int v = 0; v < 4; v++) _mm256_storeu_ps(lane + 8 * v, a[v]);
    return butterfly32(lane);
}

__attribute__((target("avx512f"))) static float canonical_avx512(const float *wt, const float *xt, int nb) {
    __m512 a0 = _mm512_setzero_ps(), a1 = _mm512_setzero_ps();
    for (int k = 0; k < nb * 8; k++) {
        a0 = _mm512_fmadd_ps(_mm512_loadu_ps(wt + k * 32), _mm512_loadu_ps(xt + k * 32), a0);
        a1 = _mm512_fmadd_ps(_mm512_loadu_ps(wt + k * 32 + 16), _mm512_loadu_ps(xt + k * 32 + 16), a1);
    }
    float lane[32];
    _mm512_storeu_ps(lane, a0);
    _mm512_storeu_ps(lane + 16, a1);
    return butterfly32(lane);
}

/* Router row e (of the transposed rows t) with the transposed activation xt, canonical order:
   bit-identical to oc_dot_canonical (each lane's fma chain in the same order, the same butterfly). */
static float canonical_row(const float *t, int e, const float *xt, int D) {
    const int nb = D / 256;
    const float *wt = t + (size_t)e * D;
    switch (isa()) {
    case ISA_AVX512: return canonical_avx512(wt, xt, nb);
    case ISA_AVX2: return canonical_avx2(wt, xt, nb);
    default: return canonical_scalar(wt, xt, nb);
    }
}

/* ---------------------------------------------------------------- layers */

oc_cpu_layer *oc_cpu_prepare(const oc_layer *L) {
    oc_cpu_layer *P = (oc_cpu_layer *)calloc(1, sizeof(oc_cpu_layer));
    if (!P) return NULL;
    P->L = *L;
    P->router_t = transpose_router(&L->router);
    P->route_t = transpose_router(&L->shared_route);
    if (!P->router_t || !P->route_t) {
        oc_cpu_release(P);
        return NULL;
    }
    return P;
}

void oc_cpu_release(oc_cpu_layer *P) {
    if (!P) return;
    free(P->router_t);
    free(P->route_t);
    free(P);
}

static float sigmoid_c(float x) { return 1.0f / (1.0f + expf(-x)); }  /* Qwen36Model.cs:272 */
static float silu_c(float x) { return x * sigmoid_c(x); }            /* Qwen36Model.cs:273 */

/* A share of n rows for thread tid of nt (all of them when nt == 1). */
static void share(int n, int tid, int nt, int *lo, int *hi) {
    *lo = (int)((int64_t)n * tid / nt);
    *hi = (int)((int64_t)n * (tid + 1) / nt);
}

/* Barrier of the enclosing team (a no-op for a token computed by one thread). */
static void team_barrier(int nt) {
    if (nt > 1) {
#pragma omp barrier
    }
}

/* This thread's share of the rows of expert e of m times x into y. */
static void gemv_rows(const oc_qmatrix *m, int e, const float *x, float *y, int tid, int nt) {
    int lo, hi;
    share(m->rows, tid, nt, &lo, &hi);
    for (int r = lo; r < hi; r++) y[r] = dot_row(m, e, r, x);
}

/* Scratch of one token: xt [D], logits [E + 1], shared gate/up [2 I], expert gate/up [2 I] x 8,
   expert outputs [8 D]. */
static size_t token_scratch(const oc_layer *L) {
    const size_t E = L->router.rows, D = L->gate.cols, I = L->gate.rows;
    return D + E + 1 + 2 * I + 16 * I + 8 * D + 64;
}

/* Qwen36Model.Moe for one token (x f32 [D]) -> out [D], ids, probs. nt > 1: every thread of the
   enclosing team calls it with the same arguments and its own tid, and the rows of each GEMV are
   shared out; nt == 1: one thread computes the whole token. Returns 0, or -1 on non-finite
   router logits (the same value on every thread). */
static int cpu_token(const oc_cpu_layer *P, const float *x, float *out, int32_t *ids, float *probs, float *scratch,
                     int tid, int nt, int *status) {
    const oc_layer *L = &P->L;
    const int E = L->router.rows, D = L->gate.cols, I = L->gate.rows;
    float *xt = scratch, *lg = xt + D, *sg = lg + E + 1, *su = sg + I, *eg = su + I, *eu = eg + 8 * I;
    float *ey = eu + 8 * I;
    int lo, hi;
    /* stage 1: router (canonical order), shared gate/up, shared route (Qwen36Model.cs:221-222) */
    if (tid == 0) transpose_x(x, D, xt);
    team_barrier(nt);
    share(E + 1, tid, nt, &lo, &hi);
    for (int e = lo; e < hi; e++)
        lg[e] = e < E ? canonical_row(P->router_t, e, xt, D) + (L->router_bias ? L->router_bias[e] : 0.0f)
                      : canonical_row(P->route_t, 0, xt, D);
    gemv_rows(&L->shared_gate, 0, x, sg, tid, nt);
    gemv_rows(&L->shared_up, 0, x, su, tid, nt);
    team_barrier(nt);
    if (tid == 0) {
        if (oc_select_experts(lg, E, ids, probs)) *status = -1;      /* Qwen36Model.cs:223, :246-262 */
        for (int i = 0; i < I; i++) sg[i] = silu_c(sg[i]) * su[i];  /* Qwen36Model.cs:230 */
    }
    team_barrier(nt);
    if (*status) return -1;
    /* stage 2: ExpertMlp -- gate/up of the 8 experts, SwiGLU, down; shared down (Qwen36Model.cs:231-233) */
    for (int k = 0; k < 8; k++) {
        gemv_rows(&L->gate, ids[k], x, eg + (size_t)k * I, tid, nt);
        gemv_rows(&L->up, ids[k], x, eu + (size_t)k * I, tid, nt);
    }
    team_barrier(nt);
    share(8 * I, tid, nt, &lo, &hi);
    for (int i = lo; i < hi; i++) eg[i] = silu_c(eg[i]) * eu[i];
    team_barrier(nt);
    for (int k = 0; k < 8; k++) gemv_rows(&L->down, ids[k], eg + (size_t)k * I, ey + (size_t)k * D, tid, nt);
    gemv_rows(&L->shared_down, 0, sg, out, tid, nt);
    team_barrier(nt);
    /* Output *= sigmoid(route); Output += p_k * expert_k (AddScaled, Qwen36Model.cs:241-244) */
    const float scale = sigmoid_c(lg[E]);
    share(D, tid, nt, &lo, &hi);
    for (int d = lo; d < hi; d++) {
        float o = out[d] * scale;
        for (int k = 0; k < 8; k++) o += probs[k] * ey[(size_t)k * D + d];
        out[d] = o;
    }
    team_barrier(nt);
    return 0;
}

static int run_threads(int threads) {
#ifdef _OPENMP
    return threads > 0 ? threads : omp_get_max_threads();
#else
    (void)threads;
    return 1;
#endif
}

/* x bf16 [T, D] -> out f32 [T, D], ids [T, 8], probs [T, 8]. Returns 0, or -1 on non-finite
   router logits. */
int oc_cpu_block(const oc_cpu_layer *P, const uint16_t *x, int T, float *out, int32_t *ids, float *probs,
                 int threads) {
    const oc_layer *L = &P->L;
    const int D = L->gate.cols, nt = run_threads(threads);
    int status = 0;
    if (T >= nt) {
        /* independent tokens, one per thread at a time */
#pragma omp parallel num_threads(nt)
        {
            float *xf = (float *)malloc(sizeof(float) * (size_t)D);
            float *scratch = (float *)malloc(sizeof(float) * token_scratch(L));
#pragma omp for schedule(dynamic, 1)
            for (int t = 0; t < T; t++) {
                int st = 0;
                for (int d = 0; d < D; d++) xf[d] = oc_bf16_to_f32(x[(int64_t)t * D + d]);
                if (cpu_token(P, xf, out + (int64_t)t * D, ids + (int64_t)t * 8, probs + (int64_t)t * 8, scratch, 0, 1,
                              &st)) {
#pragma omp atomic write
                    status = -1;
                }
            }
            free(scratch);
            free(xf);
        }
        return status;
    }
    /* fewer tokens than threads: each GEMV's rows are shared out */
    float *xf = (float *)malloc(sizeof(float) * (size_t)D);
    float *scratch = (float *)malloc(sizeof(float) * token_scratch(L));
    for (int t = 0; t < T && !status; t++) {
        for (int d = 0; d < D; d++) xf[d] = oc_bf16_to_f32(x[(int64_t)t * D + d]);
#pragma omp parallel num_threads(nt)
        {
            int tid = 0;
#ifdef _OPENMP
            tid = omp_get_thread_num();
#endif
            cpu_token(P, xf, out + (int64_t)t * D, ids + (int64_t)t * 8, probs + (int64_t)t * 8, scratch, tid, nt,
                      &status);
        }
    }
    free(scratch);
    free(xf);
    return status;
}

/* The residual stack of n prepared layers over x f32 [T, D] (in place): h = bf16(RMSNorm(x) * w_l),
   x += block_l(h) (gpu_graph.mm:48-61; oc_moe_stack's arithmetic). ids_out optional [n, T, 8]. */
int oc_cpu_stack(const oc_cpu_layer *const *P, const float *norms, int n_layers, float eps, float *x, int T,
                 int32_t *ids_out, int threads) {
    const int D = P[0]->L.gate.cols;
    uint16_t *h = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)T * D);
    float *y = (float *)malloc(sizeof(float) * (size_t)T * D);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * 8);
    float *probs = (float *)malloc(sizeof(float) * (size_t)T * 8);
    int rc = 0;
    for (int l = 0; l < n_layers && !rc; l++) {
        for (int t = 0; t < T; t++) oc_rmsnorm_bf16(x + (int64_t)t * D, norms + (int64_t)l * D, D, eps, h + (int64_t)t * D);
        rc = oc_cpu_block(P[l], h, T, y, ids, probs, threads);
        for (int64_t i = 0; i < (int64_t)T * D; i++) x[i] = x[i] + y[i];
        if (ids_out) memcpy(ids_out + (int64_t)l * T * 8, ids, sizeof(int32_t) * (size_t)T * 8);
    }
    free(h);
    free(y);
    free(ids);
    free(probs);
    return rc;
}
