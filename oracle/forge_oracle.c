/*
 * forge_oracle.c — CPU restatement of ForgeLM's reference decode path
 * (TitanUranus67/forge-lm; file:line citations are relative to that project).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * Nothing in the B200 product library links, loads or calls this code.
 *
 * Build with -ffp-contract=off and without fast-math: every float operation
 * must round separately, as the C# code does (RyuJIT does not contract
 * Vector<float> multiply+add into FMA).
 *
 * Loop orders follow src/LLM.Core/Tensor/CpuBackend.cs:
 *   - MatMulNN (y = a*b) accumulates sequentially over k into each output row
 *     with a separate multiply and add (CpuBackend.cs:118-164, 175-194), so its
 *     result does not depend on the SIMD width.
 *   - MatMulNT (y = a*b^T) uses 8-lane dot products (CpuBackend.cs:196-220);
 *     the horizontal sum of the 8 lanes is an implementation detail of .NET's
 *     Vector.Sum.  This file sums ((l0+l4)+(l1+l5))+((l2+l6)+(l3+l7)); the
 *     order is not pinned and only affects the last bits.
 *   - Matmuls with M*K*N above 8,000,000 run their rows in parallel
 *     (CpuBackend.cs:29, 97, 146); OpenMP stands in for Parallel.For.  Row
 *     results do not depend on the thread count.
 */
#include "forge_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define SMALL_MATMUL_WORK 8000000LL /* CpuBackend.cs:29 */

typedef float f8 __attribute__((vector_size(32)));

/* ====================================================================== */
/* System.Random, compat seeded variant (published Knuth subtractive       */
/* generator; .NET seeds it as below and NextDouble = sample / MaxValue).   */
/* ====================================================================== */
#define ORC_MBIG 2147483647
#define ORC_MSEED 161803398

/* C# int arithmetic wraps (unchecked context); so does this. */
static inline int32_t wsub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
static inline int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

void orc_random_init(orc_dotnet_random* r, int32_t seed) {
    int32_t* sa = r->seed_array;
    memset(sa, 0, sizeof(r->seed_array));
    int32_t subtraction = (seed == INT32_MIN) ? ORC_MBIG : (seed < 0 ? -seed : seed);
    int32_t mj = ORC_MSEED - subtraction;
    sa[55] = mj;
    int32_t mk = 1;
    int32_t ii = 0;
    for (int i = 1; i < 55; i++) {
        ii += 21;
        if (ii >= 55) ii -= 55;
        sa[ii] = mk;
        mk = wsub(mj, mk);
        if (mk < 0) mk = wadd(mk, ORC_MBIG);
        mj = sa[ii];
    }
    for (int k = 1; k < 5; k++) {
        for (int i = 1; i < 56; i++) {
            int n = i + 30;
            if (n >= 55) n -= 55;
            sa[i] = wsub(sa[i], sa[1 + n]);
            if (sa[i] < 0) sa[i] = wadd(sa[i], ORC_MBIG);
        }
    }
    r->inext = 0;
    r->inextp = 21;
}

int32_t orc_random_internal_sample(orc_dotnet_random* r) {
    int32_t a = r->inext + 1;
    if (a >= 56) a = 1;
    int32_t b = r->inextp + 1;
    if (b >= 56) b = 1;
    int32_t v = wsub(r->seed_array[a], r->seed_array[b]);
    if (v == ORC_MBIG) v--;
    if (v < 0) v = wadd(v, ORC_MBIG);
    r->seed_array[a] = v;
    r->inext = a;
    r->inextp = b;
    return v;
}

double orc_random_next_double(orc_dotnet_random* r) {
    return orc_random_internal_sample(r) * (1.0 / ORC_MBIG);
}

void orc_random_next_doubles(orc_dotnet_random* r, double* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = orc_random_next_double(r);
}

/* ====================================================================== */
/* Parameter registry (GptModel.cs:47-98, Parameters.cs:109-129)            */
/* ====================================================================== */
static const char* const kBlockNames[12] = {
    "ln1.w", "ln1.b", "attn.qkv.w", "attn.qkv.b", "attn.proj.w", "attn.proj.b",
    "ln2.w", "ln2.b", "mlp.fc.w", "mlp.fc.b", "mlp.proj.w", "mlp.proj.b"};

int32_t orc_param_count(const orc_config* c) { return 4 + 12 * c->n_layers; }

int64_t orc_param_numel(const orc_config* c, int32_t index) {
    int64_t d = c->d_model, f = 4LL * c->d_model;
    int32_t n = orc_param_count(c);
    if (index < 0 || index >= n) return -1;
    if (index == 0) return (int64_t)c->vocab_size * d;
    if (index == 1) return (int64_t)c->context_length * d;
    if (index >= n - 2) return d;
    switch ((index - 2) % 12) {
    case 0: case 1: case 5: case 6: case 7: case 11: return d;
    case 2: return d * 3 * d;
    case 3: return 3 * d;
    case 4: return d * d;
    case 8: return d * f;
    case 9: return f;
    case 10: return f * d;
    }
    return -1;
}

int64_t orc_total_params(const orc_config* c) {
    int64_t s = 0;
    for (int32_t i = 0; i < orc_param_count(c); i++) s += orc_param_numel(c, i);
    return s;
}

int32_t orc_param_name(const orc_config* c, int32_t index, char* buf, int32_t buflen) {
    int32_t n = orc_param_count(c);
    if (index < 0 || index >= n || buflen <= 0) return -1;
    if (index == 0) snprintf(buf, buflen, "tok_emb");
    else if (index == 1) snprintf(buf, buflen, "pos_emb");
    else if (index == n - 2) snprintf(buf, buflen, "ln_f.w");
    else if (index == n - 1) snprintf(buf, buflen, "ln_f.b");
    else snprintf(buf, buflen, "blocks.%d.%s", (index - 2) / 12, kBlockNames[(index - 2) % 12]);
    return 0;
}

/* Tensor.FillNormal (Tensor.cs:79-91): Box-Muller in double, pairs. */
static void fill_normal(float* data, int64_t n, orc_dotnet_random* rng, float std) {
    for (int64_t i = 0; i < n; i += 2) {
        double u1 = 1.0 - orc_random_next_double(rng);
        double u2 = orc_random_next_double(rng);
        double r = sqrt(-2.0 * log(u1));
        data[i] = (float)(r * cos(2 * M_PI * u2) * (double)std);
        if (i + 1 < n) data[i + 1] = (float)(r * sin(2 * M_PI * u2) * (double)std);
    }
}

/* GptModel ctor (GptModel.cs:47-98): init order = registration order. */
void orc_model_init(const orc_config* c, int32_t seed, float* const* params) {
    orc_dotnet_random rng;
    orc_random_init(&rng, seed);
    float std = 0.02f;
    float resid_std = 0.02f / sqrtf(2.0f * (float)c->n_layers); /* GptModel.cs:50 */
    int32_t n = orc_param_count(c);
    for (int32_t i = 0; i < n; i++) {
        int64_t numel = orc_param_numel(c, i);
        float* p = params[i];
        if (i < 2) { fill_normal(p, numel, &rng, std); continue; }
        if (i >= n - 2) { /* ln_f.w = 1, ln_f.b = 0 (GptModel.cs:90-91) */
            for (int64_t j = 0; j < numel; j++) p[j] = (i == n - 2) ? 1.0f : 0.0f;
            continue;
        }
        switch ((i - 2) % 12) {
        case 0: case 6: /* ln.w = 1 (GptModel.cs:65) */
            for (int64_t j = 0; j < numel; j++) p[j] = 1.0f;
            break;
        case 2: case 8: fill_normal(p, numel, &rng, std); break;       /* qkv.w, fc.w */
        case 4: case 10: fill_normal(p, numel, &rng, resid_std); break; /* proj.w */
        default: memset(p, 0, (size_t)numel * sizeof(float)); break;    /* biases, ln.b */
        }
    }
}

/* ====================================================================== */
/* CpuBackend kernels                                                       */
/* ====================================================================== */
static inline f8 ld8(const float* p) { f8 v; memcpy(&v, p, sizeof(v)); return v; }
static inline void st8(float* p, f8 v) { memcpy(p, &v, sizeof(v)); }

/* AddScaled (CpuBackend.cs:175-194): dst[i] += scale * src[i]. */
static inline void add_scaled(float* dst, const float* src, float s, int n) {
    int i = 0;
    f8 vs = {s, s, s, s, s, s, s, s};
    for (; i <= n - 8; i += 8) st8(dst + i, ld8(dst + i) + vs * ld8(src + i));
    for (; i < n; i++) dst[i] += s * src[i];
}

/* Dot (CpuBackend.cs:196-220). */
static inline float dot8(const float* x, const float* y, int n) {
    int i = 0;
    f8 acc = {0, 0, 0, 0, 0, 0, 0, 0};
    for (; i <= n - 8; i += 8) acc += ld8(x + i) * ld8(y + i);
    float sum = ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
    for (; i < n; i++) sum += x[i] * y[i];
    return sum;
}

/* MatMulNN (CpuBackend.cs:49-57, 118-164): y[M,N] = a[M,K] * b[K,N]. */
static void matmul_nn(const float* a, const float* b, float* y, int M, int K, int N) {
    long long work = (long long)M * K * N;
    if (work <= SMALL_MATMUL_WORK) {
        for (int m = 0; m < M; m++) {
            float* yr = y + (size_t)m * N;
            memset(yr, 0, (size_t)N * sizeof(float));
            for (int k = 0; k < K; k++) add_scaled(yr, b + (size_t)k * N, a[(size_t)m * K + k], N);
        }
        return;
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < M; m++) {
        float* yr = y + (size_t)m * N;
        memset(yr, 0, (size_t)N * sizeof(float));
        for (int k = 0; k < K; k++) add_scaled(yr, b + (size_t)k * N, a[(size_t)m * K + k], N);
    }
}

/* MatMulNT (CpuBackend.cs:71-115): y[M,N] = a[M,K] * b[N,K]^T. */
static void matmul_nt(const float* a, const float* b, float* y, int M, int K, int N) {
    long long work = (long long)M * K * N;
    if (work <= SMALL_MATMUL_WORK) {
        for (int m = 0; m < M; m++)
            for (int n = 0; n < N; n++) y[(size_t)m * N + n] = dot8(a + (size_t)m * K, b + (size_t)n * K, K);
        return;
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) y[(size_t)m * N + n] = dot8(a + (size_t)m * K, b + (size_t)n * K, K);
}

/* AddBias (CpuBackend.cs:281-289). */
static void add_bias(float* y, const float* bias, int rows, int cols) {
    for (int r = 0; r < rows; r++)
        for (int c = 0; c < cols; c++) y[(size_t)r * cols + c] += bias[c];
}

/* AddInPlace (CpuBackend.cs:307-318). */
static void add_in_place(float* dst, const float* src, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] += src[i];
}

/* LayerNormForward (CpuBackend.cs:377-398), eps = 1e-5f (Layers.cs:106). */
static void layer_norm(const float* x, const float* w, const float* b, float* out, int rows, int cols) {
    const float eps = 1e-5f;
    for (int r = 0; r < rows; r++) {
        const float* xr = x + (size_t)r * cols;
        float* o = out + (size_t)r * cols;
        float sum = 0.0f;
        for (int c = 0; c < cols; c++) sum += xr[c];
        float mu = sum / (float)cols;
        float var_sum = 0.0f;
        for (int c = 0; c < cols; c++) { float d = xr[c] - mu; var_sum += d * d; }
        float rs = 1.0f / sqrtf(var_sum / (float)cols + eps);
        for (int c = 0; c < cols; c++) o[c] = (xr[c] - mu) * rs * w[c] + b[c];
    }
}

/* SoftmaxForward (CpuBackend.cs:446-458), in place, row-wise. */
static void softmax_rows(float* x, int rows, int cols) {
    for (int r = 0; r < rows; r++) {
        float* row = x + (size_t)r * cols;
        float mx = row[0];
        for (int c = 1; c < cols; c++) mx = (row[c] > mx) ? row[c] : mx;
        float sum = 0.0f;
        for (int c = 0; c < cols; c++) { row[c] = expf(row[c] - mx); sum += row[c]; }
        float inv = 1.0f / sum;
        for (int c = 0; c < cols; c++) row[c] *= inv;
    }
}

/* Gelu (CpuBackend.cs:25-26, 510-514): tanh approximation. */
static inline float gelu(float v) {
    const float gelu_c = sqrtf(2.0f / (float)M_PI);
    const float coeff = 0.044715f;
    float u = gelu_c * (v + coeff * v * v * v);
    return 0.5f * v * (1.0f + tanhf(u));
}

/* ====================================================================== */
/* GptModel forward (GptModel.cs:212-222; Layers.cs)                        */
/* ====================================================================== */
typedef struct {
    const float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
    const float *ln2_w, *ln2_b, *fc_w, *fc_b, *mproj_w, *mproj_b;
} block_params;

static block_params get_block(const float* const* params, int layer) {
    const float* const* p = params + 2 + 12 * layer;
    block_params b = {p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7], p[8], p[9], p[10], p[11]};
    return b;
}

static int validate_config(const orc_config* c) {
    if (!c || c->vocab_size <= 0 || c->context_length <= 0 || c->d_model <= 0 || c->n_layers <= 0 ||
        c->n_heads <= 0 || c->d_model % c->n_heads != 0)
        return -1;
    return 0;
}

/* head_all_rows = 1 reproduces the reference cost (logits for every row,
 * Layers.cs:80-86); 0 computes only the last row (identical values there). */
static int32_t forward_impl(const orc_config* c, const float* const* params, const int32_t* tokens,
                            int32_t T, float* logits, int head_all_rows) {
    if (validate_config(c) || !params || !tokens || !logits || T <= 0 || T > c->context_length) return -1;
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= c->vocab_size) return -1; /* GptModel.cs:288-299 */
    const int D = c->d_model, H = c->n_heads, hd = D / H, F = 4 * D, V = c->vocab_size;
    const float inv_scale = 1.0f / sqrtf((float)hd); /* Layers.cs:174 */
    size_t td = (size_t)T * D;
    float* x = malloc(td * sizeof(float));
    float* ln = malloc(td * sizeof(float));
    float* qkv = malloc(td * 3 * sizeof(float));
    float* q = malloc(td * sizeof(float));
    float* k = malloc(td * sizeof(float));
    float* v = malloc(td * sizeof(float));
    float* probs = malloc((size_t)H * T * T * sizeof(float));
    float* ctx = malloc(td * sizeof(float));
    float* concat = malloc(td * sizeof(float));
    float* a = malloc(td * sizeof(float));
    float* f = malloc((size_t)T * F * sizeof(float));
    float* hbuf = malloc((size_t)T * F * sizeof(float));
    float* m = malloc(td * sizeof(float));
    if (!x || !ln || !qkv || !q || !k || !v || !probs || !ctx || !concat || !a || !f || !hbuf || !m) {
        free(x); free(ln); free(qkv); free(q); free(k); free(v); free(probs);
        free(ctx); free(concat); free(a); free(f); free(hbuf); free(m);
        return -1;
    }
    const float* tok_emb = params[0];
    const float* pos_emb = params[1];
    /* Embedding.Forward x2 + AddInPlace (GptModel.cs:217-218). */
    for (int t = 0; t < T; t++) {
        memcpy(x + (size_t)t * D, tok_emb + (size_t)tokens[t] * D, D * sizeof(float));
        add_in_place(x + (size_t)t * D, pos_emb + (size_t)t * D, D);
    }
    for (int l = 0; l < c->n_layers; l++) {
        block_params bp = get_block(params, l);
        /* TransformerBlock.Forward (Layers.cs:384-392); MHA (Layers.cs:191-229). */
        layer_norm(x, bp.ln1_w, bp.ln1_b, ln, T, D);
        matmul_nn(ln, bp.qkv_w, qkv, T, D, 3 * D);
        add_bias(qkv, bp.qkv_b, T, 3 * D);
        /* PackQkvHeads (ITensorBackend.cs:58-65; CpuBackend.cs:251-262). */
        for (int h = 0; h < H; h++)
            for (int t = 0; t < T; t++) {
                const float* row = qkv + (size_t)t * 3 * D;
                memcpy(q + ((size_t)h * T + t) * hd, row + h * hd, hd * sizeof(float));
                memcpy(k + ((size_t)h * T + t) * hd, row + D + h * hd, hd * sizeof(float));
                memcpy(v + ((size_t)h * T + t) * hd, row + 2 * D + h * hd, hd * sizeof(float));
            }
        /* BatchedMatMulNT, then Scale -> CausalMask -> SoftmaxForward
         * (ITensorBackend.cs:117-122; CpuBackend.cs:233-238, 338-346, 547-553). */
        for (int h = 0; h < H; h++)
            matmul_nt(q + (size_t)h * T * hd, k + (size_t)h * T * hd, probs + (size_t)h * T * T, T, hd, T);
        size_t np = (size_t)H * T * T;
        for (size_t i = 0; i < np; i++) probs[i] *= inv_scale;
        for (int h = 0; h < H; h++)
            for (int i = 0; i < T; i++)
                for (int j = i + 1; j < T; j++) probs[(size_t)h * T * T + (size_t)i * T + j] = -INFINITY;
        softmax_rows(probs, H * T, T);
        /* BatchedMatMulNN (CpuBackend.cs:225-230), then UnpackHeads. */
        for (int h = 0; h < H; h++)
            matmul_nn(probs + (size_t)h * T * T, v + (size_t)h * T * hd, ctx + (size_t)h * T * hd, T, T, hd);
        for (int h = 0; h < H; h++)
            for (int t = 0; t < T; t++)
                memcpy(concat + (size_t)t * D + h * hd, ctx + ((size_t)h * T + t) * hd, hd * sizeof(float));
        matmul_nn(concat, bp.proj_w, a, T, D, D);
        add_bias(a, bp.proj_b, T, D);
        add_in_place(a, x, td); /* a += x (Layers.cs:387) */
        /* Mlp.Forward (Layers.cs:306-313). */
        layer_norm(a, bp.ln2_w, bp.ln2_b, ln, T, D);
        matmul_nn(ln, bp.fc_w, f, T, D, F);
        add_bias(f, bp.fc_b, T, F);
        for (size_t i = 0; i < (size_t)T * F; i++) hbuf[i] = gelu(f[i]);
        matmul_nn(hbuf, bp.mproj_w, m, T, F, D);
        add_bias(m, bp.mproj_b, T, D);
        add_in_place(m, a, td); /* m += x2 (Layers.cs:390) */
        float* tmp = x; x = m; m = tmp;
    }
    /* Final LN + TiedOutputProjection (GptModel.cs:221; Layers.cs:80-86). */
    const float* lnf_w = params[2 + 12 * c->n_layers];
    const float* lnf_b = params[3 + 12 * c->n_layers];
    layer_norm(x, lnf_w, lnf_b, ln, T, D);
    if (head_all_rows) {
        matmul_nt(ln, tok_emb, logits, T, D, V);
    } else {
        const float* last = ln + (size_t)(T - 1) * D;
#pragma omp parallel for schedule(static)
        for (int n = 0; n < V; n++) logits[n] = dot8(last, tok_emb + (size_t)n * D, D);
    }
    free(x); free(ln); free(qkv); free(q); free(k); free(v); free(probs);
    free(ctx); free(concat); free(a); free(f); free(hbuf); free(m);
    return 0;
}

int32_t orc_forward(const orc_config* c, const float* const* params, const int32_t* tokens, int32_t T,
                    float* logits) {
    return forward_impl(c, params, tokens, T, logits, 1);
}

int32_t orc_forward_last(const orc_config* c, const float* const* params, const int32_t* tokens,
                         int32_t T, float* logits_last) {
    return forward_impl(c, params, tokens, T, logits_last, 0);
}

/* ====================================================================== */
/* Sampler (src/LLM.Core/Inference/Sampler.cs)                              */
/* ====================================================================== */

/* Sampler.Greedy (Sampler.cs:14-20): first index of the maximum. */
int32_t orc_greedy(const float* logits, int32_t v) {
    int32_t best = 0;
    for (int32_t i = 1; i < v; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* Array.Sort<float> order: NaN first, then ascending (-0 equals +0). */
static int cmp_float(const void* pa, const void* pb) {
    float a = *(const float*)pa, b = *(const float*)pb;
    if (a < b) return -1;
    if (a > b) return 1;
    if (a == b) return 0;
    if (isnan(a)) return isnan(b) ? 0 : -1;
    return 1;
}

/* Sampler.Sample (Sampler.cs:29-69) with the NextDouble() value `u`. */
int32_t orc_sample(const float* logits, int32_t v, float temperature, int32_t top_k, double u) {
    if (!logits || v <= 0) return -1;
    if (!isfinite(temperature)) return -1;
    if (temperature <= 0.0f) return orc_greedy(logits, v);
    float* probs = malloc((size_t)v * sizeof(float));
    if (!probs) return -1;
    for (int32_t i = 0; i < v; i++) probs[i] = logits[i] / temperature;
    if (top_k > 0 && top_k < v) {
        float* sorted = malloc((size_t)v * sizeof(float));
        if (!sorted) { free(probs); return -1; }
        memcpy(sorted, probs, (size_t)v * sizeof(float));
        qsort(sorted, (size_t)v, sizeof(float), cmp_float);
        float threshold = sorted[v - top_k];
        free(sorted);
        for (int32_t i = 0; i < v; i++)
            if (probs[i] < threshold) probs[i] = -INFINITY;
    }
    float mx = -INFINITY;
    for (int32_t i = 0; i < v; i++)
        if (probs[i] > mx) mx = probs[i];
    float sum = 0.0f;
    for (int32_t i = 0; i < v; i++) {
        probs[i] = expf(probs[i] - mx);
        sum += probs[i];
    }
    float uu = (float)u * sum;
    float acc = 0.0f;
    int32_t pick = v - 1; /* rounding fallback (Sampler.cs:68) */
    for (int32_t i = 0; i < v; i++) {
        acc += probs[i];
        if (uu < acc) { pick = i; break; }
    }
    free(probs);
    return pick;
}

/* Sampler.ValidateRepetitionOptions (Sampler.cs:167-175). */
static int valid_repetition(float penalty, int32_t ngram) {
    return isfinite(penalty) && penalty >= 1.0f && ngram >= 0;
}

/* Sampler.ApplyRepetitionControls (Sampler.cs:111-165). */
int32_t orc_apply_repetition_controls(float* logits, int32_t v, const int32_t* history, int32_t n,
                                      float penalty, int32_t ngram) {
    if (!valid_repetition(penalty, ngram) || !logits || (n > 0 && !history)) return -1;
    if (penalty != 1.0f) {
        unsigned char* seen = calloc((size_t)v, 1);
        if (!seen) return -1;
        for (int32_t i = 0; i < n; i++) {
            int32_t t = history[i];
            if ((uint32_t)t >= (uint32_t)v || seen[t]) continue;
            seen[t] = 1;
            logits[t] = logits[t] < 0.0f ? logits[t] * penalty : logits[t] / penalty;
        }
        free(seen);
    }
    if (ngram <= 0 || n < ngram - 1) return 0;
    float* before = malloc((size_t)v * sizeof(float));
    if (!before) return -1;
    memcpy(before, logits, (size_t)v * sizeof(float));
    if (ngram == 1) {
        for (int32_t i = 0; i < n; i++)
            if ((uint32_t)history[i] < (uint32_t)v) logits[history[i]] = -INFINITY;
    } else {
        int32_t prefix = ngram - 1;
        int32_t suffix_start = n - prefix;
        for (int32_t start = 0; start + ngram <= n; start++) {
            int matches = 1;
            for (int32_t j = 0; j < prefix; j++)
                if (history[start + j] != history[suffix_start + j]) { matches = 0; break; }
            if (!matches) continue;
            int32_t banned = history[start + prefix];
            if ((uint32_t)banned < (uint32_t)v) logits[banned] = -INFINITY;
        }
    }
    int any = 0;
    for (int32_t i = 0; i < v; i++)
        if (!(isinf(logits[i]) && logits[i] < 0)) { any = 1; break; }
    if (!any) memcpy(logits, before, (size_t)v * sizeof(float));
    free(before);
    return 0;
}

/* One step of Sampler.Generate after the forward (Sampler.cs:96-104). */
static int32_t sample_step_u(const float* logits, int32_t v, const int32_t* window, int32_t wlen,
                             float temperature, int32_t top_k, float penalty, int32_t ngram, double u) {
    if (penalty != 1.0f || ngram > 0) {
        float* adj = malloc((size_t)v * sizeof(float));
        if (!adj) return -1;
        memcpy(adj, logits, (size_t)v * sizeof(float));
        if (orc_apply_repetition_controls(adj, v, window, wlen, penalty, ngram)) { free(adj); return -1; }
        int32_t id = orc_sample(adj, v, temperature, top_k, u);
        free(adj);
        return id;
    }
    return orc_sample(logits, v, temperature, top_k, u);
}

int32_t orc_sample_step(const float* logits, int32_t v, const int32_t* window, int32_t wlen,
                        float temperature, int32_t top_k, float penalty, int32_t ngram,
                        orc_dotnet_random* rng) {
    if (!isfinite(temperature)) return -1;
    double u = 0.0;
    if (temperature > 0.0f) u = orc_random_next_double(rng); /* Sampler.cs:61 */
    return sample_step_u(logits, v, window, wlen, temperature, top_k, penalty, ngram, u);
}

/* Sampler.Generate (Sampler.cs:78-109). */
static int32_t generate_impl(const orc_config* c, const float* const* params, const int32_t* prompt,
                             int32_t prompt_len, int32_t max_new, float temperature, int32_t top_k,
                             orc_dotnet_random* rng, const double* uniforms, int32_t eos_id,
                             float penalty, int32_t ngram, int32_t* out_tokens, float* out_logits) {
    if (validate_config(c) || !prompt || prompt_len <= 0 || max_new < 0) return -1;
    if (eos_id >= c->vocab_size) return -1;
    if (!valid_repetition(penalty, ngram)) return -1;
    if (!isfinite(temperature)) return -1;
    const int32_t V = c->vocab_size, ctx = c->context_length;
    int32_t cap = prompt_len + max_new;
    int32_t* window = malloc((size_t)cap * sizeof(int32_t));
    float* logits_all = malloc((size_t)ctx * V * sizeof(float));
    if (!window || !logits_all) { free(window); free(logits_all); return -1; }
    memcpy(window, prompt, (size_t)prompt_len * sizeof(int32_t));
    int32_t wlen = prompt_len, count = 0, used = 0;
    for (int32_t n = 0; n < max_new; n++) {
        if (wlen > ctx) { /* Sampler.cs:93-94 */
            memmove(window, window + (wlen - ctx), (size_t)ctx * sizeof(int32_t));
            wlen = ctx;
        }
        if (forward_impl(c, params, window, wlen, logits_all, 1)) { count = -1; break; }
        const float* last = logits_all + (size_t)(wlen - 1) * V; /* GptModel.cs:202-209 */
        if (out_logits) memcpy(out_logits + (size_t)n * V, last, (size_t)V * sizeof(float));
        double u = 0.0;
        if (temperature > 0.0f) u = uniforms ? uniforms[used++] : orc_random_next_double(rng);
        int32_t next = sample_step_u(last, V, window, wlen, temperature, top_k, penalty, ngram, u);
        if (next < 0) { count = -1; break; }
        out_tokens[count++] = next;
        window[wlen++] = next;
        if (eos_id >= 0 && next == eos_id) break;
    }
    free(window);
    free(logits_all);
    return count;
}

int32_t orc_generate(const orc_config* c, const float* const* params, const int32_t* prompt,
                     int32_t prompt_len, int32_t max_new, float temperature, int32_t top_k,
                     orc_dotnet_random* rng, int32_t eos_id, float penalty, int32_t ngram,
                     int32_t* out_tokens, float* out_logits) {
    if (!rng) return -1;
    return generate_impl(c, params, prompt, prompt_len, max_new, temperature, top_k, rng, NULL, eos_id,
                         penalty, ngram, out_tokens, out_logits);
}

int32_t orc_generate_uniforms(const orc_config* c, const float* const* params, const int32_t* prompt,
                              int32_t prompt_len, int32_t max_new, float temperature, int32_t top_k,
                              const double* uniforms, int32_t eos_id, float penalty, int32_t ngram,
                              int32_t* out_tokens, float* out_logits) {
    if (!uniforms && temperature > 0.0f) return -1;
    return generate_impl(c, params, prompt, prompt_len, max_new, temperature, top_k, NULL, uniforms,
                         eos_id, penalty, ngram, out_tokens, out_logits);
}

void orc_gelu_array(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = gelu(x[i]);
}

void orc_layer_norm_rows(const float* x, const float* w, const float* b, float* out, int32_t rows,
                         int32_t cols) {
    layer_norm(x, w, b, out, rows, cols);
}

void orc_softmax_rows(float* x, int32_t rows, int32_t cols) { softmax_rows(x, rows, cols); }

void orc_set_threads(int32_t n) {
#ifdef _OPENMP
    if (n <= 0) n = omp_get_num_procs();
    omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int32_t orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_expf_array(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

int64_t orc_expf_vs_double_scan(uint32_t lo_bits, uint32_t hi_bits, uint32_t* out_bits, int64_t max_out) {
    int64_t found = 0;
    for (uint64_t b = lo_bits; b <= hi_bits; b++) {
        uint32_t bits = (uint32_t)b;
        float x;
        memcpy(&x, &bits, sizeof(x));
        float e1 = expf(x);
        float e2 = (float)exp((double)x);
        if (memcmp(&e1, &e2, sizeof(float)) != 0) {
            if (found < max_out && out_bits) out_bits[found] = bits;
            found++;
        }
    }
    return found;
}

void orc_expf_hash(uint32_t lo_bits, int32_t nchunks, uint64_t* hashes) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int32_t c = 0; c < nchunks; c++) {
        uint64_t h = 0;
        for (uint32_t j = 0; j < (1u << 20); j++) {
            uint32_t bits = lo_bits + (uint32_t)c * (1u << 20) + j;
            float x;
            memcpy(&x, &bits, 4);
            uint32_t o = 0;
            if (!isnan(x)) {
                float e = expf(x);
                memcpy(&o, &e, 4);
            }
            uint64_t v = ((uint64_t)o * 0x9E3779B97F4A7C15ull) ^ ((uint64_t)bits << 17);
            h += v * 0xBF58476D1CE4E5B9ull + (v >> 29);
        }
        hashes[c] = h;
    }
}
