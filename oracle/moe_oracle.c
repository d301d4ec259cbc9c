/*
 * moe_oracle.c -- CPU restatement of the GPT-OSS MoE block of lutikk/airllm.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  Not part of the product library.
 *
 * Arithmetic follows the reference Go code exactly:
 *   - every dot product accumulates float64(x)*float64(w) sequentially over the
 *     input index and rounds to float32 once (primitives.go:23-30); a product of
 *     two float32 values is exact in float64, so contraction into FMA cannot
 *     change a result;
 *   - biases are added in float32 after that rounding (primitives.go:43-45);
 *   - MXFP4 weights are float32(scale) * table[nibble] (tensor.go:152-159);
 *   - the top-k order is a stable descending order with ties to the lower
 *     expert id, the softmax runs in float64 over the selected logits only
 *     (moe.go:20-39);
 *   - the expert mixture accumulates float64(p)*float64(y) in slot order and is
 *     added to the pre-norm row in float32 (layer.go:109-121).
 * Compile without -ffast-math (denormal MXFP4 scales must not be flushed).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* E2M1 code -> value, internal/model/gptoss/tensor.go:167-170 */
static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* E8M0 block scale, tensor.go:152-155: 2^(b-127), 0xff is NaN. */
static inline float e8m0_scale(uint8_t b) {
    if (b == 0xff) return NAN;
    return (float)ldexp(1.0, (int)b - 127);
}

int64_t oracle_mxfp4_encoded_size(int64_t elements) {
    /* reader.go:442-449 */
    if (elements < 0 || elements % 32 != 0) return -1;
    return elements / 32 * 17;
}

int oracle_mxfp4_decode(const uint8_t *data, int64_t nbytes, int64_t elements, float *out) {
    /* tensor.go:145-160: 17-byte blocks; byte j (1..16) low nibble -> element
     * 2(j-1), high nibble -> element 2(j-1)+1. */
    if (elements % 32 != 0 || nbytes != elements / 32 * 17) return -1;
    for (int64_t blk = 0; blk < elements / 32; ++blk) {
        const uint8_t *enc = data + blk * 17;
        float scale = e8m0_scale(enc[0]);
        for (int i = 0; i < 16; ++i) {
            uint8_t packed = enc[1 + i];
            out[blk * 32 + 2 * i] = scale * kE2M1[packed & 0x0f];
            out[blk * 32 + 2 * i + 1] = scale * kE2M1[packed >> 4];
        }
    }
    return 0;
}

int oracle_rmsnorm(const float *x, const float *g, int n, float eps, float *out) {
    /* primitives.go:50-72 */
    if (n <= 0) return -1;
    if (!(eps > 0.0f)) return -1; /* also rejects NaN */
    double sum_squares = 0.0;
    for (int i = 0; i < n; ++i) sum_squares += (double)x[i] * (double)x[i];
    double inverse_rms = 1.0 / sqrt(sum_squares / (double)n + (double)eps);
    for (int i = 0; i < n; ++i) out[i] = (float)((double)x[i] * inverse_rms * (double)g[i]);
    return 0;
}

int oracle_linear_bias(const float *x, const float *w, const float *b, int in_dim,
                       int out_dim, float *y) {
    /* primitives.go:11-47 */
    if (in_dim <= 0 || out_dim <= 0) return -1;
    for (int o = 0; o < out_dim; ++o) {
        const float *row = w + (int64_t)o * in_dim;
        double sum = 0.0;
        for (int i = 0; i < in_dim; ++i) sum += (double)x[i] * (double)row[i];
        y[o] = (float)sum;
    }
    if (b)
        for (int o = 0; o < out_dim; ++o) y[o] += b[o];
    return 0;
}

int oracle_router_topk(const float *logits, int n, int k, int32_t *idx, float *w) {
    /* moe.go:12-41.  The first k entries of a stable descending sort equal k
     * rounds of "largest remaining value, lowest index among equals" for
     * ordered (non-NaN) inputs; NaN logits have no defined order in either. */
    if (n <= 0 || k <= 0 || k > n) return -1;
    unsigned char used_stack[1024];
    unsigned char *used = n <= 1024 ? used_stack : (unsigned char *)calloc((size_t)n, 1);
    if (!used) return -1;
    memset(used, 0, (size_t)n);
    for (int s = 0; s < k; ++s) {
        int best = -1;
        for (int e = 0; e < n; ++e) {
            if (used[e]) continue;
            if (best < 0 || logits[e] > logits[best]) best = e;
        }
        used[best] = 1;
        idx[s] = best;
    }
    if (used != used_stack) free(used);
    double max_logit = (double)logits[idx[0]];
    double denominator = 0.0;
    for (int s = 0; s < k; ++s) {
        double weight = exp((double)logits[idx[s]] - max_logit);
        w[s] = (float)weight;
        denominator += weight;
    }
    for (int s = 0; s < k; ++s) w[s] = (float)((double)w[s] / denominator);
    return 0;
}

/* Go math.Min / math.Max semantics for the operands used here: NaN wins. */
static inline double go_min(double a, double b) {
    if (isnan(a) || isnan(b)) return NAN;
    return a < b ? a : b;
}
static inline double go_max(double a, double b) {
    if (isnan(a) || isnan(b)) return NAN;
    return a > b ? a : b;
}

int oracle_swiglu(const float *gate, const float *up, int n, float *out) {
    /* primitives.go:138-149 */
    for (int i = 0; i < n; ++i) {
        double g = go_min((double)gate[i], 7.0);
        double u = go_max(-7.0, go_min(7.0, (double)up[i]));
        out[i] = (float)(g / (1.0 + exp(-1.702 * g)) * (u + 1.0));
    }
    return 0;
}

/* Dot product of float32 x with one MXFP4 row decoded on the fly; identical
 * to decoding the row first and calling Linear.  Four rows are interleaved to
 * give the CPU independent dependency chains; each chain keeps the sequential
 * input order, so results are bit-identical to one row at a time. */
static void mxfp4_rows4(const float *x, const uint8_t *rows, int64_t row_bytes, int nrows,
                        int in_dim, double *sums) {
    double s[4] = {0, 0, 0, 0};
    const int nblk = in_dim / 32;
    for (int blk = 0; blk < nblk; ++blk) {
        float scale[4];
        const uint8_t *enc[4];
        for (int r = 0; r < nrows; ++r) {
            enc[r] = rows + r * row_bytes + (int64_t)blk * 17;
            scale[r] = e8m0_scale(enc[r][0]);
        }
        const float *xb = x + blk * 32;
        for (int i = 0; i < 16; ++i) {
            double x0 = (double)xb[2 * i], x1 = (double)xb[2 * i + 1];
            for (int r = 0; r < nrows; ++r) {
                uint8_t p = enc[r][1 + i];
                s[r] += x0 * (double)(scale[r] * kE2M1[p & 0x0f]);
                s[r] += x1 * (double)(scale[r] * kE2M1[p >> 4]);
            }
        }
    }
    for (int r = 0; r < nrows; ++r) sums[r] = s[r];
}

static void linear_bias_mxfp4(const float *x, const uint8_t *w, const float *b, int in_dim,
                              int out_dim, float *y) {
    const int64_t row_bytes = (int64_t)in_dim / 32 * 17;
    for (int o = 0; o < out_dim; o += 4) {
        int nrows = out_dim - o < 4 ? out_dim - o : 4;
        double sums[4];
        mxfp4_rows4(x, w + (int64_t)o * row_bytes, row_bytes, nrows, in_dim, sums);
        for (int r = 0; r < nrows; ++r) y[o + r] = (float)sums[r];
    }
    for (int o = 0; o < out_dim; ++o) y[o] += b[o];
}

typedef struct {
    float *normalized, *logits, *gate_up, *gate, *up, *act, *down;
    double *mixture;
    float *wgu, *wdn; /* faithful mode: one decoded expert */
} scratch;

static int scratch_init(scratch *s, const oracle_layer *L, int faithful) {
    const int H = L->hidden, I = L->intermediate, E = L->experts;
    memset(s, 0, sizeof(*s));
    s->normalized = (float *)malloc(sizeof(float) * H);
    s->logits = (float *)malloc(sizeof(float) * E);
    s->gate_up = (float *)malloc(sizeof(float) * 2 * I);
    s->gate = (float *)malloc(sizeof(float) * I);
    s->up = (float *)malloc(sizeof(float) * I);
    s->act = (float *)malloc(sizeof(float) * I);
    s->down = (float *)malloc(sizeof(float) * H);
    s->mixture = (double *)malloc(sizeof(double) * H);
    if (faithful) {
        s->wgu = (float *)malloc(sizeof(float) * (size_t)2 * I * H);
        s->wdn = (float *)malloc(sizeof(float) * (size_t)H * I);
    }
    return (s->normalized && s->logits && s->gate_up && s->gate && s->up && s->act &&
            s->down && s->mixture && (!faithful || (s->wgu && s->wdn)))
               ? 0
               : -1;
}

static void scratch_free(scratch *s) {
    free(s->normalized); free(s->logits); free(s->gate_up); free(s->gate); free(s->up);
    free(s->act); free(s->down); free(s->mixture); free(s->wgu); free(s->wdn);
}

/* forwardExpert, layer.go:126-188 (fused gate_up dialect, layer.go:130-148). */
static int forward_expert(const oracle_layer *L, const float *hidden, int expert, int faithful,
                          scratch *s) {
    const int H = L->hidden, I = L->intermediate;
    const int64_t gu_bytes = (int64_t)2 * I * (H / 32) * 17;
    const int64_t dn_bytes = (int64_t)H * (I / 32) * 17;
    const uint8_t *gu = L->gate_up + (int64_t)expert * gu_bytes; /* tensor.go:101-103 */
    const uint8_t *dn = L->down + (int64_t)expert * dn_bytes;
    const float *gub = L->gate_up_b + (int64_t)expert * 2 * I;
    const float *dnb = L->down_b + (int64_t)expert * H;
    if (faithful) {
        if (oracle_mxfp4_decode(gu, gu_bytes, (int64_t)2 * I * H, s->wgu)) return -1;
        oracle_linear_bias(hidden, s->wgu, gub, H, 2 * I, s->gate_up);
    } else {
        linear_bias_mxfp4(hidden, gu, gub, H, 2 * I, s->gate_up);
    }
    for (int i = 0; i < I; ++i) { /* layer.go:145-148 */
        s->gate[i] = s->gate_up[2 * i];
        s->up[i] = s->gate_up[2 * i + 1];
    }
    oracle_swiglu(s->gate, s->up, I, s->act);
    if (faithful) {
        if (oracle_mxfp4_decode(dn, dn_bytes, (int64_t)H * I, s->wdn)) return -1;
        oracle_linear_bias(s->act, s->wdn, dnb, I, H, s->down);
    } else {
        linear_bias_mxfp4(s->act, dn, dnb, I, H, s->down);
    }
    return 0;
}

static int validate(const oracle_layer *L) {
    if (!L || L->hidden <= 0 || L->intermediate <= 0 || L->experts <= 0) return -1;
    if (L->hidden % 32 || L->intermediate % 32) return -1;
    if (L->top_k <= 0 || L->top_k > L->experts) return -1;
    return 0;
}

static int route_row(const oracle_layer *L, const float *row, scratch *s, int32_t *idx,
                     float *w) {
    if (oracle_rmsnorm(row, L->norm_gain, L->hidden, L->eps, s->normalized)) return -1;
    oracle_linear_bias(s->normalized, L->router_w, L->router_b, L->hidden, L->experts,
                       s->logits);
    return oracle_router_topk(s->logits, L->experts, L->top_k, idx, w);
}

int oracle_route(const oracle_layer *L, const float *residual, int T, float *logits,
                 int32_t *topk_idx, float *topk_w, int threads) {
    if (validate(L) || T < 0) return -1;
    int status = 0;
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
    {
        scratch s;
        int ok = scratch_init(&s, L, 0) == 0;
        if (!ok) {
#pragma omp atomic write
            status = -1;
        }
#pragma omp for schedule(static)
        for (int t = 0; t < T; ++t) {
            if (!ok) continue;
            const float *row = residual + (int64_t)t * L->hidden;
            if (route_row(L, row, &s, topk_idx + (int64_t)t * L->top_k,
                          topk_w + (int64_t)t * L->top_k)) {
#pragma omp atomic write
                status = -1;
            }
            if (logits) memcpy(logits + (int64_t)t * L->experts, s.logits, sizeof(float) * L->experts);
        }
        scratch_free(&s);
    }
    return status;
}

int oracle_moe_block(const oracle_layer *L, const float *residual, int T, float *out,
                     int32_t *topk_idx, float *topk_w, float *logits, const int32_t *tokens,
                     int n_tokens, int faithful, int threads) {
    if (validate(L) || T < 0) return -1;
    const int H = L->hidden, k = L->top_k;
    const int n = tokens ? n_tokens : T;
    int status = 0;
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
    {
        scratch s;
        int ok = scratch_init(&s, L, faithful) == 0;
        if (!ok) {
#pragma omp atomic write
            status = -1;
        }
        int32_t idx[256];
        float w[256];
#pragma omp for schedule(dynamic, 1)
        for (int j = 0; j < n; ++j) {
            if (!ok) continue;
            const int t = tokens ? tokens[j] : j;
            if (t < 0 || t >= T || k > 256) {
#pragma omp atomic write
                status = -1;
                continue;
            }
            const float *row = residual + (int64_t)t * H; /* layer.go:96 */
            if (route_row(L, row, &s, idx, w)) {          /* layer.go:97-108 */
#pragma omp atomic write
                status = -1;
                continue;
            }
            for (int i = 0; i < H; ++i) s.mixture[i] = 0.0;
            for (int slot = 0; slot < k; ++slot) { /* layer.go:110-118 */
                if (forward_expert(L, s.normalized, idx[slot], faithful, &s)) {
#pragma omp atomic write
                    status = -1;
                    break;
                }
                for (int i = 0; i < H; ++i) s.mixture[i] += (double)w[slot] * (double)s.down[i];
            }
            for (int i = 0; i < H; ++i) /* layer.go:119-121 */
                out[(int64_t)t * H + i] = row[i] + (float)s.mixture[i];
            if (topk_idx) memcpy(topk_idx + (int64_t)t * k, idx, sizeof(int32_t) * k);
            if (topk_w) memcpy(topk_w + (int64_t)t * k, w, sizeof(float) * k);
            if (logits) memcpy(logits + (int64_t)t * L->experts, s.logits, sizeof(float) * L->experts);
        }
        scratch_free(&s);
    }
    return status;
}

int oracle_expert_rows(const oracle_layer *L, int expert, const float *x, int n, float *y, int threads) {
    if (validate(L) || expert < 0 || expert >= L->experts || n < 0) return -1;
    int status = 0;
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
    {
        scratch s;
        int ok = scratch_init(&s, L, 0) == 0;
#pragma omp for schedule(dynamic, 1)
        for (int j = 0; j < n; ++j) {
            if (!ok || forward_expert(L, x + (int64_t)j * L->hidden, expert, 0, &s)) {
#pragma omp atomic write
                status = -1;
                continue;
            }
            memcpy(y + (int64_t)j * L->hidden, s.down, sizeof(float) * L->hidden);
        }
        scratch_free(&s);
    }
    return status;
}

int oracle_permute(const int32_t *topk_idx, int T, int k, int E, int32_t *perm_pair,
                   int32_t *counts, int32_t *offsets, int32_t *inv) {
    if (T < 0 || k <= 0 || E <= 0) return -1;
    for (int e = 0; e < E; ++e) counts[e] = 0;
    for (int64_t p = 0; p < (int64_t)T * k; ++p) {
        int e = topk_idx[p];
        if (e < 0 || e >= E) return -1;
        counts[e]++;
    }
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *cursor = (int32_t *)malloc(sizeof(int32_t) * E);
    if (!cursor) return -1;
    memcpy(cursor, offsets, sizeof(int32_t) * E);
    /* pairs visited in (t, s) order: a stable counting sort by expert */
    for (int64_t p = 0; p < (int64_t)T * k; ++p) {
        int e = topk_idx[p];
        int32_t pos = cursor[e]++;
        perm_pair[pos] = (int32_t)p;
        inv[p] = pos;
    }
    free(cursor);
    return 0;
}

/* ---- block-scaled FP4 activation terms (see moe_oracle.h) ---------------------- */

/* E2M1 code of v (|v| <= 6 after saturation), round to nearest, ties to the even
 * mantissa: the grid is 0, .5, 1, 1.5, 2, 3, 4, 6 (codes 0..7, sign in bit 3). */
static uint8_t e2m1_rne(float v) {
    static const float grid[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const uint8_t sign = (v < 0.0f) ? 8u : 0u;
    float a = fabsf(v);
    if (a >= 6.0f) return (uint8_t)(sign | 7u);
    int lo = 0;
    while (lo < 7 && grid[lo + 1] <= a) ++lo;
    if (lo == 7 || a == grid[lo]) return (uint8_t)(sign | (uint8_t)lo);
    const float dl = a - grid[lo], dh = grid[lo + 1] - a;
    int code;
    if (dl < dh) code = lo;
    else if (dh < dl) code = lo + 1;
    else code = (lo & 1) ? lo + 1 : lo; /* tie: the code with an even mantissa bit */
    if (code == 0) return 0; /* no negative zero code */
    return (uint8_t)(sign | (uint8_t)code);
}

static float e2m1_value(uint8_t code) {
    static const float grid[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    return (code & 8u) ? -grid[code & 7u] : grid[code & 7u];
}

int oracle_e2m1_terms(const float *x, int64_t n, int terms, uint8_t *codes, uint8_t *scales) {
    if (!x || !codes || !scales || n <= 0 || n % 32 != 0 || terms < 1) return -1;
    for (int64_t i = 0; i < n; ++i)
        if (!isfinite(x[i])) return -1;
    const int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        float r[32];
        memcpy(r, x + b * 32, sizeof(r));
        for (int j = 0; j < terms; ++j) {
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(r[i]));
            int e = 0;
            if (amax > 0.0f) {
                int p;
                const float m = frexpf(amax, &p); /* amax = m 2^p, m in [0.5, 1) */
                e = (m * 8.0f <= 6.0f) ? p - 3 : p - 2;
            }
            if (e < -127) e = -127; /* the smallest E8M0 scale */
            if (e > 127) return -1;
            scales[(int64_t)j * nb + b] = (uint8_t)(e + 127);
            uint8_t *cj = codes + (int64_t)j * (n / 2) + b * 16;
            for (int i = 0; i < 32; i += 2) {
                const uint8_t c0 = e2m1_rne(ldexpf(r[i], -e)), c1 = e2m1_rne(ldexpf(r[i + 1], -e));
                cj[i / 2] = (uint8_t)(c0 | (c1 << 4));
                r[i] = r[i] - ldexpf(e2m1_value(c0), e);
                r[i + 1] = r[i + 1] - ldexpf(e2m1_value(c1), e);
            }
        }
    }
    return 0;
}


/* ---- expert-major evaluation (same arithmetic, all experts at once) ------------------
 *
 * oracle_moe_block_grouped computes exactly what oracle_moe_block computes, with
 * the work reordered so that every expert's MXFP4 rows are decoded once per call
 * instead of once per (token, expert): each output element is still the float64
 * sum of float64(x_i) * float64(w_i) in increasing i from 0.0, rounded to float32
 * once, then the float32 bias (primitives.go:23-30, 43-45); SwiGLU, the slot-order
 * mixture and the residual add are the per-token code's.  A product of two
 * float32 values is exact in float64, so vectorising over tokens (each token
 * keeping its own sequential chain) changes no bit.  Used to check full
 * prefill-sized outputs in seconds; tests pin it to oracle_moe_block. */

#define GROUP_ROWS 16  /* weight rows decoded per work item */
#define GROUP_TOK 8    /* tokens whose dot products run side by side */

/* acc[r][j] = sum_i xt[i][j] * w[r][i] (sequential in i, from 0.0) for GROUP_ROWS
 * rows of decoded weights w (nrows, a multiple of 8) and GROUP_TOK token columns
 * xt: eight rows by eight tokens per pass, one float64 chain per (row, token). */
typedef double v8d __attribute__((vector_size(64)));
#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
__attribute__((target_clones("avx512f", "avx2", "default")))
#endif
static void dot_block(const double *xt, const double *w, int in_dim, int nrows, double acc[GROUP_ROWS][GROUP_TOK]) {
    for (int r = 0; r < nrows; r += 8) {
        v8d a[8];
        for (int q = 0; q < 8; ++q) a[q] = (v8d){0, 0, 0, 0, 0, 0, 0, 0};
        const double *wr = w + (int64_t)r * in_dim;
        for (int i = 0; i < in_dim; ++i) {
            v8d x;
            memcpy(&x, xt + (int64_t)i * GROUP_TOK, sizeof(x));
            for (int q = 0; q < 8; ++q) a[q] += x * wr[(int64_t)q * in_dim + i];
        }
        for (int q = 0; q < 8; ++q) memcpy(acc[r + q], &a[q], sizeof(v8d));
    }
}

/* Decodes rows [r0, r0 + n) of one expert's MXFP4 tensor into float64 (via the
 * float32 value scale * table[nibble], tensor.go:152-159).  Rows past n are zero. */
static void decode_rows_f64(const uint8_t *w, int in_dim, int r0, int n, double *out) {
    const int64_t row_bytes = (int64_t)in_dim / 32 * 17;
    for (int r = 0; r < GROUP_ROWS; ++r) {
        double *o = out + (int64_t)r * in_dim;
        if (r >= n) {
            memset(o, 0, sizeof(double) * (size_t)in_dim);
            continue;
        }
        const uint8_t *row = w + (int64_t)(r0 + r) * row_bytes;
        for (int b = 0; b < in_dim / 32; ++b) {
            const uint8_t *enc = row + (int64_t)b * 17;
            const float scale = e8m0_scale(enc[0]);
            for (int i = 0; i < 16; ++i) {
                o[b * 32 + 2 * i] = (double)(scale * kE2M1[enc[1 + i] & 0x0f]);
                o[b * 32 + 2 * i + 1] = (double)(scale * kE2M1[enc[1 + i] >> 4]);
            }
        }
    }
}

/* One linear layer over an expert's pairs: y[pair][o] = f32(sum) + b[o] for output
 * rows [r0, r0 + GROUP_ROWS), x rows taken from x + rowsel[j] * in_dim. */
static void expert_rows_block(const double *wdec, int in_dim, int r0, int nrows, const float *b,
                              const float *x, const int64_t *rowsel, int npairs, float *y, int64_t y_pitch,
                              double *xt) {
    double acc[GROUP_ROWS][GROUP_TOK];
    for (int j0 = 0; j0 < npairs; j0 += GROUP_TOK) {
        const int nt = npairs - j0 < GROUP_TOK ? npairs - j0 : GROUP_TOK;
        for (int j = 0; j < GROUP_TOK; ++j) {
            const float *xr = j < nt ? x + rowsel[j0 + j] * in_dim : NULL;
            for (int i = 0; i < in_dim; ++i) xt[(int64_t)i * GROUP_TOK + j] = xr ? (double)xr[i] : 0.0;
        }
        dot_block(xt, wdec, in_dim, (nrows + 7) & ~7, acc);
        for (int j = 0; j < nt; ++j) {
            float *yr = y + (int64_t)(j0 + j) * y_pitch;
            for (int r = 0; r < nrows; ++r) yr[r0 + r] = (float)acc[r][j];
        }
    }
    for (int j = 0; j < npairs; ++j) {
        float *yr = y + (int64_t)j * y_pitch;
        for (int r = 0; r < nrows; ++r) yr[r0 + r] += b[r0 + r];
    }
}

int oracle_moe_block_grouped(const oracle_layer *L, const float *residual, int T, float *out,
                             int32_t *topk_idx, float *topk_w, float *logits, const int32_t *tokens,
                             int n_tokens, int threads) {
    if (validate(L) || T < 0 || L->top_k > 256) return -1;
    const int H = L->hidden, I = L->intermediate, E = L->experts, k = L->top_k;
    const int n = tokens ? n_tokens : T;
    const int nth = threads > 0 ? threads : 1;
    if (n < 0) return -1;
    for (int j = 0; j < n; ++j)
        if (tokens && (tokens[j] < 0 || tokens[j] >= T)) return -1;
    const int64_t P = (int64_t)n * k;
    float *xn = (float *)malloc(sizeof(float) * ((size_t)n * H + 1));
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * ((size_t)P + 1));
    float *w = (float *)malloc(sizeof(float) * ((size_t)P + 1));
    float *lg = (float *)malloc(sizeof(float) * ((size_t)n * E + 1));
    int64_t *order = (int64_t *)malloc(sizeof(int64_t) * ((size_t)P + 1)); /* pairs, expert-major */
    int64_t *tok_of = (int64_t *)malloc(sizeof(int64_t) * ((size_t)P + 1)); /* x row of each sorted pair */
    int64_t *start = (int64_t *)calloc((size_t)E + 1, sizeof(int64_t));
    float *act = (float *)malloc(sizeof(float) * ((size_t)P * I + 1)); /* by sorted position */
    float *y = (float *)malloc(sizeof(float) * ((size_t)P * H + 1));   /* by sorted position */
    int status = 0;
    if (!xn || !idx || !w || !lg || !order || !tok_of || !start || !act || !y) status = -1;
    /* 1. routing (layer.go:96-108) */
#pragma omp parallel num_threads(nth)
    {
        scratch s;
        int ok = status == 0 && scratch_init(&s, L, 0) == 0;
#pragma omp for schedule(static)
        for (int j = 0; j < n; ++j) {
            if (!ok) continue;
            const int t = tokens ? tokens[j] : j;
            if (route_row(L, residual + (int64_t)t * H, &s, idx + (int64_t)j * k, w + (int64_t)j * k)) {
#pragma omp atomic write
                status = -1;
                continue;
            }
            memcpy(xn + (int64_t)j * H, s.normalized, sizeof(float) * H);
            memcpy(lg + (int64_t)j * E, s.logits, sizeof(float) * E);
        }
        if (ok) scratch_free(&s);
        else {
#pragma omp atomic write
            status = -1;
        }
    }
    if (status == 0) {
        /* 2. pairs grouped by expert, (token, slot) order within an expert */
        for (int64_t p = 0; p < P; ++p) start[idx[p] + 1]++;
        for (int e = 0; e < E; ++e) start[e + 1] += start[e];
        int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * ((size_t)E + 1));
        if (!cur) status = -1;
        else {
            memcpy(cur, start, sizeof(int64_t) * (size_t)E);
            for (int64_t p = 0; p < P; ++p) {
                const int64_t pos = cur[idx[p]]++;
                order[pos] = p;
                tok_of[pos] = p / k;
            }
            free(cur);
        }
    }
    if (status == 0) {
        const int64_t gu_bytes = (int64_t)2 * I * (H / 32) * 17, dn_bytes = (int64_t)H * (I / 32) * 17;
        const int gu_blocks = (2 * I + GROUP_ROWS - 1) / GROUP_ROWS, dn_blocks = (H + GROUP_ROWS - 1) / GROUP_ROWS;
        const int kmax = H > I ? H : I;
        /* 3. gate_up + SwiGLU (layer.go:126-175), then 4. down (layer.go:179-187) */
        for (int phase = 0; phase < 2 && status == 0; ++phase) {
            const int nblk = phase == 0 ? gu_blocks : dn_blocks;
#pragma omp parallel num_threads(nth)
            {
                double *wdec = (double *)malloc(sizeof(double) * (size_t)GROUP_ROWS * kmax);
                double *xt = (double *)malloc(sizeof(double) * (size_t)GROUP_TOK * kmax);
                float *gu = (float *)malloc(sizeof(float) * (size_t)GROUP_TOK * GROUP_ROWS);
                int64_t *rowsel = (int64_t *)malloc(sizeof(int64_t) * (size_t)GROUP_TOK);
                const int ok = wdec && xt && gu && rowsel;
                if (!ok) {
#pragma omp atomic write
                    status = -1;
                }
#pragma omp for schedule(dynamic, 1)
                for (int64_t item = 0; item < (int64_t)E * nblk; ++item) {
                    const int e = (int)(item / nblk), blk = (int)(item % nblk);
                    const int64_t p0 = start[e], np = start[e + 1] - start[e];
                    if (!ok || np == 0) continue;
                    if (phase == 0) {
                        const int r0 = blk * GROUP_ROWS;
                        const int nr = 2 * I - r0 < GROUP_ROWS ? 2 * I - r0 : GROUP_ROWS;
                        decode_rows_f64(L->gate_up + (int64_t)e * gu_bytes, H, r0, nr, wdec);
                        const float *bias = L->gate_up_b + (int64_t)e * 2 * I;
                        for (int64_t j0 = 0; j0 < np; j0 += GROUP_TOK) {
                            const int nt = np - j0 < GROUP_TOK ? (int)(np - j0) : GROUP_TOK;
                            for (int j = 0; j < nt; ++j) rowsel[j] = tok_of[p0 + j0 + j];
                            /* gu[j][r]: rows r0.. of pair j (bias included) */
                            expert_rows_block(wdec, H, 0, nr, bias + r0, xn, rowsel, nt, gu, GROUP_ROWS, xt);
                            for (int j = 0; j < nt; ++j) {
                                float *a = act + (p0 + j0 + j) * I;
                                for (int r = 0; r + 1 < nr; r += 2) { /* layer.go:145-148 */
                                    const int i = (r0 + r) / 2;
                                    oracle_swiglu(&gu[j * GROUP_ROWS + r], &gu[j * GROUP_ROWS + r + 1], 1, &a[i]);
                                }
                            }
                        }
                    } else {
                        const int r0 = blk * GROUP_ROWS;
                        const int nr = H - r0 < GROUP_ROWS ? H - r0 : GROUP_ROWS;
                        decode_rows_f64(L->down + (int64_t)e * dn_bytes, I, r0, nr, wdec);
                        for (int64_t j0 = 0; j0 < np; j0 += GROUP_TOK) {
                            const int nt = np - j0 < GROUP_TOK ? (int)(np - j0) : GROUP_TOK;
                            for (int j = 0; j < nt; ++j) rowsel[j] = p0 + j0 + j;
                            expert_rows_block(wdec, I, 0, nr, L->down_b + (int64_t)e * H + r0, act, rowsel, nt,
                                              y + (p0 + j0) * H + r0, H, xt);
                        }
                    }
                }
                free(wdec);
                free(xt);
                free(gu);
                free(rowsel);
            }
        }
    }
    if (status == 0) {
        /* 5. slot-order mixture and residual (layer.go:109-121) */
        int64_t *pos_of = tok_of; /* reuse: pair id -> sorted position */
        for (int64_t q = 0; q < P; ++q) pos_of[order[q]] = q;
#pragma omp parallel num_threads(nth)
        {
            double *mix = (double *)malloc(sizeof(double) * (size_t)H);
#pragma omp for schedule(static)
            for (int j = 0; j < n; ++j) {
                if (!mix) continue;
                const int t = tokens ? tokens[j] : j;
                for (int i = 0; i < H; ++i) mix[i] = 0.0;
                for (int s = 0; s < k; ++s) {
                    const float *yr = y + pos_of[(int64_t)j * k + s] * H;
                    const double ws = (double)w[(int64_t)j * k + s];
                    for (int i = 0; i < H; ++i) mix[i] += ws * (double)yr[i];
                }
                const float *row = residual + (int64_t)t * H;
                for (int i = 0; i < H; ++i) out[(int64_t)t * H + i] = row[i] + (float)mix[i];
                if (topk_idx) memcpy(topk_idx + (int64_t)t * k, idx + (int64_t)j * k, sizeof(int32_t) * k);
                if (topk_w) memcpy(topk_w + (int64_t)t * k, w + (int64_t)j * k, sizeof(float) * k);
                if (logits) memcpy(logits + (int64_t)t * E, lg + (int64_t)j * E, sizeof(float) * E);
            }
            if (!mix) {
#pragma omp atomic write
                status = -1;
            }
            free(mix);
        }
    }
    free(xn); free(idx); free(w); free(lg); free(order); free(tok_of); free(start); free(act); free(y);
    return status;
}

/* ---- the model head: Runtime.nextToken, internal/model/gptoss/runtime.go:234-250 ---- */

int oracle_next_token(const float *hidden, int H, const float *gain, float eps, const float *lm_head, int V,
                      float *logits, int32_t *token) {
    if (!hidden || !gain || !lm_head || !token || H <= 0 || V <= 0) return -1;
    float *normalized = (float *)malloc(sizeof(float) * (size_t)H);
    float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)V);
    if (!normalized || !lg) {
        free(normalized);
        if (!logits) free(lg);
        return -1;
    }
    int rc = oracle_rmsnorm(hidden, gain, H, eps, normalized); /* runtime.go:235 */
    if (rc == 0) rc = oracle_linear_bias(normalized, lm_head, NULL, H, V, lg); /* runtime.go:239, no bias */
    if (rc == 0) {
        int best = 0; /* runtime.go:243-248: strict >, so the first of equal maxima wins */
        for (int i = 1; i < V; ++i)
            if (lg[i] > lg[best]) best = i;
        *token = best;
    }
    free(normalized);
    if (!logits) free(lg);
    return rc;
}
