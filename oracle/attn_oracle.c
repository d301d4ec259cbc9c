/* attn_oracle.c -- TEST INFRASTRUCTURE ONLY (see attn_oracle.h).
 *
 * Restates the reference's rounding points: angles, sines and cosines, dot
 * products, softmax terms and weighted sums in float64, rounded to float32
 * where the Go code stores a []float32.  Loop orders follow the Go loops, so
 * the float64 sums add in the same order. */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

static const double kPi = 3.14159265358979323846;

/* yarnCorrectionDimension (rope.go:46-48) */
static double yarn_correction_dimension(double beta, int head_dim, double theta, double original_max) {
    return (double)head_dim * log(original_max / (beta * 2.0 * kPi)) / (2.0 * log(theta));
}

int oracle_rope(const float *in, int64_t n, int head_dim, int pos_offset, double theta, int yarn, float *out) {
    /* validation order of rope() (rope.go:50-62); YaRNRoPE checks head_dim and theta first */
    if (head_dim <= 0 || head_dim % 2 != 0) return -1;
    if (yarn && (theta <= 0 || isnan(theta) || isinf(theta))) return -3;
    if (pos_offset < 0) return -2;
    if (theta <= 0 || isnan(theta) || isinf(theta)) return -3;
    if (n % head_dim != 0) return -4;
    const int half = head_dim / 2;
    double *freq = (double *)malloc(sizeof(double) * (size_t)half);
    if (!freq) return -100;
    double concentration = 1.0;
    if (yarn) {
        /* YaRNRoPE (rope.go:17-44): factor 32, original context 4096, beta fast 32, slow 1 */
        const double factor = 32.0, original_max = 4096.0, beta_fast = 32.0, beta_slow = 1.0;
        const double low = fmax(0.0, floor(yarn_correction_dimension(beta_fast, head_dim, theta, original_max)));
        const double high =
            fmin((double)(half - 1), ceil(yarn_correction_dimension(beta_slow, head_dim, theta, original_max)));
        for (int i = 0; i < half; ++i) {
            const double base = pow(theta, -2.0 * (double)i / (double)head_dim);
            double ramp = 0.0;
            if (high != low) ramp = ((double)i - low) / (high - low);
            ramp = fmax(0.0, fmin(1.0, ramp));
            freq[i] = base * (ramp + (1.0 - ramp) / factor);
        }
        concentration = 1.0 + 0.1 * log(factor);
    } else {
        for (int i = 0; i < half; ++i) freq[i] = pow(theta, -2.0 * (double)i / (double)head_dim);
    }
    const int64_t tokens = n / head_dim;
    for (int64_t t = 0; t < tokens; ++t) {
        const double position = (double)(pos_offset + t);
        const float *row = in + t * head_dim;
        float *o = out + t * head_dim;
        for (int i = 0; i < half; ++i) {
            const double angle = position * freq[i];
            const double s = sin(angle) * concentration, c = cos(angle) * concentration;
            const double first = (double)row[i], second = (double)row[i + half];
            o[i] = (float)(first * c - second * s);
            o[i + half] = (float)(second * c + first * s);
        }
    }
    free(freq);
    return 0;
}

int oracle_causal_attention(const float *q, int64_t nq, int q_heads, const float *keys, const float *values,
                            int kv_len, int kv_heads, int head_dim, const float *sinks, int n_sinks, int window,
                            double pre_scalar, double softcap, float *out) {
    /* validation order of attention.go:86-111 */
    if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0) return -1;
    if (n_sinks != 0 && n_sinks != q_heads) return -2;
    if (window < 0) return -3;
    if (pre_scalar < 0 || isnan(pre_scalar) || isinf(pre_scalar)) return -4;
    if (softcap < 0 || isnan(softcap) || isinf(softcap)) return -5;
    const int64_t q_stride = (int64_t)q_heads * head_dim;
    if (nq == 0 || nq % q_stride != 0) return -6;
    const int q_len = (int)(nq / q_stride);
    if (q_len > kv_len) return -7;

    const int64_t kv_stride = (int64_t)kv_heads * head_dim;
    const int heads_per_kv = q_heads / kv_heads;
    double scale = 1.0 / sqrt((double)head_dim);
    if (pre_scalar > 0) scale = 1.0 / sqrt(pre_scalar);
    double *scores = (double *)malloc(sizeof(double) * (size_t)(kv_len > 0 ? kv_len : 1));
    if (!scores) return -100;
    const int first_query_position = kv_len - q_len;
    for (int qi = 0; qi < q_len; ++qi) {
        const int position = first_query_position + qi;
        int first_key = 0;
        if (window > 0 && position >= window) first_key = position - window + 1;
        for (int h = 0; h < q_heads; ++h) {
            const int kvh = h / heads_per_kv;
            const float *qv = q + qi * q_stride + (int64_t)h * head_dim;
            double max_score = -INFINITY;
            if (n_sinks != 0) max_score = (double)sinks[h];
            for (int kp = first_key; kp <= position; ++kp) {
                const float *k = keys + kp * kv_stride + (int64_t)kvh * head_dim;
                double dot = 0.0;
                for (int d = 0; d < head_dim; ++d) dot += (double)qv[d] * (double)k[d];
                scores[kp] = dot * scale;
                if (softcap > 0) scores[kp] = softcap * tanh(scores[kp] / softcap);
                if (scores[kp] > max_score) max_score = scores[kp];
            }
            double denominator = 0.0;
            for (int kp = first_key; kp <= position; ++kp) {
                scores[kp] = exp(scores[kp] - max_score);
                denominator += scores[kp];
            }
            if (n_sinks != 0) denominator += exp((double)sinks[h] - max_score);
            float *o = out + qi * q_stride + (int64_t)h * head_dim;
            for (int d = 0; d < head_dim; ++d) {
                double sum = 0.0;
                for (int kp = first_key; kp <= position; ++kp)
                    sum += scores[kp] * (double)values[kp * kv_stride + (int64_t)kvh * head_dim + d];
                o[d] = (float)(sum / denominator);
            }
        }
    }
    free(scores);
    return 0;
}

/* yarnHeads (layer.go:189-207): each head's sequence rotated on its own */
static int yarn_heads(float *x, int T, int heads, int head_dim, int pos_offset, double theta) {
    const int width = heads * head_dim;
    float *seq = (float *)malloc(sizeof(float) * (size_t)T * head_dim * 2);
    if (!seq) return -100;
    float *rot = seq + (size_t)T * head_dim;
    int rc = 0;
    for (int h = 0; h < heads && rc == 0; ++h) {
        for (int t = 0; t < T; ++t) memcpy(seq + t * head_dim, x + t * width + h * head_dim, sizeof(float) * head_dim);
        rc = oracle_rope(seq, (int64_t)T * head_dim, head_dim, pos_offset, theta, 1, rot);
        for (int t = 0; t < T && rc == 0; ++t)
            memcpy(x + t * width + h * head_dim, rot + t * head_dim, sizeof(float) * head_dim);
    }
    free(seq);
    return rc;
}

int oracle_attention_half(const oracle_attn_layer *L, const float *input, int T, float *keys, float *values,
                          int *kv_len, int capacity, int window, float *out) {
    if (T <= 0) return -10;
    const int H = L->hidden, qw = L->heads * L->head_dim, kvw = L->kv_heads * L->head_dim;
    const int pos = *kv_len;
    if (pos + T > capacity) return -11;
    float *q = (float *)malloc(sizeof(float) * (size_t)T * (qw + 2 * kvw + qw + H + qw + 2 * kvw));
    if (!q) return -100;
    float *k = q + (size_t)T * qw, *v = k + (size_t)T * kvw, *att = v + (size_t)T * kvw;
    float *normed = att + (size_t)T * qw, *qkv = normed + H;
    int rc = 0;
    for (int t = 0; t < T && rc == 0; ++t) {
        rc = oracle_rmsnorm(input + (size_t)t * H, L->norm1, H, L->eps, normed);
        if (rc == 0) rc = oracle_linear_bias(normed, L->qkv_w, L->qkv_b, H, qw + 2 * kvw, qkv);
        if (rc == 0) {
            memcpy(q + (size_t)t * qw, qkv, sizeof(float) * qw);
            memcpy(k + (size_t)t * kvw, qkv + qw, sizeof(float) * kvw);
            memcpy(v + (size_t)t * kvw, qkv + qw + kvw, sizeof(float) * kvw);
        }
    }
    if (rc == 0) rc = yarn_heads(q, T, L->heads, L->head_dim, pos, L->theta);
    if (rc == 0) rc = yarn_heads(k, T, L->kv_heads, L->head_dim, pos, L->theta);
    if (rc == 0) {
        /* KVCache.Append (attention.go:40-59) */
        memcpy(keys + (size_t)pos * kvw, k, sizeof(float) * (size_t)T * kvw);
        memcpy(values + (size_t)pos * kvw, v, sizeof(float) * (size_t)T * kvw);
        *kv_len = pos + T;
        rc = oracle_causal_attention(q, (int64_t)T * qw, L->heads, keys, values, *kv_len, L->kv_heads, L->head_dim,
                                     L->sinks, L->sinks ? L->heads : 0, window, 0.0, 0.0, att);
    }
    for (int t = 0; t < T && rc == 0; ++t) {
        float *proj = normed;  /* reuse: [H] */
        rc = oracle_linear_bias(att + (size_t)t * qw, L->out_w, L->out_b, qw, H, proj);
        for (int i = 0; i < H && rc == 0; ++i) out[(size_t)t * H + i] = input[(size_t)t * H + i] + proj[i];
    }
    free(q);
    return rc;
}
