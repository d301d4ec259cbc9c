/* attn_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * C restatement of the reference's GPT-OSS attention half, the checker for a
 * GPU attention path: rotary embeddings (plain and YaRN), causal attention over
 * a GQA KV cache with learned sinks and a sliding window, and the attention half
 * of the decoder layer.  Each function cites the Go code it follows (paths
 * relative to the reference project root).  Return 0 on success, a negative
 * code on an argument the reference rejects. */
#ifndef ATTN_ORACLE_H
#define ATTN_ORACLE_H

#include <stdint.h>

/* RoPE / YaRNRoPE (internal/backend/cpuref/rope.go:10-86) over n values laid out
 * [tokens][head_dim]; yarn != 0 selects the gpt-oss YaRN frequencies.
 * Errors: -1 head_dim not positive and even, -2 negative position offset,
 * -3 theta not finite and positive, -4 n not a multiple of head_dim. */
int oracle_rope(const float *in, int64_t n, int head_dim, int pos_offset, double theta, int yarn, float *out);

/* CausalAttentionWithConfig (internal/backend/cpuref/attention.go:82-171).
 * q [q_len][q_heads][head_dim]; the cache holds kv_len tokens as
 * keys/values [kv_len][kv_heads][head_dim]; the queries are the last q_len of
 * them.  sinks: q_heads learned logits or NULL; window 0 = none;
 * pre_scalar 0 = scale 1/sqrt(head_dim); softcap 0 = none.
 * Errors: -1 q_heads not a positive multiple of kv_heads, -2 sinks length,
 * -3 negative window, -4 pre_scalar, -5 softcap, -6 query length, -7 more
 * queries than cached tokens. */
int oracle_causal_attention(const float *q, int64_t nq, int q_heads, const float *keys, const float *values,
                            int kv_len, int kv_heads, int head_dim, const float *sinks, int n_sinks, int window,
                            double pre_scalar, double softcap, float *out);

typedef struct {
    int hidden, heads, kv_heads, head_dim;
    float eps;
    double theta;
    const float *norm1;   /* [hidden] */
    const float *qkv_w;   /* [(heads + 2 kv_heads) head_dim][hidden] */
    const float *qkv_b;   /* [(heads + 2 kv_heads) head_dim] */
    const float *out_w;   /* [hidden][heads head_dim] */
    const float *out_b;   /* [hidden] */
    const float *sinks;   /* [heads] */
} oracle_attn_layer;

/* The attention half of DecoderLayer.forward (internal/model/gptoss/layer.go:31-92):
 * per token RMSNorm(norm1) and the QKV projection, YaRN on the query and key
 * heads at the cache's position, the cache append, causal attention with the
 * layer's sinks and window, the output projection and the residual add.
 * keys/values: the cache [capacity][kv_heads][head_dim], *kv_len tokens filled
 * (advanced by T).  Errors: -10 T not positive, -11 cache capacity, or a
 * callee's code. */
int oracle_attention_half(const oracle_attn_layer *L, const float *input, int T, float *keys, float *values,
                          int *kv_len, int capacity, int window, float *out);

#endif
