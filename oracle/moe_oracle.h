/*
 * moe_oracle.h -- CPU restatement of the GPT-OSS MoE block of lutikk/airllm.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library (airllm_b200/libamoe.so).  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference legs use it.
 *
 * Every function restates the reference Go code it cites (paths relative to the
 * reference project root) with the same arithmetic: float64 accumulation in the
 * same order, float32 rounding at the same points.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One MoE layer in the reference's GGUF storage layout.
 *   norm_gain   [H]                      ffn_norm.weight         (weights.go:80)
 *   router_w    [E x H] row-major        ffn_gate_inp.weight     (weights.go:53)
 *   router_b    [E]                      ffn_gate_inp.bias       (weights.go:54)
 *   gate_up     E x (2I rows x H/32 blocks x 17 B)  ffn_gate_up_exps.weight, MXFP4
 *   gate_up_b   [E x 2I]                 ffn_gate_up_exps.bias   (weights.go:88)
 *   down        E x (H rows x I/32 blocks x 17 B)   ffn_down_exps.weight, MXFP4
 *   down_b      [E x H]                  ffn_down_exps.bias      (weights.go:112)
 */
typedef struct {
    int32_t hidden, intermediate, experts, top_k;
    float eps;
    const float *norm_gain, *router_w, *router_b;
    const uint8_t *gate_up;
    const float *gate_up_b;
    const uint8_t *down;
    const float *down_b;
} oracle_layer;

/* internal/backend/cpuref/primitives.go:50-72 */
int oracle_rmsnorm(const float *x, const float *g, int n, float eps, float *out);
/* internal/backend/cpuref/primitives.go:11-47 */
int oracle_linear_bias(const float *x, const float *w, const float *b, int in_dim,
                       int out_dim, float *y);
/* internal/backend/cpuref/moe.go:12-41 */
int oracle_router_topk(const float *logits, int n, int k, int32_t *idx, float *w);
/* internal/backend/cpuref/primitives.go:138-149 */
int oracle_swiglu(const float *gate, const float *up, int n, float *out);
/* internal/model/gptoss/tensor.go:145-160 and reader.go:442-449 */
int oracle_mxfp4_decode(const uint8_t *blocks, int64_t nbytes, int64_t elements, float *out);
/* internal/gguf/reader.go:442-449: bytes for an MXFP4 tensor, -1 on a partial block */
int64_t oracle_mxfp4_encoded_size(int64_t elements);
/* Activations as `terms` E2M1 terms with E8M0 scales per 32 elements, the operand
 * form of a block-scaled FP4 (mxf4) expert GEMM.  No reference counterpart: it
 * defines, bit for bit, what a GPU quantizer must produce.  Per 32-element block,
 * term j takes the remainder r_j (r_0 = x, f32), the smallest scale 2^e with
 * max|r_j| / 2^e <= 6 (E8M0 byte e + 127; 127 for an all-zero remainder), codes
 * round-to-nearest-even of r_j / 2^e on the E2M1 grid, saturated at +-6, and
 * r_{j+1} = r_j - q_j 2^e in f32.  A value that rounds to zero gets code 0 whatever
 * its sign, never 8 (E2M1's negative zero): a GPU quantizer whose hardware conversion
 * keeps the sign of zero must clear it to match.  codes [terms][n / 2]: two codes per byte, the
 * lower element in the low nibble; scales [terms][n / 32].  n must be a multiple
 * of 32 and every value finite.  Returns -1 on bad arguments. */
int oracle_e2m1_terms(const float *x, int64_t n, int terms, uint8_t *codes, uint8_t *scales);

/* The MoE half of DecoderLayer.forward, internal/model/gptoss/layer.go:94-123,
 * with forwardExpert layer.go:126-188 for each selected expert.
 *   residual  [T x H]  the pre-norm row (the layer's residual stream)
 *   out       [T x H]  residual + mixture
 *   topk_idx  [T x k]  (nullable) selected experts in slot order
 *   topk_w    [T x k]  (nullable) routing weights
 *   logits    [T x E]  (nullable) router logits
 *   tokens    (nullable) list of n_tokens row indices to compute; NULL = all T rows.
 *             Rows not listed are left untouched in out/topk_*.
 *   faithful  1: decode each selected expert's whole MXFP4 tensor into a float
 *             buffer for every (token, expert), as readExpert (tensor.go:94-111)
 *             does on every call; 0: decode weights on the fly inside the dot
 *             product.  Both give bit-identical results.
 *   threads   OpenMP threads over tokens (1 = the reference's single thread).
 */
int oracle_moe_block(const oracle_layer *L, const float *residual, int T, float *out,
                     int32_t *topk_idx, float *topk_w, float *logits,
                     const int32_t *tokens, int n_tokens, int faithful, int threads);

/* oracle_moe_block with the work in expert-major order: each routed expert's MXFP4
 * rows are decoded once per call and multiplied with all of its tokens, every
 * output element keeping the reference's sequential float64 sum (layer.go:94-188,
 * primitives.go:11-47).  Outputs are bit-identical to oracle_moe_block (tested);
 * used to check full prefill-sized outputs.  Same arguments without `faithful`. */
int oracle_moe_block_grouped(const oracle_layer *L, const float *residual, int T, float *out,
                             int32_t *topk_idx, float *topk_w, float *logits,
                             const int32_t *tokens, int n_tokens, int threads);

/* Runtime.nextToken (internal/model/gptoss/runtime.go:234-250): RMSNorm of one
 * hidden row with the final norm gain, logits = Linear(normalized, lm_head) with
 * lm_head [V x H] row-major and no bias, token = the first index of the largest
 * logit (a later logit must be strictly larger to win; a NaN never wins, and a
 * NaN at index 0 is never replaced).  logits [V] nullable. */
int oracle_next_token(const float *hidden, int H, const float *gain, float eps, const float *lm_head, int V,
                      float *logits, int32_t *token);

/* forwardExpert (layer.go:126-188) of expert e on n normalized rows x [n x H]:
 * y [n x H] = down(SwiGLU(gate_up(x))) with biases. */
int oracle_expert_rows(const oracle_layer *L, int expert, const float *x, int n, float *y, int threads);

/* Router only (RMSNorm + LinearBias + top-k + selected softmax) for all T rows. */
int oracle_route(const oracle_layer *L, const float *residual, int T, float *logits,
                 int32_t *topk_idx, float *topk_w, int threads);

/* Token->expert permutation (no reference function; the order the GPU path uses):
 * pairs (t, s) sorted stably by (expert, t, s).
 *   perm_pair [T*k]  position -> pair id t*k+s
 *   counts    [E], offsets [E+1] (exclusive scan of counts)
 *   inv       [T*k]  pair id -> position                                   */
int oracle_permute(const int32_t *topk_idx, int T, int k, int E, int32_t *perm_pair,
                   int32_t *counts, int32_t *offsets, int32_t *inv);

#ifdef __cplusplus
}
#endif
#endif
