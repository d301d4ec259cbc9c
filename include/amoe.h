/*
 * amoe.h -- C ABI of the B200 GPT-OSS mixture-of-experts block.
 *
 * This is the drop-in boundary for the MoE half of the reference's
 * DecoderLayer.forward (internal/model/gptoss/layer.go:94-123 plus
 * forwardExpert, layer.go:126-188).  A Go cgo shim binds these entry points;
 * plain pointers and sizes only, no C++ or torch types.
 *
 * Conventions
 *  - Every entry point returns AMOE_OK (0) or a negative AMOE_ERR_* code and
 *    never aborts; amoe_last_error() describes the last failure.
 *  - Host pointers are only read/written during the call (cgo forbids C from
 *    retaining Go pointers); the context copies what it keeps.
 *  - A context is thread-compatible, not thread-safe (the reference serialises
 *    generation with Runtime.mu, runtime.go:108-109).  Each call makes the
 *    context's device current, because cgo calls may land on any OS thread.
 *  - Shapes: hidden and intermediate must be multiples of 64 (GPT-OSS: 2880).
 */
#ifndef AMOE_H
#define AMOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AMOE_ABI_VERSION 1

#if defined(__GNUC__)
#define AMOE_API __attribute__((visibility("default")))
#else
#define AMOE_API
#endif

enum {
    AMOE_OK = 0,
    AMOE_ERR_INVALID = -1, /* bad argument or shape (mirrors the reference's length checks) */
    AMOE_ERR_CUDA = -2,    /* a CUDA runtime call failed */
    AMOE_ERR_NCCL = -3,    /* an NCCL call failed (expert-parallel mode) */
    AMOE_ERR_TIMEOUT = -4, /* a bounded wait gave up */
    AMOE_ERR_STATE = -5,   /* e.g. layer not uploaded, wrong mode */
    AMOE_ERR_NOMEM = -6    /* device or pinned-host allocation failed */
};

/* Expert-GEMM implementation selector (amoe_config.path). */
enum {
    AMOE_PATH_AUTO = 0,   /* GEMV for small token counts, tcgen05 grouped GEMM otherwise */
    AMOE_PATH_GEMV = 1,   /* always the MXFP4 GEMV kernels */
    AMOE_PATH_TENSOR = 2  /* always the tcgen05 grouped GEMM */
};

typedef struct amoe_ctx amoe_ctx;

typedef struct amoe_config {
    int32_t hidden;          /* H (GPT-OSS gptoss.embedding_length) */
    int32_t intermediate;    /* I (gptoss.expert_feed_forward_length) */
    int32_t experts;         /* E (gptoss.expert_count), 1..256 */
    int32_t top_k;           /* k (gptoss.expert_used_count), 1..min(E, 32) */
    int32_t layers;          /* number of layer slots (gptoss.block_count) */
    float rms_eps;           /* gptoss.attention.layer_norm_rms_epsilon, > 0 */
    float swiglu_alpha;      /* must be 1.702: hard-coded in primitives.go:146 */
    float swiglu_limit;      /* must be 7: hard-coded in primitives.go:144-145 */
    int32_t max_tokens;      /* largest T passed to one forward call (sizes scratch) */
    int32_t device;          /* CUDA device ordinal */
    int32_t stream_slots;    /* 0: every layer resident in HBM.  n >= 2: weights live in
                                pinned host memory, n device slots are filled on a copy stream;
                                streamed layers hold only the tensor-core planes (path AUTO or
                                TENSOR) */
    int32_t ep_size;         /* expert-parallel group size; 1 = single GPU */
    int32_t ep_rank;         /* this process's rank in the expert-parallel group */
    const void *nccl_id;     /* 128-byte ncclUniqueId shared by the group (ep_size > 1) */
    int32_t path;            /* AMOE_PATH_* */
    int32_t stream_experts;  /* with stream_slots >= 2: 1 = each forward routes first and copies
                                only the experts its tokens selected (the reference reads only
                                those too: tensor.go:94-111) instead of whole layers */
} amoe_config;

/* Replaces: gptoss.Open's per-runtime setup (runtime.go:37-60).  Allocates the
 * per-layer device (or pinned-host) weight storage and the scratch for
 * max_tokens tokens. */
AMOE_API int amoe_create(const amoe_config *cfg, amoe_ctx **out);

/* Releases everything the context owns.  NULL is a no-op. */
AMOE_API void amoe_destroy(amoe_ctx *ctx);

/* Description of the last failure on ctx (ctx NULL: the last failure of a
 * context-free call -- amoe_create, amoe_route_noalloc -- on this thread).
 * Valid until the next call on the same context. */
AMOE_API const char *amoe_last_error(const amoe_ctx *ctx);

/* Replaces: loadDecoderLayer's MoE tensors (weights.go:52-54, 80, 84-116) and
 * the per-call readExpert decode (tensor.go:94-111).  Takes one layer's tensors
 * in their GGUF storage layout and keeps them on the device in a tiled MXFP4
 * layout (a lossless byte shuffle: no dequantisation).
 *   norm_gain  [H] f32                          ffn_norm.weight
 *   router_w   [E x H] f32 row-major            ffn_gate_inp.weight
 *   router_b   [E] f32                          ffn_gate_inp.bias
 *   gate_up    E*2I*(H/32)*17 bytes, MXFP4      ffn_gate_up_exps.weight (rows interleave gate, up)
 *   gate_up_b  [E x 2I] f32                     ffn_gate_up_exps.bias
 *   down       E*H*(I/32)*17 bytes, MXFP4       ffn_down_exps.weight
 *   down_b     [E x H] f32                      ffn_down_exps.bias                    */
AMOE_API int amoe_upload_layer(amoe_ctx *ctx, int32_t layer, const float *norm_gain,
                      const float *router_w, const float *router_b, const uint8_t *gate_up,
                      const float *gate_up_b, const uint8_t *down, const float *down_b);

/* Replaces: the MoE loop of DecoderLayer.forward, layer.go:94-123.
 * residual [T x H] host f32 (the pre-norm rows); out [T x H] host f32 receives
 * residual + sum_k p_k * expert_k(RMSNorm(residual)).  topk_idx [T x k] and
 * topk_w [T x k] (both nullable) receive the routing (MoERouterTopK, moe.go:12-41).
 * Synchronous.  1 <= T <= max_tokens. */
AMOE_API int amoe_forward(amoe_ctx *ctx, int32_t layer, const float *residual, int32_t T, float *out,
                 int32_t *topk_idx, float *topk_w);

/* Same computation on device buffers, enqueued on `stream` (a cudaStream_t;
 * NULL = the context's own stream); returns without synchronising. */
AMOE_API int amoe_forward_device(amoe_ctx *ctx, int32_t layer, const float *residual, int32_t T,
                        float *out, int32_t *topk_idx, float *topk_w, void *stream);

/* Waits for all work the context enqueued. */
AMOE_API int amoe_synchronize(amoe_ctx *ctx);

/* Streaming mode (stream_slots >= 2): starts copying `layer` from pinned host
 * memory into the least recently used device slot on the copy stream.  A later
 * forward of that layer waits for the copy on the device (an event), not on
 * the host.  After every forward of layer L the context itself starts copying
 * layer (L+1) mod layers, so a sequential layer loop needs no explicit call.
 * Replaces the synchronous per-layer reload of Generate, runtime.go:146-199. */
AMOE_API int amoe_prefetch_layer(amoe_ctx *ctx, int32_t layer);

/* Test/diagnostic hook: copies the routing of the last forward to host.
 *   logits [T x E] f32 (router logits incl. bias), perm_pair [T*k] (position ->
 *   pair id t*k+s, pairs ordered stably by expert), counts [E], offsets [E+1].
 * Any pointer may be NULL. */
AMOE_API int amoe_last_routing(amoe_ctx *ctx, float *logits, int32_t *perm_pair, int32_t *counts,
                      int32_t *offsets);

/* Per-stage device timing (CUDA events on the launch stream) and launch count.
 * Stages: 0 route (RMSNorm+router+top-k), 1 expert-offset scan (+ scatter on
 * the GEMV path), 2 gate_up (+SwiGLU), 3 down, 4 combine, 5 scatter + gather
 * of the expert-sorted rows (tensor path), 6 fused decode expert stage (gate_up,
 * down and combine in one launch, T <= 4), 7 reserved. */
#define AMOE_STAGES 8
typedef struct amoe_stats {
    int64_t launches;               /* kernels this context has launched */
    int64_t forwards;               /* forward calls */
    int64_t timed_forwards;         /* forwards with profiling on, summed in stage_ms */
    double stage_ms[AMOE_STAGES];   /* summed event time per stage (profiling on) */
    int32_t last_path;              /* AMOE_PATH_GEMV or AMOE_PATH_TENSOR of the last forward */
    int64_t layer_bytes;            /* device-format bytes of one layer (what a streamed layer visit copies) */
} amoe_stats;

/* Turns per-stage event timing on (1) or off (0).  Timing adds event records
 * between kernels; leave it off when measuring whole-forward throughput. */
AMOE_API int amoe_set_profiling(amoe_ctx *ctx, int32_t on);

/* Synchronises, folds finished stage timings into the counters and copies
 * them out; reset != 0 clears the counters afterwards. */
AMOE_API int amoe_get_stats(amoe_ctx *ctx, amoe_stats *out, int32_t reset);

/* No counterpart in the reference: the routing step (RMSNorm, router
 * LinearBias, top-k, selected softmax -- the same kernels and results as the
 * routing inside amoe_forward) for callers that cannot allocate device memory,
 * e.g. a runtime that plans all device memory up front and hands out fixed
 * regions, or a process whose GPU memory is already reserved by another
 * allocator.  It needs no context and calls no cudaMalloc/cudaFree: its scratch
 * is one fixed device array of 2.1 MB that every GPU loading this library holds
 * until exit.  Limits: 1 <= T <= 64, hidden a multiple of 64 up to 4096,
 * experts <= 128, top_k <= min(experts, 32); larger sizes return
 * AMOE_ERR_INVALID with a message in amoe_last_error(NULL).
 *   residual [T x H], norm_gain [H], router_w [E x H] (GGUF layout), router_b [E]:
 *     device inputs;  logits [T x E], topk_idx [T x k], topk_w [T x k]: device outputs.
 * Enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 * The first call on a device resolves the array's device address; make that
 * first call before any stream capture.  The calling thread's current device is
 * the same after the call as before it.  All calls share the array and it
 * keeps the last call's contents (the counters that must start at zero are
 * cleared by each call), so calls that overlap on the GPU race. */
AMOE_API int amoe_route_noalloc(int32_t device, int32_t hidden, int32_t experts, int32_t top_k,
                                float rms_eps, const float *residual, int32_t T,
                                const float *norm_gain, const float *router_w, const float *router_b,
                                float *logits, int32_t *topk_idx, float *topk_w, void *stream);

/* Expert parallelism (ep_size > 1, at most 8 GPUs of one box): experts
 * [r*E/N, (r+1)*E/N) live on rank r; each rank routes its own tokens.  Rows move
 * by stores into the other ranks' device memory over NVLink (CUDA IPC windows
 * mapped at amoe_create), ordered by per-source epoch flags, with no host
 * synchronisation inside a forward (no counterpart in the reference, which is
 * single-process CPU code).  NCCL is used once, at amoe_create, to exchange the
 * windows' IPC handles.  All ranks must call amoe_forward* for the same layer in
 * the same order with the same max_tokens; a wait that runs out (a rank failed
 * or never called) returns AMOE_ERR_TIMEOUT and the group must be recreated.
 * amoe_ep_unique_id fills the 128-byte ncclUniqueId that rank 0 creates and
 * passes to the others (amoe_config.nccl_id). */
AMOE_API int amoe_ep_unique_id(void *out);

/* Layout of one expert-parallel exchange as rank `rank` derives it on the device
 * from the all-gathered count table (no GPU needed here):
 *   table [N][E], E = N*El: pairs each source rank routes to each global expert.
 * Out (each nullable):
 *   send_base [E]: row, in the owning rank's expert-major receive buffer, of
 *                  this rank's first pair for expert e;
 *   offsets_loc [El+1]: expert-major row ranges of this rank's experts;
 *   seg_start [El][N]: first expert-major row of source s's rows for local expert el;
 *   src_pos [El][N]: sorted position of those rows on source s (where outputs return). */
AMOE_API int amoe_ep_layout(int32_t n_ranks, int32_t experts_per_rank, int32_t rank,
                            const int32_t *table, int32_t *send_base, int32_t *offsets_loc,
                            int32_t *seg_start, int32_t *src_pos);

/* The fused decode kernel's work table (T <= 4; no GPU needed): the units each of
 * `ctas` CTAs runs, built the way the context builds it.  CTA b's row holds
 * AMOE_DECODE_SCHED_WORDS int32 words: S + 1 offsets (S = min(experts, 4 * top_k)),
 * then for n = 1..S active experts the units at words [n - 1]..[n] of the row.
 * A unit is bit 30: phase (0 gate_up, 1 down), bits 20-29: active-slot index,
 * bits 8-19: 128-row weight tile, bit 0: K half (down units).
 * rows: [ctas][AMOE_DECODE_SCHED_WORDS], nullable (then the shape is only checked).
 * AMOE_ERR_INVALID if the decode kernel does not run this shape. */
#define AMOE_DECODE_SCHED_WORDS 1024
AMOE_API int amoe_decode_schedule(int32_t hidden, int32_t intermediate, int32_t experts, int32_t top_k,
                                  int32_t ctas, int32_t *rows);

/* ---- GGUF files ------------------------------------------------------------------
 * GGUF tensor encodings (internal/gguf/reader.go:17-27). */
enum {
    AMOE_GGUF_F32 = 0,
    AMOE_GGUF_F16 = 1,
    AMOE_GGUF_Q4_0 = 2,
    AMOE_GGUF_Q8_0 = 8,
    AMOE_GGUF_Q4_K = 12,
    AMOE_GGUF_Q5_K = 13,
    AMOE_GGUF_Q6_K = 14,
    AMOE_GGUF_BF16 = 30,
    AMOE_GGUF_MXFP4 = 39
};

typedef struct amoe_gguf amoe_gguf;

/* Replaces: gguf.Open (internal/gguf/reader.go:74-86, 300-410).  Maps the file
 * read-only and parses the little-endian GGUF v2/v3 header, metadata and tensor
 * index; rejects bad magic or version, duplicate keys or tensors, unknown value
 * or tensor types, and any tensor whose data range passes the end of the file.
 * Errors: AMOE_ERR_INVALID with the reason in amoe_last_error(NULL). */
AMOE_API int amoe_gguf_open(const char *path, amoe_gguf **out);
AMOE_API void amoe_gguf_close(amoe_gguf *g);

/* Replaces: Reader.Tensor (reader.go:130-133).  One tensor of the index: its
 * encoding (AMOE_GGUF_*), GGUF shape (dims[0] varies fastest; up to 4 entries
 * written), absolute data offset in the file and encoded size.  Each output is
 * nullable.  AMOE_ERR_INVALID if the tensor is absent. */
AMOE_API int amoe_gguf_tensor(const amoe_gguf *g, const char *name, int32_t *type, int32_t *ndims,
                              int64_t *dims, int64_t *offset, int64_t *bytes);

/* Replaces: GPTOSSMetadata (internal/gguf/gptoss.go:35-95) for the MoE fields:
 * hidden, intermediate, experts, top_k, layers and rms_eps of *cfg come from the
 * "gptoss." or "gpt-oss." metadata (embedding_length, expert_feed_forward_length,
 * expert_count, expert_used_count, block_count, attention.layer_norm_rms_epsilon).
 * The other fields of *cfg are left as they are.  Nothing changes on error. */
AMOE_API int amoe_gguf_moe_config(const amoe_gguf *g, amoe_config *cfg);

/* Replaces: loadDecoderLayer's MoE tensors (internal/model/gptoss/weights.go:35-124)
 * and the per-call readExpert (tensor.go:94-111): uploads layer `layer` of the file
 * into slot `layer` of the context, as amoe_upload_layer does with host arrays.
 * Reads blk.<layer>.ffn_norm.weight (or post_attention_norm.weight),
 * ffn_gate_inp.weight/.bias, ffn_gate_up_exps.weight/.bias (or ffn_gate_exps +
 * ffn_up_exps, interleaved into the fused row order) and ffn_down_exps.weight/.bias,
 * with exactly the reference's GGUF shapes.  Vectors may be f32, f16 or bf16;
 * expert weights must be MXFP4.  The expert bytes go from the mapped file to the
 * device without a host-side decode. */
AMOE_API int amoe_upload_layer_gguf(amoe_ctx *ctx, const amoe_gguf *g, int32_t layer);

/* ---- the model head ----------------------------------------------------------------
 * Replaces: Runtime.nextToken (internal/model/gptoss/runtime.go:234-250) with the head
 * weights of loadResidentWeights (weights.go:19-33): RMSNorm of each hidden row with the
 * final norm gain (output_norm.weight), logits = lm_head . normalized (output.weight,
 * [V x H] row-major, no bias; the dot products accumulate in float64 and round to f32 once,
 * as cpuref.Linear does), and the token = the first index of the largest logit (a later
 * logit must be strictly larger; a NaN never wins; a NaN at index 0 gives token 0).  The
 * lm head stays on the device in its GGUF encoding (F32, F16 or BF16) and is streamed once
 * per call for every row of the call.  A head is independent of the MoE contexts (the
 * reference keeps these weights resident while it streams the layers). */
typedef struct amoe_head amoe_head;

/* Replaces: the finalNorm / lmHead fields of Runtime (runtime.go:27-28).  hidden >= 1,
 * vocab >= 1, rms_eps > 0; the head's buffers for up to 16 rows per call. */
AMOE_API int amoe_head_create(int32_t hidden, int32_t vocab, float rms_eps, int32_t device, amoe_head **out);
AMOE_API void amoe_head_destroy(amoe_head *h);

/* Description of the last failure on h (h NULL: of the last amoe_head_create on this thread). */
AMOE_API const char *amoe_head_last_error(const amoe_head *h);

/* Replaces: loadResidentWeights (weights.go:19-33).  final_norm [H] f32; lm_head [V x H] in
 * the encoding `type` (AMOE_GGUF_F32, AMOE_GGUF_F16 or AMOE_GGUF_BF16), host memory. */
AMOE_API int amoe_head_upload(amoe_head *h, const float *final_norm, const void *lm_head, int32_t type);

/* The same from an open GGUF file: output_norm.weight and output.weight, or token_embd.weight
 * when the file has no output.weight (weights.go:27-31), with the reference's GGUF shapes
 * ([H] and [H, V]). */
AMOE_API int amoe_head_upload_gguf(amoe_head *h, const amoe_gguf *g);

/* Replaces: Runtime.nextToken (runtime.go:234-250) for T rows at once (1 <= T <= 16):
 * hidden [T x H] f32 host rows (the last layer's outputs), tokens [T] receives each row's
 * token, logits [T x V] (nullable) the logits.  Synchronous. */
AMOE_API int amoe_head_next_token(amoe_head *h, const float *hidden, int32_t T, int32_t *tokens, float *logits);

/* The same on device buffers, enqueued on `stream` (NULL = the head's own stream). */
AMOE_API int amoe_head_next_token_device(amoe_head *h, const float *hidden, int32_t T, int32_t *tokens,
                                         float *logits, void *stream);

/* ABI version (AMOE_ABI_VERSION). */
AMOE_API int amoe_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* AMOE_H */
