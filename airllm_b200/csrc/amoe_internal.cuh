// amoe_internal.cuh -- shared definitions of the B200 MoE-block library.
//
// Device data layout (per layer) and the kernel launchers that the C-ABI in
// ctx.cu strings together.  See include/amoe.h for the public boundary.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <nccl.h>

#include <string>
#include <vector>

struct amoe_gguf;  // include/amoe.h: an open GGUF file (gguf.cu)

namespace amoe {

// ---------------------------------------------------------------------------
// Tiled MXFP4 weight layout ("fragment tiles")
//
// The GGUF tensor stores, per expert, R rows of K values as K/32 blocks of
// 17 bytes (1 E8M0 scale byte + 16 bytes of E2M1 nibbles, low nibble = even
// element).  Upload shuffles those bytes, losslessly, into two planes:
//
//   q[e][rt][kt][lane][16 B]   rt = R/16 row tiles, kt = K/64 k tiles
//   s[e][rt][kt][32 B]
//
// A tile is 16 rows x 64 values (2 scale blocks).  Lane (g = lane/4,
// c = lane%4) holds, in order:
//   bytes 0-3   tile row g,   block 0, nibble bytes 4c..4c+3
//   bytes 4-7   tile row g+8, block 0, nibble bytes 4c..4c+3
//   bytes 8-11  tile row g,   block 1
//   bytes 12-15 tile row g+8, block 1
// which is exactly the A-fragment of two m16n8k16 MMAs per block once each
// byte goes through cvt.rn.f16x2.e2m1x2 (the k order inside a block is
// permuted consistently with the activation fragment).  Scale byte
// s[...][4*g + 2*h + b] belongs to tile row g + 8*h, block b.
//
// gate_up rows are additionally re-ordered so that tile row g holds the gate
// row of pair p = 8*rt + g (GGUF row 2p) and tile row g+8 its up row (GGUF
// row 2p+1): the fused SwiGLU pairs sit in the same thread / TMEM lane + 8.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 16;
constexpr int kTileK = 64;
constexpr int kTileQBytes = 512;
constexpr int kTileSBytes = 32;

struct LayerDev {
    float *norm_gain = nullptr;   // [H]
    float *router_w = nullptr;    // [E x H]  (GGUF layout)
    float *router_b = nullptr;    // [E]
    uint8_t *gu_q = nullptr;      // [E][2I/16][H/64][512]
    uint8_t *gu_s = nullptr;      // [E][2I/16][H/64][32]
    float *gu_b = nullptr;        // [E][2I]  GGUF row order
    uint8_t *dn_q = nullptr;      // [E][H/16][I/64][512]
    uint8_t *dn_s = nullptr;      // [E][H/16][I/64][32]
    float *dn_b = nullptr;        // [E][H]
    // Box planes of the tensor-core GEMMs and the decode kernel (see "Box planes" below)
    uint8_t *gu_tq = nullptr;     // [E][2I/128][Hp/128] boxes of kBoxStride bytes, rows in fragment order
    uint8_t *dn_tq = nullptr;     // [E][ceil(H/128)][Ip/128] boxes of kBoxStride bytes
};

// ---------------------------------------------------------------------------
// Box planes for the block-scaled tensor-core path (tcgen05.mma kind::mxf4:
// E2M1 weights x E2M1 activation terms, E8M0 scales) and the decode kernel.
//
//   tq[e][m][kb]    box (m, kb): rows 128m..128m+127, elements 128kb..128kb+127,
//                   kBoxStride = 8704 contiguous bytes:
//     bytes 0..8191     the 128 rows' GGUF nibble bytes (64 per row; byte j: low
//                       nibble element 2j, high nibble 2j+1), each row's four
//                       16-byte chunks in the 64-byte swizzle order (chunk c at
//                       position c ^ ((r / 2) % 4)), the K-major layout the tensor
//                       core reads;
//     bytes 8192..8703  the rows' E8M0 bytes, block j of row r at
//                       (r % 32) * 16 + (r / 32) * 4 + j: the scale-factor chunk
//                       that tcgen05.cp.32x128b.warpx4 spreads over the 128 TMEM
//                       lanes (lane r, column base + r / 32, byte j).
//   So one box -- weights and scales -- reaches shared memory as one copy: a TMA
//   copy costs tens of cycles of fixed work per copy in the SM's copy engine, so
//   the pipelines move few, large pieces.  K is padded with zeros to Kp = K
//   rounded up to 128; rows past R are zero; padding scales are 127 (2^0).
// gate_up rows use the fragment order of the tiled planes (row 16t + j, j < 8:
// gate of pair 8t + j; j >= 8: its up row), so a SwiGLU pair sits in TMEM
// lanes 8 apart.
// ---------------------------------------------------------------------------
constexpr int kTmaBoxK = 128;
constexpr size_t kBoxData = 128 * 64;                  // the box's E2M1 rows
constexpr size_t kBoxStride = kBoxData + 512;          // ... then its E8M0 chunk
inline int kpad128(int K) { return (K + kTmaBoxK - 1) / kTmaBoxK * kTmaBoxK; }
inline size_t box_plane_bytes(int E, int R, int K) {
    return (size_t)E * ((R + 127) / 128) * (kpad128(K) / kTmaBoxK) * kBoxStride;
}
cudaError_t launch_repack_tma(const uint8_t *gguf, int E, int R, int K, bool pair_rows, uint8_t *tq, cudaStream_t st);

struct Dims {
    int H, I, E, k;
    float eps;
};

// Routing kernels ------------------------------------------------------------
constexpr int kRouteTokens = 8;  // tokens per routing CTA (one "chunk")
constexpr int kRouteWarps = 8;

struct RouteOut {
    __half *x_hi, *x_lo;     // [T][H] fp16 split of RMSNorm(residual): x ~= hi + lo
    float *logits;           // [T][E]
    int32_t *topk_idx;       // [T][k]
    float *topk_w;           // [T][k]
    int32_t *hist;           // [nchunk][E]
    int32_t *chunk_base;     // [nchunk][E]
    int32_t *counts;         // [E]
    int32_t *offsets;        // [E+1]
    int32_t *active;         // [E] experts with counts > 0, ascending; then n_active at [E]
    int32_t *perm_pair;      // [T*k] position -> pair id
    int32_t *inv;            // [T*k] pair id -> position
};

// Optional per-stage timing callback: hook(arg, stage) after a stage's launch.
typedef void (*StageHook)(void *arg, int stage);

// partial/arrivals: split-K scratch for small T (nullable: no split).
cudaError_t launch_route_impl(const Dims &d, const LayerDev &L, const float *residual, int T,
                              const RouteOut &o, double *partial, int32_t *arrivals,
                              cudaStream_t st, StageHook hook = nullptr, void *hook_arg = nullptr);
// Stable token->expert positions (perm_pair, inv) from the chunk bases; with
// gather, also the expert-sorted copy of x_hi/x_lo.  Needed when T > 8 (the
// router writes the permutation itself for a single chunk) or for the gather.
cudaError_t launch_scatter(const Dims &d, int T, const RouteOut &o, bool gather, __half *xp_hi,
                           __half *xp_lo, cudaStream_t st);
// Largest number of doubles the split-K partial buffer needs for any T <= max_tokens.
size_t route_partial_elems(int max_tokens, int H, int E);

// Weight upload ----------------------------------------------------------------
// gguf: E*R*(K/32)*17 bytes on the device.  pair_rows: gate_up row re-order.
cudaError_t launch_repack(const uint8_t *gguf, int E, int R, int K, bool pair_rows,
                          uint8_t *q, uint8_t *s, cudaStream_t st);

struct EpReturn;  // expert-parallel down epilogue (below)

// Expert GEMV (decode) ---------------------------------------------------------
// Expert-sorted rows the GEMV stages work on.
struct GemvRows {
    const __half *x_hi, *x_lo;  // gate_up input rows: by token (perm_pair) or by position
    const int32_t *perm_pair;   // position -> pair id (t*k+s); NULL: x rows are positions
    const int32_t *offsets;     // [E+1] expert row ranges
    const int32_t *active;      // [E] experts with rows, then their count at [E]
    const int32_t *y_rows;      // down output row per position (NULL: the position)
    int max_active;             // grid bound on the active list
    const int32_t *gate = nullptr;  // if set, the launch does nothing unless *gate == gate_want
    int gate_want = 0;
};
// Fused decode step (decode.cu): routing, gate_up + SwiGLU, down and the combine in
// one cooperative launch for T <= kDecodeMaxTokens.  Its cross-CTA flags carry the
// launch count, which each CTA keeps here.
constexpr int kDecodeMaxTokens = 4;
constexpr int kDecodeMaxCtas = 1024;
struct DecodeBarrier {
    unsigned epoch[kDecodeMaxCtas];   // launches CTA b has completed (written only by CTA b)
};
bool decode_supported(const Dims &d, int T, int device);
// scratch: decode_scratch_bytes(), prepared once by init_decode_scratch()
size_t decode_scratch_bytes(const Dims &d, int device);
cudaError_t init_decode_scratch(const Dims &d, int device, void *scratch, cudaStream_t st);
cudaError_t launch_decode(const Dims &d, const LayerDev &L, const RouteOut &r, const float *residual, int T,
                          void *scratch, float *out, DecodeBarrier *bar, int32_t *err, int device, cudaStream_t st);

// T: upper bound on any expert's row count (sizes the token groups per pass).
cudaError_t launch_gemv_gate_up(const Dims &d, const LayerDev &L, const GemvRows &rows, int T,
                                __half *act_hi, __half *act_lo, int32_t *err, cudaStream_t st);
cudaError_t launch_gemv_down(const Dims &d, const LayerDev &L, const GemvRows &rows, int T,
                             const __half *act_hi, const __half *act_lo, float *y, int32_t *err,
                             cudaStream_t st, const EpReturn *ret = nullptr);

// tcgen05 grouped GEMMs (prefill) -------------------------------------------------
// True on an sm_100 device once the TMA tensor-map encoder is resolved.
bool tc_supported();
// Block-scaled grouped GEMMs (gemm_bs.cu): gate_up(+SwiGLU) and down over
// expert-sorted rows.  Rows come from (x_hi, x_lo) [*][H] through perm (position
// -> pair id, token = pair / k; `tokens` rows, each quantized once) or, with perm
// NULL, by position; rows_cap bounds the positions, tok_cap the tokens.  Outputs
// go to y[y_rows ? y_rows[pos] : pos][H] (with ret: the source rank's y, see
// EpReturn).  scratch: bs_scratch_bytes(), prepared once by init_bs_scratch().
size_t bs_scratch_bytes(int rows_cap, int tok_cap, int E, int H, int I);
// Each of `tokens` rows of (x_hi, x_lo) [tokens][H] as five-term E2M1 records in the
// scratch's token-record arrays (returned in *tq, *ts); nothing to do unless *gate == 1
// (gate NULL: always).
cudaError_t launch_tok_quant(const __half *x_hi, const __half *x_lo, int tokens, int H, int I, void *scratch,
                             int rows_cap, int tok_cap, int scratch_e, const int32_t *gate, cudaStream_t st,
                             const uint4 **tq, const uint2 **ts);
cudaError_t init_bs_scratch(void *scratch, int rows_cap, int tok_cap, int E, int H, int I);
// scratch_e: the expert count the scratch was sized for (bs_scratch_bytes), >= d.E.
cudaError_t launch_bs_experts(const Dims &d, const LayerDev &L, const int32_t *offsets, const __half *x_hi,
                              const __half *x_lo, const int32_t *perm, int tokens, int rows_cap, int tok_cap,
                              void *scratch, int scratch_e, float *y, const int32_t *y_rows, int32_t *err,
                              cudaStream_t st, StageHook hook, void *hook_arg, int *launches,
                              const EpReturn *ret = nullptr, const int32_t *gate = nullptr, int gate_want = 0,
                              const uint4 *rec_q = nullptr, const uint2 *rec_s = nullptr);
// (rec_q, rec_s: the rows already as token records, row = position; x_hi/x_lo unused)
// Combine --------------------------------------------------------------------
cudaError_t launch_combine(const Dims &d, const float *residual, const RouteOut &r,
                           const float *y, int T, float *out, cudaStream_t st);

// Expert parallelism --------------------------------------------------------------
// Rank r of N owns experts [r*El, (r+1)*El).  Every rank exports one device
// window to its peers (CUDA IPC, mapped over NVLink); all data moves as stores
// into the receiver's window, and per-source epoch flags order them:
//   1. count kernel: this rank's per-expert pair counts go into row `me` of every
//      rank's count table; once all N rows are in, each rank derives the whole
//      exchange layout (where its rows land, its expert-major row ranges, where
//      each received row returns to) on the device;
//   2. dispatch kernel: each routed row (fp16 hi/lo of the normalized token) is
//      stored straight into the owner's receive buffer, expert-major;
//   3. the expert GEMMs run on the receive buffer; the down epilogue stores each
//      output row into its source rank's window at the row's local sorted
//      position, where the source's combine reads it.
// No host synchronisation and no collective library on the data path; NCCL
// only exchanges the IPC handles when the context is created.
constexpr int kMaxEpRanks = 8;
constexpr int kEpRowShift = 28;  // y_rows entry: (source rank << 28) | row in that rank's y
constexpr uint32_t kEpRowMask = (1u << kEpRowShift) - 1;
enum { kEpFlagCount = 0, kEpFlagDispatch = 1, kEpFlagReturn = 2 };

// Byte offsets inside each rank's window (identical on every rank).
struct EpWindow {
    size_t flags;             // int32 [3][kMaxEpRanks]: count / dispatch / return flag per source rank
    size_t table;             // int32 [N][E]: pairs source s routes to global expert e
    size_t recv_hi, recv_lo;  // fp16 [r_cap][H]: rows for this rank's experts, expert-major (GEMV path);
                              // the tcgen05 path receives token records from recv_hi on (ep_recv_records)
    size_t y;                 // f32 [p_cap][H]: outputs for this rank's pairs, at their sorted position
    size_t bytes;
};
EpWindow ep_window(int N, int E, int H, int p_cap, int r_cap);

// Device scratch of the exchange (local to each rank).
struct EpMeta {
    int32_t *send_base;    // [E] receive row of this rank's first pair of expert e (in e's owner)
    int32_t *offsets_loc;  // [El+1] expert-major row ranges of this rank's experts
    int32_t *active_loc;   // [El+1] local experts with rows, then their count at [El]
    int32_t *seg_start;    // [El][N] first expert-major row of source s's rows for local expert el
    int32_t *src_pos;      // [El][N] sorted position of those rows in source s
    int32_t *y_rows;       // [r_cap] return target of each received row: (source << 28) | position
    int32_t *status;       // [1] 1 while this exchange is intact, 0 after a failed wait
    int32_t *mode;         // [1] expert path of this exchange: 1 tcgen05 GEMM, 0 GEMV
    unsigned *arrive;      // [2] CTA arrival counters (dispatch kernel, down GEMM)
    uint8_t **win;         // [kMaxEpRanks] every rank's window as mapped here
    float **ret_y;         // [kMaxEpRanks] every rank's y (inside its window)
    int32_t **ret_flag;    // [kMaxEpRanks] this rank's return flag inside every rank's window
};

struct EpArgs {
    int N, me, E, El, H, k, r_cap, p_cap, epoch;
    int path;               // 1 GEMV, 2 tcgen05, 0 auto: tcgen05 once the group has >= 32 pairs per expert
    long long count_limit_ns;  // bound on the count exchange (absorbs the ranks' host-side skew)
    long long limit_ns;        // bound on the dispatch and return waits (device progress only)
    EpWindow w;
    EpMeta m;
    const int32_t *counts, *offsets, *topk_idx, *perm_pair;  // this rank's routing
    const __half *x_hi, *x_lo;                                // its normalized rows, by token
    // the same rows as five-term token records (tok_quant_kernel), sent instead of the
    // fp16 rows when the group takes the tcgen05 path (*m.mode == 1); NULL: never
    const uint4 *tq;
    const uint2 *ts;
    int nkb;
    int32_t *err;
};

// Where the tcgen05 path's received token records sit in a window: the codes of row
// p at q + p * nkb * 4 * 5 (uint4), its scale words at s + p * nkb * 4 (uint2).
__host__ __device__ inline void ep_recv_records(uint8_t *win, const EpWindow &w, int r_cap, int H, uint4 **q,
                                                uint2 **s) {
    const size_t nkb = (size_t)(H + 127) / 128;
    *q = reinterpret_cast<uint4 *>(win + w.recv_hi);
    *s = reinterpret_cast<uint2 *>(win + w.recv_hi + (size_t)r_cap * nkb * 4 * 5 * 16);
}

// Down-GEMM epilogue of an expert-parallel step: output row y_rows[pos] goes to
// ret_y[rank] at its position; the last CTA to finish publishes `epoch` in
// every source's return flag (only while *status is 1).
struct EpReturn {
    float *const *y = nullptr;
    int32_t *const *flag = nullptr;
    unsigned *arrive = nullptr;
    const int32_t *status = nullptr;
    int n = 0, epoch = 0;
};

// Layout of one exchange from the count table (host restatement of the count
// kernel's arithmetic, for tests): returns 0, or -1 on negative counts.
int ep_layout(int N, int El, int me, const int32_t *table, int32_t *send_base, int32_t *offsets_loc,
              int32_t *seg_start, int32_t *src_pos);

cudaError_t launch_ep_counts(const EpArgs &a, cudaStream_t st);
cudaError_t launch_ep_dispatch(const EpArgs &a, int grid, cudaStream_t st);
// Waits (bounded) for flags[0..n) >= epoch; on timeout records `code`, clears
// *status and, when offsets_loc is set, empties the expert ranges.
cudaError_t launch_ep_wait(const EpArgs &a, int which, int code, cudaStream_t st);

struct NcclApi {
    ncclResult_t (*ncclGetUniqueId)(ncclUniqueId *);
    ncclResult_t (*ncclCommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*ncclCommDestroy)(ncclComm_t);
    ncclResult_t (*ncclAllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char *(*ncclGetErrorString)(ncclResult_t);
};
extern NcclApi g_nccl;
// Resolves NCCL from libnccl.so.2 once; false (with a reason) if unavailable.
bool nccl_load(std::string *err);

// GGUF (gguf.cu) ---------------------------------------------------------------------
// One layer's MoE tensors as host pointers (into the mapped file, or into the
// buffers below when a vector was widened to f32 or split gate/up was interleaved).
struct GgufLayer {
    const float *norm = nullptr, *router_w = nullptr, *router_b = nullptr, *gu_b = nullptr, *dn_b = nullptr;
    const uint8_t *gu = nullptr, *dn = nullptr;
    std::vector<float> buf[5];
    std::vector<uint8_t> gu_buf;
};
// 0, or -1 with a message in *err.
int gguf_layer(const ::amoe_gguf *g, int layer, int H, int I, int E, GgufLayer *L, std::string *err);

// The head's tensors: output_norm.weight widened to f32, and the lm head's bytes as
// stored (output.weight, or token_embd.weight when the file ties them), F32/F16/BF16.
struct GgufHead {
    const float *norm = nullptr;
    const void *lm_head = nullptr;
    int type = 0;
    std::vector<float> buf;
    std::vector<uint8_t> head_buf;
};
int gguf_head(const ::amoe_gguf *g, int H, int V, GgufHead *h, std::string *err);

// Sets the message amoe_last_error(NULL) returns on the calling thread.
void set_thread_error(const std::string &msg);

// Shared device helpers ---------------------------------------------------------
__device__ __forceinline__ float e8m0_to_float(uint32_t b) {
    // 2^(b-127); b == 0 is the subnormal 2^-127; b == 255 is NaN (tensor.go:152-155)
    uint32_t bits = b == 0 ? 0x00400000u : (b == 255 ? 0x7fc00000u : (b << 23));
    return __uint_as_float(bits);
}

// Four E8M0 bytes -> 2^(b-127) each.  Fast path (no byte is 0 or 255): the byte
// shifted into the f32 exponent field; otherwise the exact per-byte rule.
__device__ __forceinline__ void e8m0x4_to_float(uint32_t sv, float (&f)[4]) {
    const uint32_t zero = (sv - 0x01010101u) & ~sv & 0x80808080u;  // some byte == 0x00
    const uint32_t ones = (~sv - 0x01010101u) & sv & 0x80808080u;  // some byte == 0xFF
    if ((zero | ones) == 0u) {
        f[0] = __uint_as_float((sv << 23) & 0x7f800000u);
        f[1] = __uint_as_float((sv << 15) & 0x7f800000u);
        f[2] = __uint_as_float((sv << 7) & 0x7f800000u);
        f[3] = __uint_as_float((sv >> 1) & 0x7f800000u);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = e8m0_to_float((sv >> (8 * j)) & 0xffu);
    }
}

// Eight E2M1 values (four bytes, low nibble first) -> four f16x2, one per byte.
__device__ __forceinline__ uint4 e2m1x8_to_f16(uint32_t w) {
    uint4 o;
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
        : "=r"(o.x), "=r"(o.y), "=r"(o.z), "=r"(o.w)
        : "r"(w));
    return o;
}

__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    uint32_t r;
    asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(r) : "r"(byte));
    return r;
}

// Expert-parallel epilogue helpers ------------------------------------------------
__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Output row base for down-GEMM position `pos`: the local y (row y_rows[pos] or
// pos), or, expert-parallel, the source rank's y at the packed row.
__device__ __forceinline__ float *ep_out_row(float *y, const int32_t *y_rows, const EpReturn &ret, int pos,
                                             int R) {
    if (!y_rows) return y + (size_t)pos * R;
    const uint32_t v = (uint32_t)y_rows[pos];
    if (ret.n == 0) return y + (size_t)v * R;
    return ret.y[v >> kEpRowShift] + (size_t)(v & kEpRowMask) * R;
}

// Called by every thread of every CTA of an expert-parallel down GEMM once its
// last store is issued: the CTA's stores to peer memory are fenced at system
// scope, and the last CTA to arrive (the counter wraps to 0 for the next
// launch) publishes the epoch in every source rank's return flag.
__device__ __forceinline__ void ep_return_done(const EpReturn &ret) {
    if (ret.n == 0) return;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        if (atomicInc(ret.arrive, total - 1) == total - 1) {
            __threadfence_system();
            if (*reinterpret_cast<const volatile int32_t *>(ret.status) == 1)
                for (int q = 0; q < ret.n; ++q) st_release_sys(ret.flag[q], ret.epoch);
        }
    }
}

}  // namespace amoe
