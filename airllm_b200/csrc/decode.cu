// decode.cu -- K9: a decode step (T <= kDecodeMaxTokens) as ONE cooperative
// persistent kernel: routing, gate_up + SwiGLU, down and the combine.
//
//   routing  RMSNorm, router logits, top-k, softmax     (primitives.go:11-72, moe.go:12-41)
//   gate_up  act = SwiGLU(x . W_gu^T + b_gu)              (layer.go:139-148, 175; primitives.go:138-149)
//   down     y = act . W_dn^T + b_dn                      (layer.go:179-187)
//   combine  out = residual + f32(sum_s f64(w_s) * f64(y_s))  (layer.go:109-121)
//
// A decode step is a batched matrix-vector product over the selected experts'
// MXFP4 weights (53 MB per token for the 20B shape): the bound is HBM, and the
// design goal is to keep every SM streaming weight boxes from the moment the
// routing is known to the end, with next to no instructions per weight.
//
// Work.  A unit is one 128-row weight tile of one selected expert over its K
// range: every gate_up tile over all of K (SwiGLU needs the whole sum), every
// down tile over one half of K.  A host-built table (longest-processing-time
// first over the units' box counts, one table per number of active experts)
// gives each CTA its units: gate_up units first, then down units, both in
// slot order.  No unit is shared between CTAs, so no tile needs a cross-CTA
// reduction.  Two hand-offs cross CTAs, both through L2:
//   - the last gate_up unit of a slot to finish publishes the slot's
//     activation (a per-slot flag carrying the launch epoch); a down unit's
//     activation operand is copied in once the flag is up (its weights are
//     already streaming into the ring meanwhile);
//   - the last down unit of a 128-row output tile to finish combines that
//     tile for every token (self-resetting arrival counters).
//
// Tensor cores.  The weights never leave their packed form: each unit's boxes
// (128 rows x 64 B of E2M1 codes per 128-element K box, plus the box's 512-byte
// E8M0 chunk, stored together in the 64-byte swizzle order) stream by bulk copy
// into a ring of 17 KB stages, two boxes per stage, and go straight into
// tcgen05.mma kind::mxf4 (M = 128, K = 64, two per box) with the E8M0 chunk as
// the hardware block scales.  The tokens are the N columns, each as five
// block-scaled E2M1 terms (fp4_terms.cuh): N = 8, 16 or 32 for 1, 2-3 or 4
// tokens.  gate_up's operand (the normalized tokens) is quantized once per CTA
// into shared memory; gate_up's epilogue writes down's operand, the SwiGLU
// outputs' terms, to global memory in the same box form, and a down unit copies
// its K half of it in one bulk copy.
//
// Roles after the routing: warp 0 lane 0 streams the ring (waiting for the
// MMAs to release a stage), warp 1 issues the MMAs into two TMEM accumulators
// (the epilogue of one unit overlaps the next unit's MMAs), warp 2 lane 0
// copies the down units' operands as their flags come up, warps 4-15 first
// quantize gate_up's operand (while the first stages are in flight) and warps
// 4-7 (one per TMEM lane quadrant) then run the unit epilogues.
//
// The routing is a chain of short dependent steps, so it is written for
// latency: every global load in flight at once, warp-uniform control flow around
// every shuffle (a warp split by a lane-0-only branch pays for each full-mask
// shuffle), one warp per token for the top-k and one warp for the permutation.
//
// Every wait is bounded (~1 s of clock): it records a code (50-59) in the error
// flag, marks the CTA dead (later waits return at once, no further copy is
// issued, the copies and MMAs in flight are waited for) and the kernel winds
// down through the same barriers.
#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/amoe.h"
#include "fp4_terms.cuh"
#include "tc_ptx.cuh"

namespace amoe {

namespace {

using namespace bs;

constexpr int kDecThreads = 512;                // 16 warps: the routing spreads H over all of them
constexpr int kProdWarp = 0, kMmaWarp = 1, kLoadWarp = 2, kEpiWarp0 = 4;
constexpr int kEpiThreads = 128;                // warps 4-7, one per TMEM lane quadrant
constexpr int kBuildThreads = kDecThreads - kEpiWarp0 * 32;  // warps 4-15 quantize gate_up's operand
constexpr int kTerms = fp4::kTerms;
constexpr uint32_t kBoxBytes = 128 * 64;        // one packed box: 128 rows x 128 E2M1 values
constexpr uint32_t kBoxStep = (uint32_t)kBoxStride;  // a box's rows and its scale chunk, as stored
constexpr uint32_t kStageBytes = 2 * kBoxStep;       // two boxes, each followed by its scale chunk
constexpr uint32_t kSfChunk = 512;              // E8M0 chunk of 128 rows x 4 blocks
constexpr int kMaxStages = 12;
constexpr int kMinStages = 4;
constexpr int kMaxUnits = 64;                   // units per CTA
constexpr int kSchedWords = 1024;               // one CTA's schedule rows (int32)
static_assert(kSchedWords == AMOE_DECODE_SCHED_WORDS, "the table row size is part of the C ABI");
constexpr int kMaxCtaStages = kMaxUnits * 16;   // ring stages of one CTA (a unit has <= 16: K <= 4096)
constexpr size_t kSmemBudget = 232448;          // dynamic shared memory per block (227 KB)
constexpr uint32_t kTmemCols = 128;             // accumulators at columns 0 and 32, scale slots at 64 and 80
constexpr uint32_t kAccCols = 32;
constexpr uint32_t kSfCol = 64;

static_assert(kStageBytes % 1024 == 0 && kBoxStep % 512 == 0, "64-byte swizzle atoms start on 512 B");
static_assert((size_t)kMinStages * kStageBytes >= 4 * kSchedWords, "the routing stages the schedule rows in the ring");

// An activation operand box: N rows x 64 B of codes (swizzled like the weights),
// then the N rows' E8M0 bytes in a 512-byte chunk (byte 16 n + j: row n, block j).
__host__ __device__ constexpr uint32_t bbox_bytes(int ncol) { return (uint32_t)ncol * 64u + kSfChunk; }

// Unit encoding in the schedule table.
__host__ __device__ constexpr int32_t unit_code(int phase, int slot, int mt, int kpart) {
    return (phase << 30) | (slot << 20) | (mt << 8) | kpart;
}

struct DecodeParams {
    const float *residual;
    float *out;
    const float *gain, *router_w, *router_b;  // RMSNorm gain [H], router [E][H] and bias [E]
    float eps;
    RouteOut route;             // routing outputs (logits doubles as the cross-CTA exchange buffer)
    unsigned *rcnt;             // [2] CTAs whose router dot products are stored: the launch with epoch e
                                //     counts on [e % 2] and clears [(e + 1) % 2] for the next launch
    const uint8_t *gu_tq, *dn_tq;    // box planes: per box its swizzled rows, then its scale chunk
    const float *gu_b, *dn_b;
    uint8_t *aq;                // [S][nkb2] down operand boxes: the five E2M1 terms of every token's activation
    float *yb;                  // [S][2][T][H] down outputs, one plane per K half
    uint32_t *cnt_gu;           // [S] self-resetting arrival counters of the gate_up units
    uint32_t *cnt_dn;           // [nmt2] ... of the down units per output tile
    unsigned *aflag;            // [S] launch epoch once the slot's activation is complete
    const int32_t *sched;       // [G][kSchedWords]: per CTA, [n - 1]..[n] delimit its units when n slots are active
    DecodeBarrier *bar;
    int32_t *err;
    int T, H, I, E, k, Hp, Ip, S;
    int stages;
};

// Boxes of the longest down unit (one K half, or all of K when it is one box).
__host__ __device__ inline int down_boxes(int Ip) {
    const int nkb2 = Ip / 128;
    return nkb2 >= 2 ? (nkb2 + 1) / 2 : nkb2;
}

// Shared-memory layout (offsets from a 1 KB-aligned base).
struct DecLayout {
    uint32_t ring, bx, bd, actst, units, stg, rel, offs, act, perm, inv, w, sl, rms, lg, tk, amask, misc, bars, tslot,
        total;
};

__host__ __device__ inline DecLayout dec_layout(int T, int Hp, int Ip, int E, int k, int stages, int ncol) {
    DecLayout L;
    uint32_t o = 0;
    const uint32_t P = (uint32_t)(T * k);
    L.ring = o;
    o += (uint32_t)stages * kStageBytes;
    L.bx = o;  // gate_up operand: every K box of the normalized tokens' terms
    o += (uint32_t)(Hp / 128) * bbox_bytes(ncol);
    L.bd = o;  // down operand: two buffers of one unit's K boxes; first the normalized tokens [T][Hp] f32
    {
        const uint32_t boxes = 2u * (uint32_t)down_boxes(Ip) * bbox_bytes(ncol), xn = (uint32_t)(T * Hp) * 4u;
        o += ((boxes > xn ? boxes : xn) + 511u) & ~511u;
    }
    L.actst = o;  // [T][64] SwiGLU outputs of one gate_up tile
    o += (uint32_t)T * 64 * 4;
    L.units = o;
    o += kMaxUnits * 4;
    L.stg = o;  // [kMaxCtaStages] this CTA's ring stages: phase << 31 | (boxes - 1) << 30 | first box
    o += kMaxCtaStages * 4;
    L.rel = o;  // [stages] last stage issued into each ring slot
    o += (uint32_t)stages * 4;
    L.offs = o;
    o += (uint32_t)(E + 1) * 4;
    L.act = o;
    o += (uint32_t)(E + 1) * 4;
    L.perm = o;
    o += P * 4;
    L.inv = o;
    o += P * 4;
    L.w = o;
    o += P * 4;
    L.sl = o;  // [P] active-slot index of each (token, slot) pair
    o += P * 4;
    o = (o + 7u) & ~7u;
    L.rms = o;  // [4] inverse RMS per token, then [warps][4] partial sums (f64)
    o += (uint32_t)(4 + (kDecThreads / 32) * 4) * 8;
    L.lg = o;  // [T*E] router logits
    o += (uint32_t)(T * E) * 4;
    L.tk = o;  // [P] selected experts in slot order
    o += P * 4;
    L.amask = o;  // [8] active-expert bit mask
    o += 32;
    L.misc = o;  // broadcast words
    o += 64;
    o = (o + 7u) & ~7u;
    L.bars = o;  // full[stages], empty[stages], accfull[2], accempty[2], bfull[2], bempty[2], done, bxready
    o += (uint32_t)(2 * stages + 10) * 8;
    L.tslot = o;
    o += 16;
    L.total = o + 1024;  // base alignment slack
    return L;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }
__device__ __forceinline__ void build_bar() { asm volatile("bar.sync 2, %0;" ::"n"(kBuildThreads) : "memory"); }

// Bounded mbarrier wait that returns at once once the CTA is dead.
__device__ __forceinline__ bool ring_wait(uint64_t *bar, uint32_t parity, volatile int *dead, int32_t *err,
                                          int code) {
    if (*dead) return false;
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (*dead) return false;
        if (clock64() - t0 > kWaitLimit) {
            atomicCAS(err, 0, code);
            *dead = 1;
            return false;
        }
    }
}

// ---- tcgen05, one CTA (M = 128) ----
__device__ __forceinline__ void sf_copy(uint32_t tmem_col, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc_sf(saddr)) : "memory");
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                     uint32_t sfb) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
// Arrives on `bar` once the MMAs (and scale copies) issued so far complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Instruction descriptor, kind::mxf4 block-scaled, M = 128: A and B E2M1,
// K-major, E8M0 scales; sf_id is the first of the two scale bytes (32-element
// blocks) the K = 64 MMA uses.
__device__ __forceinline__ uint32_t idesc_dec(uint32_t sf_id, int n) {
    return (sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
           (sf_id << 29);
}
template <int NCOL>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[NCOL]) {
    if constexpr (NCOL == 8) tmem_ld8(taddr, v);
    else if constexpr (NCOL == 16) tmem_ld16(taddr, v);
    else tmem_ld32(taddr, v);
}
__device__ __forceinline__ uint32_t elect_one() {
    uint32_t e;
    asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(e));
    return e;
}

// Orders (logit, expert) as moe.go:20-27 does: larger value first, ties to the
// lower id, NaN after every number; -0 ties with +0.  The largest key wins.
__device__ __forceinline__ uint64_t topk_key(float v, int e) {
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
    const uint32_t ord = isnan(v) ? 1u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return ((uint64_t)ord << 32) | (uint64_t)(0xffffffffu - (uint32_t)e);
}

// Writes the five E2M1 terms of eight elements (this lane's part `sub` of 32-element
// block jb, token t) into an operand box: codes of row 5 t + j, and the scale bytes
// (each lane of the block writes the scales of the terms j % 4 == sub).
__device__ __forceinline__ void put_terms(uint8_t *box, uint32_t cb, int t, int jb, int sub,
                                          const uint32_t (&codes)[kTerms][1], const uint32_t (&sbyte)[kTerms]) {
#pragma unroll
    for (int j = 0; j < kTerms; ++j) {
        const int n = kTerms * t + j;
        *reinterpret_cast<uint32_t *>(box + n * 64 + ((jb ^ ((n >> 1) & 3)) << 4) + 4 * sub) = codes[j][0];
        if (j % 4 == sub) box[cb + n * 16 + jb] = (uint8_t)sbyte[j];
    }
}

template <int NCOL>
__launch_bounds__(kDecThreads, 1) __global__
    void decode_kernel(DecodeParams p) {
    static_assert(NCOL == 8 || NCOL == 16 || NCOL == 32, "MMA N");
    constexpr uint32_t kCb = NCOL * 64;               // codes of one operand box
    constexpr uint32_t kBb = bbox_bytes(NCOL);        // codes + scale chunk
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    const DecLayout lay = dec_layout(p.T, p.Hp, p.Ip, p.E, p.k, p.stages, NCOL);
    uint8_t *ring = sm + lay.ring;
    uint8_t *bx = sm + lay.bx;
    uint8_t *bd = sm + lay.bd;
    float *actst = reinterpret_cast<float *>(sm + lay.actst);
    int32_t *units_s = reinterpret_cast<int32_t *>(sm + lay.units);
    int32_t *offs_s = reinterpret_cast<int32_t *>(sm + lay.offs);
    int32_t *act_s = reinterpret_cast<int32_t *>(sm + lay.act);
    int32_t *perm_s = reinterpret_cast<int32_t *>(sm + lay.perm);
    int32_t *inv_s = reinterpret_cast<int32_t *>(sm + lay.inv);
    float *w_s = reinterpret_cast<float *>(sm + lay.w);
    int32_t *sl_s = reinterpret_cast<int32_t *>(sm + lay.sl);
    volatile int *misc = reinterpret_cast<volatile int *>(sm + lay.misc);  // [0] dead, [1] last, [2] units, [3] stages
    int32_t *stg_s = reinterpret_cast<int32_t *>(sm + lay.stg);
    int *rel_s = reinterpret_cast<int *>(sm + lay.rel);  // [R] last stage issued into each slot
    const int R = p.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + lay.bars);
    uint64_t *empty = full + R;
    uint64_t *accfull = empty + R;
    uint64_t *accempty = accfull + 2;
    uint64_t *bfull = accempty + 2;
    uint64_t *bempty = bfull + 2;
    uint64_t *done = bempty + 2;
    uint64_t *bxready = done + 1;  // gate_up's operand is in shared memory (one arrival per builder warp)
    uint32_t *tslot = reinterpret_cast<uint32_t *>(sm + lay.tslot);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, P = p.T * p.k, G = gridDim.x;
    const unsigned epoch = p.bar->epoch[blockIdx.x] + 1u;

    if (tid == 0) {
        misc[0] = 0;
        for (int s = 0; s < R; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
            rel_s[s] = -1;
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accfull + b, 1);
            mbar_init(accempty + b, kEpiThreads);
            mbar_init(bfull + b, 1);
            mbar_init(bempty + b, 1);
        }
        mbar_init(done, 1);
        mbar_init(bxready, kBuildThreads / 32);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "n"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    // ---------------- routing, in every CTA ----------------
    // RMSNorm (primitives.go:50-72), router logits (primitives.go:11-47), top-k and
    // softmax over the selected logits (moe.go:12-41), stable (expert, token, slot)
    // permutation.  The T x E router dot products are spread over the CTAs; each
    // counts itself in once its logits are stored, and every CTA then reads all
    // logits and derives the same routing.
    {
        constexpr int kWarps = kDecThreads / 32;
        constexpr int kPer = (4096 / 4 + kDecThreads - 1) / kDecThreads;  // float4 per thread, H <= 4096
        constexpr int kSchedPer = kSchedWords / kDecThreads;
        double *rms_s = reinterpret_cast<double *>(sm + lay.rms);
        double *red_s = rms_s + 4;
        float *lg_s = reinterpret_cast<float *>(sm + lay.lg);
        int *tk_s = reinterpret_cast<int *>(sm + lay.tk);
        uint32_t *amask_s = reinterpret_cast<uint32_t *>(sm + lay.amask);
        int32_t *sched_s = reinterpret_cast<int32_t *>(ring);  // read before any copy lands in the ring
        float *xn_s = reinterpret_cast<float *>(bd);           // [T][Hp]: bd is idle until the first down unit
        const int T = p.T, H = p.H, Hp = p.Hp;
        const int ndots = T * E, dot_ctas = min(G, ndots);
        if (blockIdx.x == 0 && tid == 0) p.rcnt[(epoch + 1u) & 1u] = 0u;  // the previous launch is over
        // (0) every global input of the routing in flight at once: this CTA's schedule
        //     rows for every number of active slots, the T residual rows, the gain
        //     and, for a CTA that owns a router dot product, the first router row
        //     (elements 4 (tid + 512 r) .. + 3 of each row)
        int32_t sv[kSchedPer];
        float4 wv[kPer], gv[kPer], xv[kDecodeMaxTokens][kPer];
        {
            const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const int e0 = (int)blockIdx.x < ndots ? (int)blockIdx.x % E : 0;
#pragma unroll
            for (int r = 0; r < kSchedPer; ++r)
                sv[r] = __ldg(p.sched + (size_t)blockIdx.x * kSchedWords + tid + r * kDecThreads);
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i4 = tid + r * kDecThreads;
                const bool in = 4 * i4 < H;
                wv[r] = in && (int)blockIdx.x < ndots
                            ? __ldg(reinterpret_cast<const float4 *>(p.router_w + (size_t)e0 * H) + i4)
                            : z;
                gv[r] = in ? __ldg(reinterpret_cast<const float4 *>(p.gain) + i4) : z;
#pragma unroll
                for (int t = 0; t < kDecodeMaxTokens; ++t)
                    xv[t][r] = in && t < T ? __ldg(reinterpret_cast<const float4 *>(p.residual + (size_t)t * H) + i4) : z;
            }
#pragma unroll
            for (int r = 0; r < kSchedPer; ++r) sched_s[tid + r * kDecThreads] = sv[r];
        }
        // (1) float64 sums of squares of the T residual rows
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t) {
            double v = 0.0;
#pragma unroll
            for (int r = 0; r < kPer; ++r)
                v += (double)xv[t][r].x * (double)xv[t][r].x + (double)xv[t][r].y * (double)xv[t][r].y +
                     (double)xv[t][r].z * (double)xv[t][r].z + (double)xv[t][r].w * (double)xv[t][r].w;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red_s[warp * 4 + t] = v;
        }
        __syncthreads();
        if (tid < T) {
            double sum = 0.0;
            for (int w = 0; w < kWarps; ++w) sum += red_s[w * 4 + tid];
            rms_s[tid] = 1.0 / sqrt(sum / (double)H + (double)p.eps);
        }
        __syncthreads();
        // (2) the normalized rows, rounded to f32 as RMSNorm stores them
        //     (primitives.go:68-70), zero past H; then the router dot products, one
        //     per CTA (dot d on CTA d mod G): logit = f32(sum f64(x_n) f64(W)) + b,
        //     partials added in a fixed order.  Each thread reads back only its own
        //     elements of xn_s.
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t) {
            if (t < T) {
                const double inv = rms_s[t];
#pragma unroll
                for (int r = 0; r < kPer; ++r) {
                    const int i4 = tid + r * kDecThreads;
                    if (4 * i4 < Hp) {
                        const float4 x = xv[t][r], g = gv[r];
                        const bool in = 4 * i4 < H;
                        float4 n;
                        n.x = in ? (float)((double)x.x * inv * (double)g.x) : 0.0f;
                        n.y = in ? (float)((double)x.y * inv * (double)g.y) : 0.0f;
                        n.z = in ? (float)((double)x.z * inv * (double)g.z) : 0.0f;
                        n.w = in ? (float)((double)x.w * inv * (double)g.w) : 0.0f;
                        reinterpret_cast<float4 *>(xn_s + (size_t)t * Hp)[i4] = n;
                    }
                }
            }
        }
        for (int dd = blockIdx.x; dd < ndots; dd += G) {
            const int t = dd / E, e = dd - t * E;
            double acc = 0.0;
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i4 = tid + r * kDecThreads;
                if (4 * i4 < H) {
                    const float4 w = dd == (int)blockIdx.x
                                         ? wv[r]
                                         : __ldg(reinterpret_cast<const float4 *>(p.router_w + (size_t)e * H) + i4);
                    const float4 x = reinterpret_cast<const float4 *>(xn_s + (size_t)t * Hp)[i4];
                    acc = fma((double)x.x, (double)w.x, acc);
                    acc = fma((double)x.y, (double)w.y, acc);
                    acc = fma((double)x.z, (double)w.z, acc);
                    acc = fma((double)x.w, (double)w.w, acc);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            __syncthreads();  // red_s reuse
            if (lane == 0) red_s[warp] = acc;
            __syncthreads();
            if (tid == 0) {
                double sum = 0.0;
                for (int w = 0; w < kWarps; ++w) sum += red_s[w];
                p.route.logits[dd] = (float)sum + p.router_b[e];
            }
        }
        if (tid == 0 && (int)blockIdx.x < dot_ctas) {  // this CTA's logits are stored
            __threadfence();
            atomicAdd(p.rcnt + (epoch & 1u), 1u);
        }
        // (3) one warp per token: its E logits, then the top-k as k rounds of a warp
        //     argmax over 64-bit keys ordered as moe.go:20-27 orders the experts
        //     (value descending, ties to the lower id, NaN after every number), then
        //     the softmax over the selected logits (moe.go:29-39): the k exponentials
        //     in parallel, the denominator summed in slot order.  The whole warp polls
        //     (one request per poll) so that it stays converged.
        if (warp < T) {
            const int t = warp;
            {
                const long long t0 = clock64();
                for (;;) {
                    const bool ready = ld_acquire(p.rcnt + (epoch & 1u)) >= (unsigned)dot_ctas;
                    if (__all_sync(0xffffffffu, ready)) break;
                    if (__shfl_sync(0xffffffffu, (int)(clock64() - t0 > kWaitLimit), 0)) {
                        if (lane == 0) atomicCAS(p.err, 0, 53);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            uint64_t key[8];  // lane holds experts lane + 32 j (E <= 256)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = lane + 32 * j;
                const bool in = e < E;
                const float v = __ldcg(p.route.logits + (size_t)t * E + (in ? e : 0));
                if (in) lg_s[t * E + e] = v;
                key[j] = in ? topk_key(v, e) : 0ull;
            }
            __syncwarp();
            int my_e = 0;
            for (int s = 0; s < p.k; ++s) {
                uint64_t b = key[0];
#pragma unroll
                for (int j = 1; j < 8; ++j) b = key[j] > b ? key[j] : b;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const uint64_t ob = __shfl_xor_sync(0xffffffffu, b, o);
                    b = ob > b ? ob : b;
                }
                const int es = (int)(0xffffffffu - (uint32_t)b);
                my_e = lane == s ? es : my_e;
#pragma unroll
                for (int j = 0; j < 8; ++j) key[j] = lane + 32 * j == es ? 0ull : key[j];
            }
            if (lane < p.k) tk_s[t * p.k + lane] = my_e;
            const double maxv = (double)lg_s[t * E + __shfl_sync(0xffffffffu, my_e, 0)];
            const double ex_all = exp((double)lg_s[t * E + my_e] - maxv);
            const double ex = lane < p.k ? ex_all : 0.0;
            double den = 0.0;
            for (int sl = 0; sl < p.k; ++sl) den += __shfl_sync(0xffffffffu, ex, sl);
            if (lane < p.k) w_s[t * p.k + lane] = (float)((double)(float)ex / den);
        }
        __syncthreads();
        // (4) one warp: counts, offsets, active experts, the stable permutation, each
        //     pair's active slot, and this CTA's units for this number of active slots
        if (warp == 0) {
            for (int e0 = 0; e0 <= E; e0 += 32)
                if (e0 + lane <= E) offs_s[e0 + lane] = 0;
            if (lane < 8) amask_s[lane] = 0u;
            __syncwarp();
            for (int q0 = 0; q0 < P; q0 += 32) {
                const int q = q0 + lane;
                if (q < P) {
                    const int e = tk_s[q];
                    atomicAdd(&offs_s[e], 1);
                    atomicOr(&amask_s[e >> 5], 1u << (e & 31));
                }
            }
            __syncwarp();
            // warp scan over experts (lane owns experts 8 lane .. 8 lane + 7; E <= 256)
            int c[8], a[8];
            int cs = 0, as = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = 8 * lane + j;
                c[j] = e < E ? offs_s[e] : 0;
                a[j] = c[j] > 0;
                cs += c[j];
                as += a[j];
            }
            int cx = cs, ax = as;  // inclusive warp prefix sums
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int cu = __shfl_up_sync(0xffffffffu, cx, o), au = __shfl_up_sync(0xffffffffu, ax, o);
                cx += lane >= o ? cu : 0;
                ax += lane >= o ? au : 0;
            }
            int co = cx - cs, ao = ax - as;
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = 8 * lane + j;
                if (e < E) {
                    offs_s[e] = co;
                    if (a[j]) act_s[ao] = e;
                }
                co += c[j];
                ao += a[j];
            }
            if (lane == 31) {
                offs_s[E] = cx;
                act_s[E] = ax;
            }
            const int na = __shfl_sync(0xffffffffu, ax, 31);  // active experts (>= 1)
            __syncwarp();
            for (int q0 = 0; q0 < P; q0 += 32) {  // pairs in (token, slot) order land stably
                const int q = q0 + lane;
                const int e = tk_s[q < P ? q : 0];
                int pos = offs_s[e];
                for (int r = 0; r < P; ++r) pos += (r < q) & (tk_s[r] == e);
                int slot = __popc(amask_s[e >> 5] & ((1u << (e & 31)) - 1u));  // active experts below e
#pragma unroll
                for (int w = 0; w < 8; ++w) slot += w < (e >> 5) ? __popc(amask_s[w]) : 0;
                if (q < P) {
                    perm_s[pos] = q;
                    inv_s[q] = pos;
                    sl_s[q] = slot;
                }
            }
            const int u0 = sched_s[na - 1], u1 = sched_s[na];
            const int n = min(u1 - u0, kMaxUnits);
            for (int u0w = 0; u0w < n; u0w += 32)
                if (u0w + lane < n) units_s[u0w + lane] = sched_s[u0 + u0w + lane];
            if (lane == 0) misc[2] = n;
        }
        __syncthreads();
        if (blockIdx.x == 0) {  // the routing the C ABI reports
            for (int q = tid; q < P; q += kDecThreads) {
                p.route.topk_idx[q] = tk_s[q];
                p.route.topk_w[q] = w_s[q];
                p.route.perm_pair[q] = perm_s[q];
                p.route.inv[q] = inv_s[q];
            }
            for (int e = tid; e <= E; e += kDecThreads) {
                p.route.offsets[e] = offs_s[e];
                p.route.active[e] = act_s[e];
                if (e < E) p.route.counts[e] = offs_s[e + 1] - offs_s[e];
            }
        }
    }

    const int n_active = act_s[E];
    const int nunits = misc[2];
    const int nkb1 = p.Hp / 128, nkb2 = p.Ip / 128;
    const int nmt1 = 2 * p.I / 128, nmt2 = (p.H + 127) / 128;
    const int nkp = nkb2 >= 2 ? 2 : 1, half2 = (nkb2 + 1) / 2;  // down units: K halves
    const int dmax = down_boxes(p.Ip);
    // a unit's phase (0 gate_up, 1 down), slot, weight tile, K part and box range
    auto unit_span = [&](int32_t code, int &phase, int &slot, int &mt, int &kpart, int &kb0, int &kb1) {
        phase = (code >> 30) & 1;
        slot = (code >> 20) & 1023;
        mt = (code >> 8) & 4095;
        kpart = code & 1;
        kb0 = phase == 0 || kpart == 0 ? 0 : half2;
        kb1 = phase == 0 ? nkb1 : (nkp == 1 || kpart == 1 ? nkb2 : half2);
    };

    // ---------------- the ring: this CTA's stages, two boxes each ----------------
    // Stage j is filled into slot j % R once the MMAs of stage j - R released it.
    auto issue = [&](int j) {
        const int32_t code = stg_s[j];
        const int phase = (int)(((uint32_t)code >> 31) & 1u), nb = ((code >> 30) & 1) + 1;
        const size_t box = (size_t)(code & 0x3fffffff);  // plane row of the first box: 128 * box
        const int sl = j % R;
        uint8_t *st = ring + (size_t)sl * kStageBytes;
        mbar_expect_tx(full + sl, (uint32_t)nb * kBoxStep);
        bulk_g2s(st, (phase ? p.dn_tq : p.gu_tq) + box * kBoxStep, (uint32_t)nb * kBoxStep, full + sl);
        rel_s[sl] = j;
    };
    if (tid == 0) {
        int j = 0;
        for (int u = 0; u < nunits; ++u) {
            int phase, slot, mt, kpart, kb0, kb1;
            unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
            const int e = act_s[slot];
            const int nmt = phase ? nmt2 : nmt1, nkb = phase ? nkb2 : nkb1;
            for (int kb = kb0; kb < kb1 && j < kMaxCtaStages; kb += 2, ++j)
                stg_s[j] = (int32_t)(((uint32_t)phase << 31) | ((uint32_t)(min(2, kb1 - kb) - 1) << 30) |
                                     (uint32_t)(((size_t)e * nmt + mt) * nkb + kb));
        }
        misc[3] = j;
        // the routing's staged rows in the ring are read by now (barrier above)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int i = 0; i < min(R, j); ++i) issue(i);
    }
    __syncthreads();
    tc_fence_after();
    const int nst = misc[3];
    const uint32_t tmem = *tslot;

    if (warp >= kEpiWarp0) {
        // ---------------- gate_up's operand, while the first stages stream in ----------------
        // every token's normalized row as five E2M1 terms per 32-element block, row
        // 5 t + j of every K box; rows of absent tokens and K past H read as zero
        // codes at unit scale
        const int bt = tid - kEpiWarp0 * 32;
        const float *xn_s = reinterpret_cast<const float *>(bd);
        for (uint32_t o = 16u * (uint32_t)bt; o < (uint32_t)nkb1 * kBb; o += 16u * kBuildThreads)
            *reinterpret_cast<uint4 *>(bx + o) =
                o % kBb < kCb ? make_uint4(0u, 0u, 0u, 0u) : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
        build_bar();
        const int nblk = p.Hp / 32, total = 4 * p.T * nblk;  // four lanes per (token, 32-element block)
        for (int base = (warp - kEpiWarp0) * 32; base < total; base += kBuildThreads) {  // whole warps
            const int it = base + lane;
            const bool live = it < total;
            const int unit = it >> 2, sub = it & 3;
            const int t = live ? unit / nblk : 0, blk = live ? unit - t * nblk : 0;
            float x[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) x[q] = live ? xn_s[(size_t)t * p.Hp + 32 * blk + 8 * sub + q] : 0.0f;
            uint32_t codes[kTerms][1], sbyte[kTerms];
            fp4::quantize<8, 4>(x, codes, sbyte);
            if (live) put_terms(bx + (size_t)(blk >> 2) * kBb, kCb, t, blk & 3, sub, codes, sbyte);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // read by the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(bxready);
    }

    if (warp == kProdWarp) {
        // ---------------- producer: refill each slot once its MMAs are done ----------------
        if (lane == 0) {
            for (int j = R; j < nst; ++j)
                if (!ring_wait(empty + j % R, ((j / R) - 1) & 1, misc, p.err, 51)) break;
                else issue(j);
            // copies in flight (only after a failed wait) land before the CTA exits
            for (int sl = 0; sl < R; ++sl)
                if (rel_s[sl] >= 0) mbar_wait(full + sl, (rel_s[sl] / R) & 1, p.err, 54);
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        const uint32_t elected = elect_one();
        const uint32_t idesc0 = idesc_dec(0, NCOL), idesc1 = idesc_dec(2, NCOL);
        const uint32_t ring_a = smem_u32(ring), bx_a = smem_u32(bx), bd_a = smem_u32(bd);
        int i = 0, dn = 0, nbox = 0;
        bool ok = true, bx_ready = false;
        for (int u = 0; u < nunits && ok; ++u) {
            int phase, slot, mt, kpart, kb0, kb1;
            unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
            const int buf = u & 1, ub = dn & 1;
            if (phase == 0 && !bx_ready) {
                if (!ring_wait(bxready, 0, misc, p.err, 50)) break;
                bx_ready = true;
            }
            if (u >= 2 && !ring_wait(accempty + buf, ((u >> 1) - 1) & 1, misc, p.err, 55)) break;
            if (phase == 1 && !ring_wait(bfull + ub, (dn >> 1) & 1, misc, p.err, 56)) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)buf * kAccCols;
            const uint32_t bbase = phase ? bd_a + (uint32_t)(ub * dmax) * kBb : bx_a;
            const int kbase = phase ? kb0 : 0;
            for (int kb = kb0; kb < kb1; kb += 2, ++i) {
                const int s = i % R, nb = min(2, kb1 - kb);
                if (!ring_wait(full + s, (i / R) & 1, misc, p.err, 51)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int b = 0; b < nb; ++b, ++nbox) {
                    if (elected) {
                        // tcgen05.cp and tcgen05.mma issued by this thread execute in issue
                        // order, so a scale slot is rewritten only after the MMAs that read it
                        const uint32_t a = ring_a + (uint32_t)s * kStageBytes + (uint32_t)b * kBoxStep;
                        const uint32_t bq = bbase + (uint32_t)(kb + b - kbase) * kBb;
                        const uint32_t sf = tmem + kSfCol + 16u * (uint32_t)(nbox & 1);
                        sf_copy(sf, a + kBoxBytes);  // the weights' E8M0 chunk
                        sf_copy(sf + 4, bq + kCb);   // the tokens' term scales
                        umma(d, desc_sw64(a), desc_sw64(bq), idesc0, (kb + b > kb0) ? 1u : 0u, sf, sf + 4);
                        umma(d, desc_sw64(a + 32), desc_sw64(bq + 32), idesc1, 1u, sf, sf + 4);
                    }
                }
                if (elected) mma_commit(empty + s);
                __syncwarp();
            }
            if (!ok) break;
            if (elected) {
                mma_commit(accfull + buf);
                if (phase == 1) mma_commit(bempty + ub);
            }
            __syncwarp();
            if (phase == 1) ++dn;
        }
        // every MMA issued so far completes before the TMEM is released
        if (elected) mma_commit(done);
        __syncwarp();
        mbar_wait(done, 0, p.err, 59);
    } else if (warp == kLoadWarp) {
        // ---------------- down operands: one bulk copy per unit once the slot is published ----------------
        if (lane == 0) {
            int dn = 0, last[2] = {-1, -1};
            bool bx_ready = false;
            for (int u = 0; u < nunits && !misc[0]; ++u) {
                int phase, slot, mt, kpart, kb0, kb1;
                unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
                if (phase == 0) continue;
                // bd holds the normalized tokens until gate_up's operand is built from them
                if (!bx_ready && !ring_wait(bxready, 0, misc, p.err, 50)) break;
                bx_ready = true;
                const int ub = dn & 1;
                if (dn >= 2 && !ring_wait(bempty + ub, ((dn >> 1) - 1) & 1, misc, p.err, 57)) break;
                const long long t0 = clock64();
                while ((int)(ld_acquire(p.aflag + slot) - epoch) < 0 && !misc[0]) {
                    if (clock64() - t0 > kWaitLimit) {
                        atomicCAS(p.err, 0, 52);
                        misc[0] = 1;
                    }
                    __nanosleep(32);
                }
                if (misc[0]) break;
                asm volatile("fence.proxy.async.global;" ::: "memory");  // generic stores of other CTAs -> bulk copy
                const uint32_t bytes = (uint32_t)(kb1 - kb0) * kBb;
                mbar_expect_tx(bfull + ub, bytes);
                bulk_g2s(bd + (size_t)(ub * dmax) * kBb, p.aq + ((size_t)slot * nkb2 + kb0) * kBb, bytes, bfull + ub);
                last[ub] = dn;
                ++dn;
            }
            for (int b = 0; b < 2; ++b)
                if (last[b] >= 0) mbar_wait(bfull + b, (last[b] >> 1) & 1, p.err, 54);
        }
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
        // ---------------- unit epilogues (one thread per tile row; the same barriers on every path) ----------------
        const int quad = warp & 3, row = quad * 32 + lane, et = tid - kEpiWarp0 * 32;
        // gate_up: rows 16 g + j (j < 8) hold the gate of pair 8 g + j, row + 8 its up row
        const int j16 = row & 15;
        const bool gate_lane = j16 < 8;
        const int pl = 8 * (row >> 4) + (j16 & 7);  // pair within the tile (0..63)
        for (int u = 0; u < nunits; ++u) {
            int phase, slot, mt, kpart, kb0, kb1;
            unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
            const int e = act_s[slot];
            const int buf = u & 1, h = 128 * mt + row;
            // the bias first: its load overlaps the wait
            float bias;
            if (phase == 0) bias = __ldg(p.gu_b + (size_t)e * 2 * p.I + 2 * (64 * mt + pl) + (gate_lane ? 0 : 1));
            else bias = kpart == 0 && h < p.H ? __ldg(p.dn_b + (size_t)e * p.H + h) : 0.0f;
            float v[kDecodeMaxTokens] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (ring_wait(accfull + buf, (u >> 1) & 1, misc, p.err, 58)) {
                tc_fence_after();
                float a[NCOL];
                tmem_ld_cols<NCOL>(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)buf * kAccCols, a);
#pragma unroll
                for (int t = 0; t < kDecodeMaxTokens; ++t)
                    if (kTerms * (t + 1) <= NCOL && t < p.T) {
                        float s = 0.0f;
#pragma unroll
                        for (int j = 0; j < kTerms; ++j) s += a[kTerms * t + j];
                        v[t] = s;
                    }
            }
            tc_fence_before();
            mbar_arrive(accempty + buf);
            if (phase == 0) {
                // SwiGLU of the tile's 64 pairs (partner lanes 8 apart swap values)
#pragma unroll
                for (int t = 0; t < kDecodeMaxTokens; ++t) {
                    if (t < p.T) {  // uniform
                        const float val = v[t] + bias;
                        const float other = __shfl_xor_sync(0xffffffffu, val, 8);
                        if (gate_lane) actst[t * 64 + pl] = swiglu(val, other);
                    }
                }
                epi_bar();
                if (warp == kEpiWarp0) {
                    // four lanes per (token, 32-pair block): the five E2M1 terms and their
                    // scales into down's operand, blocks 2 (mt % 2) + b of box mt / 2
                    const int unitq = lane >> 2, sub = lane & 3, t = unitq >> 1, b = unitq & 1;
                    const bool live = t < p.T;
                    float x[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) x[q] = live ? actst[t * 64 + 32 * b + 8 * sub + q] : 0.0f;
                    uint32_t codes[kTerms][1], sbyte[kTerms];
                    fp4::quantize<8, 4>(x, codes, sbyte);
                    uint8_t *box = p.aq + ((size_t)slot * nkb2 + (mt >> 1)) * kBb;
                    if (live) put_terms(box, kCb, t, 2 * (mt & 1) + b, sub, codes, sbyte);
                    if (mt == nmt1 - 1 && (mt & 1) == 0) {
                        // K past I (blocks 2 and 3 of the last box): zero codes at unit scale
                        for (int q = lane; q < 2 * NCOL; q += 32) {
                            const int n = q >> 1, jz = 2 + (q & 1);
                            *reinterpret_cast<uint4 *>(box + n * 64 + ((jz ^ ((n >> 1) & 3)) << 4)) =
                                make_uint4(0u, 0u, 0u, 0u);
                            box[kCb + n * 16 + jz] = 127;
                        }
                    }
                    asm volatile("fence.proxy.async.global;" ::: "memory");  // read by other CTAs' bulk copies
                    __threadfence();
                }
            } else {
                if (h < p.H) {
                    float *yrow = p.yb + ((size_t)slot * 2 + kpart) * p.T * p.H + h;
#pragma unroll
                    for (int t = 0; t < kDecodeMaxTokens; ++t)
                        if (t < p.T) yrow[(size_t)t * p.H] = v[t] + bias;
                }
                __threadfence();
            }
            epi_bar();
            if (et == 0) {
                const unsigned n = phase == 0 ? (unsigned)nmt1 : (unsigned)(nkp * n_active);
                unsigned *cnt = phase == 0 ? p.cnt_gu + slot : p.cnt_dn + mt;
                const unsigned old = atomicInc(cnt, n - 1u);
                misc[1] = old == n - 1u;
                if (old == n - 1u && phase == 0) publish(p.aflag + slot, epoch);
            }
            epi_bar();
            if (phase == 1 && misc[1]) {
                // the last down unit of output tile mt: combine its rows for every token in
                // slot order (layer.go:109-121)
                __threadfence();
                for (int it = et; it < p.T * 128; it += kEpiThreads) {
                    const int t = it >> 7, hh = 128 * mt + (it & 127);
                    if (hh >= p.H) continue;
                    double m = 0.0;
                    for (int s = 0; s < p.k; ++s) {
                        const int q = t * p.k + s;
                        const float *yp = p.yb + ((size_t)sl_s[q] * 2 * p.T + t) * p.H + hh;
                        float yv = __ldcg(yp);
                        if (nkp == 2) yv += __ldcg(yp + (size_t)p.T * p.H);
                        m += (double)w_s[q] * (double)yv;
                    }
                    p.out[(size_t)t * p.H + hh] = p.residual[(size_t)t * p.H + hh] + (float)m;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kTmemCols));
    }
    if (tid == 0) p.bar->epoch[blockIdx.x] = epoch;
}

// ---- host side -------------------------------------------------------------------------
struct DecodeCaps {
    int sms = 0;
    bool coop = false;
};
DecodeCaps g_caps[64];
std::once_flag g_caps_once[64];

const DecodeCaps &caps(int device) {
    std::call_once(g_caps_once[device], [device]() {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) == cudaSuccess) g_caps[device].sms = v;
        v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrCooperativeLaunch, device) == cudaSuccess)
            g_caps[device].coop = v != 0;
    });
    return g_caps[device];
}

int dec_ncol(int T) { return T <= 1 ? 8 : (T <= 3 ? 16 : 32); }

// Ring stages that fit beside the operand boxes.
int dec_stages(int T, int Hp, int Ip, int E, int k) {
    const DecLayout none = dec_layout(T, Hp, Ip, E, k, 0, dec_ncol(T));
    if (none.total + 64 >= kSmemBudget) return 0;
    // a slot, its index and two barriers per stage; 64 bytes for the layout's alignment rounding
    const int st = (int)((kSmemBudget - none.total - 64) / (kStageBytes + 4 + 16));
    return std::min(st, kMaxStages);
}

int dec_slots(const Dims &d) { return d.E < kDecodeMaxTokens * d.k ? d.E : kDecodeMaxTokens * d.k; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The units of every CTA for each number of active slots n = 1..S: longest
// processing time first over the units' box counts (all units of a phase are
// the same size, so this is a balanced round over the least-loaded CTAs),
// gate_up units before down units, each in slot order.  CTA b's rows sit in
// words [b * kSchedWords, (b + 1) * kSchedWords): S + 1 offsets (relative to
// the row start), then the unit lists for n = 1..S.
struct Schedule {
    std::vector<int32_t> rows;   // [G][kSchedWords]
    int max_units = 0;           // most units of one CTA for one n
    int max_words = 0;           // most words of one CTA's rows
};

Schedule build_schedule(const Dims &d, int G) {
    Schedule s;
    const int S = dec_slots(d);
    const int nkb1 = kpad128(d.H) / 128, nkb2 = kpad128(d.I) / 128;
    const int nmt1 = 2 * d.I / 128, nmt2 = (d.H + 127) / 128;
    const int nkp = nkb2 >= 2 ? 2 : 1, half2 = (nkb2 + 1) / 2;
    std::vector<std::vector<int32_t>> rows(G, std::vector<int32_t>(S + 1, 0));
    std::vector<std::vector<int32_t>> lists(G);
    std::vector<long long> load(G);
    for (int b = 0; b < G; ++b) rows[b][0] = S + 1;
    for (int n = 1; n <= S; ++n) {
        for (auto &l : lists) l.clear();
        std::fill(load.begin(), load.end(), 0);
        auto place = [&](int32_t code, int cost) {
            int best = 0;
            for (int b = 1; b < G; ++b)
                if (load[b] < load[best]) best = b;
            lists[best].push_back(code);
            load[best] += cost;
        };
        for (int sl = 0; sl < n; ++sl)
            for (int m = 0; m < nmt1; ++m) place(unit_code(0, sl, m, 0), nkb1);
        for (int sl = 0; sl < n; ++sl)
            for (int m = 0; m < nmt2; ++m)
                for (int kp = 0; kp < nkp; ++kp)
                    place(unit_code(1, sl, m, kp), nkp == 1 ? nkb2 : (kp ? nkb2 - half2 : half2));
        for (int b = 0; b < G; ++b) {
            rows[b].insert(rows[b].end(), lists[b].begin(), lists[b].end());
            rows[b][n] = (int32_t)rows[b].size();
            s.max_units = std::max(s.max_units, (int)lists[b].size());
        }
    }
    s.rows.assign((size_t)G * kSchedWords, 0);
    for (int b = 0; b < G; ++b) {
        s.max_words = std::max(s.max_words, (int)rows[b].size());
        std::copy_n(rows[b].begin(), std::min<size_t>(rows[b].size(), kSchedWords), s.rows.begin() + (size_t)b * kSchedWords);
    }
    return s;
}

struct DecScratch {
    size_t aq, yb, cnt_gu, cnt_dn, aflag, rcnt, sched, total;
};

DecScratch dec_scratch(const Dims &d, int G, const Schedule &s) {
    const int S = dec_slots(d), Ip = kpad128(d.I), nmt2 = (d.H + 127) / 128;
    DecScratch L;
    size_t o = 0;
    L.aq = o;  // down operand boxes, laid out for the widest N
    o += align256((size_t)S * (Ip / 128) * bbox_bytes(32));
    L.yb = o;
    o += align256((size_t)S * 2 * kDecodeMaxTokens * d.H * 4);
    L.cnt_gu = o;
    o += align256((size_t)S * 4);
    L.cnt_dn = o;
    o += align256((size_t)nmt2 * 4);
    L.aflag = o;
    o += align256((size_t)S * 4);
    L.rcnt = o;
    o += align256(2 * 4);
    L.sched = o;
    o += align256(s.rows.size() * 4);
    L.total = o;
    return L;
}

int grid_of(int device) { return device >= 0 && device < 64 && caps(device).sms > 0 ? caps(device).sms : 1; }

}  // namespace

size_t decode_scratch_bytes(const Dims &d, int device) {
    const int G = grid_of(device);
    return dec_scratch(d, G, build_schedule(d, G)).total;
}

cudaError_t init_decode_scratch(const Dims &d, int device, void *scratch, cudaStream_t st) {
    (void)st;
    const int G = grid_of(device);
    const Schedule s = build_schedule(d, G);
    const DecScratch L = dec_scratch(d, G, s);
    uint8_t *b = static_cast<uint8_t *>(scratch);
    cudaError_t e = cudaMemset(b, 0, L.total);  // activation padding, counters and flags start at 0
    if (e == cudaSuccess) e = cudaMemcpy(b + L.sched, s.rows.data(), s.rows.size() * 4, cudaMemcpyHostToDevice);
    return e;
}

bool decode_supported(const Dims &d, int T, int device) {
    if (T < 1 || T > kDecodeMaxTokens || device < 0 || device >= 64) return false;
    const DecodeCaps &cp = caps(device);
    if (!cp.coop || cp.sms <= 0 || cp.sms > kDecodeMaxCtas) return false;
    if ((2 * d.I) % 128 || d.H % 4 || d.H > 4096 || d.I > 4096 || d.E > 256 || d.k > 32 || dec_slots(d) > 1023) return false;
    if (2 * d.I / 128 > 4095 || (d.H + 127) / 128 > 4095) return false;
    if (dec_stages(T, kpad128(d.H), kpad128(d.I), d.E, d.k) < kMinStages) return false;
    static thread_local Dims last{};
    static thread_local int last_dev = -1;
    static thread_local bool last_ok = false;
    if (last_dev != device || last.H != d.H || last.I != d.I || last.E != d.E || last.k != d.k) {
        last = d;
        last_dev = device;
        const Schedule s = build_schedule(d, cp.sms);
        last_ok = s.max_units <= kMaxUnits && s.max_words <= kSchedWords;
    }
    return last_ok;
}

cudaError_t launch_decode(const Dims &d, const LayerDev &L, const RouteOut &r, const float *residual, int T,
                          void *scratch, float *out, DecodeBarrier *bar, int32_t *err, int device, cudaStream_t st) {
    const int S = dec_slots(d), Hp = kpad128(d.H), Ip = kpad128(d.I);
    const int G = caps(device).sms;
    const int ncol = dec_ncol(T);
    // the scratch layout depends only on the shape and the grid: recompute the offsets
    static thread_local Dims last{};
    static thread_local int last_dev = -1;
    static thread_local DecScratch lay{};
    if (last_dev != device || last.H != d.H || last.I != d.I || last.E != d.E || last.k != d.k) {
        last = d;
        last_dev = device;
        lay = dec_scratch(d, G, build_schedule(d, G));
    }
    uint8_t *b = static_cast<uint8_t *>(scratch);
    DecodeParams p{};
    p.residual = residual;
    p.out = out;
    p.gain = L.norm_gain;
    p.router_w = L.router_w;
    p.router_b = L.router_b;
    p.eps = d.eps;
    p.route = r;
    p.rcnt = reinterpret_cast<unsigned *>(b + lay.rcnt);
    p.gu_tq = L.gu_tq;
    p.dn_tq = L.dn_tq;
    p.gu_b = L.gu_b;
    p.dn_b = L.dn_b;
    p.aq = b + lay.aq;
    p.yb = reinterpret_cast<float *>(b + lay.yb);
    p.cnt_gu = reinterpret_cast<uint32_t *>(b + lay.cnt_gu);
    p.cnt_dn = reinterpret_cast<uint32_t *>(b + lay.cnt_dn);
    p.aflag = reinterpret_cast<unsigned *>(b + lay.aflag);
    p.sched = reinterpret_cast<const int32_t *>(b + lay.sched);
    p.bar = bar;
    p.err = err;
    p.T = T;
    p.H = d.H;
    p.I = d.I;
    p.E = d.E;
    p.k = d.k;
    p.Hp = Hp;
    p.Ip = Ip;
    p.S = S;
    p.stages = dec_stages(T, Hp, Ip, d.E, d.k);
    if (p.stages < kMinStages) return cudaErrorInvalidValue;
    const size_t smem = dec_layout(T, Hp, Ip, d.E, d.k, p.stages, ncol).total;
    auto kern = ncol == 8 ? decode_kernel<8> : (ncol == 16 ? decode_kernel<16> : decode_kernel<32>);
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace amoe

// The decode kernel's work table, as the context builds it (host arithmetic only).
extern "C" AMOE_API int amoe_decode_schedule(int32_t hidden, int32_t intermediate, int32_t experts, int32_t top_k,
                                             int32_t ctas, int32_t *rows) {
    using namespace amoe;
    if (hidden < 64 || hidden % 64 || hidden > 4096 || intermediate < 64 || intermediate % 64 ||
        intermediate > 4096 || experts < 1 || experts > 256 || top_k < 1 || top_k > experts || top_k > 32 ||
        ctas < 1 || ctas > kDecodeMaxCtas) {
        set_thread_error("decode schedule: hidden and intermediate must be multiples of 64 up to 4096, "
                         "1 <= top_k <= min(experts, 32), experts <= 256, 1 <= ctas <= 1024");
        return AMOE_ERR_INVALID;
    }
    const Dims d{hidden, intermediate, experts, top_k, 1e-5f};
    const Schedule s = build_schedule(d, ctas);
    if (s.max_units > kMaxUnits || s.max_words > kSchedWords) {
        set_thread_error("decode schedule: a CTA would get more units than its table row holds");
        return AMOE_ERR_INVALID;
    }
    if (rows) std::memcpy(rows, s.rows.data(), s.rows.size() * sizeof(int32_t));
    return AMOE_OK;
}
