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
// Work.  A unit is a K range of one 128-row weight tile of one selected expert.
// A host-built table (one per number of active experts) gives each CTA its units:
// the down tiles as K halves, placed longest-processing-time first, then the
// gate_up boxes in (slot, tile, K) order cut into contiguous ranges so that every
// CTA's total box count comes out even (stream-K).  A gate_up tile whose range
// spans CTAs becomes pieces: the later pieces store their partial sums, and piece
// 0 (the end of an earlier CTA's range, so the last to run) adds them in piece
// order.  Within a CTA the gate_up pieces run first.  The hand-offs between CTAs
// go through L2:
//   - every finished gate_up tile counts itself into its slot's counter; a down
//     unit's activation operand is copied in once the counter is complete (its
//     weights are already streaming into the ring meanwhile);
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
// Roles once the CTA's units are known: warp 0 issues the ring's first stages at
// once, one stage per lane, then lane 0 streams the rest (a slot refilled once the
// MMAs released it), warp 1 issues the MMAs into two TMEM
// accumulators, warp 2 lane 0 copies the down units' operands as their counters
// complete, warp 3 finishes the routing that only the combine needs (softmax
// weights, permutation, slots), and two epilogue groups of four warps (one per
// TMEM lane quadrant) run the unit epilogues: warps 4-7 take the units of
// accumulator 0, warps 8-11 those of accumulator 1, so two epilogues (each a chain
// of global round trips) and the next unit's MMAs overlap.  Before that, while
// warps 0-3 select the experts, warps 4-15 quantize gate_up's operand.
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
constexpr int kProdWarp = 0, kMmaWarp = 1, kLoadWarp = 2, kRestWarp = 3, kEpiWarp0 = 4;
constexpr int kEpiThreads = 128;                // an epilogue group: four warps, one per TMEM lane quadrant
constexpr int kEpiGroups = 2;                   // warps 4-7 take the units of accumulator 0, warps 8-11 those of 1
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
constexpr size_t kSmemBudget = 232448;          // dynamic shared memory per block (227 KB)
constexpr uint32_t kTmemCols = 128;             // accumulators at columns 0 and 32, scale slots at 64 and 80
constexpr uint32_t kAccCols = 32;
constexpr uint32_t kSfCol = 64;

static_assert(kStageBytes % 1024 == 0 && kBoxStep % 512 == 0, "64-byte swizzle atoms start on 512 B");
static_assert((size_t)kMinStages * kStageBytes >= 4 * kSchedWords, "the routing stages the schedule rows in the ring");

// An activation operand box: N rows x 64 B of codes (swizzled like the weights),
// then the N rows' E8M0 bytes in a 512-byte chunk (byte 16 n + j: row n, block j).
__host__ __device__ constexpr uint32_t bbox_bytes(int ncol) { return (uint32_t)ncol * 64u + kSfChunk; }

// A unit in the schedule table is two words:
//   w0 = phase << 31 | slot << 20 | tile << 8 | piece << 4 | pieces
//   w1 = first K box << 24 | end K box << 16 | split index
// gate_up tiles cut between CTAs (pieces > 1) meet through the partial-sum
// buffer of their split index; a down unit's piece is its K half.
constexpr int kMaxPieces = 4;
__host__ __device__ constexpr int32_t unit_w0(int phase, int slot, int mt, int piece, int pieces) {
    return (int32_t)(((uint32_t)phase << 31) | ((uint32_t)slot << 20) | ((uint32_t)mt << 8) | ((uint32_t)piece << 4) |
                     (uint32_t)pieces);
}
__host__ __device__ constexpr int32_t unit_w1(int kb0, int kb1, int split) {
    return (int32_t)(((uint32_t)kb0 << 24) | ((uint32_t)kb1 << 16) | (uint32_t)split);
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
    uint32_t *cnt_gu;           // [2][S] finished gate_up tiles per slot: the launch with epoch e counts
                                //     on [e % 2] and clears [(e + 1) % 2] for the next launch
    float *gpart;               // [G][kMaxPieces][4][128] partial sums of the gate_up tiles cut between CTAs
    uint32_t *cnt_split;        // [2][G] pieces of those tiles stored besides piece 0 (epoch parity as cnt_gu)
    uint32_t *cnt_dn;           // [nmt2] ... of the down units per output tile
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
    uint32_t ring, bx, bd, actst, units, rel, offs, act, perm, inv, w, sl, rms, lg, tk, amask, misc, bars, tslot,
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
    L.actst = o;  // [group][T][64] SwiGLU outputs of one gate_up tile
    o += (uint32_t)kEpiGroups * T * 64 * 4;
    L.units = o;  // [kMaxUnits][2] this CTA's units
    o += kMaxUnits * 8;
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
    L.bars = o;  // full[stages], empty[stages], accfull[2], accempty[2], bfull[2], bempty[2], done, bxready, rdone
    o += (uint32_t)(2 * stages + 11) * 8;
    L.tslot = o;
    o += 16;
    L.total = o + 1024;  // base alignment slack
    return L;
}

// Barrier of epilogue group g (named barriers 4 and 5).
__device__ __forceinline__ void epi_bar(int g) { asm volatile("bar.sync %0, %1;" ::"r"(4 + g), "n"(kEpiThreads) : "memory"); }
// Arrival on a cross-CTA counter (wraps to 0 after `lim`): release for the
// stores that precede it in this CTA (ordered by a barrier), acquire for the
// other CTAs' stores that precede their arrivals.
__device__ __forceinline__ unsigned atom_inc_acq_rel(unsigned *p, unsigned lim) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(lim) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_release(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void route_bar() { asm volatile("bar.sync 3, %0;" ::"n"(kEpiWarp0 * 32) : "memory"); }
__device__ __forceinline__ void build_bar() { asm volatile("bar.sync 2, %0;" ::"n"(kBuildThreads) : "memory"); }

// Bounded mbarrier wait that returns at once once the CTA is dead (a phase that
// has already completed is taken first: the common case costs one poll).
__device__ __forceinline__ bool ring_wait(uint64_t *bar, uint32_t parity, volatile int *dead, int32_t *err,
                                          int code) {
    {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
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
__device__ __forceinline__ void sf_copy(uint32_t tmem_col, uint64_t desc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc) : "memory");
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
    volatile int *misc = reinterpret_cast<volatile int *>(sm + lay.misc);  // [0] dead, [1] last, [2] units, [3] stages, [4] last piece
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
    uint64_t *rdone = bxready + 1;  // the softmax weights and each pair's slot are in shared memory (for the combine)
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
        mbar_init(rdone, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "n"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    const int nkb1 = p.Hp / 128, nkb2 = p.Ip / 128;
    const int nmt1 = 2 * p.I / 128, nmt2 = (p.H + 127) / 128;
    const int nkp = nkb2 >= 2 ? 2 : 1;  // down units: K halves
    const int dmax = down_boxes(p.Ip);
    // unit u's phase (0 gate_up, 1 down), slot, weight tile, piece (a down unit's K
    // half), pieces of its tile, K box range and split index
    auto unit_span = [&](int u, int &phase, int &slot, int &mt, int &kpart, int &np, int &kb0, int &kb1, int &split) {
        const uint32_t w0 = (uint32_t)units_s[2 * u], w1 = (uint32_t)units_s[2 * u + 1];
        phase = (int)(w0 >> 31);
        slot = (int)((w0 >> 20) & 1023u);
        mt = (int)((w0 >> 8) & 4095u);
        kpart = (int)((w0 >> 4) & 15u);
        np = (int)(w0 & 15u);
        kb0 = (int)(w1 >> 24);
        kb1 = (int)((w1 >> 16) & 255u);
        split = (int)(w1 & 0xffffu);
    };

    // ---------------- the ring: this CTA's stages, two boxes each ----------------
    // Stage j (the units' K ranges in order, two boxes a stage) is filled into slot
    // j % R once the MMAs of stage j - R released it.
    auto issue = [&](int j, int u, int kb) {  // boxes kb, kb + 1 (kb alone at the range's end) of unit u
        int phase, slot, mt, kpart, np, kb0, kb1, split;
        unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
        const size_t e = (size_t)act_s[slot];
        const uint32_t nb = (uint32_t)min(2, kb1 - kb);
        const size_t box = phase ? (e * nmt2 + mt) * nkb2 + kb : (e * nmt1 + mt) * nkb1 + kb;
        const int sl = j % R;
        mbar_expect_tx(full + sl, nb * kBoxStep);
        bulk_g2s(ring + (size_t)sl * kStageBytes, (phase ? p.dn_tq : p.gu_tq) + box * kBoxStep, nb * kBoxStep, full + sl);
        rel_s[sl] = j;
    };

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
        if (blockIdx.x == 0) {  // the previous launch is over: clear the next one's counters
            if (tid == 0) p.rcnt[(epoch + 1u) & 1u] = 0u;
            for (int i = tid; i < p.S; i += kDecThreads) p.cnt_gu[((epoch + 1u) & 1u) * p.S + i] = 0u;
            for (int i = tid; i < G; i += kDecThreads) p.cnt_split[((epoch + 1u) & 1u) * G + i] = 0u;
        }
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
        __syncthreads();  // the operand builders read every thread's rows
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
        if (tid == 0 && (int)blockIdx.x < dot_ctas)  // this CTA's logits are stored (release orders them first)
            red_add_release(p.rcnt + (epoch & 1u), 1u);
        if (warp >= kEpiWarp0) {
            // ---------------- gate_up's operand, while warps 0-3 finish the routing ----------------
            // every token's normalized row as five E2M1 terms per 32-element block, row
            // 5 t + j of every K box; rows of absent tokens and K past H read as zero
            // codes at unit scale
            const int bt = tid - kEpiWarp0 * 32;
            for (uint32_t o = 16u * (uint32_t)bt; o < (uint32_t)nkb1 * kBb; o += 16u * kBuildThreads)
                *reinterpret_cast<uint4 *>(bx + o) = o % kBb < kCb ? make_uint4(0u, 0u, 0u, 0u)
                                                                   : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
            build_bar();
            const int nblk = Hp / 32, total = 4 * T * nblk;  // four lanes per (token, 32-element block)
            for (int base = (warp - kEpiWarp0) * 32; base < total; base += kBuildThreads) {  // whole warps
                const int it = base + lane;
                const bool live = it < total;
                const int unit = it >> 2, sub = it & 3;
                const int t = live ? unit / nblk : 0, blk = live ? unit - t * nblk : 0;
                float x[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) x[q] = live ? xn_s[(size_t)t * Hp + 32 * blk + 8 * sub + q] : 0.0f;
                uint32_t codes[kTerms][1], sbyte[kTerms];
                fp4::quantize<8, 4>(x, codes, sbyte);
                if (live) put_terms(bx + (size_t)(blk >> 2) * kBb, kCb, t, blk & 3, sub, codes, sbyte);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // read by the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(bxready);
        } else {
            // (3) one warp per token: its E logits, then the top-k as k rounds of a warp
            //     argmax over 64-bit keys ordered as moe.go:20-27 orders the experts
            //     (value descending, ties to the lower id, NaN after every number).  The
            //     whole warp spins on the counter (one request per poll): it stays
            //     converged, and a warp that slept runs its shuffles slowly afterwards.
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
                if (E <= 32) {
                    // one expert per lane (e = lane): per round one 32-bit max reduction and a
                    // ballot; equal keys go to the lowest lane, i.e. the lower id
                    uint32_t ord = (uint32_t)(key[0] >> 32);
                    for (int s = 0; s < p.k; ++s) {
                        const uint32_t m = __reduce_max_sync(0xffffffffu, ord);
                        const int win = __ffs(__ballot_sync(0xffffffffu, ord == m)) - 1;
                        my_e = lane == s ? win : my_e;
                        ord = lane == win ? 0u : ord;
                    }
                }
                for (int s = 0; s < (E <= 32 ? 0 : p.k); ++s) {
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
            }
            route_bar();
            // (4) one warp: the active experts (their slots in ascending id order), this
            //     CTA's units for that many, and the first copies.  Everything else of
            //     the routing is needed only by the combine and the reported routing.
            if (warp == 0) {
                if (lane < 8) amask_s[lane] = 0u;
                __syncwarp();
                for (int q0 = 0; q0 < P; q0 += 32) {
                    const int q = q0 + lane;
                    if (q < P) atomicOr(&amask_s[tk_s[q] >> 5], 1u << (tk_s[q] & 31));
                }
                __syncwarp();
                const uint32_t word = lane < 8 ? amask_s[lane] : 0u;
                int pre = __popc(word);  // inclusive scan of the words' counts
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    const int x = __shfl_up_sync(0xffffffffu, pre, o);
                    pre += lane >= o ? x : 0;
                }
                const int na = __shfl_sync(0xffffffffu, pre, 7);  // active experts (>= 1)
                int pos = pre - __popc(word);
                for (int bit = 0; bit < 32; ++bit)
                    if ((word >> bit) & 1u) act_s[pos++] = 32 * lane + bit;
                if (lane == 0) act_s[E] = na;
                const int u0 = sched_s[na - 1], u1 = sched_s[na];
                const int n = min((u1 - u0) / 2, kMaxUnits);
                for (int w0 = 0; w0 < 2 * n; w0 += 32)
                    if (w0 + lane < 2 * n) units_s[w0 + lane] = sched_s[u0 + w0 + lane];
                if (lane == 0) misc[2] = n;
                __syncwarp();
                {  // the first copies: stage j < R from lane j
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the staged schedule rows are read
                    int j = 0, mine_u = -1, mine_kb = 0;
                    for (int u = 0; u < n && j < R; ++u) {
                        int phase, slot, mt, kpart, np, kb0, kb1, split;
                        unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
                        const int ns = (kb1 - kb0 + 1) >> 1;  // the unit's stages
                        if (lane >= j && lane < j + ns) {
                            mine_u = u;
                            mine_kb = kb0 + 2 * (lane - j);
                        }
                        j += ns;
                    }
                    if (mine_u >= 0 && lane < R) issue(lane, mine_u, mine_kb);
                    if (lane == 0) misc[3] = min(j, R);  // stages issued
                }
            }
        }
    }
    __syncthreads();
    tc_fence_after();
    const int n_active = act_s[E];
    const int nunits = misc[2];
    const int issued = misc[3];
    const uint32_t tmem = *tslot;

    if (warp == kProdWarp) {
        // ---------------- producer: the rest of the stages, in order ----------------
        if (lane == 0) {
            bool ok = true;
            int j = 0;
            for (int u = 0; u < nunits && ok; ++u) {
                int phase, slot, mt, kpart, np, kb0, kb1, split;
                unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
                for (int kb = kb0; kb < kb1; kb += 2, ++j) {
                    if (j < issued) continue;
                    // the MMAs released stage j - R's slot
                    if (j >= R && !ring_wait(empty + j % R, ((j / R) - 1) & 1, misc, p.err, 51)) {
                        ok = false;
                        break;
                    }
                    issue(j, u, kb);
                }
            }
            // copies in flight (only after a failed wait) land before the CTA exits
            for (int sl = 0; sl < R; ++sl)
                if (rel_s[sl] >= 0) mbar_wait(full + sl, (rel_s[sl] / R) & 1, p.err, 54);
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        // The loop issues few instructions per box: every descriptor is its base plus
        // an offset in the start-address field (bits 0-13, 16-byte units; shared
        // addresses stay below 256 KB, so no carry leaves the field).
        const uint32_t elected = elect_one();
        const uint32_t idesc0 = idesc_dec(0, NCOL), idesc1 = idesc_dec(2, NCOL);
        const uint32_t ring_a = smem_u32(ring), bx_a = smem_u32(bx), bd_a = smem_u32(bd);
        const uint64_t da = desc_sw64(ring_a), fa = desc_sf(ring_a + kBoxBytes);  // stage 0, box 0
        const uint64_t dbx = desc_sw64(bx_a), fbx = desc_sf(bx_a + kCb);         // gate_up's operand
        const uint64_t dbd = desc_sw64(bd_a), fbd = desc_sf(bd_a + kCb);         // down's, buffer 0
        int i = 0, dn = 0, nbox = 0, s = 0;
        uint32_t ph = 0;  // parity of the ring's current pass
        bool ok = true, bx_ready = false;
        for (int u = 0; u < nunits && ok; ++u) {
            int phase, slot, mt, kpart, np, kb0, kb1, split;
            unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
            const int buf = u & 1, ub = dn & 1;
            if (phase == 0 && !bx_ready) {
                if (!ring_wait(bxready, 0, misc, p.err, 50)) break;
                bx_ready = true;
            }
            if (u >= 2 && !ring_wait(accempty + buf, ((u >> 1) - 1) & 1, misc, p.err, 55)) break;
            if (phase == 1 && !ring_wait(bfull + ub, (dn >> 1) & 1, misc, p.err, 56)) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)buf * kAccCols;
            const uint32_t bo0 = phase ? (uint32_t)(ub * dmax) * (kBb >> 4) : 0u;
            const uint64_t db = (phase ? dbd : dbx) + bo0, fb = (phase ? fbd : fbx) + bo0;
            const int kbase = phase ? kb0 : 0;
            for (int kb = kb0; kb < kb1; kb += 2, ++i) {
                const int nb = min(2, kb1 - kb);
                if (!ring_wait(full + s, ph, misc, p.err, 51)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int b = 0; b < nb; ++b, ++nbox) {
                    if (elected) {
                        // tcgen05.cp and tcgen05.mma issued by this thread execute in issue
                        // order, so a scale slot is rewritten only after the MMAs that read it
                        const uint32_t ao = (uint32_t)s * (kStageBytes >> 4) + (uint32_t)b * (kBoxStep >> 4);
                        const uint32_t bo = (uint32_t)(kb + b - kbase) * (kBb >> 4);
                        const uint32_t sf = tmem + kSfCol + 16u * (uint32_t)(nbox & 1);
                        sf_copy(sf, fa + ao);      // the weights' E8M0 chunk
                        sf_copy(sf + 4, fb + bo);  // the tokens' term scales
                        umma(d, da + ao, db + bo, idesc0, (kb + b > kb0) ? 1u : 0u, sf, sf + 4);
                        umma(d, da + ao + 2, db + bo + 2, idesc1, 1u, sf, sf + 4);
                    }
                }
                if (elected) mma_commit(empty + s);
                __syncwarp();
                if (++s == R) {
                    s = 0;
                    ph ^= 1u;
                }
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
    } else if (warp == kRestWarp) {
        // ---------------- the rest of the routing, off the critical path ----------------
        // the softmax over each token's selected logits (moe.go:29-39): the k
        // exponentials in parallel, the denominator summed in slot order
        const float *lg_s = reinterpret_cast<const float *>(sm + lay.lg);
        const int *tk_s = reinterpret_cast<const int *>(sm + lay.tk);
        const uint32_t *amask_s = reinterpret_cast<const uint32_t *>(sm + lay.amask);
        for (int t = 0; t < p.T; ++t) {
            const int my_e = tk_s[t * p.k + (lane < p.k ? lane : 0)];
            const double maxv = (double)lg_s[t * E + tk_s[t * p.k]];
            const double ex_all = exp((double)lg_s[t * E + my_e] - maxv);
            const double ex = lane < p.k ? ex_all : 0.0;
            double den = 0.0;
            for (int sl = 0; sl < p.k; ++sl) den += __shfl_sync(0xffffffffu, ex, sl);
            if (lane < p.k) w_s[t * p.k + lane] = (float)((double)(float)ex / den);
        }
        // counts, offsets, the stable permutation and each pair's active slot
        for (int e0 = 0; e0 <= E; e0 += 32)
            if (e0 + lane <= E) offs_s[e0 + lane] = 0;
        __syncwarp();
        for (int q0 = 0; q0 < P; q0 += 32) {
            const int q = q0 + lane;
            if (q < P) atomicAdd(&offs_s[tk_s[q]], 1);
        }
        __syncwarp();
        int c[8];  // warp scan over experts (lane owns experts 8 lane .. 8 lane + 7; E <= 256)
        int cs = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = 8 * lane + j;
            c[j] = e < E ? offs_s[e] : 0;
            cs += c[j];
        }
        int cx = cs;  // inclusive warp prefix sum
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int cu = __shfl_up_sync(0xffffffffu, cx, o);
            cx += lane >= o ? cu : 0;
        }
        int co = cx - cs;
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = 8 * lane + j;
            if (e < E) offs_s[e] = co;
            co += c[j];
        }
        if (lane == 31) offs_s[E] = cx;
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
        __syncwarp();
        if (blockIdx.x == 0) {  // the routing the C ABI reports
            for (int q = lane; q < P; q += 32) {
                p.route.topk_idx[q] = tk_s[q];
                p.route.topk_w[q] = w_s[q];
                p.route.perm_pair[q] = perm_s[q];
                p.route.inv[q] = inv_s[q];
            }
            for (int e = lane; e <= E; e += 32) {
                p.route.offsets[e] = offs_s[e];
                p.route.active[e] = act_s[e];
                if (e < E) p.route.counts[e] = offs_s[e + 1] - offs_s[e];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(rdone);
    } else if (warp == kLoadWarp) {
        // ---------------- down operands: one bulk copy per unit once the slot is published ----------------
        if (lane == 0) {
            int dn = 0, last[2] = {-1, -1};
            bool bx_ready = false;
            for (int u = 0; u < nunits && !misc[0]; ++u) {
                int phase, slot, mt, kpart, np, kb0, kb1, split;
                unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
                if (phase == 0) continue;
                // bd holds the normalized tokens until gate_up's operand is built from them
                if (!bx_ready && !ring_wait(bxready, 0, misc, p.err, 50)) break;
                bx_ready = true;
                const int ub = dn & 1;
                if (dn >= 2 && !ring_wait(bempty + ub, ((dn >> 1) - 1) & 1, misc, p.err, 57)) break;
                const long long t0 = clock64();
                // the slot's gate_up tiles all finished (spins: a sleep slows the warp after)
                while (ld_acquire(p.cnt_gu + (epoch & 1u) * p.S + slot) < (unsigned)nmt1 && !misc[0]) {
                    if (clock64() - t0 > kWaitLimit) {
                        atomicCAS(p.err, 0, 52);
                        misc[0] = 1;
                    }
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
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4 * kEpiGroups) {
        // ---------------- unit epilogues (one thread per tile row; the same barriers on every path) ----------------
        // group grp takes the units of accumulator grp (u = grp, grp + 2, ...), so two
        // epilogues, each a chain of global round trips, run at once
        const int grp = (warp - kEpiWarp0) >> 2;
        const int quad = warp & 3, row = quad * 32 + lane, et = tid - (kEpiWarp0 + 4 * grp) * 32;
        volatile int *gmisc = misc + 8 + grp;  // the group's unit was the last down unit of its output tile
        float *actg = actst + grp * p.T * 64;
        // gate_up: rows 16 g + j (j < 8) hold the gate of pair 8 g + j, row + 8 its up row
        const int j16 = row & 15;
        const bool gate_lane = j16 < 8;
        const int pl = 8 * (row >> 4) + (j16 & 7);  // pair within the tile (0..63)
        bool rdone_seen = false;
        // this thread's bias of unit u: loaded a unit ahead, so its latency hides behind a whole unit
        auto unit_bias = [&](int u) {
            if (u >= nunits) return 0.0f;
            int phase, slot, mt, kpart, np, kb0, kb1, split;
            unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
            const size_t e = (size_t)act_s[slot];
            const int h = 128 * mt + row;
            if (phase == 0) return __ldg(p.gu_b + e * 2 * p.I + 2 * (64 * mt + pl) + (gate_lane ? 0 : 1));
            return kpart == 0 && h < p.H ? __ldg(p.dn_b + e * p.H + h) : 0.0f;
        };
        float bias_next = unit_bias(grp);
        for (int u = grp; u < nunits; u += kEpiGroups) {
            int phase, slot, mt, kpart, np, kb0, kb1, split;
            unit_span(u, phase, slot, mt, kpart, np, kb0, kb1, split);
            const int buf = u & 1, h = 128 * mt + row;
            const float bias = bias_next;
            bias_next = unit_bias(u + kEpiGroups);
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
            bool finish = true;  // this unit completes its tile (uniform over the epilogue threads)
            if (phase == 0 && np > 1) {
                // a tile cut between CTAs: pieces 1.. store their partial sums and count
                // themselves in without waiting; piece 0, the end of an earlier CTA's range
                // and so the last to run, waits for them and adds all in piece order
                float *gp = p.gpart + (size_t)split * kMaxPieces * kDecodeMaxTokens * 128 + row;
                unsigned *cs = p.cnt_split + (epoch & 1u) * G + split;
                finish = kpart == 0;
                if (!finish) {
#pragma unroll
                    for (int t = 0; t < kDecodeMaxTokens; ++t)
                        if (t < p.T) gp[(kpart * kDecodeMaxTokens + t) * 128] = v[t];
                    epi_bar(grp);  // every thread's partials before the release below
                    if (et == 0) red_add_release(cs, 1u);
                } else {
                    if (et == 0) {
                        const long long t0 = clock64();
                        while (ld_acquire(cs) < (unsigned)np - 1u && !misc[0])
                            if (clock64() - t0 > kWaitLimit) {
                                atomicCAS(p.err, 0, 57);
                                misc[0] = 1;
                            }
                    }
                    epi_bar(grp);  // the acquire above orders the other pieces' partials before the reads
#pragma unroll
                    for (int t = 0; t < kDecodeMaxTokens; ++t) {
                        if (t < p.T) {
                            float sum = v[t];
                            for (int pc = 1; pc < np; ++pc) sum += __ldcg(gp + (pc * kDecodeMaxTokens + t) * 128);
                            v[t] = sum;
                        }
                    }
                }
            }
            if (phase == 0 && finish) {
                // SwiGLU of the tile's 64 pairs (partner lanes 8 apart swap values)
#pragma unroll
                for (int t = 0; t < kDecodeMaxTokens; ++t) {
                    if (t < p.T) {  // uniform
                        const float val = v[t] + bias;
                        const float other = __shfl_xor_sync(0xffffffffu, val, 8);
                        if (gate_lane) actg[t * 64 + pl] = swiglu(val, other);
                    }
                }
                epi_bar(grp);
                if (quad < p.T) {  // warp t: token t (uniform per warp)
                    // sixteen lanes per (token, 32-pair block), two pairs each (the terms are a
                    // dependent chain: fewer elements a lane shorten it): the five E2M1 terms
                    // and their scales into down's operand, blocks 2 (mt % 2) + b of box mt / 2
                    const int t = quad, b = lane >> 4, sub = lane & 15, jb = 2 * (mt & 1) + b;
                    float x[2] = {actg[t * 64 + 32 * b + 2 * sub], actg[t * 64 + 32 * b + 2 * sub + 1]};
                    uint32_t codes[kTerms][1], sbyte[kTerms];
                    fp4::quantize<2, 16>(x, codes, sbyte);
                    uint8_t *box = p.aq + ((size_t)slot * nkb2 + (mt >> 1)) * kBb;
#pragma unroll
                    for (int j = 0; j < kTerms; ++j) {
                        const int n = kTerms * t + j;
                        box[n * 64 + ((jb ^ ((n >> 1) & 3)) << 4) + sub] = (uint8_t)codes[j][0];
                        if (sub == j) box[kCb + n * 16 + jb] = (uint8_t)sbyte[j];
                    }
                }
                if (quad == 0 && mt == nmt1 - 1 && (mt & 1) == 0) {
                    // K past I (blocks 2 and 3 of the last box): zero codes at unit scale
                    uint8_t *box = p.aq + ((size_t)slot * nkb2 + (mt >> 1)) * kBb;
                    for (int q = lane; q < 2 * NCOL; q += 32) {
                        const int n = q >> 1, jz = 2 + (q & 1);
                        *reinterpret_cast<uint4 *>(box + n * 64 + ((jz ^ ((n >> 1) & 3)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                        box[kCb + n * 16 + jz] = 127;
                    }
                }
                if (quad < p.T || quad == 0)
                    asm volatile("fence.proxy.async.global;" ::: "memory");  // read by other CTAs' bulk copies
            } else if (phase == 1) {
                if (h < p.H) {
                    float *yrow = p.yb + ((size_t)slot * 2 + kpart) * p.T * p.H + h;
#pragma unroll
                    for (int t = 0; t < kDecodeMaxTokens; ++t)
                        if (t < p.T) yrow[(size_t)t * p.H] = v[t] + bias;
                }
            }
            epi_bar(grp);
            // the barrier above orders every epilogue thread's stores before this thread's
            // release; a down unit's acquire orders the other CTAs' outputs before the combine
            if (et == 0 && finish && phase == 0) red_add_release(p.cnt_gu + (epoch & 1u) * p.S + slot, 1u);
            if (et == 0 && phase == 1) {
                const unsigned n = (unsigned)(nkp * n_active);
                gmisc[0] = atom_inc_acq_rel(p.cnt_dn + mt, n - 1u) == n - 1u;
            }
            epi_bar(grp);
            if (phase == 1 && gmisc[0] && (rdone_seen || ring_wait(rdone, 0, misc, p.err, 50))) {
                // the last down unit of output tile mt: combine its rows for every token in
                // slot order (layer.go:109-121)
                rdone_seen = true;
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

// The units of every CTA for each number of active slots n = 1..S.  Down units
// (one per output tile and K half) go first to the least-loaded CTAs; then the
// gate_up boxes, in (slot, tile, K box) order, are cut into contiguous ranges so
// that every CTA's total box count comes out even: CTA b takes the next
// (target - its down boxes) boxes.  A tile whose range spans CTAs becomes pieces
// (at most kMaxPieces) joined through a split index.  Within a CTA the gate_up
// pieces run first.  CTA b's rows sit in words [b * kSchedWords, (b + 1) *
// kSchedWords): S + 1 offsets (relative to the row start), then the unit lists for
// n = 1..S, two words per unit.  Should a tile need more pieces than allowed, the
// gate_up tiles of that n are placed whole, longest processing time first.
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
    std::vector<std::vector<int32_t>> gu(G), dn(G);
    std::vector<long long> load(G), quota(G);
    for (int b = 0; b < G; ++b) rows[b][0] = S + 1;
    auto least = [&]() {
        int best = 0;
        for (int b = 1; b < G; ++b)
            if (load[b] < load[best]) best = b;
        return best;
    };
    auto push = [](std::vector<int32_t> &l, int32_t w0, int32_t w1) {
        l.push_back(w0);
        l.push_back(w1);
    };
    for (int n = 1; n <= S; ++n) {
        for (int b = 0; b < G; ++b) {
            gu[b].clear();
            dn[b].clear();
            load[b] = 0;
        }
        for (int sl = 0; sl < n; ++sl)
            for (int m = 0; m < nmt2; ++m)
                for (int kp = 0; kp < nkp; ++kp) {
                    const int kb0 = kp ? half2 : 0, kb1 = nkp == 1 || kp ? nkb2 : half2;
                    const int b = least();
                    push(dn[b], unit_w0(1, sl, m, kp, nkp), unit_w1(kb0, kb1, 0));
                    load[b] += kb1 - kb0;
                }
        // water level L: the smallest with sum max(0, L - load) >= the gate_up boxes;
        // the surplus comes off the first CTAs that have a share
        const long long gu_total = (long long)n * nmt1 * nkb1;
        auto fill = [&](long long L) {
            long long f = 0;
            for (int c = 0; c < G; ++c) f += std::max(0LL, L - load[c]);
            return f;
        };
        long long lo = 0, hi = gu_total + *std::max_element(load.begin(), load.end());
        while (lo < hi) {
            const long long mid = (lo + hi) / 2;
            if (fill(mid) >= gu_total) hi = mid;
            else lo = mid + 1;
        }
        long long surplus = fill(lo) - gu_total;
        for (int c = 0; c < G; ++c) {
            quota[c] = std::max(0LL, lo - load[c]);
            if (surplus > 0 && quota[c] > 0) {
                --quota[c];
                --surplus;
            }
        }
        int b = 0, nsplit = 0;
        long long rem = quota[0];
        bool ok = true;
        for (int sl = 0; sl < n && ok; ++sl)
            for (int m = 0; m < nmt1 && ok; ++m) {
                int cta[kMaxPieces + 1], k0[kMaxPieces + 1], k1[kMaxPieces + 1], np = 0;
                for (int kb = 0; kb < nkb1;) {
                    while (rem == 0 && b < G - 1) rem = quota[++b];
                    const int take = rem == 0 ? nkb1 - kb : (int)std::min<long long>(rem, nkb1 - kb);  // the last CTA takes any rest
                    if (np == kMaxPieces) {
                        ok = false;
                        break;
                    }
                    cta[np] = b;
                    k0[np] = kb;
                    k1[np] = kb + take;
                    ++np;
                    kb += take;
                    rem -= std::min<long long>(rem, take);
                }
                if (!ok) break;
                const int split = np > 1 ? nsplit++ : 0;
                for (int pc = 0; pc < np; ++pc) push(gu[cta[pc]], unit_w0(0, sl, m, pc, np), unit_w1(k0[pc], k1[pc], split));
            }
        if (!ok || nsplit >= G) {
            for (int c = 0; c < G; ++c) gu[c].clear();
            for (int sl = 0; sl < n; ++sl)
                for (int m = 0; m < nmt1; ++m) {
                    const int c = least();
                    push(gu[c], unit_w0(0, sl, m, 0, 1), unit_w1(0, nkb1, 0));
                    load[c] += nkb1;
                }
        }
        for (int c = 0; c < G; ++c) {
            rows[c].insert(rows[c].end(), gu[c].begin(), gu[c].end());
            rows[c].insert(rows[c].end(), dn[c].begin(), dn[c].end());
            rows[c][n] = (int32_t)rows[c].size();
            s.max_units = std::max(s.max_units, (int)(gu[c].size() + dn[c].size()) / 2);
        }
    }
    s.rows.assign((size_t)G * kSchedWords, 0);
    for (int c = 0; c < G; ++c) {
        s.max_words = std::max(s.max_words, (int)rows[c].size());
        std::copy_n(rows[c].begin(), std::min<size_t>(rows[c].size(), kSchedWords), s.rows.begin() + (size_t)c * kSchedWords);
    }
    return s;
}

struct DecScratch {
    size_t aq, yb, cnt_gu, cnt_dn, rcnt, gpart, cnt_split, sched, total;
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
    o += align256((size_t)2 * S * 4);
    L.cnt_dn = o;
    o += align256((size_t)nmt2 * 4);
    L.rcnt = o;
    o += align256(2 * 4);
    L.gpart = o;
    o += align256((size_t)G * kMaxPieces * kDecodeMaxTokens * 128 * 4);
    L.cnt_split = o;
    o += align256((size_t)2 * G * 4);
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
    p.gpart = reinterpret_cast<float *>(b + lay.gpart);
    p.cnt_split = reinterpret_cast<uint32_t *>(b + lay.cnt_split);
    p.cnt_dn = reinterpret_cast<uint32_t *>(b + lay.cnt_dn);
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
    const int var = ncol == 8 ? 0 : (ncol == 16 ? 1 : 2);
    auto kern = var == 0 ? decode_kernel<8> : (var == 1 ? decode_kernel<16> : decode_kernel<32>);
    // the shared-memory ceiling once per device and variant (a driver call on every
    // step would sit between the step's start and its launch)
    static thread_local bool attr_set[64][3] = {};
    if (!attr_set[device][var]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
        if (e != cudaSuccess) return e;
        attr_set[device][var] = true;
    }
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
