// gemm_bs.cu -- K4/K5: the grouped expert GEMMs of prefill on the block-scaled
// FP4 rate of the 5th-generation tensor cores (tcgen05.mma kind::mxf4).
//
// Per expert e with m_e routed rows (positions offsets[e]..offsets[e+1] of the
// expert-sorted pairs):
//   gate_up: act = SwiGLU(W_gu . x + b_gu)   (layer.go:139-148, 175; primitives.go:138-149)
//   down:    y   = W_dn . act + b_dn          (layer.go:179-187)
//
// A = the MXFP4 weights exactly as stored: the box-tiled E2M1 planes (64-byte
//     rows of 128 packed elements, kept in global memory in the 64-byte swizzle
//     order the tensor core reads) with the GGUF E8M0 bytes as the hardware block
//     scales.
// B = the activations as five E2M1 terms per element with their own E8M0 scale
//     per 32 elements and term (fp4_terms.cuh), one term per MMA column: a tile
//     of 48 tokens is N = 240 columns, and the epilogue adds each token's five
//     columns.  The tensor core multiplies E2M1 x E2M1 exactly and accumulates in
//     f32.
//
// Tokens are tiled per expert (48 per tile, the last tile of an expert ragged).
// The B operand of every (tile, 128-element K box) sits in global memory as 240
// rows of 64 bytes (row 5i + j: token i, term j), also in the swizzle order:
// each CTA's 120 rows followed by the 1 KB of scale chunks of all 240 rows.  gate_up's epilogue writes down's B
// operand in the same form: SwiGLU, then the five terms of every (token, 32-pair
// block).  gate_up's own B operand comes from token-major records: each token is
// quantized once (tok_quant_kernel; with expert parallelism the source rank does it
// and sends the records) and every tile gathers its tokens' rows (bs_gather_kernel).
//
// Every operand therefore reaches shared memory as one plain copy (TMA without
// swizzle) of data and scales stored side by side: a stage is two copies of
// 17 KB per CTA: two adjacent A boxes, and this CTA's parts of the same two B
// boxes.  Each TMA copy costs the SM's copy engine about 50-60 cycles of fixed
// work besides its bytes, and a copy's latency is long, so the pipeline moves few,
// large copies: rows and scales in separate small copies fed the FP4 MMAs at half
// their rate.
//
// The MMAs are 2-SM (tcgen05 cta_group::2): a cluster of two CTAs computes a
// 256-row weight tile x 48 tokens.  Each CTA loads its own 128-row A box, its
// half of the B rows (120) and the full B scales; every load signals the leader
// CTA's barrier, the leader issues the MMAs (M = 256, N = 240, K = 64, two per
// box) and commits to both CTAs' barriers, and each CTA's epilogue reads the
// accumulator rows in its own TMEM.
//
// Work item = (token tile, 256-row weight pair), clusters striding over items.
// Roles per CTA (16 warps): warp 0 TMA producer, warp 1 MMA issuer (leader) and TMEM
// owner.  down: warps 2-13, three groups of four (one warp per TMEM lane quadrant),
// each group reading a third of the tile's tokens from TMEM and storing the outputs.
// gate_up runs a pipeline instead: warps 12-15 (one per quadrant) read the
// accumulator 8 tokens at a time, apply bias and SwiGLU, and fill a ring of three
// 16-token slots (chunks) in shared memory; two groups of four quantizer warps
// (warps 2-5 and 6-9) take alternate chunks and write down's B operand.  The
// quantization of one item thus overlaps the SwiGLU of the next, and both overlap
// the MMAs.  TMEM: two
// 240-column accumulators (the epilogue of one item overlaps the next item's MMAs)
// and two 12-column scale-factor slots used alternately.  Every wait is bounded; on
// timeout the kernel records a code in the error flag and winds down.
#include "fp4_terms.cuh"
#include "tc_ptx.cuh"

namespace amoe {

namespace {

using namespace bs;

constexpr int kTerms = fp4::kTerms;               // E2M1 terms per activation value
constexpr int kTok = 48;                          // tokens per tile
constexpr int kN = kTerms * kTok;                 // MMA N: 240
constexpr int kHalfRows = kN / 2;                 // B rows per CTA of a pair
constexpr uint32_t kRow = 64;                     // one 128-element K box of a row, packed E2M1
constexpr uint32_t kABytes = 128 * kRow;          // A box rows
constexpr uint32_t kBHalf = kHalfRows * kRow;     // this CTA's B rows of a box
constexpr uint32_t kBSf = 1024;                   // B scale chunks of one (tile, box): rows 0-127, 128-239
constexpr uint32_t kBPart = kBHalf + kBSf;        // what one CTA copies of a B blob: its rows, then all scales
// Stage: two K boxes.  The A boxes as stored (rows, then the scale chunk, each),
// then this CTA's B parts of the same two boxes.
constexpr int kBoxes = 2;
constexpr uint32_t kStageA = kBoxes * (uint32_t)kBoxStride;   // 17 KB
constexpr uint32_t kStageBytes = kStageA + kBoxes * kBPart;   // 34 KB
constexpr int kStages = 6;
constexpr uint32_t kCopyRow = 512;                // TMA row width: both copies of a stage are whole rows
constexpr int kProdWarp = 0, kMmaWarp = 1, kEpiWarp0 = 2;
constexpr int kEpiGroups = 3;                     // down: warps 2-13, groups of one warp per TMEM lane quadrant
constexpr int kEpiWarps = 4 * kEpiGroups;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kSwiWarp0 = 12;                     // gate_up: warps 12-15 read the accumulators
constexpr int kSwiThreads = 4 * 32;
constexpr int kQuantGroups = 2;                   // gate_up: warps 2-5 and 6-9 quantize alternate chunks
constexpr int kThreads = 16 * 32;
constexpr int kGroupTok = kTok / kEpiGroups;      // tokens per group (down) and per chunk (gate_up): 16
constexpr int kSlots = kTok / kGroupTok;          // gate_up staging ring: one slot per chunk of an item
constexpr uint32_t kSfCol = 2 * kN;               // TMEM column of scale-factor slot 0 (slot 1: +16)
constexpr int kActPitch = 68;                     // a slot: [16 tokens][64 pairs] f32, padded rows
constexpr int kSlotFloats = kGroupTok * kActPitch;
constexpr uint32_t kOutStage = kSlots * kSlotFloats * 4;
constexpr size_t kSmem = 1024 + kStages * kStageBytes + kOutStage + 32 * 8 + 16;

static_assert(kN % 16 == 0 && kN <= 256, "MMA N for M = 256");
static_assert(kStageA % 1024 == 0 && kStageBytes % 1024 == 0 && kBoxStride % 512 == 0 && kBPart % 512 == 0,
              "64-byte swizzle atoms start on 512 B");
static_assert(kSfCol + 16 + 12 <= 512, "TMEM budget");
static_assert(kSmem <= 232448, "shared memory budget");
static_assert(kGroupTok == 16, "a down warp reads its tokens from TMEM as two halves of 8 (tmem_ld40)");
static_assert(kThreads == (kEpiWarp0 + kEpiWarps + 2) * 32 && kSwiWarp0 % 4 == 0 &&
              kEpiWarp0 + 4 * kQuantGroups <= kSwiWarp0, "warp roles");
static_assert(4 * 32 == 4 * 2 * kGroupTok, "a quantizer group: four lanes per (token, 32-pair block) of a chunk");
static_assert(kActPitch % 32 == 4, "tokens 4 apart (one SwiGLU store) fall 16 banks apart");
static_assert(kBoxStride % kCopyRow == 0 && kBPart % kCopyRow == 0 && kHalfRows % 8 == 0, "copies of whole rows");
constexpr uint32_t kARows = (uint32_t)kBoxStride / kCopyRow, kBRows = kBPart / kCopyRow;

struct BsParams {
    const int4 *tiles;     // [tiles] {expert, first position, tokens, 0}
    const int32_t *ntiles;
    const float *bias;     // [E][R], GGUF row order
    int R, nmt, nkb;
    int gate_up;
    // gate_up: down's B operand
    uint8_t *oq;
    int onkb;
    // down
    float *y;
    const int32_t *y_rows;
    EpReturn ret;
    int32_t *err;
    const int32_t *gate;   // if set: nothing to do unless *gate == gate_want (path chosen on the device)
    int gate_want;
};

// Scale byte of B row n, 32-element block jb of a box, inside its 1 KB of chunks
// (chunk n / 128 in the layout tcgen05.cp.32x128b.warpx4 spreads over TMEM).
__device__ __forceinline__ uint32_t sf_at(int n, int jb) {
    return (uint32_t)(n >> 7) * 512u + (uint32_t)(n & 31) * 16u + (uint32_t)((n & 127) >> 5) * 4u + (uint32_t)jb;
}

// B operand in global memory: part (t, kb, h) -- CTA h's 120 rows of tile t's K
// box kb, then the scale chunks of all 240 rows -- is kBPart bytes at index
// ((t * nkb2 + kb / 2) * 2 + h) * 2 + kb % 2 (nkb2: boxes rounded up to pairs), so
// that a CTA's parts of a stage's two boxes are adjacent: one copy.
__device__ __forceinline__ size_t bpart_index(int t, int kb, int h, int nkb2) {
    return (((size_t)t * nkb2 + (kb >> 1)) * 2 + h) * kBoxes + (kb & 1);
}
__device__ __forceinline__ uint8_t *bpart(uint8_t *b, int t, int kb, int h, int nkb2) {
    return b + bpart_index(t, kb, h, nkb2) * kBPart;
}
// Byte offset of 16-byte chunk c of B row r (0..119) inside its part: the rows are
// stored in the 64-byte swizzle order (chunk c at c ^ ((r / 2) % 4)).
__device__ __forceinline__ uint32_t brow_at(int r, int c) {
    return (uint32_t)r * kRow + (uint32_t)((c ^ ((r >> 1) & 3)) << 4);
}
// Stores the codes of row n (token n / 5, term n % 5), 32-element block jb, bytes
// [NB sub, NB (sub + 1)) of the block's 16.
template <int NB>
__device__ __forceinline__ void put_codes(uint8_t *b, int t, int kb, int nkb2, int n, int jb, int sub,
                                          const uint32_t (&w)[NB / 4]) {
    const int h = n >= kHalfRows, r = n - kHalfRows * h;
    uint8_t *dst = bpart(b, t, kb, h, nkb2) + brow_at(r, jb) + sub * NB;
    if (NB == 16) *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    else if (NB == 8) *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint32_t *>(dst) = w[0];
}
// The scale byte of row n, block jb, into both CTA parts of the blob.
__device__ __forceinline__ void put_scale(uint8_t *b, int t, int kb, int nkb2, int n, int jb, uint32_t sbyte) {
    bpart(b, t, kb, 0, nkb2)[kBHalf + sf_at(n, jb)] = (uint8_t)sbyte;
    bpart(b, t, kb, 1, nkb2)[kBHalf + sf_at(n, jb)] = (uint8_t)sbyte;
}

// Token tiles of every expert: tile t = {e, first position, tokens}.
__global__ void __launch_bounds__(256) bs_plan_kernel(const int32_t *__restrict__ offsets, int E, int4 *tiles,
                                                      int32_t *ntiles, int max_tiles, int32_t *err) {
    __shared__ int start[257];
    const int e = threadIdx.x;
    const int cnt = e < E ? offsets[e + 1] - offsets[e] : 0;
    const int n = (cnt + kTok - 1) / kTok;
    if (e < 256) start[e + 1] = n;
    __syncthreads();
    if (e == 0) {
        start[0] = 0;
        for (int i = 0; i < 256; ++i) start[i + 1] += start[i];
        *ntiles = min(start[256], max_tiles);
        if (start[256] > max_tiles) atomicCAS(err, 0, 46);
    }
    __syncthreads();
    for (int j = 0; j < n; ++j) {
        const int t = start[e] + j;
        if (t < max_tiles) tiles[t] = make_int4(e, offsets[e] + kTok * j, min(kTok, cnt - kTok * j), 0);
    }
}

// The gate_up B operand: one CTA per (tile, K box), one thread per (token, 32-element
// block).  Rows are the fp16 hi + lo split of the normalized tokens, gathered
// through the permutation (or, with perm NULL, already by position).  Tokens past
// the tile's count and elements past K are zeros.
// Token-major quantized rows (single-GPU prefill, where each token feeds k pairs):
// record (token, K box kb, 32-element block jb) = the five 16-byte code words of
// the block (80 B at tq + 80 r) and its five E8M0 bytes (at ts + 8 r, 3 bytes
// unused), r = (token * nkb + kb) * 4 + jb.  One thread per record; elements past
// K quantize as zeros, exactly as bs_quant_kernel treats them.
__global__ void __launch_bounds__(256) tok_quant_kernel(const __half *__restrict__ x_hi,
                                                        const __half *__restrict__ x_lo, int tokens, int K,
                                                        int nkb, uint4 *tq, uint2 *ts, const int32_t *gate) {
    if (gate && *gate != 1) return;  // the other expert path runs this step
    const size_t r = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= (size_t)tokens * nkb * 4) return;
    const int jb = (int)(r & 3);
    const size_t tk = r >> 2;
    const int tok = (int)(tk / nkb), kb = (int)(tk - (size_t)tok * nkb);
    const int k0 = kb * 128 + jb * 32;
    float x[32];
    if (k0 < K) {
        const uint4 *h = reinterpret_cast<const uint4 *>(x_hi + (size_t)tok * K + k0);
        const uint4 *l = reinterpret_cast<const uint4 *>(x_lo + (size_t)tok * K + k0);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 hv = __ldg(h + c), lv = __ldg(l + c);
            const __half2 *hh = reinterpret_cast<const __half2 *>(&hv);
            const __half2 *ll = reinterpret_cast<const __half2 *>(&lv);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 a = __half22float2(hh[q]), b = __half22float2(ll[q]);
                x[8 * c + 2 * q] = a.x + b.x;
                x[8 * c + 2 * q + 1] = a.y + b.y;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = 0.0f;
    }
    uint32_t codes[kTerms][4], sbyte[kTerms];
    fp4::quantize<32, 1>(x, codes, sbyte);
#pragma unroll
    for (int term = 0; term < kTerms; ++term)
        tq[r * kTerms + term] = make_uint4(codes[term][0], codes[term][1], codes[term][2], codes[term][3]);
    static_assert(kTerms == 5, "five scale bytes in one 8-byte word");
    ts[r] = make_uint2(sbyte[0] | sbyte[1] << 8 | sbyte[2] << 16 | sbyte[3] << 24, sbyte[4]);
}

// The gate_up B operand from the token-major records: one CTA per (tile, K box),
// one thread per (token, 32-element block), the token found through the
// permutation (perm NULL: record row = the pair's position, as expert parallelism
// receives them).  Tokens past the tile's count get zero codes with a unit scale,
// as quantized zeros do.  The code words go straight to their rows; the scale
// bytes are gathered into the box's 1 KB chunk in shared memory, which then goes
// out to both CTA parts as 16-byte stores (rows 240-255 of the chunk, which no MMA
// reads, are zero).
__global__ void __launch_bounds__(kTok * 4) bs_gather_kernel(const uint4 *__restrict__ tq,
                                                             const uint2 *__restrict__ ts,
                                                             const int32_t *__restrict__ perm, int k, int nkb,
                                                             const int4 *__restrict__ tiles, const int32_t *ntiles,
                                                             uint8_t *bq) {
    __shared__ __align__(16) uint8_t sf_s[kBSf];
    const int t = blockIdx.x / nkb, kb = blockIdx.x - t * nkb;
    if (t >= *ntiles) return;  // uniform over the CTA
    for (int i = threadIdx.x; i < (int)(kBSf / 16); i += blockDim.x)
        reinterpret_cast<uint4 *>(sf_s)[i] = make_uint4(0u, 0u, 0u, 0u);
    const int4 ti = tiles[t];
    const int i = threadIdx.x >> 2, jb = threadIdx.x & 3;
    uint4 w[kTerms];
    uint2 sc = make_uint2(0x7f7f7f7fu, 0x7fu);
    if (i < ti.z) {
        const size_t r = ((size_t)(perm ? perm[ti.y + i] / k : ti.y + i) * nkb + kb) * 4 + jb;
#pragma unroll
        for (int term = 0; term < kTerms; ++term) w[term] = __ldg(tq + r * kTerms + term);
        sc = __ldg(ts + r);
    } else {
#pragma unroll
        for (int term = 0; term < kTerms; ++term) w[term] = make_uint4(0u, 0u, 0u, 0u);
    }
    const int nkb2 = (nkb + 1) >> 1;
    __syncthreads();  // the chunk is zeroed
#pragma unroll
    for (int term = 0; term < kTerms; ++term) {
        const uint32_t words[4] = {w[term].x, w[term].y, w[term].z, w[term].w};
        put_codes<16>(bq, t, kb, nkb2, kTerms * i + term, jb, 0, words);
        sf_s[sf_at(kTerms * i + term, jb)] = (uint8_t)(term < 4 ? (sc.x >> (8 * term)) & 0xffu : sc.y & 0xffu);
    }
    __syncthreads();
    constexpr int kChunk16 = (int)(kBSf / 16);
    for (int q = threadIdx.x; q < 2 * kChunk16; q += blockDim.x) {
        const int h = q / kChunk16, c = q - h * kChunk16;
        reinterpret_cast<uint4 *>(bpart(bq, t, kb, h, nkb2) + kBHalf)[c] = reinterpret_cast<const uint4 *>(sf_s)[c];
    }
}

__global__ void __launch_bounds__(kTok * 4) bs_quant_kernel(const __half *__restrict__ x_hi,
                                                            const __half *__restrict__ x_lo,
                                                            const int32_t *__restrict__ perm, int k, int K, int nkb,
                                                            const int4 *__restrict__ tiles, const int32_t *ntiles,
                                                            uint8_t *bq) {
    const int t = blockIdx.x / nkb, kb = blockIdx.x - t * nkb;
    if (t >= *ntiles) return;  // uniform over the CTA
    const int4 ti = tiles[t];
    const int i = threadIdx.x >> 2, jb = threadIdx.x & 3;
    const int k0 = kb * 128 + jb * 32;
    float x[32];
    const bool live = i < ti.z && k0 < K;
    if (live) {
        const int pos = ti.y + i;
        const size_t row = perm ? (size_t)(perm[pos] / k) : (size_t)pos;
        const uint4 *h = reinterpret_cast<const uint4 *>(x_hi + row * K + k0);
        const uint4 *l = reinterpret_cast<const uint4 *>(x_lo + row * K + k0);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 hv = __ldg(h + c), lv = __ldg(l + c);
            const __half2 *hh = reinterpret_cast<const __half2 *>(&hv);
            const __half2 *ll = reinterpret_cast<const __half2 *>(&lv);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 a = __half22float2(hh[q]), b = __half22float2(ll[q]);
                x[8 * c + 2 * q] = a.x + b.x;
                x[8 * c + 2 * q + 1] = a.y + b.y;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = 0.0f;
    }
    uint32_t codes[kTerms][4], sbyte[kTerms];
    fp4::quantize<32, 1>(x, codes, sbyte);
    const int nkb2 = (nkb + 1) >> 1;
#pragma unroll
    for (int term = 0; term < kTerms; ++term) {
        put_codes<16>(bq, t, kb, nkb2, kTerms * i + term, jb, 0, codes[term]);
        put_scale(bq, t, kb, nkb2, kTerms * i + term, jb, sbyte[term]);
    }
}


// GPT-OSS clamped SwiGLU (primitives.go:144-146; NaN propagates) with the fast
// exponential and division: the result is carried by five E2M1 terms right
// after (about 2^-12 of its block maximum), far coarser than their error.
__device__ __forceinline__ float swiglu_fast(float gate, float up) {
    const float g = isnan(gate) ? gate : fminf(gate, 7.0f);
    const float u = isnan(up) ? up : fminf(fmaxf(up, -7.0f), 7.0f);
    return __fdividef(g, 1.0f + __expf(-1.702f * g)) * (u + 1.0f);
}

// ---- the CTA pair -----------------------------------------------------------------
__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// This CTA's shared address `a` as seen in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t a, uint32_t rank) {
    uint32_t o;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(rank));
    return o;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D TMA load into this CTA's shared memory, completing on the leader CTA's barrier.
__device__ __forceinline__ void tma_pair(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void sf_copy_pair(uint32_t tmem_col, uint64_t desc) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc) : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                          uint32_t sfb) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
// Arrives on the barrier at shared::cluster address `bar` once the MMAs issued so far complete.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Frees an accumulator: the arrive follows tcgen05.wait::ld (the TMEM reads are
// complete) and tcgen05.fence::before_thread_sync.  It is relaxed: a release would
// first wait until this thread's global stores of the previous item are visible
// at cluster scope, and nothing the MMA warp does next depends on them.
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Instruction descriptor, kind::mxf4 block-scaled, the pair (M = 256): A and B
// E2M1, K-major, E8M0 scales; sf_id is the first of the two scale bytes (32-element
// blocks) the K = 64 MMA uses.
__device__ __forceinline__ uint32_t idesc_pair(uint32_t sf_id, int n) {
    return (sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((256u >> 4) << 24) |
           (sf_id << 29);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    bs_gemm_kernel(const __grid_constant__ CUtensorMap tm_a1, const __grid_constant__ CUtensorMap tm_a2,
                   const __grid_constant__ CUtensorMap tm_b1, const __grid_constant__ CUtensorMap tm_b2, BsParams p) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    if (p.gate && *p.gate != p.gate_want) return;  // the other expert path runs this step (both CTAs)
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = sm;
    float *act_s = reinterpret_cast<float *>(ring + kStages * kStageBytes);  // gate_up SwiGLU outputs
    uint64_t *full = reinterpret_cast<uint64_t *>(act_s + kOutStage / 4);
    uint64_t *empty = full + kStages;
    uint64_t *accfull = empty + kStages;  // [2]
    uint64_t *accempty = accfull + 2;     // [2] (the leader's counts both CTAs' epilogues)
    uint64_t *slot_full = accempty + 2;   // [kSlots] gate_up staging ring
    uint64_t *slot_empty = slot_full + kSlots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(slot_empty + kSlots);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cta_rank();
    const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const int nmp = (p.nmt + 1) >> 1;  // 256-row weight pairs
    const int items = *p.ntiles * nmp;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accfull + b, 1);
            mbar_init(accempty + b, 2 * (p.gate_up ? kSwiThreads : kEpiThreads));
        }
        for (int k = 0; k < kSlots; ++k) {
            mbar_init(slot_full + k, 4);   // lane 0 of each accumulator reader
            mbar_init(slot_empty + k, 4);  // lane 0 of each warp of the quantizer group
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any load or commit names them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lead_full = peer_addr(smem_u32(full), 0);  // full[s] of the leader: + 8 s

    if (warp == kProdWarp) {
        // ---------------- TMA producer (both CTAs; one thread, stages in order) ----------------
        // The two control warps share their SM sub-partitions with busy epilogue warps,
        // so their loops keep few instructions per stage: addresses advance by constants,
        // and the next item's expert id is loaded an item ahead.
        if (lane == 0) {
            const uint32_t ring_a = smem_u32(ring);
            const int nkb2 = (p.nkb + 1) >> 1;
            int s = 0;
            uint32_t ph = 0;  // parity of the ring's current pass
            bool ok = true, first = true;
            int e_next = cl < items ? p.tiles[cl / nmp].x : 0;
            for (int w = cl; w < items && ok; w += ncl) {
                const int t = w / nmp, mp = w - t * nmp;
                const int m = 2 * mp + (int)rank;  // m == nmt: no such tile (odd nmt); its rows are not stored
                const int e = e_next;
                if (w + ncl < items) e_next = p.tiles[(w + ncl) / nmp].x;
                int arow = (e * p.nmt + m) * p.nkb * (int)kARows;  // the stage's first A box, in copy rows
                int brow = (int)bpart_index(t, 0, (int)rank, nkb2) * (int)kBRows;
                for (int kb = 0; kb < p.nkb; kb += kBoxes) {
                    const bool two = kb + 1 < p.nkb;
                    if (!first && !mbar_wait(empty + s, ph ^ 1u, p.err, 40)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = ring_a + (uint32_t)s * kStageBytes;
                    const uint32_t bar = lead_full + 8u * (uint32_t)s;
                    if (rank == 0) mbar_expect_tx(full + s, two ? 4u * (kBoxStride + kBPart) : 2u * (kBoxStride + kBPart));
                    tma_pair(st, two ? &tm_a2 : &tm_a1, bar, 0, arow);
                    tma_pair(st + kStageA, two ? &tm_b2 : &tm_b1, bar, 0, brow);
                    arow += kBoxes * (int)kARows;
                    brow += 2 * kBoxes * (int)kBRows;  // the other CTA's parts sit between
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1u;
                        first = false;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (the leader CTA) ----------------
        if (rank == 0) {
            uint32_t elected;
            asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(elected));
            const uint32_t idesc0 = idesc_pair(0, kN), idesc1 = idesc_pair(2, kN);
            // stage s, box b: the descriptors of stage 0 box 0 plus the start-address field
            // (bits 0-13, 16-byte units; shared addresses stay below 256 KB, so no carry)
            const uint32_t ring_a = smem_u32(ring);
            const uint64_t da = desc_sw64(ring_a), db = desc_sw64(ring_a + kStageA);
            const uint64_t sa = desc_sf(ring_a + kABytes), sb = desc_sf(ring_a + kStageA + kBHalf);
            const uint32_t sf0 = tmem + kSfCol, sf1 = sf0 + 16u;  // the boxes of a stage alternate slots
            const uint32_t empty_l = peer_addr(smem_u32(empty), 0), empty_r = peer_addr(smem_u32(empty), 1);
            const uint32_t accfull_l = peer_addr(smem_u32(accfull), 0), accfull_r = peer_addr(smem_u32(accfull), 1);
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            bool ok = true;
            for (int w = cl; w < items && ok; w += ncl, ++it) {
                const int buf = it & 1;
                if (!mbar_wait(accempty + buf, ((it >> 1) & 1) ^ 1, p.err, 41)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * kN);
                for (int kb = 0; kb < p.nkb; kb += kBoxes) {
                    // tcgen05.cp and tcgen05.mma issued by this thread execute in issue order,
                    // so a scale-factor slot is rewritten only after the MMAs that read it
                    if (!mbar_wait(full + s, ph, p.err, 42)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (elected) {
                        const uint64_t so = (uint64_t)((uint32_t)s * (kStageBytes >> 4));
                        const uint64_t a0 = da + so, b0 = db + so, fa = sa + so, fb = sb + so;
                        sf_copy_pair(sf0, fa);                        // A scales (each CTA its 128 rows)
                        sf_copy_pair(sf0 + 4, fb);                    // B scales, rows 0-127 (both CTAs)
                        sf_copy_pair(sf0 + 8, fb + (512 >> 4));       // rows 128-239
                        umma_pair(d, a0, b0, idesc0, kb ? 1u : 0u, sf0, sf0 + 4);
                        umma_pair(d, a0 + 2, b0 + 2, idesc1, 1u, sf0, sf0 + 4);
                        if (kb + 1 < p.nkb) {
                            constexpr uint32_t oa = kBoxStride >> 4, ob = kBPart >> 4;
                            sf_copy_pair(sf1, fa + oa);
                            sf_copy_pair(sf1 + 4, fb + ob);
                            sf_copy_pair(sf1 + 8, fb + ob + (512 >> 4));
                            umma_pair(d, a0 + oa, b0 + ob, idesc0, 1u, sf1, sf1 + 4);
                            umma_pair(d, a0 + oa + 2, b0 + ob + 2, idesc1, 1u, sf1, sf1 + 4);
                        }
                        commit_pair(empty_l + 8u * (uint32_t)s);
                        commit_pair(empty_r + 8u * (uint32_t)s);
                    }
                    __syncwarp();
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                if (elected) {
                    commit_pair(accfull_l + 8u * (uint32_t)buf);
                    commit_pair(accfull_r + 8u * (uint32_t)buf);
                }
                __syncwarp();
            }
        }
    } else if (!p.gate_up ? warp < kEpiWarp0 + kEpiWarps : warp < kEpiWarp0 + 4 * kQuantGroups) {
        // ---------------- down's epilogue (warps 2-13), gate_up's quantizers (warps 2-9) ----------------
        const int quad = warp & 3;
        const int row = quad * 32 + lane;  // row of this CTA's 128-row weight tile
        const int et = tid - kEpiWarp0 * 32;
        const int g = et >> 7;             // group: down's tokens 16g.., gate_up's chunk parity
        if (!p.gate_up) {
            const uint32_t lead_accempty = peer_addr(smem_u32(accempty), 0);
            // an item's tile and this thread's bias, loaded one item ahead (global latency
            // would otherwise sit in every item)
            auto item_tile = [&](int w) { return w < items ? p.tiles[w / nmp] : make_int4(0, 0, 0, 0); };
            auto item_bias = [&](int w, const int4 &ti) {
                if (w >= items) return 0.0f;
                const int h = 128 * (2 * (w % nmp) + (int)rank) + row;
                return h < p.R ? __ldg(p.bias + (size_t)ti.x * p.R + h) : 0.0f;
            };
            const int c0 = g * kGroupTok;
            int4 ti_next = item_tile(cl);
            float bias_next = item_bias(cl, ti_next);
            int it = 0;
            for (int w = cl; w < items; w += ncl, ++it) {
                const int m = 2 * (w % nmp) + (int)rank;
                const int4 ti = ti_next;
                const float bias = bias_next;
                const int buf = it & 1;
                if (!mbar_wait(accfull + buf, (it >> 1) & 1, p.err, 44)) break;
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kN + kTerms * c0);
                float a[2][8 * kTerms];  // this warp's columns, two halves of 8 tokens: five terms per token
                tmem_ld40(ta, a[0]);
                tmem_ld40(ta + 8u * kTerms, a[1]);
                tc_fence_before();
                arrive_remote(lead_accempty + 8u * (uint32_t)buf);
                ti_next = item_tile(w + ncl);
                bias_next = item_bias(w + ncl, ti_next);
                const int nc = min(kGroupTok, ti.z - c0);
                const int h = 128 * m + row;  // m == nmt (no such tile) gives h >= R
                if (h < p.R) {
#pragma unroll
                    for (int c = 0; c < kGroupTok; ++c) {
                        float sum = 0.0f;
#pragma unroll
                        for (int j = 0; j < kTerms; ++j) sum += a[c >> 3][kTerms * (c & 7) + j];
                        if (c < nc) ep_out_row(p.y, p.y_rows, p.ret, ti.y + c0 + c, p.R)[h] = sum + bias;
                    }
                }
            }
        } else {
            // gate_up: chunk q = 3 (item) + k (slot k, tokens 16k..) goes to group q % 2.
            // Four threads per (token, 32-pair block), 8 pairs each: five E2M1 terms and
            // their scales into down's B operand (pairs 64 (m % 2).. of box m / 2).  Block 1
            // reads its two halves in the other order: the eight threads of one
            // shared-memory phase (a token's two blocks) then hit 32 different banks.
            const int ut = et & 127, unit = ut >> 2, sub = ut & 3;
            const int c = unit >> 1, b = unit & 1;
            const int onkb2 = (p.onkb + 1) >> 1;
            int it = 0, k = g;  // this group's first chunk: slot g of item 0
            for (int w = cl; w < items;) {
                const int t = w / nmp;
                const int m = 2 * (w - t * nmp) + (int)rank;
                const bool live = m < p.nmt;  // every lane takes part in the shuffles inside quantize
                const int c0 = k * kGroupTok;
                const float4 *src =
                    reinterpret_cast<const float4 *>(act_s + k * kSlotFloats + c * kActPitch + 32 * b + 8 * sub);
                if (!mbar_wait(slot_full + k, it & 1, p.err, 47)) break;
                const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                const float4 f0 = live ? src[b] : z, f1 = live ? src[b ^ 1] : z;
                const float4 lo = b ? f1 : f0, hi = b ? f0 : f1;
                float x[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                __syncwarp();
                if (lane == 0) mbar_arrive(slot_empty + k);  // a release: the warp's reads of the slot are done
                uint32_t codes[kTerms][1], sbyte[kTerms];
                fp4::quantize<8, 4>(x, codes, sbyte);
                const int jb = 2 * (m & 1) + b, n0 = kTerms * (c0 + c);
                if (live) {
#pragma unroll
                    for (int term = 0; term < kTerms; ++term) {
                        put_codes<4>(p.oq, t, m >> 1, onkb2, n0 + term, jb, sub, codes[term]);
                        if (term % 4 == sub) put_scale(p.oq, t, m >> 1, onkb2, n0 + term, jb, sbyte[term]);
                    }
                }
                k += kQuantGroups;  // the group's next chunk
                for (; k >= kSlots; k -= kSlots) {
                    w += ncl;
                    ++it;
                }
            }
        }
    } else if (p.gate_up && warp >= kSwiWarp0) {
        // ---------------- warps 12-15 (gate_up): accumulator -> bias, SwiGLU -> the slots ----------------
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lead_accempty = peer_addr(smem_u32(accempty), 0);
        // rows 16g + j (j < 8) hold the gate of pair 8g + j, row + 8 its up row
        const int j16 = row & 15;
        const bool gate_lane = j16 < 8;
        const int pl = 8 * (row >> 4) + (j16 & 7);  // pair within this tile (0..63)
        auto item_tile = [&](int w) { return w < items ? p.tiles[w / nmp] : make_int4(0, 0, 0, 0); };
        auto item_bias = [&](int w, const int4 &ti) {
            if (w >= items) return 0.0f;
            const int m = 2 * (w % nmp) + (int)rank;
            if (m >= p.nmt) return 0.0f;
            return __ldg(p.bias + (size_t)ti.x * p.R + 2 * (64 * m + pl) + (gate_lane ? 0 : 1));
        };
        int4 ti_next = item_tile(cl);
        float bias_next = item_bias(cl, ti_next);
        int it = 0;
        bool ok = true;
        for (int w = cl; w < items && ok; w += ncl, ++it) {
            const int4 ti = ti_next;
            const float bias = bias_next;
            const int buf = it & 1;
            if (!mbar_wait(accfull + buf, (it >> 1) & 1, p.err, 44)) break;
            tc_fence_after();
            ti_next = item_tile(w + ncl);
            bias_next = item_bias(w + ncl, ti_next);
            const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kN);
            for (int k = 0; k < kSlots; ++k) {
                if (it > 0 && !mbar_wait(slot_empty + k, (it - 1) & 1, p.err, 48)) {
                    ok = false;
                    break;
                }
                float *slot = act_s + k * kSlotFloats;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int tok0 = kGroupTok * k + 8 * hf;  // first of this half's 8 tokens
                    float a[8 * kTerms];
                    tmem_ld40(ta + (uint32_t)(kTerms * tok0), a);
                    if (k == kSlots - 1 && hf == 1) {  // the item's last columns are read
                        tc_fence_before();
                        arrive_remote(lead_accempty + 8u * (uint32_t)buf);
                    }
                    float v[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        float sum = 0.0f;
#pragma unroll
                        for (int j = 0; j < kTerms; ++j) sum += a[kTerms * c + j];
                        v[c] = sum + bias;
                    }
                    // the gate lane finishes tokens 0-3 of the half, its partner (the up lane,
                    // 8 lanes away) tokens 4-7: one exchange per token pair hands each lane the
                    // partner's value it needs
                    const int nc = ti.z - tok0;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float got = __shfl_xor_sync(0xffffffffu, gate_lane ? v[c + 4] : v[c], 8);
                        const int cc = gate_lane ? c : c + 4;
                        const float r = swiglu_fast(gate_lane ? v[c] : got, gate_lane ? got : v[c + 4]);
                        slot[(8 * hf + cc) * kActPitch + pl] = cc < nc ? r : 0.0f;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(slot_full + k);  // a release: the warp's slot stores
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer is done with the pair's TMEM and barriers
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
    ep_return_done(p.ret);  // expert-parallel down: outputs are in the source ranks' windows
}

}  // namespace

// ---- host side ------------------------------------------------------------------

namespace {

struct BsScratch {
    int4 *tiles;
    int32_t *ntiles;
    uint8_t *xq;  // gate_up's B operand (the quantized tokens)
    uint8_t *aq;  // down's B operand (the quantized activations)
    uint4 *tq;    // token-major quantized rows (tok_quant_kernel), tok_cap tokens
    uint2 *ts;
    int max_tiles;
};

inline size_t up1k(size_t v) { return (v + 1023) & ~size_t(1023); }
// B operand bytes of `tiles` tiles of nkb K boxes (boxes rounded up to pairs, two parts each).
inline size_t b_bytes(size_t tiles, size_t nkb) { return tiles * ((nkb + 1) / 2) * 2 * kBoxes * kBPart; }

BsScratch carve_bs(void *base, int rows_cap, int tok_cap, int E, int H, int I) {
    BsScratch s{};
    s.max_tiles = (rows_cap + kTok - 1) / kTok + E;
    const size_t nkb_gu = kpad128(H) / 128, nkb_dn = kpad128(I) / 128;
    uint8_t *p = static_cast<uint8_t *>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *at = p + off;
        off = up1k(off + bytes);
        return at;
    };
    s.tiles = reinterpret_cast<int4 *>(take((size_t)s.max_tiles * sizeof(int4)));
    s.ntiles = reinterpret_cast<int32_t *>(take(16));
    s.xq = take(b_bytes(s.max_tiles, nkb_gu));
    s.aq = take(b_bytes(s.max_tiles, nkb_dn));
    s.tq = reinterpret_cast<uint4 *>(take((size_t)tok_cap * nkb_gu * 4 * kTerms * 16));
    s.ts = reinterpret_cast<uint2 *>(take((size_t)tok_cap * nkb_gu * 4 * 8));
    return s;
}

}  // namespace

bool tc_supported() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    static int known[64];  // per device: 0 not asked yet, 1 yes, 2 no (idempotent writes)
    if (!known[dev]) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        known[dev] = major == 10 && minor == 0 && get_encode() ? 1 : 2;
    }
    return known[dev] == 1;
}

size_t bs_scratch_bytes(int rows_cap, int tok_cap, int E, int H, int I) {
    const size_t max_tiles = (size_t)(rows_cap + kTok - 1) / kTok + E;
    const size_t nkb_gu = kpad128(H) / 128, nkb_dn = kpad128(I) / 128;
    return up1k(max_tiles * sizeof(int4)) + 1024 + up1k(b_bytes(max_tiles, nkb_gu)) + up1k(b_bytes(max_tiles, nkb_dn)) +
           up1k((size_t)tok_cap * nkb_gu * 4 * kTerms * 16) + up1k((size_t)tok_cap * nkb_gu * 4 * 8);
}

cudaError_t launch_tok_quant(const __half *x_hi, const __half *x_lo, int tokens, int H, int I, void *scratch,
                             int rows_cap, int tok_cap, int scratch_e, const int32_t *gate, cudaStream_t st,
                             const uint4 **tq, const uint2 **ts) {
    const BsScratch s = carve_bs(scratch, rows_cap, tok_cap, scratch_e, H, I);
    *tq = s.tq;
    *ts = s.ts;
    if (tokens <= 0 || tokens > tok_cap) return cudaErrorInvalidValue;
    const int nkb = kpad128(H) / 128;
    const size_t recs = (size_t)tokens * nkb * 4;
    tok_quant_kernel<<<(unsigned)((recs + 255) / 256), 256, 0, st>>>(x_hi, x_lo, tokens, H, nkb, s.tq, s.ts, gate);
    return cudaGetLastError();
}

cudaError_t init_bs_scratch(void *scratch, int rows_cap, int tok_cap, int E, int H, int I) {
    // down's B operand: rows no gate_up tile writes (K padding past I) must read as
    // zero codes with a unit scale
    const BsScratch s = carve_bs(scratch, rows_cap, tok_cap, E, H, I);
    const size_t parts = b_bytes(s.max_tiles, kpad128(I) / 128) / kBPart;
    cudaError_t e = cudaMemset(s.aq, 0, parts * kBPart);
    if (e == cudaSuccess) e = cudaMemset2D(s.aq + kBHalf, kBPart, 127, kBSf, parts);
    return e;
}

namespace {

// A byte array seen as rows of `row_bytes` (a multiple of 8) moved by TMA as
// 8-byte elements, `box_rows` rows per copy, no swizzle: the bytes land in
// shared memory exactly as stored.
cudaError_t map_rows(CUtensorMap *tm, const void *base, size_t bytes, uint32_t row_bytes, uint32_t box_rows) {
    cuuint64_t dims[2] = {row_bytes / 8, bytes / row_bytes};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {row_bytes / 8, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn()(tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(base), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// CTA pairs that can run at once (one pair per two SMs of a GPC), as an even grid.
int pair_grid(int dev) {
    static int known[64];
    if (dev < 0 || dev >= 64) return 2;
    if (!known[dev]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2, 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = kSmem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, bs_gemm_kernel, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            int sms = 148;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            n = sms / 2;
        }
        known[dev] = 2 * n;
    }
    return known[dev];
}

}  // namespace

cudaError_t launch_bs_experts(const Dims &d, const LayerDev &L, const int32_t *offsets, const __half *x_hi,
                              const __half *x_lo, const int32_t *perm, int tokens, int rows_cap, int tok_cap,
                              void *scratch, int scratch_e, float *y, const int32_t *y_rows, int32_t *err,
                              cudaStream_t st, StageHook hook, void *hook_arg, int *launches, const EpReturn *ret,
                              const int32_t *gate, int gate_want, const uint4 *rec_q, const uint2 *rec_s) {
    if (!get_encode()) return cudaErrorNotSupported;
    int dev = 0;
    cudaGetDevice(&dev);
    static int attr_set[64];  // the kernel's shared-memory ceiling, once per device (idempotent writes)
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(bs_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = 1;
    }
    const int grid = pair_grid(dev);
    const BsScratch s = carve_bs(scratch, rows_cap, tok_cap, scratch_e, d.H, d.I);
    const int nkb_gu = kpad128(d.H) / 128, nkb_dn = kpad128(d.I) / 128;
    const int nmt_gu = (2 * d.I + 127) / 128, nmt_dn = (d.H + 127) / 128;
    *launches = 0;
    // 1. token tiles, then the gate_up B operand
    bs_plan_kernel<<<1, 256, 0, st>>>(offsets, d.E, s.tiles, s.ntiles, s.max_tiles, err);
    if (rec_q && rec_s) {
        // the rows arrived as token records (expert parallelism): gather them by position
        bs_gather_kernel<<<s.max_tiles * nkb_gu, kTok * 4, 0, st>>>(rec_q, rec_s, nullptr, 1, nkb_gu, s.tiles,
                                                                    s.ntiles, s.xq);
        *launches += 2;
    } else if (perm && tokens > 0 && tokens <= tok_cap) {
        // each token feeds k pairs: quantize it once, then gather the tiles' rows
        const size_t recs = (size_t)tokens * nkb_gu * 4;
        tok_quant_kernel<<<(unsigned)((recs + 255) / 256), 256, 0, st>>>(x_hi, x_lo, tokens, d.H, nkb_gu, s.tq, s.ts,
                                                                         nullptr);
        bs_gather_kernel<<<s.max_tiles * nkb_gu, kTok * 4, 0, st>>>(s.tq, s.ts, perm, d.k, nkb_gu, s.tiles, s.ntiles,
                                                                    s.xq);
        *launches += 3;
    } else {
        bs_quant_kernel<<<s.max_tiles * nkb_gu, kTok * 4, 0, st>>>(x_hi, x_lo, perm, d.k, d.H, nkb_gu, s.tiles,
                                                                   s.ntiles, s.xq);
        *launches += 2;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (hook) hook(hook_arg, 5);
    // 2. gate_up + SwiGLU, writing down's B operand
    CUtensorMap tm_gu1, tm_gu2, tm_dn1, tm_dn2, tm_xq1, tm_xq2, tm_aq1, tm_aq2;
    const size_t gu_bytes = box_plane_bytes(d.E, 2 * d.I, d.H), dn_bytes = box_plane_bytes(d.E, d.H, d.I);
    const size_t xq_bytes = b_bytes(s.max_tiles, nkb_gu), aq_bytes = b_bytes(s.max_tiles, nkb_dn);
    e = map_rows(&tm_gu1, L.gu_tq, gu_bytes, kCopyRow, kARows);
    if (e == cudaSuccess) e = map_rows(&tm_gu2, L.gu_tq, gu_bytes, kCopyRow, 2 * kARows);
    if (e == cudaSuccess) e = map_rows(&tm_dn1, L.dn_tq, dn_bytes, kCopyRow, kARows);
    if (e == cudaSuccess) e = map_rows(&tm_dn2, L.dn_tq, dn_bytes, kCopyRow, 2 * kARows);
    if (e == cudaSuccess) e = map_rows(&tm_xq1, s.xq, xq_bytes, kCopyRow, kBRows);
    if (e == cudaSuccess) e = map_rows(&tm_xq2, s.xq, xq_bytes, kCopyRow, 2 * kBRows);
    if (e == cudaSuccess) e = map_rows(&tm_aq1, s.aq, aq_bytes, kCopyRow, kBRows);
    if (e == cudaSuccess) e = map_rows(&tm_aq2, s.aq, aq_bytes, kCopyRow, 2 * kBRows);
    if (e != cudaSuccess) return e;
    BsParams p{};
    p.tiles = s.tiles;
    p.ntiles = s.ntiles;
    p.err = err;
    p.gate = gate;
    p.gate_want = gate_want;
    p.bias = L.gu_b;
    p.R = 2 * d.I;
    p.nmt = nmt_gu;
    p.nkb = nkb_gu;
    p.gate_up = 1;
    p.oq = s.aq;
    p.onkb = nkb_dn;
    bs_gemm_kernel<<<grid, kThreads, kSmem, st>>>(tm_gu1, tm_gu2, tm_xq1, tm_xq2, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
    if (hook) hook(hook_arg, 2);
    // 3. down
    p.bias = L.dn_b;
    p.R = d.H;
    p.nmt = nmt_dn;
    p.nkb = nkb_dn;
    p.gate_up = 0;
    p.oq = nullptr;
    p.y = y;
    p.y_rows = y_rows;
    if (ret) p.ret = *ret;
    bs_gemm_kernel<<<grid, kThreads, kSmem, st>>>(tm_dn1, tm_dn2, tm_aq1, tm_aq2, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
    if (hook) hook(hook_arg, 3);
    return cudaSuccess;
}

}  // namespace amoe
