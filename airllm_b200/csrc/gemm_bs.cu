// gemm_bs.cu -- K4/K5: the grouped expert GEMMs of prefill on the block-scaled
// 5th-generation tensor cores (tcgen05.mma kind::mxf8f6f4.block_scale).
//
// Per expert e with m_e routed rows (positions offsets[e]..offsets[e+1] of the
// expert-sorted pairs):
//   gate_up: act = SwiGLU(W_gu . x + b_gu)   (layer.go:139-148, 175; primitives.go:138-149)
//   down:    y   = W_dn . act + b_dn          (layer.go:179-187)
//
// A = the MXFP4 weights as stored: E2M1 nibbles from the box-tiled TMA planes
//     (TMA unpacks them into the tensor core's shared-memory format) with the
//     GGUF E8M0 bytes as the hardware block scales -- no conversion pass.
// B = the activations as four E4M3 terms per element, x ~= sum_j q_j 2^(e0-4j)
//     per 32-element block (e0 from the block's largest magnitude), one term per
//     MMA column: a tile of 60 tokens is N = 240 columns, and the epilogue adds
//     each token's four columns.  Four terms carry ~16 significant bits; the
//     tensor core accumulates in f32.
//
// Tokens are tiled per expert (60 per tile, the last tile of an expert ragged).
// The B operand of every (tile, 128-element K box) sits in global memory as one
// 32 KB blob of two halves, one per CTA of a pair: the box's E8M0 scale chunks
// (1 KB), then 120 pre-swizzled rows of E4M3 terms.  gate_up's epilogue writes
// down's B operand in the same form: SwiGLU, block maxima, quantization to four
// terms, 16-byte swizzled stores.
//
// The MMAs are 2-SM (tcgen05 cta_group::2): a cluster of two CTAs computes a
// 256-row weight tile x 60 tokens.  Each CTA loads its own 128-row A box, its
// half of the B rows and the full B scales; every load signals the leader CTA's
// barrier, the leader issues the MMAs (M = 256, N = 240) and commits to both
// CTAs' barriers, and each CTA's epilogue reads the accumulator rows in its own
// TMEM.  Each SM thus loads half of every B tile it multiplies, which halves the
// operand traffic per MMA compared with one CTA per 128-row tile.
//
// Work item = (token tile, 256-row weight pair), clusters striding over items.
// Roles per CTA: warps 0-5 TMA producers (stage i by warp i % 6: one warp per
// ring slot), warp 6 MMA issuer (leader) and TMEM owner, warps 7-14 epilogue
// (two per TMEM lane quadrant, splitting the tile's tokens).  TMEM: two
// 240-column accumulators (the epilogue of one item overlaps the next item's
// MMAs) and two 12-column scale-factor slots.  Every wait is bounded; on timeout
// the kernel records a code in the error flag and winds down.
#include "tc_ptx.cuh"

namespace amoe {

namespace {

using namespace bs;

constexpr int kTok = 60;                          // tokens per tile
constexpr int kN = 4 * kTok;                      // MMA N: four E4M3 terms per token
constexpr int kHalfRows = kN / 2;                 // B rows per CTA of a pair
constexpr uint32_t kBSf = 1024;                   // a B box's scale chunks: rows 0-127, 128-239
constexpr uint32_t kHalf = kBSf + kHalfRows * 128;  // 16384: scales + 120 pre-swizzled rows (one TMA box)
constexpr uint32_t kBlob = 2 * kHalf;             // one (tile, K box) B operand
constexpr uint32_t kABox = 128 * 128;             // unpacked A box in shared memory
constexpr uint32_t kAPacked = 128 * 64;           // its bytes in global memory (TMA transaction size)
constexpr uint32_t kStageBytes = 33792;           // A box | B half | A scales, padded to 1 KB
constexpr int kStages = 6;
constexpr int kProdWarps = kStages;
constexpr int kMmaWarp = kProdWarps;
constexpr int kEpiWarp0 = kMmaWarp + 1;
constexpr int kEpiWarps = 8;                      // two per TMEM lane quadrant (token halves 0-31, 32-59)
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 480
constexpr uint32_t kSfCol = 2 * kN;               // TMEM column of scale-factor slot 0 (slot 1: +16)
constexpr int kActPitch = 68;                     // gate_up epilogue staging: [60 tokens][64 pairs] f32, padded rows
constexpr uint32_t kOutStage = kTok * kActPitch * 4;
constexpr size_t kSmem = 1024 + kStages * kStageBytes + kOutStage + 16 * 8 + 16;
constexpr uint32_t kStageTx = 2 * (kAPacked + kHalf + 512);  // bytes both CTAs' loads bring per stage

static_assert(kABox + kHalf + 512 <= kStageBytes && kStageBytes % 1024 == 0, "stage layout");
static_assert(kHalfRows % 8 == 0, "B halves start on a swizzle atom");
// Each producer warp owns one ring slot, so its waits on that slot's empty
// barrier are for consecutive phases (a parity wait two phases ahead would pass).
static_assert(kProdWarps == kStages, "one producer warp per ring slot");
static_assert(kSfCol + 16 + 12 <= 512, "TMEM budget");
static_assert(kSmem <= 232448, "shared memory budget");

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

// Blob byte offset of B row n (token 4i + term j), 16-byte chunk c: half n / 120,
// after its scale chunks; SWIZZLE_128B within the half (120 is a multiple of 8).
__device__ __forceinline__ uint32_t swz(int n, int c) {
    const int h = n >= kHalfRows, r = n - kHalfRows * h;
    return (uint32_t)h * kHalf + kBSf + (uint32_t)r * 128u + (uint32_t)((c ^ (r & 7)) << 4);
}

// Scale byte of B row n, 32-element block jb of a box, inside one half's chunks
// (chunk n / 128 in the layout tcgen05.cp.32x128b.warpx4 spreads over TMEM).
__device__ __forceinline__ uint32_t sf_at(int n, int jb) {
    return (uint32_t)(n >> 7) * 512u + (uint32_t)(n & 31) * 16u + (uint32_t)((n & 127) >> 5) * 4u + (uint32_t)jb;
}

__device__ __forceinline__ void put_sf(uint8_t *blob, int n, int jb, uint8_t v) {  // both halves carry the scales
    blob[sf_at(n, jb)] = v;
    blob[kHalf + sf_at(n, jb)] = v;
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
// through the permutation (or, with perm NULL, already by position).
__global__ void __launch_bounds__(256) bs_quant_kernel(const __half *__restrict__ x_hi, const __half *__restrict__ x_lo,
                                                       const int32_t *__restrict__ perm, int k, int K, int nkb,
                                                       const int4 *__restrict__ tiles, const int32_t *ntiles,
                                                       uint8_t *bq) {
    const int t = blockIdx.x / nkb, kb = blockIdx.x - t * nkb;
    if (t >= *ntiles || threadIdx.x >= kTok * 4) return;
    const int4 ti = tiles[t];
    const int i = threadIdx.x >> 2, jb = threadIdx.x & 3;
    const int k0 = kb * 128 + jb * 32;
    float x[32];
    bool live = i < ti.z && k0 < K;
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
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = live ? fmaxf(amax, fabsf(x[j])) : 0.0f;
    const int e0 = block_exp(amax);
    const TermScales ts = term_scales(e0);
    uint32_t w[4][8];  // [term][4 elements]
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        uint32_t lo[4], hi[4];
        quant4_pair(live ? x[4 * g] : 0.0f, live ? x[4 * g + 1] : 0.0f, ts, lo);
        quant4_pair(live ? x[4 * g + 2] : 0.0f, live ? x[4 * g + 3] : 0.0f, ts, hi);
#pragma unroll
        for (int term = 0; term < 4; ++term) w[term][g] = (lo[term] & 0xffffu) | (hi[term] << 16);
    }
    uint8_t *blob = bq + ((size_t)t * nkb + kb) * kBlob;
#pragma unroll
    for (int term = 0; term < 4; ++term) {
        const uint32_t *wt = w[term];
        const int r = 4 * i + term;
        *reinterpret_cast<uint4 *>(blob + swz(r, 2 * jb)) = make_uint4(wt[0], wt[1], wt[2], wt[3]);
        *reinterpret_cast<uint4 *>(blob + swz(r, 2 * jb + 1)) = make_uint4(wt[4], wt[5], wt[6], wt[7]);
        put_sf(blob, r, jb, live ? (uint8_t)term_scale_byte(e0, term) : (uint8_t)127);
    }
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

// GPT-OSS clamped SwiGLU (primitives.go:144-146; NaN propagates) with the fast
// exponential and division: the result is rounded to 16 significant bits (four
// E4M3 terms) right after, far coarser than their error.
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
__device__ __forceinline__ void tma_pair(void *dst, const CUtensorMap *tm, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void sf_copy_pair(uint32_t tmem_col, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc_sf(saddr)) : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                          uint32_t sfb) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
// Arrives on the barrier at shared::cluster address `bar` once the MMAs issued so far complete.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Instruction descriptor for the pair: M = 256.
__device__ __forceinline__ uint32_t idesc_pair(uint32_t sf_id, int n) {
    return (sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((256u >> 4) << 24) |
           (sf_id << 29);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    bs_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_sfa, BsParams p) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    if (p.gate && *p.gate != p.gate_want) return;  // the other expert path runs this step (both CTAs)
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = sm;
    float *act_s = reinterpret_cast<float *>(ring + kStages * kStageBytes);  // gate_up SwiGLU outputs
    uint64_t *full = reinterpret_cast<uint64_t *>(act_s + kTok * kActPitch);
    uint64_t *empty = full + kStages;
    uint64_t *accfull = empty + kStages;  // [2]
    uint64_t *accempty = accfull + 2;     // [2] (the leader's counts both CTAs' epilogues)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + 2);

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
            mbar_init(accempty + b, 2 * kEpiThreads);
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

    if (warp < kProdWarps) {
        // ---------------- TMA producers (both CTAs) ----------------
        if (lane == 0) {
            int i = 0;
            bool ok = true;
            for (int w = cl; w < items && ok; w += ncl) {
                const int t = w / nmp, mp = w - t * nmp;
                const int m = 2 * mp + (int)rank;  // m == nmt: no such tile (odd nmt); its rows are not stored
                const int e = p.tiles[t].x;
                for (int kb = 0; kb < p.nkb; ++kb, ++i) {
                    if (i % kProdWarps != warp) continue;
                    const int s = i % kStages;
                    if (i >= kStages && !mbar_wait(empty + s, ((i / kStages) - 1) & 1, p.err, 40)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = ring + (size_t)s * kStageBytes;
                    if (rank == 0) mbar_expect_tx(full + s, kStageTx);
                    const int box = (e * p.nmt + m) * p.nkb + kb;  // box-tiled plane: row origin 128 * box
                    const uint32_t bar = lead_full + 8u * (uint32_t)s;
                    tma_pair(st, &tm_a, bar, 0, box * 128);
                    tma_pair(st + kABox, &tm_b, bar, 0, (t * p.nkb + kb) * (int)(kBlob / 128) + (int)rank * (int)(kHalf / 128));
                    tma_pair(st + kABox + kHalf, &tm_sfa, bar, 0, box * 4);
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (the leader CTA) ----------------
        if (rank == 0) {
            uint32_t elected;
            asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(elected));
            uint32_t idesc[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) idesc[kk] = idesc_pair(kk, kN);
            const uint32_t ring_a = smem_u32(ring);
            const uint32_t empty0 = smem_u32(empty), accfull0 = smem_u32(accfull);
            int i = 0, it = 0;
            bool ok = true;
            for (int w = cl; w < items && ok; w += ncl, ++it) {
                const int buf = it & 1;
                if (!mbar_wait(accempty + buf, ((it >> 1) & 1) ^ 1, p.err, 41)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * kN);
                for (int kb = 0; kb < p.nkb; ++kb, ++i) {
                    const int s = i % kStages;
                    // scale-factor slot i % 2 is free once the MMAs of iteration i - 2 completed
                    if (!mbar_wait(full + s, (i / kStages) & 1, p.err, 42) ||
                        (i >= 2 && !mbar_wait(empty + (i - 2) % kStages, ((i - 2) / kStages) & 1, p.err, 43))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = ring_a + (uint32_t)s * kStageBytes;
                    const uint32_t sf = tmem + kSfCol + 16u * (uint32_t)(i & 1);
                    if (elected) {
                        sf_copy_pair(sf, st + kABox + kHalf);      // A scales (each CTA its 128 rows)
                        sf_copy_pair(sf + 4, st + kABox);          // B scales, rows 0-127 (both CTAs)
                        sf_copy_pair(sf + 8, st + kABox + 512);    // rows 128-239
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            umma_pair(d, desc_sw128(st + 32 * kk), desc_sw128(st + kABox + kBSf + 32 * kk), idesc[kk],
                                      (kb | kk) ? 1u : 0u, sf, sf + 4);
                        const uint32_t eb = empty0 + 8u * (uint32_t)s;
                        commit_pair(peer_addr(eb, 0));
                        commit_pair(peer_addr(eb, 1));
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (elected) {
                    commit_pair(peer_addr(accfull0 + 8u * (uint32_t)buf, 0));
                    commit_pair(peer_addr(accfull0 + 8u * (uint32_t)buf, 1));
                }
                __syncwarp();
            }
        }
    } else {
        // ---------------- epilogue (warps 7-14 of both CTAs; TMEM lane quadrant = warp % 4) ----------------
        const int quad = warp & 3;
        const int row = quad * 32 + lane;  // row of this CTA's 128-row weight tile
        const int et = tid - kEpiWarp0 * 32;
        const int c0 = (et >> 7) * 32;     // this warp's tokens: c0 .. c0 + 31 (the second half has 28)
        const uint32_t lead_accempty = peer_addr(smem_u32(accempty), 0);
        int it = 0;
        bool ok = true;
        for (int w = cl; w < items; w += ncl, ++it) {
            const int t = w / nmp, mp = w - t * nmp;
            const int m = 2 * mp + (int)rank;
            const bool real = m < p.nmt;  // an odd nmt leaves the last pair's second tile empty
            const int4 ti = p.tiles[t];
            const int e = ti.x;
            const int buf = it & 1;
            float v[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] = 0.0f;
            if (ok) ok = mbar_wait(accfull + buf, (it >> 1) & 1, p.err, 44);
            if (ok) {
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kN + 4 * c0);
#pragma unroll
                for (int g = 0; g < 4; ++g) {  // 8 tokens per load
                    if (c0 != 0 && g == 3) {
                        float r16[16];
                        tmem_ld16(ta + 96u, r16);
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            v[24 + u] = ((r16[4 * u] + r16[4 * u + 1]) + r16[4 * u + 2]) + r16[4 * u + 3];
                    } else {
                        float r32[32];
                        tmem_ld32(ta + 32u * g, r32);
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            v[8 * g + u] = ((r32[4 * u] + r32[4 * u + 1]) + r32[4 * u + 2]) + r32[4 * u + 3];
                    }
                }
                tc_fence_before();
                arrive_remote(lead_accempty + 8u * (uint32_t)buf);
            }
            const int nc = min(32, kTok - c0);
            if (!p.gate_up) {
                const int h = 128 * m + row;
                if (ok && h < p.R) {
                    const float bias = p.bias[(size_t)e * p.R + h];
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        if (c < nc && c0 + c < ti.z) ep_out_row(p.y, p.y_rows, p.ret, ti.y + c0 + c, p.R)[h] = v[c] + bias;
                }
                continue;
            }
            // gate_up: rows 16g + j (j < 8) hold the gate of pair 8g + j, row + 8 its up row
            const int j16 = row & 15;
            const bool gate_lane = j16 < 8;
            const int pl = 8 * (row >> 4) + (j16 & 7);  // pair within this tile (0..63)
            const float bias = real ? p.bias[(size_t)e * p.R + 2 * (64 * m + pl) + (gate_lane ? 0 : 1)] : 0.0f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float val = v[c] + bias;
                const float up = __shfl_down_sync(0xffffffffu, val, 8);
                if (gate_lane && c < nc) act_s[(c0 + c) * kActPitch + pl] = swiglu_fast(val, up);
            }
            epi_bar();
            // two threads per (token, 32-pair block), 16 pairs each: block maximum, four
            // E4M3 terms, their scales, written into down's B blob (pairs 64(m%2).. of box m/2)
            {
                const bool live = real && et < 4 * kTok;  // the shuffle below runs on every lane
                const int c = min(et >> 2, kTok - 1), b = (et >> 1) & 1, sub = et & 1;
                const float4 *src = reinterpret_cast<const float4 *>(act_s + c * kActPitch + 32 * b + 16 * sub);
                float x[16];
                float amax = 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 f = live ? src[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    x[4 * q] = f.x;
                    x[4 * q + 1] = f.y;
                    x[4 * q + 2] = f.z;
                    x[4 * q + 3] = f.w;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(x[j]));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                const int e0 = block_exp(amax);
                const TermScales ts = term_scales(e0);
                uint32_t wq[4][4];  // [term][4 pairs]
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t lo[4], hi[4];
                    quant4_pair(x[4 * g], x[4 * g + 1], ts, lo);
                    quant4_pair(x[4 * g + 2], x[4 * g + 3], ts, hi);
#pragma unroll
                    for (int term = 0; term < 4; ++term) wq[term][g] = (lo[term] & 0xffffu) | (hi[term] << 16);
                }
                uint8_t *blob = p.oq + ((size_t)t * p.onkb + (m >> 1)) * kBlob;
                const int chunk = 4 * (m & 1) + 2 * b + sub, jb = 2 * (m & 1) + b;
#pragma unroll
                for (int term = 0; term < 4; ++term) {
                    const int r = 4 * c + term;
                    if (live)
                        *reinterpret_cast<uint4 *>(blob + swz(r, chunk)) =
                            make_uint4(wq[term][0], wq[term][1], wq[term][2], wq[term][3]);
                    if (live && sub == 0) put_sf(blob, r, jb, (uint8_t)term_scale_byte(e0, term));
                }
            }
            epi_bar();  // act_s is rewritten by the next item
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
    uint8_t *xq, *aq;  // B blobs of gate_up (quantized tokens) and down (quantized activations)
    int max_tiles;
};

inline size_t up1k(size_t v) { return (v + 1023) & ~size_t(1023); }

BsScratch carve_bs(void *base, int rows_cap, int E, int H, int I) {
    BsScratch s{};
    s.max_tiles = (rows_cap + kTok - 1) / kTok + E;
    const size_t nkb_gu = kpad128(H) / 128, nkb_dn = kpad128(I) / 128;
    uint8_t *p = static_cast<uint8_t *>(base);
    size_t off = 0;
    s.tiles = reinterpret_cast<int4 *>(p + off);
    off = up1k(off + (size_t)s.max_tiles * sizeof(int4));
    s.ntiles = reinterpret_cast<int32_t *>(p + off);
    off = up1k(off + 16);
    s.xq = p + off;
    off = up1k(off + (size_t)s.max_tiles * nkb_gu * kBlob);
    s.aq = p + off;
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

size_t bs_scratch_bytes(int rows_cap, int E, int H, int I) {
    const size_t max_tiles = (size_t)(rows_cap + kTok - 1) / kTok + E;
    const size_t nkb_gu = kpad128(H) / 128, nkb_dn = kpad128(I) / 128;
    return up1k(max_tiles * sizeof(int4)) + 1024 + up1k(max_tiles * nkb_gu * kBlob) + up1k(max_tiles * nkb_dn * kBlob);
}

cudaError_t init_bs_scratch(void *scratch, int rows_cap, int E, int H, int I) {
    // down's B operand: bytes no gate_up tile writes (K padding past I) must read as
    // zero terms with a unit scale
    const BsScratch s = carve_bs(scratch, rows_cap, E, H, I);
    const size_t nkb_dn = kpad128(I) / 128;
    const size_t blobs = (size_t)s.max_tiles * nkb_dn;
    cudaError_t e = cudaMemset(s.aq, 0, blobs * kBlob);
    if (e == cudaSuccess) e = cudaMemset2D(s.aq, kHalf, 127, kBSf, 2 * blobs);  // both halves' scale chunks
    return e;
}

namespace {

// Rows of 128 bytes, boxes of `box_rows` rows, no swizzle (the data is stored pre-swizzled).
cudaError_t map_rows(CUtensorMap *tm, const void *base, uint64_t rows, uint32_t box_rows) {
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn()(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
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
                              const __half *x_lo, const int32_t *perm, int rows_cap, void *scratch, int scratch_e,
                              float *y,
                              const int32_t *y_rows, int32_t *err, cudaStream_t st, StageHook hook, void *hook_arg,
                              int *launches, const EpReturn *ret, const int32_t *gate, int gate_want) {
    if (!get_encode()) return cudaErrorNotSupported;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(bs_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = pair_grid(dev);
    const BsScratch s = carve_bs(scratch, rows_cap, scratch_e, d.H, d.I);
    const int nkb_gu = kpad128(d.H) / 128, nkb_dn = kpad128(d.I) / 128;
    const int nmt_gu = (2 * d.I + 127) / 128, nmt_dn = (d.H + 127) / 128;
    *launches = 0;
    // 1. token tiles, then the gate_up B operand
    bs_plan_kernel<<<1, 256, 0, st>>>(offsets, d.E, s.tiles, s.ntiles, s.max_tiles, err);
    bs_quant_kernel<<<s.max_tiles * nkb_gu, 256, 0, st>>>(x_hi, x_lo, perm, d.k, d.H, nkb_gu, s.tiles, s.ntiles,
                                                         s.xq);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    *launches += 2;
    if (hook) hook(hook_arg, 5);
    // 2. gate_up + SwiGLU, writing down's B operand
    CUtensorMap tm_gu, tm_dn, tm_xq, tm_aq, tm_gsf, tm_dsf;
    e = map_boxes(&tm_gu, L.gu_tq, tq_bytes(d.E, 2 * d.I, d.H) / 64);
    if (e == cudaSuccess) e = map_boxes(&tm_dn, L.dn_tq, tq_bytes(d.E, d.H, d.I) / 64);
    if (e == cudaSuccess) e = map_rows(&tm_xq, s.xq, (uint64_t)s.max_tiles * nkb_gu * (kBlob / 128), kHalf / 128);
    if (e == cudaSuccess) e = map_rows(&tm_aq, s.aq, (uint64_t)s.max_tiles * nkb_dn * (kBlob / 128), kHalf / 128);
    if (e == cudaSuccess) e = map_rows(&tm_gsf, L.gu_tsf, tsf_bytes(d.E, 2 * d.I, d.H) / 128, 4);
    if (e == cudaSuccess) e = map_rows(&tm_dsf, L.dn_tsf, tsf_bytes(d.E, d.H, d.I) / 128, 4);
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
    bs_gemm_kernel<<<grid, kThreads, kSmem, st>>>(tm_gu, tm_xq, tm_gsf, p);
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
    bs_gemm_kernel<<<grid, kThreads, kSmem, st>>>(tm_dn, tm_aq, tm_dsf, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
    if (hook) hook(hook_arg, 3);
    return cudaSuccess;
}

}  // namespace amoe
