// gemm_tc.cu -- K4/K5: grouped expert GEMMs on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for prefill-sized token counts.
//
// Per expert e with m_e routed tokens (rows offsets[e]..offsets[e+1] of the
// expert-sorted activation matrix), computes
//   gate_up: act = SwiGLU(W_gu . x + b_gu)   (layer.go:139-148, 175; primitives.go:138-149)
//   down:    y   = W_dn . act + b_dn          (layer.go:179-187)
// Operand roles are swapped relative to a textbook GEMM so that ragged
// per-expert token counts only pad to 16:
//   A (M = 128 weight rows per UMMA, two UMMAs per CTA tile = 256 rows)
//     = MXFP4 weights.  TMA brings the raw fragment tiles (4-bit nibbles + E8M0
//       bytes) to shared memory; sixteen converter warps expand them to fp16 in
//       the canonical K-major SWIZZLE_128B layout (cvt.rn.f16x2.e2m1x2 and one
//       f16x2 multiply by 2^(s-127-c_e)).  c_e is a per-expert power of two
//       chosen at upload so every scaled weight of a block within 27 binades of
//       the expert's largest block is exact in fp16 (blocks further below are
//       flushed to zero); the epilogue multiplies by 2^c_e again.
//   B (N = tokens of the tile, multiple of 16, <= 128)
//     = activations as an fp16 hi + lo split (x ~= hi + lo), TMA SWIZZLE_128B;
//       two MMAs (hi, lo) per k-step accumulate into the same TMEM tile.
//   D = f32 in TMEM, 128 lanes x N columns per UMMA, double-buffered.
// Warp roles: 0 TMA producer, 1 MMA issuer (+TMEM owner), 2-17 converters,
// 18-21 epilogue.  Persistent CTAs walk the tile list (expert-major, then
// 256-row weight block, then token block).  Every mbarrier wait is bounded;
// on timeout the kernel records an error code and unwinds.
#include "amoe_internal.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace amoe {

namespace {

constexpr int BM = 128;                 // weight rows per UMMA
constexpr int MT = 2;                   // UMMAs per CTA tile along M
constexpr int BN = 128;                 // max tokens per CTA tile (UMMA N)
constexpr int BK = 64;                  // K per pipeline stage (one 128-B swizzle atom)
constexpr int STAGES = 3;               // TMA ring depth
constexpr int CSTAGES = 3;              // converted-A ring depth
constexpr int ROWS = BM * MT;           // 256 weight rows per CTA tile
constexpr int ROW_TILES = ROWS / kTileRows;  // 16 fragment tiles per stage
constexpr int B_BYTES = BN * BK * 2;         // 16 KB (hi or lo)
constexpr int ARAW_BYTES = ROW_TILES * kTileQBytes;  // 8 KB
constexpr int ASC_BYTES = ROW_TILES * kTileSBytes;   // 512 B
constexpr int ACONV_MT_BYTES = BM * BK * 2;          // 16 KB per UMMA A tile
constexpr int ACONV_BYTES = MT * ACONV_MT_BYTES;     // 32 KB
constexpr int TX_BYTES = 2 * B_BYTES + ARAW_BYTES + ASC_BYTES;
constexpr int CONV_WARPS = 16;          // converter warps (four per scheduler, one chunk per thread)
constexpr int CONV_THREADS = 32 * CONV_WARPS;
constexpr int EPI_WARP0 = 2 + CONV_WARPS;  // first of the 4 epilogue warps
constexpr int NUM_THREADS = 32 * (EPI_WARP0 + 4);
constexpr int TMEM_COLS = 512;          // 2 buffers x MT x BN
constexpr int MAX_E = 256;

constexpr size_t SMEM_BYTES = 1024 /*alignment slack*/ + CSTAGES * ACONV_BYTES +
                              STAGES * (2 * B_BYTES + ARAW_BYTES + ASC_BYTES) +
                              (2 * STAGES + 2 * CSTAGES + 4) * 8 /*barriers*/ + 16 + (MAX_E + 1) * 4;

static_assert(2 * MT * BN <= TMEM_COLS, "TMEM budget");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct TcParams {
    const int32_t *offsets;  // [E+1]
    const int32_t *cexp;     // [E]
    const float *bias;       // [E][R], GGUF row order
    int R, K, E, nrt, mblocks;
    int gate_up;
    __half *act_hi, *act_lo;  // [P][R/2]
    float *y;                 // [P][R]
    const int32_t *y_rows;    // output row of each position (NULL: the position)
    int32_t *err;
    EpReturn ret;             // expert-parallel down: rows go to their source rank
    const int32_t *gate;      // if set: nothing to do unless *gate == gate_want (path chosen on the device)
    int gate_want;
};

// ---- PTX helpers ----------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: ~1 s of clock before giving up (a correct pipeline never gets close).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > 2000000000LL) {
            atomicCAS(err, 0, code);
            return false;
        }
        if (*reinterpret_cast<volatile int32_t *>(err) != 0) return false;  // another role gave up
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
    d |= (uint64_t)1u << 16;                   // leading byte offset (16 B; unused for SW128 K-major)
    d |= (uint64_t)(1024u >> 4) << 32;         // stride byte offset
    d |= (uint64_t)1u << 46;                   // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                   // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: D f32, A/B f16, both K-major.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The hi and lo MMAs of one k-step share their A tile: the first reads it from
// shared memory into the A collector buffer, the second reuses it from there, so
// the weights cross the shared-memory port once per k-step.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b_hi, uint64_t b_lo,
                                              uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.b32 p, %5, 0;\n setp.eq.b32 q, %5, %5;\n"
        " tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %1, %2, %4, p;\n"
        " tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %1, %3, %4, q;\n}" ::"r"(d_tmem),
        "l"(a), "l"(b_hi), "l"(b_lo), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ float swiglu(float gate, float up) {
    float g = isnan(gate) ? gate : fminf(gate, 7.0f);
    float u = isnan(up) ? up : fminf(fmaxf(up, -7.0f), 7.0f);
    return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
}

struct TileInfo {
    int e, mb, nb, ntok, pos0;
};

__device__ __forceinline__ TileInfo decode_tile(int t, const int *tile_start, const int32_t *offsets, int E,
                                                int mblocks) {
    int lo = 0, hi = E - 1;  // last e with tile_start[e] <= t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tile_start[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    TileInfo ti;
    ti.e = lo;
    const int count = offsets[lo + 1] - offsets[lo];
    const int nblk = (count + BN - 1) / BN;
    const int local = t - tile_start[lo];
    ti.mb = local / nblk;
    ti.nb = local % nblk;
    ti.ntok = min(BN, count - ti.nb * BN);
    ti.pos0 = offsets[lo] + ti.nb * BN;
    (void)mblocks;
    return ti;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                   const __grid_constant__ CUtensorMap tm_araw, const __grid_constant__ CUtensorMap tm_asc,
                   TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    if (p.gate && *p.gate != p.gate_want) return;  // the other expert path runs this step
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *aconv = smem;
    uint8_t *bhi = aconv + CSTAGES * ACONV_BYTES;
    uint8_t *blo = bhi + STAGES * B_BYTES;
    uint8_t *araw = blo + STAGES * B_BYTES;
    uint8_t *asc = araw + STAGES * ARAW_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(asc + STAGES * ASC_BYTES);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *cfull = bars + 2 * STAGES, *cempty = cfull + CSTAGES;
    uint64_t *afull = cempty + CSTAGES, *aempty = afull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(aempty + 2);
    int *tile_start = reinterpret_cast<int *>(tmem_slot + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = p.E;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1 + CONV_THREADS);  // MMA commit + every converter thread
        }
        for (int c = 0; c < CSTAGES; ++c) {
            mbar_init(cfull + c, CONV_THREADS);
            mbar_init(cempty + c, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(afull + b, 1);
            mbar_init(aempty + b, 128);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2 && lane == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            tile_start[e] = acc;
            const int count = p.offsets[e + 1] - p.offsets[e];
            acc += ((count + BN - 1) / BN) * p.mblocks;
        }
        tile_start[E] = acc;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = tile_start[E];
    const int nkt = p.K / BK;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int it = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                const TileInfo ti = decode_tile(t, tile_start, p.offsets, E, p.mblocks);
                const int rt0 = ti.e * p.nrt + ti.mb * ROW_TILES;
                for (int kt = 0; kt < nkt; ++kt, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(empty + s, ph ^ 1, p.err, 1)) goto done;
                    mbar_arrive_expect_tx(full + s, TX_BYTES);
                    tma_load_2d(bhi + s * B_BYTES, &tm_bhi, full + s, kt * BK, ti.pos0);
                    tma_load_2d(blo + s * B_BYTES, &tm_blo, full + s, kt * BK, ti.pos0);
                    tma_load_3d(araw + s * ARAW_BYTES, &tm_araw, full + s, 0, kt, rt0);
                    tma_load_3d(asc + s * ASC_BYTES, &tm_asc, full + s, 0, kt, rt0);
                }
            }
            // drain: the last fills must land before the CTA may exit
            for (int s = 0; s < STAGES && it > 0; ++s) {
                const int last = it - 1 - s;
                if (last < 0) break;
                if (!mbar_wait(full + (last % STAGES), (last / STAGES) & 1, p.err, 2)) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, cit = 0, tc = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
                const TileInfo ti = decode_tile(t, tile_start, p.offsets, E, p.mblocks);
                const int n16 = (ti.ntok + 15) & ~15;
                const uint32_t idesc = idesc_f16(BM, n16);
                const int buf = tc & 1;
                if (!mbar_wait(aempty + buf, ((tc >> 1) & 1) ^ 1, p.err, 3)) goto done;
                tc_fence_after();
                for (int kt = 0; kt < nkt; ++kt, ++it, ++cit) {
                    const int s = it % STAGES, cs = cit % CSTAGES;
                    if (!mbar_wait(full + s, (it / STAGES) & 1, p.err, 4)) goto done;
                    if (!mbar_wait(cfull + cs, (cit / CSTAGES) & 1, p.err, 5)) goto done;
                    tc_fence_after();
                    const uint32_t bh = smem_u32(bhi + s * B_BYTES), bl = smem_u32(blo + s * B_BYTES);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint32_t d = tmem_base + (uint32_t)((buf * MT + m) * BN);
                        const uint32_t a = smem_u32(aconv + cs * ACONV_BYTES + m * ACONV_MT_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            umma_f16_pair(d, sw128_desc(a + kk * 32), sw128_desc(bh + kk * 32),
                                          sw128_desc(bl + kk * 32), idesc, (kt | kk) != 0);
                        }
                    }
                    umma_commit(empty + s);
                    umma_commit(cempty + cs);
                }
                umma_commit(afull + buf);
            }
        }
    } else if (warp < EPI_WARP0) {
        // ---------------- converters: raw MXFP4 tiles -> fp16 SW128 A tiles ----------------
        // Thread ct owns one 16-B lane chunk (g, c) of fragment tile rtl in every stage:
        // 8 nibble bytes of rows g and g+8 per block; all its offsets are fixed.
        static_assert(ROW_TILES * 32 == CONV_THREADS, "one chunk per converter thread");
        const int ct = threadIdx.x - 64;
        const int rtl = ct >> 5, ln = ct & 31, g = ln >> 2, c = ln & 3;
        const int src_q = rtl * kTileQBytes + ln * 16, src_s = rtl * kTileSBytes + 4 * g;
        int dst[2][2];  // [h][bb]: byte offset of the 16-B chunk in a converted stage
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = (rtl & 7) * 16 + g + 8 * h;  // row within the UMMA A tile (row & 7 == g)
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                // odd rows store their blocks in the other order, so the 8 lanes of each
                // quarter-warp hit 8 distinct 16-B slots of the swizzled rows
                const int b = bb ^ (g & 1);
                dst[h][bb] = (rtl >> 3) * ACONV_MT_BYTES + row * 128 + (((4 * b + c) ^ g) << 4);
            }
        }
        int it = 0, cit = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            const TileInfo ti = decode_tile(t, tile_start, p.offsets, E, p.mblocks);
            // fp16 biased exponent of 2^(s-127-c_e) is s - K with K = c_e + 112 (<= 28 by the
            // choice of c_e); bytes at or below K are flushed to zero (>27 binades below the
            // expert's largest block), 255 is NaN.
            const int K = p.cexp[ti.e] + 112;
            const uint32_t kb = (uint32_t)(K >= 0 ? K : -K) * 0x01010101u;
            for (int kt = 0; kt < nkt; ++kt, ++it, ++cit) {
                const int s = it % STAGES, cs = cit % CSTAGES;
                if (!mbar_wait(full + s, (it / STAGES) & 1, p.err, 6)) goto done;
                if (!mbar_wait(cempty + cs, ((cit / CSTAGES) & 1) ^ 1, p.err, 7)) goto done;
                const uint4 raw = *reinterpret_cast<const uint4 *>(araw + s * ARAW_BYTES + src_q);
                const uint32_t scl = *reinterpret_cast<const uint32_t *>(asc + s * ASC_BYTES + src_s);
                const uint32_t eb = K >= 0 ? __vsubus4(scl, kb) : __vadd4(scl, kb);
                const uint32_t nan4 = __vcmpeq4(scl, 0xffffffffu);
                uint8_t *dstage = aconv + cs * ACONV_BYTES;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
#pragma unroll
                    for (int bb = 0; bb < 2; ++bb) {
                        const int b = bb ^ (g & 1);
                        const uint32_t w = b ? (h ? raw.w : raw.z) : (h ? raw.y : raw.x);
                        const uint32_t sel = (uint32_t)(2 * h + b) * 0x0101u + 0x4040u;  // byte j -> halves 0, 2
                        uint32_t sc = __byte_perm(eb, 0u, sel) << 10;
                        if (__byte_perm(nan4, 0u, sel)) sc = 0x7e007e00u;
                        uint4 o = e2m1x8_to_f16(w);
                        o.x = hmul2_bits(o.x, sc);
                        o.y = hmul2_bits(o.y, sc);
                        o.z = hmul2_bits(o.z, sc);
                        o.w = hmul2_bits(o.w, sc);
                        *reinterpret_cast<uint4 *>(dstage + dst[h][bb]) = o;
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(cfull + cs);
                mbar_arrive(empty + s);
            }
        }
    } else {
        // ---------------- epilogue: TMEM -> bias (+SwiGLU) -> global ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int g16 = lane & 15;   // row within its 16-row fragment tile
        const bool gate_lane = g16 < 8;
        int tc = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
            const TileInfo ti = decode_tile(t, tile_start, p.offsets, E, p.mblocks);
            const int buf = tc & 1;
            if (!mbar_wait(afull + buf, (tc >> 1) & 1, p.err, 8)) goto done;
            tc_fence_after();
            const float scale = ldexpf(1.0f, p.cexp[ti.e]);
            const float *bias = p.bias + (size_t)ti.e * p.R;
            const int n16 = (ti.ntok + 15) & ~15;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int rrow = ti.mb * ROWS + m * BM + 32 * q + lane;  // tile-order weight row
                const bool row_ok = rrow < p.R;
                // gate_up: a gate lane (tile row g) and the up lane 8 above it share pair pr;
                // the gate lane finishes even tokens and the up lane odd ones.
                const int pr = (rrow >> 4) * 8 + (g16 & 7);
                float bg = 0.0f, bu = 0.0f, bd = 0.0f;
                if (row_ok) {
                    if (p.gate_up) {
                        bg = bias[2 * pr];
                        bu = bias[2 * pr + 1];
                    } else {
                        bd = bias[rrow];
                    }
                }
                for (int col0 = 0; col0 < n16; col0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)((buf * MT + m) * BN + col0), v);
                    if (p.gate_up) {
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const float x0 = __uint_as_float(v[2 * jj]) * scale;
                            const float x1 = __uint_as_float(v[2 * jj + 1]) * scale;
                            const float from_up = __shfl_down_sync(0xffffffffu, x0, 8);
                            const float from_gate = __shfl_up_sync(0xffffffffu, x1, 8);
                            const float gv = gate_lane ? x0 : from_gate;
                            const float uv = gate_lane ? from_up : x1;
                            const int tok = col0 + 2 * jj + (gate_lane ? 0 : 1);
                            if (tok < ti.ntok && row_ok) {
                                const float a = swiglu(gv + bg, uv + bu);
                                const __half hi = __float2half_rn(a);
                                const __half lo = __float2half_rn(a - __half2float(hi));
                                const size_t o = (size_t)(ti.pos0 + tok) * (p.R / 2) + pr;
                                p.act_hi[o] = hi;
                                p.act_lo[o] = lo;
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int tok = col0 + j;
                            if (tok < ti.ntok && row_ok)
                                ep_out_row(p.y, p.y_rows, p.ret, ti.pos0 + tok, p.R)[rrow] =
                                    __uint_as_float(v[j]) * scale + bd;
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(aempty + buf);
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
    ep_return_done(p.ret);  // expert-parallel down: outputs are in the source ranks' windows
}

// Per-expert exponent bias for the fp16 weight expansion: c = max finite E8M0
// byte - 140, so the largest scaled E2M1 value (6 * 2^13) still fits fp16 and
// the block scales within 27 binades of it are normal fp16 numbers.
__global__ void cexp_kernel(const uint8_t *__restrict__ s_plane, size_t bytes_per_expert, int32_t *out) {
    __shared__ int mx;
    if (threadIdx.x == 0) mx = -1;
    __syncthreads();
    const uint8_t *s = s_plane + (size_t)blockIdx.x * bytes_per_expert;
    int local = -1;
    for (size_t i = threadIdx.x; i < bytes_per_expert; i += blockDim.x) {
        const int b = s[i];
        if (b != 255 && b > local) local = b;
    }
    atomicMax(&mx, local);
    __syncthreads();
    if (threadIdx.x == 0) out[blockIdx.x] = mx < 0 ? 0 : mx - 140;
}

// ---- host side ----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_num_sms = 0;

bool get_encode() {
    std::call_once(g_encode_once, []() {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

cudaError_t encode(CUtensorMap *tm, CUtensorMapDataType dt, int rank, void *base, const cuuint64_t *dims,
                   const cuuint64_t *strides_bytes, const cuuint32_t *box, CUtensorMapSwizzle sw) {
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(tm, dt, (cuuint32_t)rank, base, dims, strides_bytes, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

struct Maps {
    CUtensorMap bhi, blo, araw, asc;
};

cudaError_t make_maps(Maps &m, const __half *b_hi, const __half *b_lo, int K, int P_cap, const uint8_t *q,
                      const uint8_t *s, int E, int R) {
    const int nkt = K / BK, nrt = R / kTileRows;
    cuuint64_t bdims[2] = {(cuuint64_t)K, (cuuint64_t)P_cap};
    cuuint64_t bstr[1] = {(cuuint64_t)K * 2};
    cuuint32_t bbox[2] = {BK, BN};
    cudaError_t e = encode(&m.bhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)b_hi, bdims, bstr, bbox,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    e = encode(&m.blo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)b_lo, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    cuuint64_t qdims[3] = {kTileQBytes / 4, (cuuint64_t)nkt, (cuuint64_t)E * nrt};
    cuuint64_t qstr[2] = {kTileQBytes, (cuuint64_t)nkt * kTileQBytes};
    cuuint32_t qbox[3] = {kTileQBytes / 4, 1, ROW_TILES};
    e = encode(&m.araw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, (void *)q, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e != cudaSuccess) return e;
    cuuint64_t sdims[3] = {kTileSBytes, (cuuint64_t)nkt, (cuuint64_t)E * nrt};
    cuuint64_t sstr[2] = {kTileSBytes, (cuuint64_t)nkt * kTileSBytes};
    cuuint32_t sbox[3] = {kTileSBytes, 1, ROW_TILES};
    return encode(&m.asc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void *)s, sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_NONE);
}

struct TcScratch {
    __half *xp_hi, *xp_lo;  // [P_cap][H]
    int32_t *err;
};

TcScratch carve(void *base, int max_pairs, int H) {
    TcScratch t;
    uint8_t *b = static_cast<uint8_t *>(base);
    const size_t plane = ((size_t)max_pairs * H * 2 + 255) & ~size_t(255);
    t.xp_hi = reinterpret_cast<__half *>(b);
    t.xp_lo = reinterpret_cast<__half *>(b + plane);
    t.err = reinterpret_cast<int32_t *>(b + 2 * plane);
    return t;
}

}  // namespace

size_t tc_scratch_bytes(int max_pairs, int H, int I) {
    (void)I;
    const size_t plane = ((size_t)max_pairs * H * 2 + 255) & ~size_t(255);
    return 2 * plane + 256;
}

bool tc_supported() {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) return false;
    if (!g_num_sms) cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    return get_encode();
}

cudaError_t launch_cexp(const uint8_t *s_plane, size_t bytes_per_expert, int E, int32_t *out, cudaStream_t st) {
    cexp_kernel<<<E, 256, 0, st>>>(s_plane, bytes_per_expert, out);
    return cudaGetLastError();
}

int32_t *tc_error_flag(void *tc_scratch, int max_pairs, int H) { return carve(tc_scratch, max_pairs, H).err; }

void tc_rows(void *tc_scratch, int max_pairs, int H, __half **xp_hi, __half **xp_lo) {
    const TcScratch t = carve(tc_scratch, max_pairs, H);
    *xp_hi = t.xp_hi;
    *xp_lo = t.xp_lo;
}

cudaError_t launch_tc_experts(const Dims &d, const LayerDev &L, const int32_t *offsets, const __half *b_hi,
                              const __half *b_lo, int rows_cap, __half *act_hi, __half *act_lo, float *y,
                              const int32_t *y_rows, int32_t *err, cudaStream_t st, StageHook hook,
                              void *hook_arg, int *launches, const EpReturn *ret, const int32_t *gate,
                              int gate_want) {
    if (!tc_supported()) return cudaErrorNotSupported;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int grid = g_num_sms > 0 ? g_num_sms : 148;
    cudaError_t e;
    // gate_up + SwiGLU
    {
        Maps m;
        e = make_maps(m, b_hi, b_lo, d.H, rows_cap, L.gu_q, L.gu_s, d.E, 2 * d.I);
        if (e != cudaSuccess) return e;
        TcParams p{};
        p.offsets = offsets;
        p.cexp = L.gu_cexp;
        p.bias = L.gu_b;
        p.R = 2 * d.I;
        p.K = d.H;
        p.E = d.E;
        p.nrt = p.R / kTileRows;
        p.mblocks = (p.R + ROWS - 1) / ROWS;
        p.gate_up = 1;
        p.act_hi = act_hi;
        p.act_lo = act_lo;
        p.err = err;
        p.gate = gate;
        p.gate_want = gate_want;
        tc_gemm_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(m.bhi, m.blo, m.araw, m.asc, p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ++*launches;
        if (hook) hook(hook_arg, 2);
    }
    // down
    {
        Maps m;
        e = make_maps(m, act_hi, act_lo, d.I, rows_cap, L.dn_q, L.dn_s, d.E, d.H);
        if (e != cudaSuccess) return e;
        TcParams p{};
        p.offsets = offsets;
        p.cexp = L.dn_cexp;
        p.bias = L.dn_b;
        p.R = d.H;
        p.K = d.I;
        p.E = d.E;
        p.nrt = p.R / kTileRows;
        p.mblocks = (p.R + ROWS - 1) / ROWS;
        p.gate_up = 0;
        p.y = y;
        p.y_rows = y_rows;
        p.err = err;
        if (ret) p.ret = *ret;
        p.gate = gate;
        p.gate_want = gate_want;
        tc_gemm_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(m.bhi, m.blo, m.araw, m.asc, p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ++*launches;
        if (hook) hook(hook_arg, 3);
    }
    return cudaSuccess;
}

cudaError_t launch_tc_forward(const Dims &d, const LayerDev &L, const RouteOut &r, int T, __half *act_hi,
                              __half *act_lo, float *y, void *tc_scratch, int max_pairs, cudaStream_t st,
                              StageHook hook, void *hook_arg, int *launches) {
    if (!tc_supported()) return cudaErrorNotSupported;
    const TcScratch ts = carve(tc_scratch, max_pairs, d.H);
    *launches = 0;
    // 1. stable token->expert positions and the expert-sorted fp16 hi/lo copy of the
    //    normalized rows (the gate_up B operand)
    cudaError_t e = launch_scatter(d, T, r, true, ts.xp_hi, ts.xp_lo, st);
    if (e != cudaSuccess) return e;
    ++*launches;
    if (hook) hook(hook_arg, 5);
    // 2. the two grouped GEMMs
    int n = 0;
    e = launch_tc_experts(d, L, r.offsets, ts.xp_hi, ts.xp_lo, max_pairs, act_hi, act_lo, y, nullptr, ts.err, st,
                          hook, hook_arg, &n);
    *launches += n;
    return e;
}

}  // namespace amoe
