// decode.cu -- K9: the expert stage of a decode step (T <= kDecodeMaxTokens)
// as ONE cooperative persistent kernel on the block-scaled tensor cores:
//
//   phase 1  gate_up = x . W_gu^T + b_gu -> clamped SwiGLU      (layer.go:139-148, 175;
//                                                                primitives.go:138-149)
//   phase 2  y = act . W_dn^T + b_dn                             (layer.go:179-187)
//   phase 3  out = residual + f32(sum_s f64(w_s) * f64(y_s))      (layer.go:109-121)
//
// No grid-wide barrier: a finished tile publishes a per-launch flag; an
// expert's down tiles wait for that expert's gate_up tiles, and each 128-row
// slice of the combine waits for the down tiles of those rows.
//
// The MXFP4 experts are consumed as stored: tcgen05.mma kind::mxf8f6f4 with
// A = E2M1 weights straight from the TMA planes (TMA unpacks the nibbles into
// the tensor core's 16-byte-aligned shared-memory format) and the GGUF E8M0
// bytes as the hardware block scales of A.  The activations enter as four
// E4M3 terms x ~= sum_j q_j * 2^(e - 4j) per 32-element block (B scale
// factors), one term per MMA column, so one MMA computes all four partial
// products; the epilogue adds the columns.  Four terms carry ~16 significant
// bits; accumulation is f32 in TMEM.
//
// Work split: all selected experts' 128-row weight tiles of a phase form one
// sequence of 128-element K boxes; CTA b takes the contiguous run
// [n*b/G, n*(b+1)/G) (stream-K), so every SM streams the same number of
// bytes.  A tile cut between CTAs is summed by whichever of its CTAs arrives
// last (self-resetting counter), adding the partials in CTA order
// (deterministic).  The down boxes do not depend on phase 1, so the producers
// stream them early; only their activation operand waits for its expert.
//
// Roles: warps 0-3 TMA producers (stage i filled by warp i % 4), warp 4 MMA
// issuer and TMEM owner, warps 5-8 epilogue (TMEM lane quadrants 1, 2, 3, 0),
// warp 9 watches the gate_up tiles this CTA's down boxes depend on.
// Every wait is bounded (~1 s of clock): it records a code in the error flag
// and the kernel winds down.
#include "amoe_internal.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace amoe {

namespace {

// Copies issued by one warp are serviced one after another (~0.4 us each at
// load), so four producer warps fill the ring's stages round-robin.
constexpr int kProdWarps = 4;
constexpr int kMmaWarp = kProdWarps;
constexpr int kEpiWarp0 = kProdWarps + 1;
constexpr int kEpiWarps = 4;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kWatchWarp = kEpiWarp0 + kEpiWarps;  // polls other CTAs' tile flags
constexpr int kDecThreads = (kWatchWarp + 1) * 32;
constexpr int kNMax = 16;                       // MMA N: up to 4 tokens x 4 terms
constexpr int kBoxes = 2;                       // 128-element K boxes per pipeline stage
constexpr int kMaxStages = 6;
constexpr uint32_t kABytes = 128 * 128;         // unpacked A box in shared memory
constexpr uint32_t kAPacked = 128 * 64;         // its bytes in global memory (TMA transaction size)
constexpr uint32_t kTmemCols = 128;             // 2 accumulators + 16 scale columns per stage
constexpr long long kWaitLimit = 2000000000LL;  // clock cycles (~1 s)
constexpr size_t kSmemBudget = 225 * 1024;
constexpr int kTilesPerSlot = 64;               // tile counters per slot and phase

// Stage: kBoxes A boxes | their scale chunks | kBoxes B boxes | their scale chunks.
__host__ __device__ constexpr uint32_t b_box_bytes(int nt) { return (uint32_t)nt * 128; }
__host__ __device__ constexpr uint32_t stage_bytes(int nt) {
    return (kBoxes * kABytes + kBoxes * 512 + kBoxes * b_box_bytes(nt) + kBoxes * 512 + 1023) & ~1023u;
}

struct DecodeParams {
    const float *residual;
    float *out;
    const __half *x_hi, *x_lo;  // [T][H] normalized rows
    const int32_t *perm_pair, *offsets, *active, *inv;
    const float *topk_w;
    const uint8_t *gu_tsf, *dn_tsf;
    const float *gu_b, *dn_b;
    uint8_t *act_q;             // [S][16][Ip] E4M3 terms of each slot's activation rows
    uint8_t *act_sf;            // [S][Ip/128][512] their scale-factor chunks
    float *y;                   // [P][H]
    float *partial;             // [G][2][128][kNMax]
    uint32_t *cnt;              // [2][S][kTilesPerSlot] self-resetting tile counters
    unsigned *tflag;            // [2][S][kTilesPerSlot] launch epoch of each finished tile
    DecodeBarrier *bar;
    int32_t *err;
    int T, H, I, E, k, Hp, Ip, S;
    int stages;
    int N;                      // MMA N (8 or 16)
};

struct DecLayout {
    uint32_t ring, b1, sfb1, offs, act, perm, inv, w, ready, xchg, bars, tmem_slot, total;
};

__host__ __device__ inline DecLayout dec_layout(int T, int Hp, int E, int k, int stages, int nt) {
    DecLayout L;
    uint32_t o = 0;
    L.ring = o;
    o += (uint32_t)stages * stage_bytes(nt);
    L.b1 = o;
    o += (uint32_t)(Hp / 128) * b_box_bytes(nt);
    L.sfb1 = o;
    o += (uint32_t)(Hp / 128) * 512;
    L.offs = o;
    o += (uint32_t)(E + 1) * 4;
    L.act = o;
    o += (uint32_t)(E + 1) * 4;
    const uint32_t P = (uint32_t)(T * k);
    L.perm = o;
    o += P * 4;
    L.inv = o;
    o += P * 4;
    L.w = o;
    o += P * 4;
    L.ready = o;  // [min(E, P)] phase-2 operand of the slot complete
    o += (uint32_t)(E < (int)P ? E : (int)P) * 4;
    L.xchg = o;
    o += 64;  // block maxima of the activation quantization + flags
    o = (o + 7u) & ~7u;
    L.bars = o;
    o += (2u * (uint32_t)stages + 5u) * 8;
    L.tmem_slot = o;
    o += 16;
    L.total = o + 1024;  // base alignment slack
    return L;
}

// ---- PTX helpers -------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int code) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > kWaitLimit) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_3d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major SWIZZLE_128B operand: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Scale-factor chunk for tcgen05.cp: 32 rows of 16 B, no swizzle, 8-row core
// matrices 128 B apart.
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(128u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

__device__ __forceinline__ void sf_copy(uint32_t tmem_col, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc_sf(saddr)) : "memory");
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled: A E2M1, B E4M3, both
// K-major, E8M0 scales, M = 128, N = n; sf_id picks the byte (32-element
// block) of the scale words.
__device__ __forceinline__ uint32_t idesc_bs(uint32_t sf_id, int n) {
    return (sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
           (sf_id << 29);
}

__device__ __forceinline__ void umma_bs(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                        uint32_t sfb) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// E4M3 with round-to-nearest, saturating to +-448 (NaN stays NaN).
__device__ __forceinline__ uint32_t to_e4m3(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(r) : "f"(v));
    return r & 0xffu;
}

__device__ __forceinline__ float from_e4m3(uint32_t b) {
    uint32_t h;
    const uint16_t two = (uint16_t)(b | (b << 8));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(two));
    return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// Scale exponent of a 32-element block with largest magnitude amax: amax /
// 2^e0 lies in [128, 256) (inside E4M3's 448); term j uses 2^(e0 - 4j).
__device__ __forceinline__ int block_exp(float amax) {
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127;
    return e - 7;
}

__device__ __forceinline__ int term_scale_byte(int e0, int j) { return max(e0 - 4 * j + 127, 1); }

// Four E4M3 terms of v for block exponent e0: v ~= sum_j q_j 2^(e0 - 4j), each
// term rounding what the previous ones left.  Scale bytes clamp at 1 (2^-126):
// such blocks are ~2^-120 small.
__device__ __forceinline__ uint32_t quant4(float v, int e0) {
    uint32_t out = 0;
    float r = v;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int eb = term_scale_byte(e0, j);
        const float s = __uint_as_float((uint32_t)eb << 23);
        const float inv = __uint_as_float((uint32_t)(254 - eb) << 23);
        const uint32_t q = to_e4m3(r * inv);
        r -= from_e4m3(q) * s;
        out |= q << (8 * j);
    }
    return out;
}

// GPT-OSS clamped SwiGLU in f32 with Go's math.Min/Max NaN semantics
// (primitives.go:144-146): NaN propagates.
__device__ __forceinline__ float swiglu(float gate, float up) {
    float g = isnan(gate) ? gate : fminf(gate, 7.0f);
    float u = isnan(up) ? up : fminf(fmaxf(up, -7.0f), 7.0f);
    return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
}

// Cross-CTA dependencies are per tile: the CTA that finishes a tile publishes
// the launch epoch in the tile's flag (values grow with every launch, so no
// flag is ever reset), and whoever needs the tile polls for it.  The launch is
// cooperative, so every producing CTA is resident while others wait.
__device__ __forceinline__ void publish(unsigned *flag, unsigned v) {
    __threadfence();
    st_release(flag, v);
}

// Warp-wide: returns once flags[0..n) all reached v (lane j polls j, j+32, ...).
__device__ void wait_flags(const unsigned *flags, int n, unsigned v, int lane, int32_t *err, int code) {
    const long long t0 = clock64();
    for (int j = lane; j < n; j += 32) {
        while ((int)(ld_acquire(flags + j) - v) < 0) {
            if (clock64() - t0 > kWaitLimit) {
                atomicCAS(err, 0, code);
                return;
            }
            __nanosleep(32);
        }
    }
}

// A phase's geometry: the whole phase's box sequence and this CTA's run.
struct Phase {
    int nmt, nkb;  // 128-row tiles per expert, 128-element K boxes per tile
    int nbox;      // boxes of the whole phase
    int lo, hi;    // this CTA's boxes [lo, hi)
};

__device__ __forceinline__ int run_start(int nbox, int b, int G) { return (int)((long long)nbox * b / G); }

__device__ __forceinline__ Phase make_phase(int nmt, int nkb, int n_active) {
    Phase ph;
    ph.nmt = nmt;
    ph.nkb = nkb;
    ph.nbox = n_active * nmt * nkb;
    ph.lo = run_start(ph.nbox, blockIdx.x, gridDim.x);
    ph.hi = run_start(ph.nbox, blockIdx.x + 1, gridDim.x);
    return ph;
}

// Largest b whose run starts at or before box x (the CTA whose run holds x).
__device__ __forceinline__ int cta_of_box(int x, int nbox, int G) {
    return (int)(((long long)(x + 1) * G - 1) / nbox);
}

// Walks a CTA's run in pipeline stages: up to kBoxes consecutive boxes of one
// tile per stage, indices advanced without division.
struct Walker {
    int x, hi, nkb, nmt;
    int slot, mt, kb;  // position of box x
    __device__ __forceinline__ Walker(const Phase &q) : x(q.lo), hi(q.hi), nkb(q.nkb), nmt(q.nmt) {
        const int tile = q.nkb > 0 ? q.lo / q.nkb : 0;
        kb = q.lo - tile * q.nkb;
        slot = q.nmt > 0 ? tile / q.nmt : 0;
        mt = tile - slot * q.nmt;
    }
    __device__ __forceinline__ bool more() const { return x < hi; }
    __device__ __forceinline__ int boxes() const { return min(kBoxes, min(nkb - kb, hi - x)); }
    __device__ __forceinline__ void advance(int nb) {
        x += nb;
        kb += nb;
        if (kb == nkb) {
            kb = 0;
            if (++mt == nmt) {
                mt = 0;
                ++slot;
            }
        }
    }
};

template <int NT>
__launch_bounds__(kDecThreads, 1) __global__
    void decode_kernel(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dn,
                       const __grid_constant__ CUtensorMap tm_act, DecodeParams p) {
    constexpr uint32_t kBBox = b_box_bytes(NT);
    constexpr uint32_t kStage = stage_bytes(NT);
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    const DecLayout lay = dec_layout(p.T, p.Hp, p.E, p.k, p.stages, NT);
    uint8_t *ring = sm + lay.ring;
    uint8_t *b1 = sm + lay.b1;
    uint8_t *sfb1 = sm + lay.sfb1;
    int32_t *offs_s = reinterpret_cast<int32_t *>(sm + lay.offs);
    int32_t *act_s = reinterpret_cast<int32_t *>(sm + lay.act);
    int32_t *perm_s = reinterpret_cast<int32_t *>(sm + lay.perm);
    int32_t *inv_s = reinterpret_cast<int32_t *>(sm + lay.inv);
    float *w_s = reinterpret_cast<float *>(sm + lay.w);
    float *xchg = reinterpret_cast<float *>(sm + lay.xchg);
    volatile int *last_flag = reinterpret_cast<volatile int *>(sm + lay.xchg + 32);
    volatile int *ready_s = reinterpret_cast<volatile int *>(sm + lay.ready);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + lay.bars);
    uint64_t *empty = full + p.stages;
    uint64_t *accfull = empty + p.stages;  // [2]
    uint64_t *accempty = accfull + 2;      // [2]
    uint64_t *b1ready = accempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + lay.tmem_slot);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, P = p.T * p.k, R = p.stages, G = gridDim.x;
    const unsigned epoch = p.bar->epoch[blockIdx.x] + 1u;

    if (tid == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_gu)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_dn)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_act)) : "memory");
    }
    for (int i = tid; i <= E; i += kDecThreads) {
        offs_s[i] = p.offsets[i];
        act_s[i] = p.active[i];
    }
    for (int i = tid; i < P; i += kDecThreads) {
        perm_s[i] = p.perm_pair[i];
        inv_s[i] = p.inv[i];
        w_s[i] = p.topk_w[i];
    }
    for (int i = tid; i < (E < P ? E : P); i += kDecThreads) ready_s[i] = 0;
    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accfull + b, 1);
            mbar_init(accempty + b, kEpiThreads);
        }
        mbar_init(b1ready, kEpiThreads);
        *last_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_active = act_s[E];
    const int nkb1 = p.Hp / 128, nkb2 = p.Ip / 128;
    const int nmt1 = 2 * p.I / 128, nmt2 = (p.H + 127) / 128;
    const Phase ph[2] = {make_phase(nmt1, nkb1, n_active), make_phase(nmt2, nkb2, n_active)};

    if (warp < kProdWarps) {
        // ---------------- producers: stage i is warp i % kProdWarps's ----------------
        if (lane == 0) {
            int i = 0;
            bool dead = false;
            for (int f = 0; f < 2 && !dead; ++f) {
                const CUtensorMap *tma = f ? &tm_dn : &tm_gu;
                const uint8_t *tsf = f ? p.dn_tsf : p.gu_tsf;
                const int nmt = ph[f].nmt, nkb = ph[f].nkb;
                for (Walker w(ph[f]); w.more(); ++i) {
                    const int s = i % R, nb = w.boxes();
                    if (i % kProdWarps != warp) {
                        w.advance(nb);
                        continue;
                    }
                    if (i >= R && !mbar_wait(empty + s, ((i / R) - 1) & 1, p.err, 30)) {
                        dead = true;
                        break;
                    }
                    const int e = act_s[w.slot];
                    uint8_t *st = ring + (size_t)s * kStage;
                    mbar_expect_tx(full + s, (uint32_t)nb * (kAPacked + 512 + (f ? kBBox + 512 : 0)));
                    const int box0 = (e * nmt + w.mt) * nkb + w.kb;  // box-tiled plane: row origin 128 * box
                    for (int b = 0; b < nb; ++b) tma_2d(st + b * kABytes, tma, full + s, 0, (box0 + b) * 128);
                    bulk_g2s(st + kBoxes * kABytes, tsf + (((size_t)e * nmt + w.mt) * nkb + w.kb) * 512, nb * 512,
                             full + s);
                    if (f) {
                        // the slot's activation operand: ready once all its gate_up tiles are done
                        if (ready_s[w.slot] == 0) {
                            const long long t0 = clock64();
                            while (ready_s[w.slot] == 0) {
                                if (clock64() - t0 > kWaitLimit) {
                                    atomicCAS(p.err, 0, 31);
                                    break;
                                }
                                __nanosleep(64);
                            }
                        }
                        uint8_t *bst = st + kBoxes * (kABytes + 512);
                        for (int b = 0; b < nb; ++b) tma_3d(bst + b * kBBox, &tm_act, full + s, (w.kb + b) * 128, 0, w.slot);
                        bulk_g2s(bst + kBoxes * kBBox, p.act_sf + ((size_t)w.slot * nkb2 + w.kb) * 512, nb * 512,
                                 full + s);
                    }
                    w.advance(nb);
                }
            }
        }
    } else if (warp == kWatchWarp) {
        // ---------------- watcher: which phase-2 slots may load their operand ----------------
        const Phase &q = ph[1];
        if (q.hi > q.lo) {
            const int per_slot = q.nmt * q.nkb;
            for (int slot = q.lo / per_slot; slot <= (q.hi - 1) / per_slot; ++slot) {
                wait_flags(p.tflag + (size_t)slot * kTilesPerSlot, nmt1, epoch, lane, p.err, 36);
                __syncwarp();
                if (lane == 0) ready_s[slot] = 1;
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        // The whole warp walks the stages (warp-uniform descriptors stay in
        // uniform registers); one elected lane issues the tcgen05 operations.
        uint32_t elected;
        asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(elected));
        uint32_t idesc[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) idesc[kk] = idesc_bs(kk, NT);
        const uint32_t ring_a = smem_u32(ring), b1_a = smem_u32(b1), sfb1_a = smem_u32(sfb1);
        int i = 0, seg = 0;
        bool ok = mbar_wait(b1ready, 0, p.err, 32);
        for (int f = 0; f < 2 && ok; ++f) {
            Walker w(ph[f]);
            while (w.more() && ok) {
                // one segment: this CTA's boxes of one tile
                const int buf = seg & 1;
                if (!mbar_wait(accempty + buf, ((seg >> 1) & 1) ^ 1, p.err, 33)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * NT);
                uint32_t acc = 0;
                for (;;) {
                    const int s = i % R, nb = w.boxes();
                    if (!mbar_wait(full + s, (i / R) & 1, p.err, 34)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = ring_a + (uint32_t)s * kStage;
                    const uint32_t sfa = tmem + 32u + 16u * (uint32_t)s, sfb = sfa + 8u;
                    for (int b = 0; b < nb; ++b) {
                        const uint32_t bsrc = f ? st + kBoxes * (kABytes + 512) + b * kBBox : b1_a + (uint32_t)(w.kb + b) * kBBox;
                        const uint32_t sfb_src = f ? st + kBoxes * (kABytes + 512 + kBBox) + 512 * b
                                                   : sfb1_a + (uint32_t)(w.kb + b) * 512;
                        const uint32_t a0 = st + b * kABytes;
                        if (elected) {
                            sf_copy(sfa + 4 * b, st + kBoxes * kABytes + 512 * b);
                            sf_copy(sfb + 4 * b, sfb_src);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                umma_bs(d, desc_sw128(a0 + 32 * kk), desc_sw128(bsrc + 32 * kk), idesc[kk], acc,
                                        sfa + 4 * b, sfb + 4 * b);
                                acc = 1u;
                            }
                        }
                        acc = 1u;
                    }
                    if (elected) umma_commit(empty + s);
                    __syncwarp();
                    ++i;
                    const bool tile_end = w.kb + nb == w.nkb;
                    w.advance(nb);
                    if (tile_end || !w.more()) break;
                }
                if (elected) umma_commit(accfull + buf);
                __syncwarp();
                ++seg;
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int et = tid - kEpiWarp0 * 32;  // 0..127
        const int quad = warp & 3;         // TMEM lane quadrant
        const int row = quad * 32 + lane;  // row of the 128-row tile this thread owns
        // (a) phase-1 operand: every token's normalized row as four E4M3 terms.
        //     Item = 8 elements; four consecutive lanes hold one 32-element block.
        {
            const int n8 = p.Hp / 8, total = p.T * n8;
            constexpr int kBatch = 4;  // items per thread whose loads are in flight together
            for (int base0 = 0; base0 < total; base0 += kBatch * kEpiThreads) {
              uint4 hv[kBatch], lv[kBatch];
#pragma unroll
              for (int u = 0; u < kBatch; ++u) {
                const int it = base0 + u * kEpiThreads + et;
                const int t = it / n8, k0 = 8 * (it - t * n8);
                hv[u] = lv[u] = make_uint4(0, 0, 0, 0);
                if (it < total && k0 < p.H) {
                    hv[u] = *reinterpret_cast<const uint4 *>(p.x_hi + (size_t)t * p.H + k0);
                    lv[u] = *reinterpret_cast<const uint4 *>(p.x_lo + (size_t)t * p.H + k0);
                }
              }
#pragma unroll
              for (int u = 0; u < kBatch; ++u) {
                const int it = base0 + u * kEpiThreads + et;
                const bool valid = it < total;
                const int t = valid ? it / n8 : 0, k8 = valid ? it - t * n8 : 0;
                const int k0 = 8 * k8;
                float v[8];
                float amax = 0.0f;
                const __half2 *hh = reinterpret_cast<const __half2 *>(&hv[u]);
                const __half2 *ll = reinterpret_cast<const __half2 *>(&lv[u]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 a = __half22float2(hh[u]), bb = __half22float2(ll[u]);
                    v[2 * u] = a.x + bb.x;
                    v[2 * u + 1] = a.y + bb.y;
                    amax = fmaxf(amax, fmaxf(fabsf(v[2 * u]), fabsf(v[2 * u + 1])));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                if (!valid) continue;
                const int e0 = block_exp(amax);
                uint32_t lo4[4] = {0, 0, 0, 0}, hi4[4] = {0, 0, 0, 0};  // [term]: elements 0-3, 4-7
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t q = quant4(v[i], e0);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t byte = ((q >> (8 * j)) & 0xffu) << (8 * (i & 3));
                        if (i < 4) lo4[j] |= byte;
                        else hi4[j] |= byte;
                    }
                }
                const int box = k0 / 128, chunk = (k0 % 128) / 16, half = (k0 % 16) / 8;
                uint8_t *bx = b1 + (size_t)box * kBBox;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = 4 * t + j;  // B row: token t, term j (SWIZZLE_128B: chunk ^ row % 8)
                    uint8_t *dst = bx + (n >> 3) * 1024 + (n & 7) * 128 + ((chunk ^ (n & 7)) << 4) + 8 * half;
                    *reinterpret_cast<uint2 *>(dst) = make_uint2(lo4[j], hi4[j]);
                    if ((k8 & 3) == 0) sfb1[(size_t)box * 512 + n * 16 + (k0 % 128) / 32] = (uint8_t)term_scale_byte(e0, j);
                }
              }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(b1ready);
        }
        // (b) the CTA's tile segments, phase 1 then phase 2
        float *part = p.partial + (size_t)blockIdx.x * 2 * 128 * kNMax;
        int seg = 0;
        for (int f = 0; f < 2; ++f) {
            const Phase &q = ph[f];
            int x = q.lo;
            while (x < q.hi) {
                const int tile = x / q.nkb;
                const int tbeg = tile * q.nkb, tend_full = tbeg + q.nkb;
                const int tend = min(tend_full, q.hi);
                const int slot = tile / q.nmt, mt = tile - slot * q.nmt;
                const int e = act_s[slot];
                const int base = offs_s[e];
                int m_e = offs_s[e + 1] - base;
                if (m_e > p.T) m_e = p.T;  // at most one pair per token (distinct top-k experts)
                // this row's bias, loaded while the MMAs run
                const int grp = row >> 4, j16 = row & 15;
                const bool gate_lane = j16 < 8;
                const int pr = 64 * mt + 8 * grp + (j16 & 7);  // phase 1: SwiGLU pair = activation column
                const int h = 128 * mt + row;                   // phase 2: output row
                float bias = 0.0f;
                if (f == 0) bias = p.gu_b[(size_t)e * 2 * p.I + 2 * pr + (gate_lane ? 0 : 1)];
                else if (h < p.H) bias = p.dn_b[(size_t)e * p.H + h];
                const int buf = seg & 1;
                float v[NT];
                mbar_wait(accfull + buf, (seg >> 1) & 1, p.err, 35);
                tc_fence_after();
                {
                    float t16[16];
                    tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * NT), t16);
#pragma unroll
                    for (int c = 0; c < NT; ++c) v[c] = t16[c];
                }
                tc_fence_before();
                mbar_arrive(accempty + buf);
                ++seg;
                const bool whole = x == tbeg && tend == tend_full;
                const bool head = x == q.lo;
                x = tend;
                if (!whole) {
                    // a split tile: the last of its CTAs to arrive adds the partials in CTA order
                    const int b_first = cta_of_box(tbeg, q.nbox, G), b_last = cta_of_box(tend_full - 1, q.nbox, G);
                    float *mine = part + (size_t)(head ? 0 : 1) * 128 * kNMax + (size_t)row * kNMax;
#pragma unroll
                    for (int c = 0; c < NT; c += 4)
                        __stcg(reinterpret_cast<float4 *>(mine + c), make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]));
                    __threadfence();
                    epi_bar();
                    if (et == 0) {
                        unsigned nseg = 0;
                        for (int b = b_first; b <= b_last; ++b)
                            nseg += run_start(q.nbox, b + 1, G) > run_start(q.nbox, b, G) ? 1u : 0u;
                        const unsigned old =
                            atomicInc(p.cnt + ((size_t)f * p.S + slot) * kTilesPerSlot + mt, nseg - 1u);
                        *last_flag = old == nseg - 1u;
                    }
                    epi_bar();
                    const bool last = *last_flag != 0;
                    epi_bar();
                    if (!last) continue;
                    __threadfence();
#pragma unroll
                    for (int c = 0; c < NT; ++c) v[c] = 0.0f;
                    for (int b = b_first; b <= b_last; ++b) {
                        const int blo = run_start(q.nbox, b, G), bhi = run_start(q.nbox, b + 1, G);
                        if (bhi <= blo) continue;  // empty run: no piece
                        // CTA b's piece: the head of its run if the run starts inside this tile
                        const float *src =
                            p.partial + ((size_t)b * 2 + (blo >= tbeg ? 0 : 1)) * 128 * kNMax + (size_t)row * kNMax;
#pragma unroll
                        for (int c = 0; c < NT; c += 4) {
                            const float4 t4 = __ldcg(reinterpret_cast<const float4 *>(src + c));
                            v[c] += t4.x;
                            v[c + 1] += t4.y;
                            v[c + 2] += t4.z;
                            v[c + 3] += t4.w;
                        }
                    }
                }
                // ---- finalize the tile ----
                if (f == 0) {
                    // rows 16g'+j (j < 8) hold the gate of pair 8g'+j, row +8 its up row
                    for (int g = 0; g < m_e; ++g) {
                        const int t = perm_s[base + g] / p.k;
                        float val = 0.0f;
#pragma unroll
                        for (int c = 0; c < NT; c += 4)
                            if (c / 4 == t) val = v[c] + v[c + 1] + v[c + 2] + v[c + 3];
                        val += bias;
                        const float up = __shfl_down_sync(0xffffffffu, val, 8);
                        const float a = gate_lane ? swiglu(val, up) : 0.0f;
                        // the 32-pair block of this row: rows 0-63 (quadrants 0, 1) or 64-127 (2, 3)
                        float m = gate_lane ? fabsf(a) : 0.0f;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                        if (lane == 0) xchg[quad] = m;
                        epi_bar();
                        const float amax = fmaxf(xchg[quad & 2], xchg[(quad & 2) + 1]);
                        epi_bar();
                        const int e0 = block_exp(amax);
                        if (gate_lane) {
                            const uint32_t q4 = quant4(a, e0);
                            uint8_t *dst = p.act_q + ((size_t)slot * 16 + 4 * g) * p.Ip + pr;
#pragma unroll
                            for (int j = 0; j < 4; ++j) dst[(size_t)j * p.Ip] = (uint8_t)(q4 >> (8 * j));
                        }
                        if (lane == 0 && (quad & 1) == 0) {  // one writer per block of 32 pairs
                            const int blk = 2 * mt + (quad >> 1);
                            uint8_t *sfd = p.act_sf + ((size_t)slot * (p.Ip / 128) + blk / 4) * 512;
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                sfd[(4 * g + j) * 16 + (blk % 4)] = (uint8_t)term_scale_byte(e0, j);
                        }
                    }
                } else if (h < p.H) {
#pragma unroll
                    for (int c = 0; c < NT; c += 4)
                        if (c / 4 < m_e) p.y[(size_t)(base + c / 4) * p.H + h] = v[c] + v[c + 1] + v[c + 2] + v[c + 3] + bias;
                }
                // the tile is complete: publish it to the CTAs that consume it
                __threadfence();
                epi_bar();
                if (et == 0) publish(p.tflag + ((size_t)f * p.S + slot) * kTilesPerSlot + mt, epoch);
            }
        }
        // (c) slot-order combine with the residual: CTA b owns output rows
        //     128b..128b+127 and waits only for those rows' down tiles
        if ((int)blockIdx.x < nmt2) {
            const int mt2 = blockIdx.x;
            if (et < 32) {
                for (int s0 = 0; s0 < n_active; s0 += 32) {
                    const int ns = min(32, n_active - s0);
                    if (lane < ns)
                        wait_flags(p.tflag + ((size_t)p.S + s0 + lane) * kTilesPerSlot + mt2, 1, epoch, 0, p.err, 37);
                }
            }
            epi_bar();
            const int h = 128 * mt2 + et;
            if (h < p.H) {
                for (int t = 0; t < p.T; ++t) {
                    double m = 0.0;
                    for (int s = 0; s < p.k; ++s)
                        m += (double)w_s[t * p.k + s] * (double)__ldcg(p.y + (size_t)inv_s[t * p.k + s] * p.H + h);
                    p.out[(size_t)t * p.H + h] = p.residual[(size_t)t * p.H + h] + (float)m;
                }
            }
        }
        if (et == 0) p.bar->epoch[blockIdx.x] = epoch;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---- host side -------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

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

// Box-tiled E2M1 plane: rows of 128 packed 4-bit elements (64 B), 128-row boxes.
cudaError_t map_boxes(CUtensorMap *tm, void *base, uint64_t rows) {
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {64};
    cuuint32_t box[2] = {128, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, base, dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 3-D map over [z][y][x]: x packed 4-bit (fp4) or bytes, boxes 128 x box_y x 1,
// SWIZZLE_128B, zero fill out of bounds.
cudaError_t map3d(CUtensorMap *tm, void *base, bool fp4, uint64_t x, uint64_t y, uint64_t z, uint32_t box_y) {
    const uint64_t row_bytes = fp4 ? x / 2 : x;
    cuuint64_t dims[3] = {x, y, z};
    cuuint64_t strides[2] = {row_bytes, row_bytes * y};
    cuuint32_t box[3] = {128, box_y, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = g_encode(tm, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base,
                          dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

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

int dec_n(int T) { return 4 * T <= 8 ? 8 : 16; }

int dec_stages(int T, int Hp, int E, int k) {
    const int nt = dec_n(T);
    const DecLayout none = dec_layout(T, Hp, E, k, 0, nt);
    if (none.total >= kSmemBudget) return 0;
    const int st = (int)((kSmemBudget - none.total) / (stage_bytes(nt) + 16));
    return st > kMaxStages ? kMaxStages : st;
}

int dec_slots(const Dims &d) { return d.E < kDecodeMaxTokens * d.k ? d.E : kDecodeMaxTokens * d.k; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

size_t decode_scratch_bytes(const Dims &d, int device) {
    const int G = device >= 0 && device < 64 && caps(device).sms > 0 ? caps(device).sms : 1;
    const int S = dec_slots(d), Ip = kpad128(d.I);
    return align256((size_t)S * 16 * Ip) + align256((size_t)S * (Ip / 128) * 512) +
           align256((size_t)G * 2 * 128 * kNMax * 4) + (size_t)2 * 2 * S * kTilesPerSlot * 4;
}

cudaError_t init_decode_scratch(const Dims &d, int device, void *scratch, cudaStream_t st) {
    const int S = dec_slots(d), Ip = kpad128(d.I);
    uint8_t *b = static_cast<uint8_t *>(scratch);
    cudaError_t e = cudaMemsetAsync(b, 0, decode_scratch_bytes(d, device), st);
    if (e != cudaSuccess) return e;
    // activation scale bytes: 2^0 wherever no block is ever written (K padding)
    return cudaMemsetAsync(b + align256((size_t)S * 16 * Ip), 127, (size_t)S * (Ip / 128) * 512, st);
}

bool decode_supported(const Dims &d, int T, int device) {
    if (T < 1 || T > kDecodeMaxTokens || device < 0 || device >= 64) return false;
    const DecodeCaps &cp = caps(device);
    if (!cp.coop || cp.sms <= 0 || cp.sms > kDecodeMaxCtas || !get_encode()) return false;
    if ((2 * d.I) % 128 || 2 * d.I / 128 > kTilesPerSlot || (d.H + 127) / 128 > kTilesPerSlot) return false;
    return dec_stages(T, kpad128(d.H), d.E, d.k) >= 2;
}

cudaError_t launch_decode(const Dims &d, const LayerDev &L, const RouteOut &r, const float *residual, int T,
                          void *scratch, float *y, float *out, DecodeBarrier *bar, int32_t *err, int device,
                          cudaStream_t st) {
    const int S = dec_slots(d), Hp = kpad128(d.H), Ip = kpad128(d.I);
    const int G = caps(device).sms;
    uint8_t *b = static_cast<uint8_t *>(scratch);
    DecodeParams p{};
    p.residual = residual;
    p.out = out;
    p.x_hi = r.x_hi;
    p.x_lo = r.x_lo;
    p.perm_pair = r.perm_pair;
    p.offsets = r.offsets;
    p.active = r.active;
    p.inv = r.inv;
    p.topk_w = r.topk_w;
    p.gu_tsf = L.gu_tsf;
    p.dn_tsf = L.dn_tsf;
    p.gu_b = L.gu_b;
    p.dn_b = L.dn_b;
    p.act_q = b;
    b += align256((size_t)S * 16 * Ip);
    p.act_sf = b;
    b += align256((size_t)S * (Ip / 128) * 512);
    p.partial = reinterpret_cast<float *>(b);
    b += align256((size_t)G * 2 * 128 * kNMax * 4);
    p.cnt = reinterpret_cast<uint32_t *>(b);
    p.tflag = reinterpret_cast<unsigned *>(p.cnt + (size_t)2 * S * kTilesPerSlot);
    p.y = y;
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
    p.stages = dec_stages(T, Hp, d.E, d.k);
    p.N = dec_n(T);
    if (p.stages < 2 || !get_encode()) return cudaErrorInvalidValue;
    CUtensorMap tm_gu, tm_dn, tm_act;
    cudaError_t e = map_boxes(&tm_gu, L.gu_tq, tq_bytes(d.E, 2 * d.I, d.H) / 64);
    if (e == cudaSuccess) e = map_boxes(&tm_dn, L.dn_tq, tq_bytes(d.E, d.H, d.I) / 64);
    if (e == cudaSuccess) e = map3d(&tm_act, p.act_q, false, (uint64_t)Ip, 16, (uint64_t)S, (uint32_t)p.N);
    if (e != cudaSuccess) return e;
    const size_t smem = dec_layout(T, Hp, d.E, d.k, p.stages, p.N).total;
    auto kern = p.N == 8 ? decode_kernel<8> : decode_kernel<16>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
    return cudaLaunchKernelEx(&cfg, kern, tm_gu, tm_dn, tm_act, p);
}

}  // namespace amoe
