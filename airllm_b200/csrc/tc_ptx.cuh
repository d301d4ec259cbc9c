// tc_ptx.cuh -- device helpers shared by the block-scaled tensor-core kernels
// (decode.cu, gemm_bs.cu): mbarriers, TMA and bulk copies, tcgen05 MMA /
// scale-factor copy / TMEM load, the E4M3 multi-term activation quantizer,
// cross-CTA flags, and the host-side tensor-map encoders.
#pragma once

#include "amoe_internal.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace amoe {
namespace bs {

constexpr long long kWaitLimit = 2000000000LL;  // clock cycles (~1 s)

// ---- PTX helpers -------------------------------------------------------------------
static __device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

static __device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int code) {
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

static __device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

static __device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

static __device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

static __device__ __forceinline__ void tma_3d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

static __device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *tm, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

static __device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

static __device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
static __device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major SWIZZLE_128B operand: 8-row groups 1024 B apart.
static __device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
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
static __device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(128u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

static __device__ __forceinline__ void sf_copy(uint32_t tmem_col, uint32_t saddr) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(desc_sf(saddr)) : "memory");
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled: A E2M1, B E4M3, both
// K-major, E8M0 scales, M = 128, N = n; sf_id picks the byte (32-element
// block) of the scale words.
static __device__ __forceinline__ uint32_t idesc_bs(uint32_t sf_id, int n) {
    return (sf_id << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
           (sf_id << 29);
}

static __device__ __forceinline__ void umma_bs(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc, uint32_t sfa,
                                        uint32_t sfb) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}

static __device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

static __device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
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


// 32 consecutive TMEM columns of this warp's 32 lanes, waited for in the same
// statement (the registers are only defined after tcgen05.wait::ld).
static __device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

static __device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

static __device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// E4M3 with round-to-nearest, saturating to +-448 (NaN stays NaN).
static __device__ __forceinline__ uint32_t to_e4m3(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(r) : "f"(v));
    return r & 0xffu;
}

static __device__ __forceinline__ float from_e4m3(uint32_t b) {
    uint32_t h;
    const uint16_t two = (uint16_t)(b | (b << 8));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(two));
    return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// Scale exponent of a 32-element block with largest magnitude amax: amax /
// 2^e0 lies in [128, 256) (inside E4M3's 448); term j uses 2^(e0 - 4j).
static __device__ __forceinline__ int block_exp(float amax) {
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127;
    return e - 7;
}

static __device__ __forceinline__ int term_scale_byte(int e0, int j) { return max(e0 - 4 * j + 127, 1); }

// Four E4M3 terms of v for block exponent e0: v ~= sum_j q_j 2^(e0 - 4j), each
// term rounding what the previous ones left.  Scale bytes clamp at 1 (2^-126):
// such blocks are ~2^-120 small.
static __device__ __forceinline__ uint32_t quant4(float v, int e0) {
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

// The scales of a block's four terms (2^(e0 - 4j), clamped as in quant4) and
// their reciprocals.
struct TermScales {
    float s[4], inv[4];
};

static __device__ __forceinline__ TermScales term_scales(int e0) {
    TermScales t;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int eb = term_scale_byte(e0, j);
        t.s[j] = __uint_as_float((uint32_t)eb << 23);
        t.inv[j] = __uint_as_float((uint32_t)(254 - eb) << 23);
    }
    return t;
}

// quant4 on two elements at once (bit-identical): q[j] holds term j of a in its
// low byte and of b in its high byte.
static __device__ __forceinline__ void quant4_pair(float a, float b, const TermScales &t, uint32_t (&q)[4]) {
    float r0 = a, r1 = b;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint16_t p;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p) : "f"(r1 * t.inv[j]), "f"(r0 * t.inv[j]));
        uint32_t h;
        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(p));
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h));
        r0 = fmaf(-f.x, t.s[j], r0);
        r1 = fmaf(-f.y, t.s[j], r1);
        q[j] = p;
    }
}

// GPT-OSS clamped SwiGLU in f32 with Go's math.Min/Max NaN semantics
// (primitives.go:144-146): NaN propagates.
// (value, expert) order of the reference's stable descending sort
// (moe.go:20-27): larger logit first, ties to the lower expert id, NaN last,
// invalid entries (expert < 0) after everything.
static __device__ __forceinline__ bool topk_better(float v1, int e1, float v2, int e2) {
    if (e2 < 0) return e1 >= 0;
    if (e1 < 0) return false;
    const bool n1 = isnan(v1), n2 = isnan(v2);
    if (n1 || n2) return n1 == n2 ? e1 < e2 : n2;
    return v1 > v2 || (v1 == v2 && e1 < e2);
}

static __device__ __forceinline__ float swiglu(float gate, float up) {
    float g = isnan(gate) ? gate : fminf(gate, 7.0f);
    float u = isnan(up) ? up : fminf(fmaxf(up, -7.0f), 7.0f);
    return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
}

// Cross-CTA dependencies are per tile: the CTA that finishes a tile publishes
// the launch epoch in the tile's flag (values grow with every launch, so no
// flag is ever reset), and whoever needs the tile polls for it.  The launch is
// cooperative, so every producing CTA is resident while others wait.
static __device__ __forceinline__ void publish(unsigned *flag, unsigned v) {
    __threadfence();
    st_release(flag, v);
}

// Warp-wide: returns once flags[0..n) all reached v (lane j polls j, j+32, ...).
static __device__ void wait_flags(const unsigned *flags, int n, unsigned v, int lane, int32_t *err, int code) {
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


// ---- host side ------------------------------------------------------------------

inline PFN_cuTensorMapEncodeTiled_v12000 &encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    return fn;
}

inline bool get_encode() {
    static std::once_flag once;
    std::call_once(once, []() {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode_fn() = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return encode_fn() != nullptr;
}

// Box-tiled E2M1 plane: rows of 128 packed 4-bit elements (64 B), 128-row boxes.
inline cudaError_t map_boxes(CUtensorMap *tm, void *base, uint64_t rows) {
    cuuint64_t dims[2] = {128, rows};
    cuuint64_t strides[1] = {64};
    cuuint32_t box[2] = {128, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn()(tm, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, base, dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// 3-D map over [z][y][x]: x packed 4-bit (fp4) or bytes, boxes 128 x box_y x 1,
// SWIZZLE_128B, zero fill out of bounds.
inline cudaError_t map3d(CUtensorMap *tm, void *base, bool fp4, uint64_t x, uint64_t y, uint64_t z, uint32_t box_y) {
    const uint64_t row_bytes = fp4 ? x / 2 : x;
    cuuint64_t dims[3] = {x, y, z};
    cuuint64_t strides[2] = {row_bytes, row_bytes * y};
    cuuint32_t box[3] = {128, box_y, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = encode_fn()(tm, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base,
                          dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}


}  // namespace bs
}  // namespace amoe
