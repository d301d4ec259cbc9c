// tc_ptx.cuh -- device helpers shared by the TMA and tensor-core kernels
// (decode.cu, gemm_bs.cu, gemv.cu): mbarriers, TMA and bulk copies, tcgen05
// operand descriptors and TMEM loads, cross-CTA flags, and the host-side
// tensor-map encoder.
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

// K-major SWIZZLE_64B operand (rows of 64 bytes = 128 packed E2M1 values):
// 8-row groups 512 B apart; a K offset of 64 elements is +32 bytes.
static __device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(512u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)4u << 61;
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

// 8 consecutive TMEM columns of this warp's 32 lanes, waited for in the same statement.
static __device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive TMEM columns of this warp's 32 lanes, waited for in the same statement.
static __device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 40 consecutive TMEM columns of this warp's 32 lanes (32 + 8), one wait for both loads.
static __device__ __forceinline__ void tmem_ld40(uint32_t taddr, float (&v)[40]) {
    uint32_t r[40];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%40];\n"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%32,%33,%34,%35,%36,%37,%38,%39}, [%41];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39])
        : "r"(taddr), "r"(taddr + 32u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 40; ++i) v[i] = __uint_as_float(r[i]);
}

// 80 consecutive TMEM columns of this warp's 32 lanes (32 + 32 + 16), one wait
// for all three loads.
static __device__ __forceinline__ void tmem_ld80(uint32_t taddr, float (&v)[80]) {
    uint32_t r[80];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%80];\n"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%81];\n"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79}, "
        "[%82];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
          "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
          "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79])
        : "r"(taddr), "r"(taddr + 32u), "r"(taddr + 64u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 80; ++i) v[i] = __uint_as_float(r[i]);
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

// GPT-OSS clamped SwiGLU in f32 with Go's math.Min/Max NaN semantics
// (primitives.go:144-146): NaN propagates.
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

}  // namespace bs
}  // namespace amoe
