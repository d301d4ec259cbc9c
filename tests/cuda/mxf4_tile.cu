// Known-answer test of the FP4 tensor-core form an expert GEMM can use: one block-scaled
// tcgen05 MMA tile (kind::mxf4, M=128, N=8 or 16, K=128 as two K=64 MMAs).  A and B are packed
// E2M1 (two values per byte, low nibble first) loaded by TMA as 64-byte rows with SWIZZLE_64B,
// K-major, as the MXFP4 box planes are stored; E8M0 scales, one per 32 elements, go smem->TMEM
// with tcgen05.cp 32x128b.warpx4 in the box planes' chunk layout ((r%32)*16 + (r/32)*4 + j);
// the scale-factor id of an MMA is the byte index of its first scale (0, then 2).
// Usage: mxf4_tile N unused second_sf_id.  Prints the largest error against a float64 CPU
// product, relative to the sum of the absolute products of each dot product.  One CTA; every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <vector>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("CUDA %s at %d: %s\n", #x, __LINE__, cudaGetErrorString(e)); exit(1);} } while (0)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
        if (ok) return true;
        if (clock64() - t0 > 2000000000LL) { atomicCAS(err, 0, code); return false; }
    }
}
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {  // K-major, 64-B rows, 8-row groups 512 B apart
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(512u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)4u << 61;  // SWIZZLE_64B
    return d;
}
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {  // no swizzle, 8x16B core matrices 128 B apart
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(128u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    return d;
}

struct Args { int N; int sf2; int *err; float *D; };

__global__ void __launch_bounds__(128, 1) k(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                            const uint8_t *sfa_g, const uint8_t *sfb_g, Args a) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = sm;                 // 128 rows x 64 B packed
    uint8_t *sB = sm + 16384;         // N rows x 64 B packed (<= 2 KB)
    uint8_t *sSFA = sm + 16384 + 2048;
    uint8_t *sSFB = sSFA + 512;
    uint64_t *bar = reinterpret_cast<uint64_t *>(sSFB + 512);
    uint64_t *mbar = bar + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < 512; i += 128) { sSFA[i] = sfa_g[i]; sSFB[i] = sfb_g[i]; }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(smem_u32(tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot;
    if (tid == 0) {
        const uint32_t tx = 128u * 64u + (uint32_t)a.N * 64u;
        asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_u32(bar)), "r"(tx) : "memory");
        asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(sA)), "l"((uint64_t)&tmA), "r"(0), "r"(0), "r"(smem_u32(bar)) : "memory");
        asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(sB)), "l"((uint64_t)&tmB), "r"(0), "r"(0), "r"(smem_u32(bar)) : "memory");
        if (mbar_wait(bar, 0, a.err, 1)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // scale factors -> TMEM columns 16..19 (A) and 20..23 (B)
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem + 16), "l"(desc_sf(smem_u32(sSFA))));
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem + 20), "l"(desc_sf(smem_u32(sSFB))));
            for (int kk = 0; kk < 2; ++kk) {
                const uint32_t sf = kk ? (uint32_t)a.sf2 : 0u;  // scale-factor id: the row's byte pair
                const uint32_t idesc = (sf << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.N >> 3) << 17) | (1u << 23) |
                                       ((128u >> 4) << 24) | (sf << 29);
                const uint64_t ad = desc_sw64(smem_u32(sA) + 32 * kk), bd = desc_sw64(smem_u32(sB) + 32 * kk);
                asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                             " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}"
                             ::"r"(tmem), "l"(ad), "l"(bd), "r"(idesc), "r"((uint32_t)kk), "r"(tmem + 16), "r"(tmem + 20) : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar)) : "memory");
        }
    }
    __syncwarp();
    mbar_wait(mbar, 0, a.err, 2);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // lanes 32w..32w+31, 16 columns
    uint32_t v[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(tmem + ((uint32_t)(32 * warp) << 16)));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    const int row = tid;
    for (int n = 0; n < a.N; ++n) a.D[row * 16 + n] = __uint_as_float(v[n]);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem));
}

static float e2m1(int n) { static const float t[8] = {0, .5f, 1, 1.5f, 2, 3, 4, 6}; return (n & 8 ? -1.f : 1.f) * t[n & 7]; }

int main(int argc, char **argv) {
    const int N = argc > 1 ? atoi(argv[1]) : 8;
    const int sf2 = argc > 3 ? atoi(argv[3]) : 2;
    if (N != 8 && N != 16) { printf("N must be 8 or 16 (16 accumulator columns are read back)\n"); return 1; }
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void **)&enc, cudaEnableDefault, &q));
    srand(7);
    std::vector<uint8_t> A(128 * 64), Bm(N * 64), sfa(512), sfb(512);
    std::vector<int> sa(128 * 4), sbv(N * 4);
    for (auto &x : A) x = rand() & 0xff;
    for (auto &x : Bm) x = rand() & 0xff;
    for (int r = 0; r < 128; ++r) for (int j = 0; j < 4; ++j) sa[r * 4 + j] = 120 + rand() % 14;
    for (int n = 0; n < N; ++n) for (int j = 0; j < 4; ++j) sbv[n * 4 + j] = 120 + rand() % 14;
    memset(sfa.data(), 127, 512); memset(sfb.data(), 127, 512);
    for (int r = 0; r < 128; ++r) for (int j = 0; j < 4; ++j) sfa[(r % 32) * 16 + (r / 32) * 4 + j] = sa[r * 4 + j];
    for (int n = 0; n < N; ++n) for (int j = 0; j < 4; ++j) sfb[(n % 32) * 16 + (n / 32) * 4 + j] = sbv[n * 4 + j];
    uint8_t *dA, *dB, *dSa, *dSb; float *dD; int *dErr;
    CK(cudaMalloc(&dA, A.size())); CK(cudaMalloc(&dB, 4096)); CK(cudaMalloc(&dSa, 512)); CK(cudaMalloc(&dSb, 512));
    CK(cudaMalloc(&dD, 128 * 16 * 4)); CK(cudaMalloc(&dErr, 4));
    CK(cudaMemcpy(dA, A.data(), A.size(), cudaMemcpyHostToDevice)); CK(cudaMemset(dB, 0, 4096));
    CK(cudaMemcpy(dB, Bm.data(), Bm.size(), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dSa, sfa.data(), 512, cudaMemcpyHostToDevice)); CK(cudaMemcpy(dSb, sfb.data(), 512, cudaMemcpyHostToDevice));
    CK(cudaMemset(dD, 0, 128 * 16 * 4)); CK(cudaMemset(dErr, 0, 4));
    CUtensorMap tmA, tmB;
    cuuint64_t dimA[2] = {64, 128}, strA[1] = {64};
    cuuint32_t boxA[2] = {64, 128}, es[2] = {1, 1};
    CUresult r1 = enc(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, dA, dimA, strA, boxA, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    cuuint64_t dimB[2] = {64, (cuuint64_t)N}, strB[1] = {64};
    cuuint32_t boxB[2] = {64, (cuuint32_t)N};
    CUresult r2 = enc(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, dB, dimB, strB, boxB, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    printf("encode A %d B %d\n", (int)r1, (int)r2);
    if (r1 || r2) return 1;
    Args a{N, sf2, dErr, dD};
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 34816));
    k<<<1, 128, 34816>>>(tmA, tmB, dSa, dSb, a);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    int err = 0; CK(cudaMemcpy(&err, dErr, 4, cudaMemcpyDeviceToHost));
    std::vector<float> D(128 * 16); CK(cudaMemcpy(D.data(), dD, D.size() * 4, cudaMemcpyDeviceToHost));
    // f32 accumulation of 128 exact products: |err| <= 128 * 2^-24 * sum |a_i b_i|, so
    // the error is measured against that sum (a near-cancelling dot product has a
    // tiny |ref| but the same absolute rounding)
    double maxerr = 0; int bad = 0;
    for (int r = 0; r < 128; ++r)
        for (int n = 0; n < N; ++n) {
            double ref = 0, mag = 0;
            for (int kq = 0; kq < 128; ++kq) {
                int nib = (A[r * 64 + kq / 2] >> (4 * (kq & 1))) & 15;
                int nb = (Bm[n * 64 + kq / 2] >> (4 * (kq & 1))) & 15;
                const double t = (double)e2m1(nib) * ldexp(1.0, sa[r * 4 + kq / 32] - 127) * (double)e2m1(nb) *
                                 ldexp(1.0, sbv[n * 4 + kq / 32] - 127);
                ref += t;
                mag += fabs(t);
            }
            double g = D[r * 16 + n];
            double err = fabs(g - ref) / (mag > 0 ? mag : 1.0);
            if (err > maxerr) maxerr = err;
            if (err > 1e-5 && bad < 8) { printf("mismatch r %d n %d gpu %g ref %g\n", r, n, g, ref); ++bad; }
        }
    printf("N %d second sf id %d err %d max scaled err %.3e\n", N, sf2, err, maxerr);
    return 0;
}
