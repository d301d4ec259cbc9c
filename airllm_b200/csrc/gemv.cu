// gemv.cu -- K7: expert GEMV for small per-expert token counts (decode).
//
// Computes, for every selected (token, expert) pair,
//   gate_up = x . W_gu^T + b_gu  -> clamped SwiGLU (fused)   (layer.go:139-148, 175;
//                                                              primitives.go:138-149)
//   y       = act . W_dn^T + b_dn                             (layer.go:179-187)
// directly from the tiled MXFP4 planes (no dequantised copy in memory).
//
// Warps own a 16-row weight tile's K-range and stream it once from HBM; the
// per-expert tokens ride along as the n=8 columns of mma.sync.m16n8k16 (up to
// 8*NG tokens per pass).  Each MXFP4 byte becomes an f16x2 A-fragment register
// with one cvt.rn.f16x2.e2m1x2 (E2M1 values are exact in fp16); the E8M0 block
// scale is applied to the f32 partial of each 32-value block, so the scale
// never has to fit fp16's range.  Activations enter as an fp16 hi + lo split
// (x ~= hi + lo to ~2^-22 relative), two MMAs per k-step.  The kernel is
// HBM-bound: its work per weight byte is one cvt and a quarter MMA.
#include "amoe_internal.cuh"

namespace amoe {

namespace {

constexpr int kGemvWarps = 8;

struct GemvParams {
    const uint8_t *q;      // tiled nibbles
    const uint8_t *s;      // tiled scales
    const float *bias;     // [E][R] (GGUF row order)
    const __half *x_hi;    // activation rows [*][K]
    const __half *x_lo;
    const int32_t *perm_pair;  // gate_up: position -> pair id; NULL: rows are indexed by position
    const int32_t *y_rows;     // down: output row of each position; NULL: the position itself
    const int32_t *offsets;
    const int32_t *active;
    int R, K, E, k;
    int x_rows;    // staged activation rows the launch provides (NG == 1)
    int32_t *err;  // set when a bounded wait gives up (20) or an expert has more rows than staged (21)
    EpReturn ret;  // expert-parallel down: rows go to their source rank
    const int32_t *gate;  // if set: nothing to do unless *gate == gate_want (path chosen on the device)
    int gate_want;
    // outputs
    __half *act_hi, *act_lo;  // gate_up: [P][R/2]
    float *y;                 // down:    [P][R]
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// GPT-OSS clamped SwiGLU in f32 with Go's math.Min/Max NaN semantics
// (primitives.go:144-146): NaN propagates.
__device__ __forceinline__ float swiglu(float gate, float up) {
    float g = isnan(gate) ? gate : fminf(gate, 7.0f);
    float u = isnan(up) ? up : fminf(fmaxf(up, -7.0f), 7.0f);
    return g / (1.0f + expf(-1.702f * g)) * (u + 1.0f);
}

// CTA = kGemvTiles row tiles x kGemvKSplit warps each.  Each warp owns a
// contiguous K-range of one row tile: one elected lane brings that range's
// nibbles and scales to shared memory with two cp.async.bulk copies on the
// warp's mbarrier (a single round trip to HBM, no registers held), and the
// weights then serve every token pass.  The warps' partial sums meet in shared
// memory in a fixed order (deterministic).
constexpr int kGemvKSplit = 4;
constexpr int kGemvTiles = 2;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bounded mbarrier wait (about a second of clock); false after recording a timeout.
__device__ __forceinline__ bool gemv_wait(uint64_t *bar, int32_t *err) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(smem_addr(bar))
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > 2000000000LL) {
            atomicCAS(err, 0, 20);
            return false;
        }
    }
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// Staged activation rows (NG == 1): hi rows 0..x_rows-1, then the lo rows.  The
// 64-byte pad puts rows g and g+1 in opposite halves of the bank space, so the
// quarter-warp (g, c) loads of one k-step are conflict-free.
__host__ __device__ constexpr int gemv_x_stride(int K) { return 2 * K + 64; }

__host__ __device__ inline size_t gemv_weight_bytes(int K) {
    const int nkt = K / kTileK;
    const int per = (nkt + kGemvKSplit - 1) / kGemvKSplit;
    return (size_t)kGemvTiles * kGemvKSplit * per * (kTileQBytes + kTileSBytes) + kGemvTiles * kGemvKSplit * 8;
}

size_t gemv_smem_bytes(int K, int x_rows) {
    return gemv_weight_bytes(K) + (size_t)x_rows * 2 * gemv_x_stride(K);
}

template <bool GATE_UP, int NG>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(GemvParams p) {
    __shared__ float red[kGemvTiles][kGemvKSplit][NG][4][32];
    extern __shared__ __align__(128) uint8_t wsm[];
    if (p.gate && *p.gate != p.gate_want) return;  // the other expert path runs this step
    const int slot = blockIdx.y;
    const int n_active = p.active[p.E];
    if (slot >= n_active) {  // uniform for the whole CTA
        ep_return_done(p.ret);
        return;
    }
    const int e = p.active[slot];
    const int base = p.offsets[e];
    const int m_e = p.offsets[e + 1] - base;
    if (NG == 1 && min(8, m_e) > p.x_rows) {  // the launch bound T was violated: uniform exit
        if (threadIdx.x == 0) atomicCAS(p.err, 0, 21);
        ep_return_done(p.ret);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_local = warp / kGemvKSplit, ks = warp % kGemvKSplit;
    const int nrt = p.R / kTileRows;
    const int rt = blockIdx.x * kGemvTiles + tile_local;
    const bool live = rt < nrt;
    const int g = lane >> 2, c = lane & 3;
    const int nkt = p.K / kTileK;
    const int per = (nkt + kGemvKSplit - 1) / kGemvKSplit;
    const int kbeg = min(nkt, ks * per), kend = min(nkt, kbeg + per);
    // this warp's weights: [per][512] nibbles then [per][32] scales, then the mbarriers
    uint8_t *wq = wsm + (size_t)warp * per * (kTileQBytes + kTileSBytes);
    uint8_t *ws = wq + (size_t)per * kTileQBytes;
    uint64_t *bar = reinterpret_cast<uint64_t *>(wsm + (size_t)kGemvWarps * per * (kTileQBytes + kTileSBytes)) + warp;
    // NG == 1: the pass's (<= 8) activation rows are staged in shared memory once
    // per CTA, so the k-loop never waits on a global load.
    uint8_t *xs = wsm + gemv_weight_bytes(p.K);
    const int xstride = gemv_x_stride(p.K);
    const int nk = kend - kbeg;
    const bool issued = live && nk > 0;
    bool have = false;
    if (issued) {
        if (lane == 0) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)));
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            const size_t tile0 = ((size_t)e * nrt + rt) * nkt + kbeg;
            const uint32_t qb = (uint32_t)nk * kTileQBytes, sb = (uint32_t)nk * kTileSBytes;
            asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                             smem_addr(bar)),
                         "r"(qb + sb)
                         : "memory");
            bulk_g2s(wq, p.q + tile0 * kTileQBytes, qb, bar);
            bulk_g2s(ws, p.s + tile0 * kTileSBytes, sb, bar);
        }
        __syncwarp();
    }
    bool waited = false;

    for (int tok0 = 0; tok0 < m_e; tok0 += 8 * NG) {
        if (NG == 1) {
            // all threads: <= 8 rows x (hi, lo) x K halves, 16-B loads all in flight
            const int nv = min(8, m_e - tok0);
            const int chunks = p.K / 8;
            const int total = nv * 2 * chunks;
            for (int i0 = threadIdx.x; i0 < total; i0 += 4 * kGemvWarps * 32) {
                uint4 v[4];
                uint8_t *dst[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + u * kGemvWarps * 32;
                    dst[u] = nullptr;
                    if (i < total) {
                        const int r = i / (2 * chunks), rem = i - r * 2 * chunks;
                        const int lo = rem >= chunks, ch = rem - (lo ? chunks : 0);
                        const int tok = tok0 + r;
                        const int row = (GATE_UP && p.perm_pair) ? p.perm_pair[base + tok] / p.k : base + tok;
                        v[u] = *reinterpret_cast<const uint4 *>((lo ? p.x_lo : p.x_hi) + (size_t)row * p.K + 8 * ch);
                        dst[u] = xs + (size_t)(lo * p.x_rows + r) * xstride + 16 * ch;
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (dst[u]) *reinterpret_cast<uint4 *>(dst[u]) = v[u];
            }
            __syncthreads();
        }
        if (issued && !waited) {
            have = gemv_wait(bar, p.err);
            waited = true;
        }
        const __half *xh[NG];
        const __half *xl[NG];
        bool valid[NG];
        int ng_live = 0;
#pragma unroll
        for (int n = 0; n < NG; ++n) {
            const int tok = tok0 + 8 * n + g;
            valid[n] = tok < m_e;
            if (NG == 1) {
                xh[n] = reinterpret_cast<const __half *>(xs + (size_t)g * xstride) + 8 * c;
                xl[n] = reinterpret_cast<const __half *>(xs + (size_t)(p.x_rows + g) * xstride) + 8 * c;
            } else {
                int row = 0;
                if (valid[n]) row = (GATE_UP && p.perm_pair) ? p.perm_pair[base + tok] / p.k : base + tok;
                xh[n] = p.x_hi + (size_t)row * p.K + 8 * c;
                xl[n] = p.x_lo + (size_t)row * p.K + 8 * c;
            }
            if (tok0 + 8 * n < m_e) ng_live = n + 1;
        }
        float acc[NG][4];
#pragma unroll
        for (int n = 0; n < NG; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[n][i] = 0.0f;

        if (have) {
            for (int j = 0; j < nk; ++j) {
                const int kt = kbeg + j;
                const uint4 qv = *reinterpret_cast<const uint4 *>(wq + j * kTileQBytes + lane * 16);
                const uint32_t sv = *reinterpret_cast<const uint32_t *>(ws + j * kTileSBytes + 4 * g);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const uint32_t wg = b ? qv.z : qv.x;   // tile row g
                    const uint32_t wg8 = b ? qv.w : qv.y;  // tile row g+8
                    const uint32_t s0a0 = e2m1x2_to_f16x2(wg & 0xff);
                    const uint32_t s0a1 = e2m1x2_to_f16x2(wg8 & 0xff);
                    const uint32_t s0a2 = e2m1x2_to_f16x2((wg >> 8) & 0xff);
                    const uint32_t s0a3 = e2m1x2_to_f16x2((wg8 >> 8) & 0xff);
                    const uint32_t s1a0 = e2m1x2_to_f16x2((wg >> 16) & 0xff);
                    const uint32_t s1a1 = e2m1x2_to_f16x2((wg8 >> 16) & 0xff);
                    const uint32_t s1a2 = e2m1x2_to_f16x2(wg >> 24);
                    const uint32_t s1a3 = e2m1x2_to_f16x2(wg8 >> 24);
                    const float sc_g = e8m0_to_float((sv >> (8 * b)) & 0xff);
                    const float sc_g8 = e8m0_to_float((sv >> (8 * (2 + b))) & 0xff);
#pragma unroll
                    for (int n = 0; n < NG; ++n) {
                        if (n >= ng_live) break;
                        uint4 h = make_uint4(0, 0, 0, 0), l = make_uint4(0, 0, 0, 0);
                        if (valid[n]) {
                            h = *reinterpret_cast<const uint4 *>(xh[n] + kt * kTileK + b * 32);
                            l = *reinterpret_cast<const uint4 *>(xl[n] + kt * kTileK + b * 32);
                        }
                        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        mma16816(d, s0a0, s0a1, s0a2, s0a3, h.x, h.y);
                        mma16816(d, s0a0, s0a1, s0a2, s0a3, l.x, l.y);
                        mma16816(d, s1a0, s1a1, s1a2, s1a3, h.z, h.w);
                        mma16816(d, s1a0, s1a1, s1a2, s1a3, l.z, l.w);
                        acc[n][0] = fmaf(d[0], sc_g, acc[n][0]);
                        acc[n][1] = fmaf(d[1], sc_g, acc[n][1]);
                        acc[n][2] = fmaf(d[2], sc_g8, acc[n][2]);
                        acc[n][3] = fmaf(d[3], sc_g8, acc[n][3]);
                    }
                }
            }
        }
#pragma unroll
        for (int n = 0; n < NG; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[tile_local][ks][n][i][lane] = acc[n][i];
        __syncthreads();

        if (live && ks == 0) {
            // fixed-order sum of the K-slices, then the epilogue: thread holds rows
            // (g, g+8) for tokens 2c, 2c+1 of each n-group
#pragma unroll
            for (int n = 0; n < NG; ++n) {
                if (n >= ng_live) break;
                float v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float sum = red[tile_local][0][n][i][lane];
#pragma unroll
                    for (int q = 1; q < kGemvKSplit; ++q) sum += red[tile_local][q][n][i][lane];
                    v[i] = sum;
                }
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int tok = tok0 + 8 * n + 2 * c + j;
                    if (tok >= m_e) continue;
                    const int pos = base + tok;
                    if (GATE_UP) {
                        const int pr = 8 * rt + g;  // SwiGLU pair index
                        const float gate = v[j] + p.bias[(size_t)e * p.R + 2 * pr];
                        const float up = v[2 + j] + p.bias[(size_t)e * p.R + 2 * pr + 1];
                        const float a = swiglu(gate, up);
                        const __half hi = __float2half_rn(a);
                        const __half lo = __float2half_rn(a - __half2float(hi));
                        p.act_hi[(size_t)pos * (p.R / 2) + pr] = hi;
                        p.act_lo[(size_t)pos * (p.R / 2) + pr] = lo;
                    } else {
                        const int h = kTileRows * rt + g;
                        float *yrow = ep_out_row(p.y, p.y_rows, p.ret, pos, p.R);
                        yrow[h] = v[j] + p.bias[(size_t)e * p.R + h];
                        yrow[h + 8] = v[2 + j] + p.bias[(size_t)e * p.R + h + 8];
                    }
                }
            }
        }
        __syncthreads();  // red[] is rewritten by the next token pass
    }
    ep_return_done(p.ret);
}

template <bool GATE_UP>
cudaError_t launch(const GemvParams &p, int T, int max_active, cudaStream_t st) {
    const int nrt = p.R / kTileRows;
    dim3 grid((nrt + kGemvTiles - 1) / kGemvTiles, max_active);
    // T bounds the rows of any one expert
    GemvParams q = p;
    q.x_rows = T <= 8 ? T : 0;
    const size_t smem = gemv_smem_bytes(p.K, q.x_rows);
    cudaError_t e;
#define AMOE_GEMV(NG)                                                                              \
    do {                                                                                           \
        e = cudaFuncSetAttribute(gemv_kernel<GATE_UP, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)smem);                                                       \
        if (e != cudaSuccess) return e;                                                            \
        gemv_kernel<GATE_UP, NG><<<grid, kGemvWarps * 32, smem, st>>>(q);                          \
    } while (0)
    if (T <= 8) AMOE_GEMV(1);
    else if (T <= 16) AMOE_GEMV(2);
    else AMOE_GEMV(4);
#undef AMOE_GEMV
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemv_gate_up(const Dims &d, const LayerDev &L, const GemvRows &rows, int T,
                                __half *act_hi, __half *act_lo, int32_t *err, cudaStream_t st) {
    GemvParams p{};
    p.err = err;
    p.q = L.gu_q;
    p.s = L.gu_s;
    p.bias = L.gu_b;
    p.x_hi = rows.x_hi;
    p.x_lo = rows.x_lo;
    p.perm_pair = rows.perm_pair;
    p.gate = rows.gate;
    p.gate_want = rows.gate_want;
    p.offsets = rows.offsets;
    p.active = rows.active;
    p.R = 2 * d.I;
    p.K = d.H;
    p.E = d.E;
    p.k = d.k;
    p.act_hi = act_hi;
    p.act_lo = act_lo;
    const int max_active = rows.max_active;
    return launch<true>(p, T, max_active, st);
}

cudaError_t launch_gemv_down(const Dims &d, const LayerDev &L, const GemvRows &rows, int T,
                             const __half *act_hi, const __half *act_lo, float *y, int32_t *err,
                             cudaStream_t st, const EpReturn *ret) {
    GemvParams p{};
    p.err = err;
    p.q = L.dn_q;
    p.s = L.dn_s;
    p.bias = L.dn_b;
    p.x_hi = act_hi;
    p.x_lo = act_lo;
    p.perm_pair = nullptr;
    p.gate = rows.gate;
    p.gate_want = rows.gate_want;
    p.y_rows = rows.y_rows;
    p.offsets = rows.offsets;
    p.active = rows.active;
    p.R = d.H;
    p.K = d.I;
    p.E = d.E;
    p.k = d.k;
    p.y = y;
    if (ret) p.ret = *ret;
    const int max_active = rows.max_active;
    return launch<false>(p, T, max_active, st);
}

}  // namespace amoe
