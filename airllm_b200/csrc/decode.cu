// decode.cu -- K9: the expert stage of a decode step (T <= kDecodeMaxTokens
// tokens) as ONE cooperative persistent kernel:
//
//   phase 1  gate_up = x . W_gu^T + b_gu -> clamped SwiGLU      (layer.go:139-148, 175;
//                                                                primitives.go:138-149)
//   -------- grid barrier (every act row written)
//   phase 2  y = act . W_dn^T + b_dn                             (layer.go:179-187)
//   -------- grid barrier (every y row written)
//   phase 3  out = residual + f32(sum_s f64(w_s) * f64(y_s))      (layer.go:109-121)
//
// Why one kernel: at decode sizes each separate launch is dominated by its
// ramp-up, its tail and a few dependent memory round trips, not by its bytes.
// Here one CTA per SM streams a balanced, contiguous run of 16-row weight
// tiles (whole row tiles; gate_up tiles of every selected expert first, then
// down tiles) through a ring of shared-memory stages filled by one producer
// lane with cp.async.bulk.  The down tiles do not depend on phase 1, so the
// producer keeps HBM busy straight through the grid barrier; only the MMAs
// wait for it.
//
// Arithmetic is the GEMV kernel's (gemv.cu): each MXFP4 byte becomes an f16x2
// A-fragment with one cvt.rn.f16x2.e2m1x2; activations ride as the n=8 columns
// of mma.sync.m16n8k16 as an fp16 hi + lo split; the E8M0 block scale is
// applied to each 32-value block's f32 partial.  A stage's 16 compute warps
// take every 16th k-tile of the row tile and meet in shared memory in a fixed
// order (deterministic).
//
// Waits: every mbarrier wait and the grid barrier give up after ~1 s of clock,
// record a code in the error flag and carry on, so the kernel always ends.
#include "amoe_internal.cuh"

#include <mutex>

namespace amoe {

namespace {

constexpr int kDecWarps = 16;                      // compute warps
constexpr int kDecThreads = (kDecWarps + 1) * 32;  // + one producer warp
constexpr int kDecComputeThreads = kDecWarps * 32;
constexpr int kDecMaxStages = 8;
constexpr int kDecRed = 4;                         // reduction buffers in flight
constexpr size_t kDecSmemBudget = 220 * 1024;
constexpr long long kWaitLimit = 2000000000LL;     // clock cycles (~1 s)

struct DecodeParams {
    const float *residual;
    float *out;
    const __half *x_hi, *x_lo;  // [T][H] normalized rows
    const int32_t *perm_pair, *offsets, *active, *inv;
    const float *topk_w;
    const uint8_t *gu_q, *gu_s, *dn_q, *dn_s;
    const float *gu_b, *dn_b;
    __half *act_hi, *act_lo;  // [P][I]
    float *y;                 // [P][H]
    int T, H, I, E, k;
    int stages;
    uint32_t stage_bytes;
    int nkt_max;
    DecodeBarrier *bar;
    int32_t *err;
};

// Staged activation rows: hi rows 0..T-1, then lo rows; the stride is 2*Kmax+64
// bytes, so rows g and g+1 sit 16 banks apart (conflict-free (g, c) loads).
__host__ __device__ inline uint32_t dec_xstride(int H, int I) { return 2u * (uint32_t)(H > I ? H : I) + 64u; }

struct DecLayout {
    uint32_t ring, x, red, offs, act, perm, inv, w, bars, total;
};

__host__ __device__ inline DecLayout dec_layout(int T, int H, int I, int E, int k, int stages, uint32_t stage_bytes) {
    DecLayout L;
    uint32_t o = 0;
    L.ring = o;
    o += (uint32_t)stages * stage_bytes;
    L.x = o;
    o += 2u * (uint32_t)T * dec_xstride(H, I);
    L.red = o;
    o += (uint32_t)kDecRed * kDecWarps * 32 * 8;
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
    o = (o + 7u) & ~7u;
    L.bars = o;
    o += (2u * (uint32_t)stages + 2u * kDecRed) * 8;
    L.total = o;
    return L;
}

__host__ __device__ inline uint32_t dec_stage_bytes(int H, int I) {
    const int nkt = (H > I ? H : I) / kTileK;
    return ((uint32_t)nkt * (kTileQBytes + kTileSBytes) + 64u + 127u) & ~127u;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int32_t *err, int code) {
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

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void compute_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kDecComputeThreads) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
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

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier over the compute warps of all CTAs (the launch is cooperative,
// so every CTA is resident).  Barrier values grow monotonically across launches
// (2 per launch, from each CTA's own epoch counter), so nothing is ever reset:
// CTA b publishes its arrival in its own word; CTA 0 polls all arrival words,
// then publishes the release word that every CTA polls.  No two CTAs write the
// same word, so the barrier costs a few L2 round trips rather than a chain of
// same-address atomics.
__device__ void grid_barrier(DecodeBarrier *bar, unsigned v, int32_t *err) {
    compute_bar();
    if (threadIdx.x == 0) {
        __threadfence();
        st_release(&bar->arrive[blockIdx.x], v);
    }
    if (blockIdx.x == 0) {
        for (int j = threadIdx.x; j < (int)gridDim.x; j += kDecComputeThreads) {
            const long long t0 = clock64();
            while ((int)(ld_acquire(&bar->arrive[j]) - v) < 0) {
                if (clock64() - t0 > kWaitLimit) {
                    atomicCAS(err, 0, 32);
                    break;
                }
                __nanosleep(32);
            }
        }
        compute_bar();
        if (threadIdx.x == 0) st_release(&bar->release, v);
    }
    if (threadIdx.x == 0) {
        const long long t0 = clock64();
        while ((int)(ld_acquire(&bar->release) - v) < 0) {
            if (clock64() - t0 > kWaitLimit) {
                atomicCAS(err, 0, 32);
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
    }
    compute_bar();
}

// Per-slot facts a warp caches while it walks the CTA's tiles.
struct SlotInfo {
    int e, base, m_e, xrow;  // xrow: staged row of this lane's token (phase 1)
};

__launch_bounds__(kDecThreads, 1) __global__ void decode_kernel(DecodeParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const DecLayout lay = dec_layout(p.T, p.H, p.I, p.E, p.k, p.stages, p.stage_bytes);
    uint8_t *ring = sm + lay.ring;
    uint8_t *xs = sm + lay.x;
    float2 *red = reinterpret_cast<float2 *>(sm + lay.red);  // [kDecRed][warp][lane]
    int32_t *offs_s = reinterpret_cast<int32_t *>(sm + lay.offs);
    int32_t *act_s = reinterpret_cast<int32_t *>(sm + lay.act);
    int32_t *perm_s = reinterpret_cast<int32_t *>(sm + lay.perm);
    int32_t *inv_s = reinterpret_cast<int32_t *>(sm + lay.inv);
    float *w_s = reinterpret_cast<float *>(sm + lay.w);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + lay.bars);
    uint64_t *empty = full + p.stages;
    uint64_t *redfull = empty + p.stages;  // [kDecRed] every warp's partials written
    uint64_t *reddone = redfull + kDecRed;  // [kDecRed] the reducer has read them

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, P = p.T * p.k, R = p.stages;
    const uint32_t xstride = dec_xstride(p.H, p.I);
    // this launch's number, from the CTA's own count of completed launches
    const unsigned epoch = p.bar->epoch[blockIdx.x] + 1u;

    // routing tables (written by the router launch before this one)
    for (int i = tid; i <= E; i += kDecThreads) {
        offs_s[i] = p.offsets[i];
        act_s[i] = p.active[i];
    }
    for (int i = tid; i < P; i += kDecThreads) {
        perm_s[i] = p.perm_pair[i];
        inv_s[i] = p.inv[i];
        w_s[i] = p.topk_w[i];
    }
    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(full + s)));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(empty + s)), "r"(kDecWarps));
        }
        for (int s = 0; s < kDecRed; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(redfull + s)), "r"(kDecWarps));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(reddone + s)));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int n_active = act_s[E];
    const int nrt1 = 2 * p.I / kTileRows, nkt1 = p.H / kTileK;
    const int nrt2 = p.H / kTileRows, nkt2 = p.I / kTileK;
    const long long N1 = (long long)n_active * nrt1, N2 = (long long)n_active * nrt2;
    const int G = gridDim.x, b = blockIdx.x;
    const int lo1 = (int)(N1 * b / G), n1 = (int)(N1 * (b + 1) / G) - lo1;
    const int lo2 = (int)(N2 * b / G), n2 = (int)(N2 * (b + 1) / G) - lo2;

    if (warp == kDecWarps) {
        // ---------------- producer: one lane streams the CTA's row tiles ----------------
        if (lane == 0) {
            int i = 0;
            for (int phase = 0; phase < 2; ++phase) {
                const int n = phase ? n2 : n1, nrt = phase ? nrt2 : nrt1, nkt = phase ? nkt2 : nkt1;
                const int lo = phase ? lo2 : lo1;
                int slot = lo / nrt, rt = lo - slot * nrt;
                const uint32_t qb = (uint32_t)nkt * kTileQBytes, sb = (uint32_t)nkt * kTileSBytes;
                for (int j = 0; j < n; ++j, ++i) {
                    const int s = i % R;
                    if (i >= R && !mbar_wait_bounded(empty + s, ((i / R) - 1) & 1, p.err, 30)) return;
                    const int e = act_s[slot];
                    const size_t tile0 = ((size_t)e * nrt + rt) * nkt;
                    const uint8_t *q = (phase ? p.dn_q : p.gu_q) + tile0 * kTileQBytes;
                    const uint8_t *sc = (phase ? p.dn_s : p.gu_s) + tile0 * kTileSBytes;
                    const float *bias =
                        (phase ? p.dn_b + (size_t)e * p.H : p.gu_b + (size_t)e * 2 * p.I) + kTileRows * rt;
                    uint8_t *dst = ring + (size_t)s * p.stage_bytes;
                    asm volatile(
                        "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                            smem_u32(full + s)),
                        "r"(qb + sb + 64u)
                        : "memory");
                    bulk_g2s(dst, q, qb, full + s);
                    bulk_g2s(dst + (size_t)p.nkt_max * kTileQBytes, sc, sb, full + s);
                    bulk_g2s(dst + (size_t)p.nkt_max * (kTileQBytes + kTileSBytes), bias, 64u, full + s);
                    if (++rt == nrt) {
                        rt = 0;
                        ++slot;
                    }
                }
            }
        }
        return;
    }

    // ---------------- compute warps ----------------
    // B fragment of lane (g, c): column g = token g/2, fp16 hi (g even) or lo (g odd)
    // part of its row; D columns 2c, 2c+1 are then token c's hi and lo products.
    const int g = lane >> 2, c = lane & 3, tok = g >> 1, part = g & 1;
    {
        const int chunks = p.H / 8;
        const int total = p.T * 2 * chunks;
        for (int i = tid; i < total; i += kDecComputeThreads) {
            const int r = i / (2 * chunks), rem = i - r * 2 * chunks;
            const int lo = rem >= chunks, ch = rem - (lo ? chunks : 0);
            const uint4 v = *reinterpret_cast<const uint4 *>((lo ? p.x_lo : p.x_hi) + (size_t)r * p.H + 8 * ch);
            *reinterpret_cast<uint4 *>(xs + (size_t)(lo * p.T + r) * xstride + 16 * ch) = v;
        }
    }
    compute_bar();

    int i = 0;
    for (int phase = 0; phase < 2; ++phase) {
        const int n = phase ? n2 : n1, nrt = phase ? nrt2 : nrt1, nkt = phase ? nkt2 : nkt1;
        const int lo = phase ? lo2 : lo1;
        if (phase == 1) grid_barrier(p.bar, 2u * epoch, p.err);  // every act row of phase 1 written
        int slot = lo / nrt, rt = lo - slot * nrt;
        int cur = -1;
        SlotInfo si{0, 0, 0, 0};
        for (int j = 0; j < n; ++j, ++i) {
            if (slot != cur) {
                si.e = act_s[slot];
                si.base = offs_s[si.e];
                si.m_e = offs_s[si.e + 1] - si.base;
                if (si.m_e > p.T) {  // top-k picks distinct experts: at most one pair per token
                    if (tid == 0) atomicCAS(p.err, 0, 33);
                    si.m_e = p.T;
                }
                if (phase == 0) {
                    si.xrow = tok < si.m_e ? perm_s[si.base + tok] / p.k : 0;
                } else {
                    // restage: the slot's act rows (positions base..base+m_e-1), read from L2
                    compute_bar();
                    const int chunks = p.I / 8;
                    const int total = si.m_e * 2 * chunks;
                    for (int q = tid; q < total; q += kDecComputeThreads) {
                        const int r = q / (2 * chunks), rem = q - r * 2 * chunks;
                        const int lo_ = rem >= chunks, ch = rem - (lo_ ? chunks : 0);
                        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(
                                                   (lo_ ? p.act_lo : p.act_hi) + (size_t)(si.base + r) * p.I) +
                                               ch);
                        *reinterpret_cast<uint4 *>(xs + (size_t)(lo_ * p.T + r) * xstride + 16 * ch) = v;
                    }
                    compute_bar();
                    si.xrow = tok;
                }
                cur = slot;
            }
            const int s = i % R;
            const bool ok = mbar_wait_bounded(full + s, (i / R) & 1, p.err, 31);
            const uint8_t *stq = ring + (size_t)s * p.stage_bytes;
            const uint8_t *sts = stq + (size_t)p.nkt_max * kTileQBytes;
            const bool valid = tok < si.m_e;
            const uint8_t *xb = xs + (size_t)(part * p.T + si.xrow) * xstride + 16 * c;
            float acc0 = 0.0f, acc1 = 0.0f;  // rows g, g+8 of the tile, token c
            if (ok) {
#pragma unroll 2
                for (int kt = warp; kt < nkt; kt += kDecWarps) {
                    const uint4 qv = *reinterpret_cast<const uint4 *>(stq + kt * kTileQBytes + lane * 16);
                    float sc[4];
                    e8m0x4_to_float(*reinterpret_cast<const uint32_t *>(sts + kt * kTileSBytes + 4 * g), sc);
                    uint4 xv0 = make_uint4(0, 0, 0, 0), xv1 = make_uint4(0, 0, 0, 0);
                    if (valid) {
                        xv0 = *reinterpret_cast<const uint4 *>(xb + kt * 128);
                        xv1 = *reinterpret_cast<const uint4 *>(xb + kt * 128 + 64);
                    }
                    const uint4 a0 = e2m1x8_to_f16(qv.x), a1 = e2m1x8_to_f16(qv.y);  // block 0: rows g, g+8
                    const uint4 b0 = e2m1x8_to_f16(qv.z), b1 = e2m1x8_to_f16(qv.w);  // block 1
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    mma16816(d, a0.x, a1.x, a0.y, a1.y, xv0.x, xv0.y);
                    mma16816(d, a0.z, a1.z, a0.w, a1.w, xv0.z, xv0.w);
                    float f[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    mma16816(f, b0.x, b1.x, b0.y, b1.y, xv1.x, xv1.y);
                    mma16816(f, b0.z, b1.z, b0.w, b1.w, xv1.z, xv1.w);
                    acc0 = fmaf(d[0] + d[1], sc[0], acc0);
                    acc1 = fmaf(d[2] + d[3], sc[2], acc1);
                    acc0 = fmaf(f[0] + f[1], sc[1], acc0);
                    acc1 = fmaf(f[2] + f[3], sc[3], acc1);
                }
            }
            const int rbuf = i % kDecRed;
            if (i >= kDecRed) mbar_wait_bounded(reddone + rbuf, ((i / kDecRed) - 1) & 1, p.err, 34);
            float2 *rb = red + (size_t)rbuf * kDecWarps * 32;
            rb[warp * 32 + lane] = make_float2(acc0, acc1);
            __syncwarp();
            const bool reducer = warp == i % kDecWarps;
            if (lane == 0) {
                mbar_arrive(redfull + rbuf);
                if (!reducer) mbar_arrive(empty + s);  // done with the stage's smem
            }
            if (reducer) {
                mbar_wait_bounded(redfull + rbuf, (i / kDecRed) & 1, p.err, 35);
                float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                for (int w = 0; w < kDecWarps; ++w) {  // fixed order: deterministic
                    const float2 t = rb[w * 32 + lane];
                    v0 += t.x;
                    v1 += t.y;
                }
                const float *stb =
                    reinterpret_cast<const float *>(stq + (size_t)p.nkt_max * (kTileQBytes + kTileSBytes));
                if (c < si.m_e) {
                    const size_t pos = (size_t)si.base + c;
                    if (phase == 0) {
                        const int pr = 8 * rt + g;  // SwiGLU pair: GGUF rows 2pr (gate), 2pr+1 (up)
                        const float a = swiglu(v0 + stb[2 * g], v1 + stb[2 * g + 1]);
                        const __half hi = __float2half_rn(a);
                        const __half lo_ = __float2half_rn(a - __half2float(hi));
                        p.act_hi[pos * p.I + pr] = hi;
                        p.act_lo[pos * p.I + pr] = lo_;
                    } else {
                        const int h = kTileRows * rt + g;
                        p.y[pos * p.H + h] = v0 + stb[g];
                        p.y[pos * p.H + h + 8] = v1 + stb[g + 8];
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(reddone + rbuf);
                    mbar_arrive(empty + s);  // bias read: the stage may be refilled
                }
            }
            if (++rt == nrt) {
                rt = 0;
                ++slot;
            }
        }
    }
    grid_barrier(p.bar, 2u * epoch + 1u, p.err);  // every y row written

    // ---------------- phase 3: slot-order combine + residual ----------------
    const int H4 = p.H / 4;
    const long long items = (long long)p.T * H4;
    for (long long it = (long long)b * kDecComputeThreads + tid; it < items; it += (long long)G * kDecComputeThreads) {
        const int t = (int)(it / H4), i4 = (int)(it - (long long)t * H4);
        double m0 = 0.0, m1 = 0.0, m2 = 0.0, m3 = 0.0;
        for (int s = 0; s < p.k; ++s) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(p.y + (size_t)inv_s[t * p.k + s] * p.H) + i4);
            const double ws = (double)w_s[t * p.k + s];
            m0 += ws * (double)v.x;
            m1 += ws * (double)v.y;
            m2 += ws * (double)v.z;
            m3 += ws * (double)v.w;
        }
        const float4 r = reinterpret_cast<const float4 *>(p.residual + (size_t)t * p.H)[i4];
        reinterpret_cast<float4 *>(p.out + (size_t)t * p.H)[i4] =
            make_float4(r.x + (float)m0, r.y + (float)m1, r.z + (float)m2, r.w + (float)m3);
    }
    if (tid == 0) p.bar->epoch[blockIdx.x] = epoch;
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

int dec_stages(int T, int H, int I, int E, int k) {
    const uint32_t sb = dec_stage_bytes(H, I);
    const DecLayout none = dec_layout(T, H, I, E, k, 0, sb);
    if (none.total >= kDecSmemBudget) return 0;
    int st = (int)((kDecSmemBudget - none.total) / (sb + 16));
    return st > kDecMaxStages ? kDecMaxStages : st;
}

}  // namespace

bool decode_supported(const Dims &d, int T, int device) {
    if (T < 1 || T > kDecodeMaxTokens || device < 0 || device >= 64) return false;
    const DecodeCaps &cp = caps(device);
    return cp.coop && cp.sms > 0 && cp.sms <= kDecodeMaxCtas && dec_stages(T, d.H, d.I, d.E, d.k) >= 2;
}

cudaError_t launch_decode(const Dims &d, const LayerDev &L, const RouteOut &r, const float *residual, int T,
                          __half *act_hi, __half *act_lo, float *y, float *out, DecodeBarrier *bar, int32_t *err,
                          int device, cudaStream_t st) {
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
    p.gu_q = L.gu_q;
    p.gu_s = L.gu_s;
    p.dn_q = L.dn_q;
    p.dn_s = L.dn_s;
    p.gu_b = L.gu_b;
    p.dn_b = L.dn_b;
    p.act_hi = act_hi;
    p.act_lo = act_lo;
    p.y = y;
    p.T = T;
    p.H = d.H;
    p.I = d.I;
    p.E = d.E;
    p.k = d.k;
    p.stages = dec_stages(T, d.H, d.I, d.E, d.k);
    p.stage_bytes = dec_stage_bytes(d.H, d.I);
    p.nkt_max = (d.H > d.I ? d.H : d.I) / kTileK;
    p.bar = bar;
    p.err = err;
    if (p.stages < 2) return cudaErrorInvalidValue;
    const size_t smem = dec_layout(T, d.H, d.I, d.E, d.k, p.stages, p.stage_bytes).total;
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(caps(device).sms);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_kernel, p);
    return e;
}

}  // namespace amoe
