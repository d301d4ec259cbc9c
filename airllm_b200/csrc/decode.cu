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
// design goal is to keep every SM streaming weight boxes from the first moment
// the routing is known to the end.
//
// Work.  A unit is one 128-row weight tile of one selected expert over its K
// range: every gate_up tile over all of K (SwiGLU needs the whole sum), every
// down tile over one half of K.  A host-built table (longest-processing-time
// first over the units' box counts, one table per number of active experts)
// gives each CTA its units: gate_up units first, then down units, both in
// slot order.  No unit is shared between CTAs, so no tile needs a cross-CTA
// reduction.  Two hand-offs cross CTAs, both through L2:
//   - the last gate_up unit of a slot to finish publishes the slot's
//     activation (a per-slot flag carrying the launch epoch); a down unit
//     waits for it before it builds its operand (its weights are already
//     streaming into the ring meanwhile);
//   - the last down unit of a 128-row output tile to finish combines that
//     tile for every token (self-resetting arrival counters).
//
// Weights.  The units' boxes stream from the TMA box planes (128 rows x 64 B of
// GGUF nibble bytes per 128-element K box, 8 KB, plus the box's 512-byte E8M0
// chunk) into a ring of 17 KB stages, two boxes per stage, one bulk copy per
// stage (a box's rows and its scale chunk are stored together); the planes hold
// every row in the 64-byte swizzle order, so the fragment loads below are free
// of bank conflicts.  There is no producer
// warp: one thread fills the first stages, and afterwards the last warp to
// finish with a stage refills its slot with the stage a ring further on (all 16
// warps then fit four per SM sub-partition with 128 registers each).  The
// boxes stay packed in shared memory: 16 warps (two groups of 8
// that take alternate stages) expand them in registers with
// cvt.rn.f16x2.e2m1x2 (E2M1 is exact in fp16) and multiply on mma.sync
// m16n8k16, 16 weight rows per warp.  The activations are the n = 8 columns:
// each token as an fp16 hi + lo pair (x ~= hi + lo to ~2^-22), so one MMA
// covers up to four tokens.  Byte i of a 32-element block holds elements 2i
// and 2i+1 (tensor.go:156-158), so lane (g, c)'s four bytes of a block are
// elements 8c..8c+7: one 32-bit load per row and one 16-byte load of the
// activation column give both k-steps of the block.  Each block's two MMAs
// go to a fresh f32 accumulator that is then scaled by the row's E8M0 block
// scale, so the scale never has to fit fp16's range.
//
// Every wait is bounded (~1 s of clock): it records a code (50-54) in the error flag,
// marks the CTA dead (later waits return at once, no further stage is issued,
// the copies in flight are waited for) and the kernel winds down.
#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/amoe.h"
#include "tc_ptx.cuh"

namespace amoe {

namespace {

using namespace bs;

constexpr int kGroups = 2;                      // consumer groups, alternate stages
constexpr int kGroupWarps = 8;                  // 8 warps x 16 rows = one 128-row tile
constexpr int kComputeWarps = kGroups * kGroupWarps;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kDecThreads = kComputeWarps * 32;  // no producer warp: the last releaser of a stage refills it
constexpr uint32_t kBoxBytes = 128 * 64;        // one packed box: 128 rows x 128 E2M1 values
constexpr uint32_t kBoxStep = (uint32_t)kBoxStride;  // a box's rows and its scale chunk, as stored
constexpr uint32_t kStageBytes = 2 * kBoxStep;       // two boxes, each followed by its scale chunk
constexpr int kMaxStages = 12;
constexpr int kMaxUnits = 64;                   // units per CTA
constexpr int kSchedWords = 1024;               // one CTA's schedule rows (int32)
static_assert(kSchedWords == AMOE_DECODE_SCHED_WORDS, "the table row size is part of the C ABI");
constexpr int kMaxCtaStages = kMaxUnits * 16;   // ring stages of one CTA (a unit has <= 16: K <= 4096)
constexpr size_t kSmemBudget = 232448;          // dynamic shared memory per block (227 KB)

static_assert(kStageBytes % 1024 == 0, "stages keep the 1 KB alignment SWIZZLE_64B needs");

// Unit encoding in the schedule table.
__host__ __device__ constexpr int32_t unit_code(int phase, int slot, int mt, int kpart) {
    return (phase << 30) | (slot << 20) | (mt << 8) | kpart;
}

struct DecodeParams {
    const float *residual;
    float *out;
    const float *gain, *router_w, *router_b;  // RMSNorm gain [H], router [E][H] and bias [E]
    float eps;
    RouteOut route;             // routing outputs (logits doubles as the cross-CTA exchange buffer)
    unsigned *rflag;            // [G] launch epoch once a CTA's router dot products are stored
    const uint8_t *gu_tq, *dn_tq;    // box planes: per box its swizzled rows, then its scale chunk
    const float *gu_b, *dn_b;
    float *act;                 // [S][T][Ip] SwiGLU outputs of every token for every slot (padding stays 0)
    float *yb;                  // [S][2][T][H] down outputs, one plane per K half
    uint32_t *cnt_gu;           // [S] self-resetting arrival counters of the gate_up units
    uint32_t *cnt_dn;           // [nmt2] ... of the down units per output tile
    unsigned *aflag;            // [S] launch epoch once the slot's activation is complete
    const int32_t *sched;       // [G][kSchedWords]: per CTA, [n - 1]..[n] delimit its units when n slots are active
    DecodeBarrier *bar;
    int32_t *err;
    int T, H, I, E, k, Hp, Ip, S;
    int stages;
};

// Shared-memory layout (offsets from a 1 KB-aligned base).
__host__ __device__ constexpr uint32_t col_stride(int K) { return (uint32_t)(2 * K + 64); }  // fp16 column + pad

struct DecLayout {
    uint32_t ring, bx, bd, red, units, stg, rel, offs, act, perm, inv, w, sl, rms, lg, tk, misc, bars, total;
};

__host__ __device__ inline DecLayout dec_layout(int T, int Hp, int Ip, int E, int k, int stages, int ncol) {
    DecLayout L;
    uint32_t o = 0;
    const uint32_t P = (uint32_t)(T * k);
    L.ring = o;
    o += (uint32_t)stages * kStageBytes;
    L.bx = o;  // gate_up operand: ncol fp16 columns of Hp
    o += (uint32_t)ncol * col_stride(Hp);
    L.bd = o;  // down operand: ncol fp16 columns of Ip
    o += (uint32_t)ncol * col_stride(Ip);
    L.red = o;  // group 1's accumulators at the end of a unit
    o += (uint32_t)kGroupWarps * 32 * 4 * 4;
    L.units = o;
    o += kMaxUnits * 4;
    L.stg = o;  // [kMaxCtaStages] this CTA's ring stages: phase << 31 | (boxes - 1) << 30 | first box
    o += kMaxCtaStages * 4;
    L.rel = o;  // [stages] warps of the consuming group done with the slot; [stages] last stage issued into it
    o += 2u * (uint32_t)stages * 4;
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
    L.misc = o;  // broadcast words
    o += 64;
    o = (o + 7u) & ~7u;
    L.bars = o;  // [stages] full barriers
    o += (uint32_t)stages * 8;
    L.total = o + 1024;  // base alignment slack
    return L;
}

__device__ __forceinline__ void compute_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kComputeThreads) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Bounded mbarrier wait that returns at once once the CTA is dead.
__device__ __forceinline__ bool ring_wait(uint64_t *bar, uint32_t parity, volatile int *dead, int32_t *err,
                                          int code) {
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

// x (f32, natural order) -> fp16 hi / lo columns 2t, 2t+1 of an operand buffer.
__device__ __forceinline__ void put_split8(uint8_t *buf, uint32_t stride, int t, int k0, const float (&v)[8]) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        const float2 f = __half22float2(h);
        const __half2 l = __floats2half2_rn(v[2 * j] - f.x, v[2 * j + 1] - f.y);
        hi[j] = *reinterpret_cast<const uint32_t *>(&h);
        lo[j] = *reinterpret_cast<const uint32_t *>(&l);
    }
    *reinterpret_cast<uint4 *>(buf + (size_t)(2 * t) * stride + 2 * k0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(buf + (size_t)(2 * t + 1) * stride + 2 * k0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

template <int NCOL>
__launch_bounds__(kDecThreads, 1) __global__
    void decode_kernel(DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    const DecLayout lay = dec_layout(p.T, p.Hp, p.Ip, p.E, p.k, p.stages, NCOL);
    uint8_t *ring = sm + lay.ring;
    uint8_t *bx = sm + lay.bx;
    uint8_t *bd = sm + lay.bd;
    float *red = reinterpret_cast<float *>(sm + lay.red);
    int32_t *units_s = reinterpret_cast<int32_t *>(sm + lay.units);
    int32_t *offs_s = reinterpret_cast<int32_t *>(sm + lay.offs);
    int32_t *act_s = reinterpret_cast<int32_t *>(sm + lay.act);
    int32_t *perm_s = reinterpret_cast<int32_t *>(sm + lay.perm);
    int32_t *inv_s = reinterpret_cast<int32_t *>(sm + lay.inv);
    float *w_s = reinterpret_cast<float *>(sm + lay.w);
    int32_t *sl_s = reinterpret_cast<int32_t *>(sm + lay.sl);
    volatile int *misc = reinterpret_cast<volatile int *>(sm + lay.misc);  // [0] dead, [1] last, [2] units
    int32_t *stg_s = reinterpret_cast<int32_t *>(sm + lay.stg);
    int *rel_s = reinterpret_cast<int *>(sm + lay.rel);  // [R] releases, then [R] last stage issued per slot
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + lay.bars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, P = p.T * p.k, R = p.stages, G = gridDim.x;
    const uint32_t sx = col_stride(p.Hp), sd = col_stride(p.Ip);
    const unsigned epoch = p.bar->epoch[blockIdx.x] + 1u;

    if (tid == 0) {
        misc[0] = 0;
        for (int s = 0; s < R; ++s) {
            mbar_init(full + s, 1);
            rel_s[s] = 0;
            rel_s[R + s] = -1;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // ---------------- routing, in every CTA ----------------
    // RMSNorm (primitives.go:50-72), router logits (primitives.go:11-47), top-k and
    // softmax over the selected logits (moe.go:12-41), stable (expert, token, slot)
    // permutation.  The T x E router dot products are spread over the CTAs; each
    // publishes its flag, and every CTA then reads all logits and derives the same
    // routing.
    {
        constexpr int kWarps = kDecThreads / 32;
        double *rms_s = reinterpret_cast<double *>(sm + lay.rms);
        double *red_s = rms_s + 4;
        float *lg_s = reinterpret_cast<float *>(sm + lay.lg);
        int *tk_s = reinterpret_cast<int *>(sm + lay.tk);
        const int T = p.T, H = p.H;
        // (0) every global input of the routing in one batch, staged in the ring (no
        //     copy uses it before the routing is done): this CTA's schedule rows for
        //     every number of active slots, the T residual rows, the gain and, for a
        //     CTA that owns a router dot product, the first router row it needs.
        constexpr int kPer = (4096 + kDecThreads - 1) / kDecThreads;  // elements per thread, H <= 4096
        int32_t *sched_s = reinterpret_cast<int32_t *>(ring);
        float *xs_s = reinterpret_cast<float *>(ring + kSchedWords * 4);  // [T][Hp] residual rows
        float *gs_s = xs_s + (size_t)T * p.Hp;                            // [Hp] gain
        const int ndots = T * E;
        for (int i = tid; i < kSchedWords; i += kDecThreads)
            sched_s[i] = __ldg(p.sched + (size_t)blockIdx.x * kSchedWords + i);
        float wv[kPer];
        {
            const int e0 = (int)blockIdx.x < ndots ? (int)blockIdx.x % E : 0;
            float gv[kPer];
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i = tid + r * kDecThreads;
                const bool in = i < H;
                wv[r] = in && (int)blockIdx.x < ndots ? __ldg(p.router_w + (size_t)e0 * H + i) : 0.0f;
                gv[r] = in ? __ldg(p.gain + i) : 0.0f;
            }
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i = tid + r * kDecThreads;
                if (i < p.Hp) gs_s[i] = gv[r];
            }
        }
        // (1) float64 sums of squares of the T residual rows
        double ss[kDecodeMaxTokens];
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t) {
            ss[t] = 0.0;
            if (t < T) {
                float xv[kPer];
#pragma unroll
                for (int r = 0; r < kPer; ++r) {
                    const int i = tid + r * kDecThreads;
                    xv[r] = i < H ? __ldg(p.residual + (size_t)t * H + i) : 0.0f;
                }
#pragma unroll
                for (int r = 0; r < kPer; ++r) {
                    const int i = tid + r * kDecThreads;
                    ss[t] += (double)xv[r] * (double)xv[r];
                    if (i < p.Hp) xs_s[(size_t)t * p.Hp + i] = xv[r];
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t) {
            double v = ss[t];
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
        // (2) router dot products, one per CTA (dot d on CTA d mod G):
        //     logit = f32(sum f64(x_n) f64(W)) + b, partials added in a fixed order
        for (int dd = blockIdx.x; dd < ndots; dd += G) {
            const int t = dd / E, e = dd - t * E;
            const double inv = rms_s[t];
            double acc = 0.0;
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i = tid + r * kDecThreads;
                if (i < H) {
                    const float w = dd == (int)blockIdx.x ? wv[r] : __ldg(p.router_w + (size_t)e * H + i);
                    const float xn = (float)((double)xs_s[(size_t)t * p.Hp + i] * inv * (double)gs_s[i]);
                    acc = fma((double)xn, (double)w, acc);
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
        __syncthreads();
        if (tid == 0 && (int)blockIdx.x < min(G, ndots)) publish(p.rflag + blockIdx.x, epoch);
        // (2b) the gate_up operand, while other CTAs finish their dot products: every
        //      token's normalized row (rounded to f32 as RMSNorm stores it,
        //      primitives.go:68-70) as fp16 hi / lo columns; zero past H and in the
        //      columns of absent tokens.
        {
            const int n8 = p.Hp / 8;
            for (int it = tid; it < (NCOL / 2) * n8; it += kDecThreads) {
                const int t = it / n8, k0 = 8 * (it - t * n8);
                float v[8];
                if (t < T && k0 < H) {
                    const double inv = rms_s[t];
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        v[q] = (float)((double)xs_s[(size_t)t * p.Hp + k0 + q] * inv * (double)gs_s[k0 + q]);
                } else {
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[q] = 0.0f;
                }
                put_split8(bx, sx, t, k0, v);
            }
        }
        const int dot_ctas = min(G, ndots);
        // (3) every CTA's logits
        if (warp == 0) wait_flags(p.rflag, dot_ctas, epoch, lane, p.err, 53);
        __syncthreads();
        for (int i = tid; i < ndots; i += kDecThreads) lg_s[i] = __ldcg(p.route.logits + i);
        __syncthreads();
        // (4) top-k: the rank of every (token, expert) in the stable descending order
        //     (moe.go:20-27) in parallel; ranks below k are the selected slots.  Then
        //     the softmax over the selected logits per token (moe.go:29-39): the k
        //     exponentials in parallel, the denominator summed in slot order.
        for (int te = tid; te < ndots; te += kDecThreads) {
            const int t = te / E, e = te - t * E;
            const float v = lg_s[te];
            int rank = 0;
            for (int f2 = 0; f2 < E; ++f2) rank += topk_better(lg_s[t * E + f2], f2, v, e);
            if (rank < p.k) tk_s[t * p.k + rank] = e;
        }
        __syncthreads();
        if (warp < T) {
            const int t = warp;
            const double maxv = (double)lg_s[t * E + tk_s[t * p.k]];
            const double ex = lane < p.k ? exp((double)lg_s[t * E + tk_s[t * p.k + lane]] - maxv) : 0.0;
            double den = 0.0;
            for (int sl = 0; sl < p.k; ++sl) den += __shfl_sync(0xffffffffu, ex, sl);
            if (lane < p.k) w_s[t * p.k + lane] = (float)((double)(float)ex / den);
        }
        __syncthreads();
        // (5) counts, offsets, active experts and the stable permutation
        for (int e = tid; e <= E; e += kDecThreads) offs_s[e] = 0;
        __syncthreads();
        for (int q = tid; q < P; q += kDecThreads) atomicAdd(&offs_s[tk_s[q]], 1);
        __syncthreads();
        if (warp == 0) {
            // warp scan over experts (lane owns experts 8 lane .. 8 lane + 7; E <= 256)
            int c[8], a[8];
            int cs = 0, as = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = 8 * lane + j;
                c[j] = e < E ? offs_s[e] : 0;
                a[j] = c[j] > 0;
                cs += c[j];
                as += a[j];
            }
            int cx = cs, ax = as;  // inclusive warp prefix sums
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int cu = __shfl_up_sync(0xffffffffu, cx, o), au = __shfl_up_sync(0xffffffffu, ax, o);
                if (lane >= o) {
                    cx += cu;
                    ax += au;
                }
            }
            int co = cx - cs, ao = ax - as;
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = 8 * lane + j;
                if (e < E) {
                    offs_s[e] = co;
                    if (a[j]) act_s[ao] = e;
                }
                co += c[j];
                ao += a[j];
            }
            if (lane == 31) {
                offs_s[E] = cx;
                act_s[E] = ax;
            }
        }
        __syncthreads();
        for (int q = tid; q < P; q += kDecThreads) {  // pairs in (token, slot) order land stably
            const int e = tk_s[q];
            int pos = offs_s[e];
            for (int r = 0; r < q; ++r) pos += tk_s[r] == e;
            perm_s[pos] = q;
            inv_s[q] = pos;
            int slot = 0;
            while (act_s[slot] != e) ++slot;  // e is active, so the search ends within act_s[0..E)
            sl_s[q] = slot;
        }
        {
            // this CTA's units for this number of active slots (its staged schedule rows)
            const int n_active = act_s[E];
            const int u0 = sched_s[n_active - 1], u1 = sched_s[n_active];
            const int n = min(u1 - u0, kMaxUnits);
            for (int u = tid; u < n; u += kDecThreads) units_s[u] = sched_s[u0 + u];
            if (tid == 0) misc[2] = n;
        }
        __syncthreads();
        if (blockIdx.x == 0) {  // the routing the C ABI reports
            for (int q = tid; q < P; q += kDecThreads) {
                p.route.topk_idx[q] = tk_s[q];
                p.route.topk_w[q] = w_s[q];
                p.route.perm_pair[q] = perm_s[q];
                p.route.inv[q] = inv_s[q];
            }
            for (int e = tid; e <= E; e += kDecThreads) {
                p.route.offsets[e] = offs_s[e];
                p.route.active[e] = act_s[e];
                if (e < E) p.route.counts[e] = offs_s[e + 1] - offs_s[e];
            }
        }
    }

    const int n_active = act_s[E];
    const int nunits = misc[2];
    const int nkb1 = p.Hp / 128, nkb2 = p.Ip / 128;
    const int nmt1 = 2 * p.I / 128, nmt2 = (p.H + 127) / 128;
    const int nkp = nkb2 >= 2 ? 2 : 1, half2 = (nkb2 + 1) / 2;  // down units: K halves
    // a unit's phase (0 gate_up, 1 down), slot, weight tile, K part and box range
    auto unit_span = [&](int32_t code, int &phase, int &slot, int &mt, int &kpart, int &kb0, int &kb1) {
        phase = (code >> 30) & 1;
        slot = (code >> 20) & 1023;
        mt = (code >> 8) & 4095;
        kpart = code & 1;
        kb0 = phase == 0 || kpart == 0 ? 0 : half2;
        kb1 = phase == 0 ? nkb1 : (nkp == 1 || kpart == 1 ? nkb2 : half2);
    };

    // ---------------- the ring: this CTA's stages, two boxes each ----------------
    // Stage j is filled into slot j % R.  The first R go out now; afterwards the
    // last warp of the consuming group to finish with a slot refills it with the
    // stage R further on, so no warp ever polls for free slots.
    auto issue = [&](int j) {
        const int32_t code = stg_s[j];
        const int phase = (int)(((uint32_t)code >> 31) & 1u), nb = ((code >> 30) & 1) + 1;
        const size_t box = (size_t)(code & 0x3fffffff);  // plane row of the first box: 128 * box
        const int sl = j % R;
        uint8_t *st = ring + (size_t)sl * kStageBytes;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's reads before the copy's writes
        mbar_expect_tx(full + sl, (uint32_t)nb * kBoxStep);
        bulk_g2s(st, (phase ? p.dn_tq : p.gu_tq) + box * kBoxStep, (uint32_t)nb * kBoxStep, full + sl);
        rel_s[R + sl] = j;
    };
    if (tid == 0) {
        int j = 0;
        for (int u = 0; u < nunits; ++u) {
            int phase, slot, mt, kpart, kb0, kb1;
            unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
            const int e = act_s[slot];
            const int nmt = phase ? nmt2 : nmt1, nkb = phase ? nkb2 : nkb1;
            for (int kb = kb0; kb < kb1 && j < kMaxCtaStages; kb += 2, ++j)
                stg_s[j] = (int32_t)(((uint32_t)phase << 31) | ((uint32_t)(min(2, kb1 - kb) - 1) << 30) |
                                     (uint32_t)(((size_t)e * nmt + mt) * nkb + kb));
        }
        misc[3] = j;
        for (int i = 0; i < min(R, j); ++i) issue(i);
    }
    __syncthreads();
    const int nst = misc[3];
    {
        // ---------------- consumers: 16 warps, two groups taking alternate stages ----------------
        const int grp = warp / kGroupWarps, wl = warp % kGroupWarps;
        const int g = lane >> 2, c = lane & 3;
        const int r0 = 16 * wl + g;  // this lane's rows r0 and r0 + 8 of the 128-row tile
        const uint32_t swz = (uint32_t)((r0 >> 1) & 3);  // SWIZZLE_64B: 16-B chunk ^= (row / 2) % 4
        const uint32_t sc0 = (uint32_t)((r0 & 31) * 16 + (r0 >> 5) * 4);  // E8M0 chunk: byte (r%32)*16 + (r/32)*4 + j
        const uint32_t sc1 = (uint32_t)(((r0 + 8) & 31) * 16 + ((r0 + 8) >> 5) * 4);
        uint32_t off[4];  // this lane's 4 bytes of block q in a swizzled 64-B row
#pragma unroll
        for (int q = 0; q < 4; ++q) off[q] = (((uint32_t)q ^ swz) << 4) + 4 * c;
        int i = 0;  // stage counter, the same walk as the producer's
        for (int u = 0; u < nunits; ++u) {
            int phase, slot, mt, kpart, kb0, kb1;
            unit_span(units_s[u], phase, slot, mt, kpart, kb0, kb1);
            const int e = act_s[slot];
            if (phase == 1) {
                // the slot's activation: complete once its last gate_up unit published it
                if (tid == 0 && !misc[0]) {
                    const long long t0 = clock64();
                    while ((int)(ld_acquire(p.aflag + slot) - epoch) < 0) {
                        if (clock64() - t0 > kWaitLimit) {
                            atomicCAS(p.err, 0, 52);
                            misc[0] = 1;
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                compute_bar();
                // this unit's operand columns: the activation over its K range, fp16 hi / lo
                const int n8 = 16 * (kb1 - kb0);
                for (int it = tid; it < (NCOL / 2) * n8; it += kComputeThreads) {
                    const int t = it / n8, k0 = 128 * kb0 + 8 * (it - t * n8);
                    float v[8];
                    if (t < p.T) {
                        const float *src = p.act + ((size_t)slot * p.T + t) * p.Ip + k0;
                        const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(src));
                        const float4 a1 = __ldcg(reinterpret_cast<const float4 *>(src + 4));
                        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
                        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
                    } else {
#pragma unroll
                        for (int q = 0; q < 8; ++q) v[q] = 0.0f;
                    }
                    put_split8(bd, sd, t, k0, v);
                }
                compute_bar();
            }
            const uint8_t *bcol = (phase ? bd : bx) + (size_t)g * (phase ? sd : sx) + 16 * c;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int kb = kb0; kb < kb1; kb += 2, ++i) {
                if ((i & 1) != grp) continue;
                const int nb = min(2, kb1 - kb), s = i % R;
                ring_wait(full + s, (i / R) & 1, misc, p.err, 51);  // when dead: compute on stale data
                const uint8_t *st = ring + (size_t)s * kStageBytes;
                // all of the stage's shared-memory loads first, then up to eight independent blocks
                uint32_t w0[2][4], w1[2][4], sv0[2], sv1[2];
                uint4 bv[2][4];
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    if (b < nb) {
                        const uint8_t *rows = st + b * kBoxStep + r0 * 64;
                        const uint8_t *xk = bcol + 2 * 128 * (kb + b);
                        sv0[b] = *reinterpret_cast<const uint32_t *>(st + b * kBoxStep + kBoxBytes + sc0);
                        sv1[b] = *reinterpret_cast<const uint32_t *>(st + b * kBoxStep + kBoxBytes + sc1);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            w0[b][q] = *reinterpret_cast<const uint32_t *>(rows + off[q]);
                            w1[b][q] = *reinterpret_cast<const uint32_t *>(rows + 8 * 64 + off[q]);
                            bv[b][q] = g < NCOL ? *reinterpret_cast<const uint4 *>(xk + 64 * q) : make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    if (b < nb) {
                        float f0[4], f1[4];
                        e8m0x4_to_float(sv0[b], f0);
                        e8m0x4_to_float(sv1[b], f1);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 a = e2m1x8_to_f16(w0[b][q]), a8 = e2m1x8_to_f16(w1[b][q]);
                            // the block's two k-steps into separate accumulators: no MMA waits on another
                            float d0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                            mma16816(d0, a.x, a8.x, a.y, a8.y, bv[b][q].x, bv[b][q].y);  // elements 8c..8c+3
                            mma16816(d1, a.z, a8.z, a.w, a8.w, bv[b][q].z, bv[b][q].w);  // elements 8c+4..8c+7
                            acc[0] = fmaf(d0[0] + d1[0], f0[q], acc[0]);
                            acc[1] = fmaf(d0[1] + d1[1], f0[q], acc[1]);
                            acc[2] = fmaf(d0[2] + d1[2], f1[q], acc[2]);
                            acc[3] = fmaf(d0[3] + d1[3], f1[q], acc[3]);
                        }
                    }
                }
                // release the slot; the group's last warp refills it with stage i + R
                __syncwarp();
                if (lane == 0) {
                    if (atomicAdd(rel_s + s, 1) == kGroupWarps - 1) {
                        rel_s[s] = 0;
                        if (i + R < nst && !misc[0]) issue(i + R);
                    }
                }
                __syncwarp();
            }
            // ---- unit epilogue: group 1's sums join group 0's (fixed order) ----
            if (grp == 1)
                *reinterpret_cast<float4 *>(red + (wl * 32 + lane) * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
            compute_bar();
            if (grp == 0) {
                const float4 o = *reinterpret_cast<const float4 *>(red + (wl * 32 + lane) * 4);
                // lane (g, c) holds rows r0, r0 + 8 for columns 2c (hi) and 2c + 1 (lo): token c
                const float v0 = (acc[0] + o.x) + (acc[1] + o.y);
                const float v1 = (acc[2] + o.z) + (acc[3] + o.w);
                if (c < p.T) {
                    if (phase == 0) {
                        // rows 16w + g and 16w + g + 8 are the gate and up rows of pair 64 mt + 8w + g
                        const int pr = 64 * mt + 8 * wl + g;
                        const float gate = v0 + p.gu_b[(size_t)e * 2 * p.I + 2 * pr];
                        const float up = v1 + p.gu_b[(size_t)e * 2 * p.I + 2 * pr + 1];
                        p.act[((size_t)slot * p.T + c) * p.Ip + pr] = swiglu(gate, up);
                    } else {
                        const int h0 = 128 * mt + r0, h1 = h0 + 8;
                        float *yrow = p.yb + (((size_t)slot * 2 + kpart) * p.T + c) * p.H;
                        if (h0 < p.H) yrow[h0] = v0 + (kpart == 0 ? p.dn_b[(size_t)e * p.H + h0] : 0.0f);
                        if (h1 < p.H) yrow[h1] = v1 + (kpart == 0 ? p.dn_b[(size_t)e * p.H + h1] : 0.0f);
                    }
                }
                __threadfence();
            }
            compute_bar();
            if (tid == 0) {
                const unsigned n = phase == 0 ? (unsigned)nmt1 : (unsigned)(nkp * n_active);
                unsigned *cnt = phase == 0 ? p.cnt_gu + slot : p.cnt_dn + mt;
                const unsigned old = atomicInc(cnt, n - 1u);
                misc[1] = old == n - 1u;
                if (old == n - 1u && phase == 0) publish(p.aflag + slot, epoch);
            }
            compute_bar();
            if (phase == 1 && misc[1]) {
                // the last down unit of output tile mt: combine its rows for every token in
                // slot order (layer.go:109-121)
                __threadfence();
                for (int it = tid; it < p.T * 128; it += kComputeThreads) {
                    const int t = it >> 7, h = 128 * mt + (it & 127);
                    if (h >= p.H) continue;
                    double m = 0.0;
                    for (int s = 0; s < p.k; ++s) {
                        const int q = t * p.k + s;
                        const float *yp = p.yb + ((size_t)sl_s[q] * 2 * p.T + t) * p.H + h;
                        float yv = __ldcg(yp);
                        if (nkp == 2) yv += __ldcg(yp + (size_t)p.T * p.H);
                        m += (double)w_s[q] * (double)yv;
                    }
                    p.out[(size_t)t * p.H + h] = p.residual[(size_t)t * p.H + h] + (float)m;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        // copies still in flight (only after a failed wait) land before the CTA exits
        if (misc[0])
            for (int sl = 0; sl < R; ++sl)
                if (rel_s[R + sl] >= 0) mbar_wait(full + sl, (rel_s[R + sl] / R) & 1, p.err, 54);
        p.bar->epoch[blockIdx.x] = epoch;
    }
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

int dec_ncol(int T) { return T <= 1 ? 2 : (T <= 2 ? 4 : 8); }

// Ring stages that fit beside the operand columns (even: each slot serves one group).
int dec_stages(int T, int Hp, int Ip, int E, int k) {
    const DecLayout none = dec_layout(T, Hp, Ip, E, k, 0, dec_ncol(T));
    if (none.total >= kSmemBudget) return 0;
    int st = (int)((kSmemBudget - none.total) / (kStageBytes + 16));
    st = std::min(st, kMaxStages);
    return st & ~1;
}

int dec_slots(const Dims &d) { return d.E < kDecodeMaxTokens * d.k ? d.E : kDecodeMaxTokens * d.k; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The units of every CTA for each number of active slots n = 1..S: longest
// processing time first over the units' box counts (all units of a phase are
// the same size, so this is a balanced round over the least-loaded CTAs),
// gate_up units before down units, each in slot order.  CTA b's rows sit in
// words [b * kSchedWords, (b + 1) * kSchedWords): S + 1 offsets (relative to
// the row start), then the unit lists for n = 1..S.
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
    std::vector<std::vector<int32_t>> lists(G);
    std::vector<long long> load(G);
    for (int b = 0; b < G; ++b) rows[b][0] = S + 1;
    for (int n = 1; n <= S; ++n) {
        for (auto &l : lists) l.clear();
        std::fill(load.begin(), load.end(), 0);
        auto place = [&](int32_t code, int cost) {
            int best = 0;
            for (int b = 1; b < G; ++b)
                if (load[b] < load[best]) best = b;
            lists[best].push_back(code);
            load[best] += cost;
        };
        for (int sl = 0; sl < n; ++sl)
            for (int m = 0; m < nmt1; ++m) place(unit_code(0, sl, m, 0), nkb1);
        for (int sl = 0; sl < n; ++sl)
            for (int m = 0; m < nmt2; ++m)
                for (int kp = 0; kp < nkp; ++kp)
                    place(unit_code(1, sl, m, kp), nkp == 1 ? nkb2 : (kp ? nkb2 - half2 : half2));
        for (int b = 0; b < G; ++b) {
            rows[b].insert(rows[b].end(), lists[b].begin(), lists[b].end());
            rows[b][n] = (int32_t)rows[b].size();
            s.max_units = std::max(s.max_units, (int)lists[b].size());
        }
    }
    s.rows.assign((size_t)G * kSchedWords, 0);
    for (int b = 0; b < G; ++b) {
        s.max_words = std::max(s.max_words, (int)rows[b].size());
        std::copy_n(rows[b].begin(), std::min<size_t>(rows[b].size(), kSchedWords), s.rows.begin() + (size_t)b * kSchedWords);
    }
    return s;
}

struct DecScratch {
    size_t act, yb, cnt_gu, cnt_dn, aflag, rflag, sched, total;
};

DecScratch dec_scratch(const Dims &d, int G, const Schedule &s) {
    const int S = dec_slots(d), Ip = kpad128(d.I), nmt2 = (d.H + 127) / 128;
    DecScratch L;
    size_t o = 0;
    L.act = o;
    o += align256((size_t)S * kDecodeMaxTokens * Ip * 4);
    L.yb = o;
    o += align256((size_t)S * 2 * kDecodeMaxTokens * d.H * 4);
    L.cnt_gu = o;
    o += align256((size_t)S * 4);
    L.cnt_dn = o;
    o += align256((size_t)nmt2 * 4);
    L.aflag = o;
    o += align256((size_t)S * 4);
    L.rflag = o;
    o += align256((size_t)G * 4);
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
    if ((2 * d.I) % 128 || d.H > 4096 || d.I > 4096 || d.E > 256 || d.k > 32 || dec_slots(d) > 1023) return false;
    if (2 * d.I / 128 > 4095 || (d.H + 127) / 128 > 4095) return false;
    if (dec_stages(T, kpad128(d.H), kpad128(d.I), d.E, d.k) < 2) return false;
    // the routing stages the schedule rows, the residual rows and the gain in the ring
    const int Hp = kpad128(d.H);
    if ((size_t)dec_stages(T, Hp, kpad128(d.I), d.E, d.k) * kStageBytes <
        (size_t)4 * (kSchedWords + (size_t)(T + 1) * Hp))
        return false;
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
    p.rflag = reinterpret_cast<unsigned *>(b + lay.rflag);
    p.gu_tq = L.gu_tq;
    p.dn_tq = L.dn_tq;
    p.gu_b = L.gu_b;
    p.dn_b = L.dn_b;
    p.act = reinterpret_cast<float *>(b + lay.act);
    p.yb = reinterpret_cast<float *>(b + lay.yb);
    p.cnt_gu = reinterpret_cast<uint32_t *>(b + lay.cnt_gu);
    p.cnt_dn = reinterpret_cast<uint32_t *>(b + lay.cnt_dn);
    p.aflag = reinterpret_cast<unsigned *>(b + lay.aflag);
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
    if (p.stages < 2) return cudaErrorInvalidValue;
    const size_t smem = dec_layout(T, Hp, Ip, d.E, d.k, p.stages, ncol).total;
    auto kern = ncol == 2 ? decode_kernel<2> : (ncol == 4 ? decode_kernel<4> : decode_kernel<8>);
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
