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
#include "tc_ptx.cuh"

namespace amoe {

namespace {

using namespace bs;

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
    const float *gain, *router_w, *router_b;  // RMSNorm gain [H], router [E][H] and bias [E]
    float eps;
    RouteOut route;             // routing outputs (logits doubles as the cross-CTA exchange buffer)
    unsigned *rflag;            // [G] launch epoch once a CTA's router dot products are stored
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
    uint32_t ring, b1, sfb1, offs, act, perm, inv, w, ready, rms, lg, tk, xchg, bars, tmem_slot, total;
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
    o = (o + 7u) & ~7u;
    L.rms = o;  // [4] inverse RMS per token, then [warps][4] partial sums (f64)
    o += (uint32_t)(4 + (kDecThreads / 32) * 4) * 8;
    L.lg = o;  // [T*E] router logits
    o += (uint32_t)(T * E) * 4;
    L.tk = o;  // [P] selected experts in slot order
    o += P * 4;
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

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

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
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + lay.tmem_slot);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, P = p.T * p.k, R = p.stages, G = gridDim.x;
    const unsigned epoch = p.bar->epoch[blockIdx.x] + 1u;

    if (tid == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_gu)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_dn)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_act)) : "memory");
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
        // (1) float64 sums of squares of the T residual rows (loads unrolled: in flight together)
        constexpr int kPer = (4096 + kDecThreads - 1) / kDecThreads;  // elements per thread, H <= 4096
        double ss[kDecodeMaxTokens];
#pragma unroll
        for (int t = 0; t < kDecodeMaxTokens; ++t) {
            ss[t] = 0.0;
            if (t < T) {
                float xv[kPer];
#pragma unroll
                for (int r = 0; r < kPer; ++r) {
                    const int i = tid + r * kDecThreads;
                    xv[r] = i < H ? p.residual[(size_t)t * H + i] : 0.0f;
                }
#pragma unroll
                for (int r = 0; r < kPer; ++r) ss[t] += (double)xv[r] * (double)xv[r];
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
        const int ndots = T * E;
        for (int dd = blockIdx.x; dd < ndots; dd += G) {
            const int t = dd / E, e = dd - t * E;
            const float *xr = p.residual + (size_t)t * H;
            const float *wr = p.router_w + (size_t)e * H;
            const double inv = rms_s[t];
            float xv[kPer], gv[kPer], wv[kPer];
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const int i = tid + r * kDecThreads;
                const bool in = i < H;
                xv[r] = in ? xr[i] : 0.0f;
                gv[r] = in ? p.gain[i] : 0.0f;
                wv[r] = in ? wr[i] : 0.0f;
            }
            double acc = 0.0;
#pragma unroll
            for (int r = 0; r < kPer; ++r) {
                const float xn = (float)((double)xv[r] * inv * (double)gv[r]);
                acc = fma((double)xn, (double)wv[r], acc);
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
        // (2b) the phase-1 operand, while other CTAs finish their dot products: every
        //      token's normalized row as four E4M3 terms.  Item = 8 elements; four
        //      consecutive lanes hold one 32-element block.
        {
            const int n8 = p.Hp / 8, total = p.T * n8;
            constexpr int kBatch = 4;  // items per thread whose loads are in flight together
            for (int base0 = 0; base0 < total; base0 += kBatch * kDecThreads) {
              float4 xv[kBatch][2], gv[kBatch][2];
#pragma unroll
              for (int u = 0; u < kBatch; ++u) {
                const int it = base0 + u * kDecThreads + tid;
                const int t = it / n8, k0 = 8 * (it - t * n8);
                xv[u][0] = xv[u][1] = gv[u][0] = gv[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (it < total && k0 < p.H) {
                    xv[u][0] = *reinterpret_cast<const float4 *>(p.residual + (size_t)t * p.H + k0);
                    xv[u][1] = *reinterpret_cast<const float4 *>(p.residual + (size_t)t * p.H + k0 + 4);
                    gv[u][0] = *reinterpret_cast<const float4 *>(p.gain + k0);
                    gv[u][1] = *reinterpret_cast<const float4 *>(p.gain + k0 + 4);
                }
              }
#pragma unroll
              for (int u = 0; u < kBatch; ++u) {
                const int it = base0 + u * kDecThreads + tid;
                const bool valid = it < total;
                const int t = valid ? it / n8 : 0, k8 = valid ? it - t * n8 : 0;
                const int k0 = 8 * k8;
                // normalized row, rounded to f32 as RMSNorm stores it (primitives.go:68-70)
                const double inv = rms_s[t];
                const float xs[8] = {xv[u][0].x, xv[u][0].y, xv[u][0].z, xv[u][0].w,
                                     xv[u][1].x, xv[u][1].y, xv[u][1].z, xv[u][1].w};
                const float gs[8] = {gv[u][0].x, gv[u][0].y, gv[u][0].z, gv[u][0].w,
                                     gv[u][1].x, gv[u][1].y, gv[u][1].z, gv[u][1].w};
                float v[8];
                float amax = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    v[q] = (float)((double)xs[q] * inv * (double)gs[q]);
                    amax = fmaxf(amax, fabsf(v[q]));
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
        }
        const int dot_ctas = min(G, ndots);
        // (3) every CTA's logits
        if (warp == 0) wait_flags(p.rflag, dot_ctas, epoch, lane, p.err, 38);
        __syncthreads();
        for (int i = tid; i < ndots; i += kDecThreads) lg_s[i] = __ldcg(p.route.logits + i);
        __syncthreads();
        // (4) top-k: the rank of every (token, expert) in the stable descending order
        //     (moe.go:20-27) in parallel; ranks below k are the selected slots.  Then
        //     the softmax over the selected logits per token (moe.go:29-39).
        for (int te = tid; te < ndots; te += kDecThreads) {
            const int t = te / E, e = te - t * E;
            const float v = lg_s[te];
            int rank = 0;
            for (int f2 = 0; f2 < E; ++f2) rank += topk_better(lg_s[t * E + f2], f2, v, e);
            if (rank < p.k) tk_s[t * p.k + rank] = e;
        }
        __syncthreads();
        if (tid < T) {
            const int t = tid;
            const double maxv = (double)lg_s[t * E + tk_s[t * p.k]];
            double den = 0.0;
            for (int sl = 0; sl < p.k; ++sl) den += exp((double)lg_s[t * E + tk_s[t * p.k + sl]] - maxv);
            for (int sl = 0; sl < p.k; ++sl) {
                const float wf = (float)exp((double)lg_s[t * E + tk_s[t * p.k + sl]] - maxv);
                w_s[t * p.k + sl] = (float)((double)wf / den);
            }
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
        // With R >= kProdWarps stages, the wait for iteration i - R's slot comes after
        // this warp's wait for iteration i - kProdWarps - R, so the slot's earlier
        // phase (iteration i - 2R) has completed and the parity wait is unambiguous.
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
        bool ok = true;  // the phase-1 operand was built before the roles split
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
           align256((size_t)G * 2 * 128 * kNMax * 4) + (size_t)2 * 2 * S * kTilesPerSlot * 4 + (size_t)G * 4;
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
    // a ring of at least kProdWarps stages: producer warp w's waits on a slot's
    // empty barrier then follow the phases in order (see the producers)
    return dec_stages(T, kpad128(d.H), d.E, d.k) >= kProdWarps;
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
    p.gain = L.norm_gain;
    p.router_w = L.router_w;
    p.router_b = L.router_b;
    p.eps = d.eps;
    p.route = r;
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
    p.rflag = p.tflag + (size_t)2 * S * kTilesPerSlot;
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
    if (p.stages < kProdWarps || !get_encode()) return cudaErrorInvalidValue;
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
