// route.cu -- K1 (RMSNorm + router GEMV + top-k + selected softmax) and
// K2 (stable token->expert permutation).
//
// Reference arithmetic (paths relative to the reference project root):
//   RMSNorm        internal/backend/cpuref/primitives.go:50-72  (f64 sum of squares)
//   router logits  primitives.go:11-47  (f64 dot, f32 rounding, f32 bias add)
//   top-k          internal/backend/cpuref/moe.go:20-27  (stable descending, ties -> lower id)
//   softmax        moe.go:29-39  (f64 over the selected logits only)
// The dot products accumulate in float64 like the reference, in a different
// order; the rounded float32 logits therefore match except when the float64
// sum lies within ~1e-16 relative of a float32 rounding boundary.
#include "amoe_internal.cuh"

#include <float.h>

namespace amoe {

namespace {

constexpr int kMaxKSplit = 16;

struct RouteParams {
    const float *residual;
    const float *gain;
    const float *w;    // [E][H] router weight (GGUF layout)
    const float *bias; // [E]
    int T, H, E, k, ksplit;
    float eps;
    RouteOut o;
    double *partial;   // [ksplit][T][E] (only when ksplit > 1)
    int32_t *arrivals; // [nchunk], zero between calls
};

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// (value, expert) ordering of a stable descending sort; NaN sorts last, invalid
// entries (expert < 0) after everything.
__device__ __forceinline__ bool better(float v1, int e1, float v2, int e2) {
    if (e2 < 0) return e1 >= 0;
    if (e1 < 0) return false;
    bool n1 = isnan(v1), n2 = isnan(v2);
    if (n1 || n2) return n1 == n2 ? e1 < e2 : n2;
    return v1 > v2 || (v1 == v2 && e1 < e2);
}

__device__ __forceinline__ void dmma884(double &d0, double &d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}


// Partial router logits of the chunk's 8 tokens over k in [k0, k1) on the FP64
// tensor path (mma.m8n8k4: f64 products, f64 accumulation) for experts
// [8*nb0, 8*(nb0+NB)).  Lane (g = lane/4, c = lane%4) loads 4 consecutive k of
// token g (A) and of expert 8*nb+g (B) per 16-k group and feeds them to 4 MMAs
// as k-columns c of each: the same k permutation on both operands.  A is the
// RMSNorm output computed right here from the residual (primitives.go:68-70,
// float32(float64(x) * inverseRMS * float64(g)) left to right); the first pass
// also stores its fp16 hi/lo split for the expert GEMMs.
template <int NB>
__device__ __forceinline__ void logits_pass(const RouteParams &p, const double *inv, int t0, int nt, int k0,
                                            int k1, int nb0, int lane, bool write_split,
                                            double (&acc)[NB][2]) {
    const int g = lane >> 2, c = lane & 3;
    const int H = p.H;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) acc[nb][0] = acc[nb][1] = 0.0;
    const bool tok_ok = g < nt;
    const float *xrow = p.residual + (size_t)(t0 + g) * H;
    const double iv = inv[g];
    for (int kb = k0; kb < k1; kb += 16) {
        const int k = kb + 4 * c;
        const bool kin = k < k1;  // k1 - k0 is a multiple of 16 except at H (a multiple of 64)
        double a[4] = {0.0, 0.0, 0.0, 0.0};
        if (kin && tok_ok) {
            const float4 x = __ldg(reinterpret_cast<const float4 *>(xrow + k));
            const float4 gn = __ldg(reinterpret_cast<const float4 *>(p.gain + k));
            const float n0 = (float)((double)x.x * iv * (double)gn.x);
            const float n1 = (float)((double)x.y * iv * (double)gn.y);
            const float n2 = (float)((double)x.z * iv * (double)gn.z);
            const float n3 = (float)((double)x.w * iv * (double)gn.w);
            a[0] = n0; a[1] = n1; a[2] = n2; a[3] = n3;
            if (write_split) {
                const __half2 h01 = __floats2half2_rn(n0, n1), h23 = __floats2half2_rn(n2, n3);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                const __half2 l01 = __floats2half2_rn(n0 - f01.x, n1 - f01.y);
                const __half2 l23 = __floats2half2_rn(n2 - f23.x, n3 - f23.y);
                __half2 *dh = reinterpret_cast<__half2 *>(p.o.x_hi + (size_t)(t0 + g) * H + k);
                __half2 *dl = reinterpret_cast<__half2 *>(p.o.x_lo + (size_t)(t0 + g) * H + k);
                dh[0] = h01;
                dh[1] = h23;
                dl[0] = l01;
                dl[1] = l23;
            }
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const int e = 8 * (nb0 + nb) + g;
            float4 wv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kin && e < p.E) wv = __ldg(reinterpret_cast<const float4 *>(p.w + (size_t)e * H + k));
            dmma884(acc[nb][0], acc[nb][1], a[0], (double)wv.x);
            dmma884(acc[nb][0], acc[nb][1], a[1], (double)wv.y);
            dmma884(acc[nb][0], acc[nb][1], a[2], (double)wv.z);
            dmma884(acc[nb][0], acc[nb][1], a[3], (double)wv.w);
        }
    }
}

// One CTA = one chunk of kRouteTokens tokens x one K-slice (ksplit > 1 for
// small T spreads the router weight over more SMs).  Phases: (1) each token's
// sum of squares over its full row (primitives.go:61-65) in float64; (2) the
// slice's normalized values feed the DMMA logits directly (and their fp16 split
// is stored); (3) fixed-order reduction of the warps' partials; with ksplit > 1
// the last CTA of a chunk (arrival counter) sums the slices in slice order;
// (4) per token: logits = f32(sum) + bias, top-k, softmax over the selected.
// Every step is deterministic.
// NB: expert blocks of 8 per DMMA pass (4 for E <= 32, 8 for <= 64, 16 beyond,
// looping passes past 128 experts).
template <int NB>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(RouteParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int H = p.H, E = p.E;
    double *part = reinterpret_cast<double *>(smem);                              // [warps][8][E]
    int *hist_s = reinterpret_cast<int *>(part + kRouteWarps * kRouteTokens * E); // [E]
    __shared__ int is_last;
    __shared__ double ssq[kRouteWarps][kRouteTokens];
    __shared__ double inv_s[kRouteTokens];

    const int chunk = blockIdx.x, ks = blockIdx.y;
    const int t0 = chunk * kRouteTokens;
    const int nt = min(kRouteTokens, p.T - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // 1. float64 sums of squares of the chunk's rows (all threads, float4 loads)
    {
        const int H4 = H / 4;
        const float4 *res4 = reinterpret_cast<const float4 *>(p.residual + (size_t)t0 * H);
        double ss[kRouteTokens];
#pragma unroll
        for (int t = 0; t < kRouteTokens; ++t) ss[t] = 0.0;
        for (int i = threadIdx.x; i < H4; i += blockDim.x) {
            float4 v[kRouteTokens];
#pragma unroll
            for (int t = 0; t < kRouteTokens; ++t)
                if (t < nt) v[t] = __ldg(res4 + (size_t)t * H4 + i);
#pragma unroll
            for (int t = 0; t < kRouteTokens; ++t) {
                if (t < nt) {
                    ss[t] += (double)v[t].x * (double)v[t].x;
                    ss[t] += (double)v[t].y * (double)v[t].y;
                    ss[t] += (double)v[t].z * (double)v[t].z;
                    ss[t] += (double)v[t].w * (double)v[t].w;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kRouteTokens; ++t) {
            const double w = warp_sum_f64(ss[t]);
            if (lane == 0) ssq[warp][t] = w;
        }
        for (int e = threadIdx.x; e < E; e += blockDim.x) hist_s[e] = 0;
        __syncthreads();
        if (threadIdx.x < kRouteTokens) {
            double sum = 0.0;
            for (int w = 0; w < kRouteWarps; ++w) sum += ssq[w][threadIdx.x];
            inv_s[threadIdx.x] = 1.0 / sqrt(sum / (double)H + (double)p.eps);
        }
        __syncthreads();
    }

    // 2. partial logits over this CTA's K-slice, the slice split across warps in
    //    16-aligned ranges
    const int kslice = ((H + p.ksplit - 1) / p.ksplit + 15) & ~15;
    const int kbeg = min(H, ks * kslice), kend = min(H, kbeg + kslice);
    const int wslice = ((kend - kbeg + kRouteWarps - 1) / kRouteWarps + 15) & ~15;
    const int k0 = min(kend, kbeg + warp * wslice), k1 = min(kend, k0 + wslice);
    {
        const int g = lane >> 2, c = lane & 3;
        for (int nb0 = 0; 8 * nb0 < E; nb0 += NB) {
            double acc[NB][2];
            logits_pass<NB>(p, inv_s, t0, nt, k0, k1, nb0, lane, nb0 == 0, acc);
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int e = 8 * (nb0 + nb) + 2 * c + i;
                    if (e < E) part[(warp * kRouteTokens + g) * E + e] = acc[nb][i];
                }
        }
    }
    __syncthreads();

    if (p.ksplit > 1) {
        // publish this slice's sums (fixed warp order), then elect the last CTA
        for (int idx = threadIdx.x; idx < nt * E; idx += blockDim.x) {
            int t = idx / E, e = idx % E;
            double s = 0.0;
            for (int w = 0; w < kRouteWarps; ++w) s += part[(w * kRouteTokens + t) * E + e];
            p.partial[((size_t)ks * p.T + t0 + t) * E + e] = s;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            int prev = atomicAdd(p.arrivals + chunk, 1);
            is_last = prev == p.ksplit - 1;
            if (is_last) p.arrivals[chunk] = 0;  // ready for the next call
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
    }

    // 3. token t0 + warp: logits, top-k, softmax over the selected logits
    if (warp < nt) {
        const int t = t0 + warp;
        constexpr int EPL = 8;  // up to 256 experts, lane + 32 j
        float lg[EPL];
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            int e = lane + 32 * j;
            lg[j] = 0.0f;
            if (e < E) {
                double s = 0.0;
                if (p.ksplit > 1) {
                    double sl[kMaxKSplit];  // all slice loads in flight, then a fixed-order sum
#pragma unroll
                    for (int q = 0; q < kMaxKSplit; ++q)
                        sl[q] = q < p.ksplit ? __ldcg(p.partial + ((size_t)q * p.T + t) * E + e) : 0.0;
#pragma unroll
                    for (int q = 0; q < kMaxKSplit; ++q) s += sl[q];
                } else {
                    for (int w = 0; w < kRouteWarps; ++w) s += part[(w * kRouteTokens + warp) * E + e];
                }
                lg[j] = (float)s + p.bias[e];  // primitives.go:29 then :44
                p.o.logits[(size_t)t * E + e] = lg[j];
            }
        }
        unsigned used = 0;  // bit j: expert lane + 32 j already selected
        int my_e = -1;
        float my_v = 0.0f;
        for (int s = 0; s < p.k; ++s) {
            float bv = 0.0f;
            int be = -1;
#pragma unroll
            for (int j = 0; j < EPL; ++j) {
                int e = lane + 32 * j;
                if (e < E && !(used >> j & 1u) && better(lg[j], e, bv, be)) {
                    bv = lg[j];
                    be = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oe = __shfl_xor_sync(0xffffffffu, be, o);
                if (better(ov, oe, bv, be)) {
                    bv = ov;
                    be = oe;
                }
            }
            if (be >= 0 && (be & 31) == lane) used |= 1u << (be >> 5);
            if (lane == s) {
                my_e = be;
                my_v = bv;
            }
        }
        // softmax in float64 over the selected logits (moe.go:29-39); lane s owns slot s
        const double maxv = (double)__shfl_sync(0xffffffffu, my_v, 0);
        double wexp = lane < p.k ? exp((double)my_v - maxv) : 0.0;
        float wf = (float)wexp;
        double den = 0.0;
        for (int s = 0; s < p.k; ++s) den += __shfl_sync(0xffffffffu, wexp, s);  // slot order
        if (lane < p.k) {
            p.o.topk_idx[(size_t)t * p.k + lane] = my_e;
            p.o.topk_w[(size_t)t * p.k + lane] = (float)((double)wf / den);
            atomicAdd(hist_s + my_e, 1);
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) p.o.hist[(size_t)chunk * E + e] = hist_s[e];
    if (gridDim.x == 1) {
        // T <= kRouteTokens: this CTA holds every pair, so it also writes the
        // stable (expert, token, slot) permutation and the launch of K2 is skipped.
        __shared__ int offs[257];
        const int npairs = p.T * p.k;
        if (threadIdx.x == 0) {
            int acc = 0, na = 0;
            for (int e = 0; e < E; ++e) {
                offs[e] = acc;
                p.o.offsets[e] = acc;
                p.o.counts[e] = hist_s[e];
                p.o.chunk_base[e] = 0;  // one chunk: the expert's pairs start at its offset
                if (hist_s[e] > 0) p.o.active[na++] = e;
                acc += hist_s[e];
            }
            offs[E] = acc;
            p.o.offsets[E] = acc;
            p.o.active[E] = na;
        }
        __syncthreads();
        for (int q = threadIdx.x; q < npairs; q += blockDim.x) {
            const int ex = p.o.topk_idx[q];
            int rank = 0;
            for (int r = 0; r < q; ++r) rank += p.o.topk_idx[r] == ex;
            const int pos = offs[ex] + rank;
            p.o.perm_pair[pos] = q;
            p.o.inv[q] = pos;
        }
    }
}

// K2a: one CTA per expert e.  Its per-chunk pair counts hist[c][e], split into
// contiguous chunk ranges over the threads (loads batched, 16 in flight), become
// its chunk bases: chunk_base[c][e] = the expert's pairs in chunks before c (local
// to the expert; the scatter adds offsets[e]); counts[e] = its total.
constexpr int kScanThreads = 256;
__global__ void __launch_bounds__(kScanThreads) scan_expert_kernel(int T, int E, RouteOut o) {
    __shared__ int wsum[kScanThreads / 32];
    const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    const int per = (nchunk + kScanThreads - 1) / kScanThreads;
    const int c0 = min(nchunk, tid * per), c1 = min(nchunk, c0 + per);
    constexpr int kBatch = 16;
    int s = 0;
    for (int c = c0; c < c1; c += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) v[j] = c + j < c1 ? o.hist[(size_t)(c + j) * E + e] : 0;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) s += v[j];
    }
    // exclusive scan of the threads' sums, in thread order
    int incl = s;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, d);
        incl += lane >= d ? x : 0;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    int base = before + incl - s;
    for (int c = c0; c < c1; c += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) v[j] = c + j < c1 ? o.hist[(size_t)(c + j) * E + e] : 0;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (c + j < c1) o.chunk_base[(size_t)(c + j) * E + e] = base;
            base += v[j];
        }
    }
    if (tid == kScanThreads - 1) o.counts[e] = base;  // the last thread ends at the expert's total
}

// K2b: one thread.  Expert offsets (exclusive scan of the counts) and the
// active-expert list.
__global__ void scan_offsets_kernel(int E, RouteOut o) {
    int acc = 0, na = 0;
    for (int e = 0; e < E; ++e) {
        const int n = o.counts[e];
        o.offsets[e] = acc;
        if (n > 0) o.active[na++] = e;
        acc += n;
    }
    o.offsets[E] = acc;
    o.active[E] = na;
}

// K2c: one warp per chunk.  Pair (t, s) goes to offsets[e] + chunk_base[chunk][e] + the
// number of earlier pairs of expert e in the chunk (match_any ranks, carried across
// 32-pair rounds): a stable sort by (e, t, s).  With GATHER the warp also copies
// the chunk's normalized rows (fp16 hi/lo) to their expert-sorted positions,
// which is the B operand of the tensor-core gate_up GEMM.
constexpr int kScatterWarps = 4;

// Stable positions of one chunk's pairs, computed by one warp; returns nothing,
// writes perm_pair/inv and (if pos_s) the positions to shared memory.
__device__ __forceinline__ void chunk_positions(int chunk, int T, int E, int k, const RouteOut &o, int *carry,
                                                int *pos_s, int lane) {
    for (int e = lane; e < E; e += 32) carry[e] = 0;
    __syncwarp();
    const int first = chunk * kRouteTokens * k;
    const int last = min(T * k, first + kRouteTokens * k);
    const unsigned lt = (1u << lane) - 1u;
    for (int q0 = first; q0 < last; q0 += 32) {
        const int q = q0 + lane;
        const bool valid = q < last;
        const int ex = valid ? o.topk_idx[q] : E;  // E: sentinel group for idle lanes
        const unsigned peers = __match_any_sync(0xffffffffu, ex);
        if (valid) {
            const int pos = o.offsets[ex] + o.chunk_base[(size_t)chunk * E + ex] + carry[ex] + __popc(peers & lt);
            o.perm_pair[pos] = q;
            o.inv[q] = pos;
            if (pos_s) pos_s[q - first] = pos;
        }
        __syncwarp();
        if (valid && (peers >> lane) == 1u) carry[ex] += __popc(peers);  // last lane of its group
        __syncwarp();
    }
}

// K2c (GEMV path): one warp per chunk.  Pair (t, s) goes to offsets[e] + chunk_base[chunk][e]
// + the number of earlier pairs of expert e in the chunk: a stable sort by
// (e, t, s).
__global__ void __launch_bounds__(kScatterWarps * 32) scatter_kernel(int T, int E, int k, RouteOut o) {
    extern __shared__ int carry_all[];  // [warps][E]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    const int chunk = blockIdx.x * kScatterWarps + warp;
    if (chunk >= nchunk) return;  // whole warp
    chunk_positions(chunk, T, E, k, o, carry_all + warp * E, nullptr, lane);
}

// K2c (tensor path): one CTA per chunk.  Warp 0 computes the positions, then
// warp t copies token t's normalized row (fp16 hi/lo) to its k expert-sorted
// positions: the B operand of the tensor-core gate_up GEMM.
__global__ void __launch_bounds__(kRouteTokens * 32)
    scatter_gather_kernel(int T, int E, int k, int H, RouteOut o, __half *xp_hi, __half *xp_lo) {
    extern __shared__ int sg_smem[];  // carry [E], positions [kRouteTokens * k]
    int *carry = sg_smem, *pos_s = sg_smem + E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x;
    if (warp == 0) chunk_positions(chunk, T, E, k, o, carry, pos_s, lane);
    __syncthreads();
    const int t = chunk * kRouteTokens + warp;
    if (t >= T) return;
    const uint4 *sh = reinterpret_cast<const uint4 *>(o.x_hi + (size_t)t * H);
    const uint4 *sl = reinterpret_cast<const uint4 *>(o.x_lo + (size_t)t * H);
    const int H8 = H / 8;
    for (int i = lane; i < H8; i += 32) {
        const uint4 vh = sh[i], vl = sl[i];
        for (int sidx = 0; sidx < k; ++sidx) {
            const int pos = pos_s[warp * k + sidx];
            reinterpret_cast<uint4 *>(xp_hi + (size_t)pos * H)[i] = vh;
            reinterpret_cast<uint4 *>(xp_lo + (size_t)pos * H)[i] = vl;
        }
    }
}

}  // namespace

static int route_ksplit(int H, int nchunk) {
    int ksplit = (2 * 148 + nchunk - 1) / nchunk;
    ksplit = ksplit < 1 ? 1 : (ksplit > kMaxKSplit ? kMaxKSplit : ksplit);
    // every 16-aligned K-slice must be non-empty
    while (ksplit > 1 && (((H + ksplit - 1) / ksplit + 15) & ~15) * (ksplit - 1) >= H) --ksplit;
    return ksplit;
}

size_t route_partial_elems(int max_tokens, int H, int E) {
    size_t best = 0;
    const int max_chunks = (max_tokens + kRouteTokens - 1) / kRouteTokens;
    for (int nc = 1; nc <= max_chunks; ++nc) {
        const int ks = route_ksplit(H, nc);
        if (ks == 1) break;  // ksplit only falls as the chunk count grows
        const int T = nc * kRouteTokens < max_tokens ? nc * kRouteTokens : max_tokens;
        const size_t need = (size_t)ks * T * E;
        if (need > best) best = need;
    }
    return best;
}

cudaError_t launch_route_impl(const Dims &d, const LayerDev &L, const float *residual, int T,
                              const RouteOut &o, double *partial, int32_t *arrivals,
                              cudaStream_t st, StageHook hook, void *hook_arg) {
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    const int ksplit = (partial && arrivals) ? route_ksplit(d.H, nchunk) : 1;
    RouteParams p;
    p.residual = residual;
    p.gain = L.norm_gain;
    p.w = L.router_w;
    p.bias = L.router_b;
    p.T = T;
    p.H = d.H;
    p.E = d.E;
    p.k = d.k;
    p.ksplit = ksplit;
    p.eps = d.eps;
    p.o = o;
    p.partial = partial;
    p.arrivals = arrivals;
    const size_t smem = (size_t)kRouteWarps * kRouteTokens * d.E * sizeof(double) + d.E * sizeof(int);
    const dim3 grid(nchunk, ksplit);
    cudaError_t err;
#define AMOE_ROUTE(NB)                                                                            \
    do {                                                                                          \
        err = cudaFuncSetAttribute(route_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem);                                                    \
        if (err != cudaSuccess) return err;                                                       \
        route_kernel<NB><<<grid, kRouteWarps * 32, smem, st>>>(p);                                \
    } while (0)
    if (d.E <= 32) AMOE_ROUTE(4);
    else if (d.E <= 64) AMOE_ROUTE(8);
    else AMOE_ROUTE(16);
#undef AMOE_ROUTE
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    if (hook) hook(hook_arg, 0);
    if (nchunk == 1) return cudaSuccess;  // counts, offsets and chunk bases written by route_kernel
    scan_expert_kernel<<<d.E, kScanThreads, 0, st>>>(T, d.E, o);
    scan_offsets_kernel<<<1, 1, 0, st>>>(d.E, o);
    return cudaGetLastError();
}

cudaError_t launch_scatter(const Dims &d, int T, const RouteOut &o, bool gather, __half *xp_hi,
                           __half *xp_lo, cudaStream_t st) {
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    if (gather) {
        const size_t smem = (size_t)(d.E + kRouteTokens * d.k) * sizeof(int);
        scatter_gather_kernel<<<nchunk, kRouteTokens * 32, smem, st>>>(T, d.E, d.k, d.H, o, xp_hi, xp_lo);
    } else {
        const size_t smem = (size_t)kScatterWarps * d.E * sizeof(int);
        scatter_kernel<<<(nchunk + kScatterWarps - 1) / kScatterWarps, kScatterWarps * 32, smem, st>>>(T, d.E,
                                                                                                   d.k, o);
    }
    return cudaGetLastError();
}

}  // namespace amoe
