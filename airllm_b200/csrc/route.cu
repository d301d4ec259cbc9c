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
    const float *wt;   // [H][E]
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

template <int NT, int EPL>
__device__ __forceinline__ void partial_logits(const float *xn, int H, const float *wt, int E,
                                               int k0, int k1, int lane, double (&acc)[EPL][NT]) {
    // U router rows in flight per batch: the loads of a batch are independent
    constexpr int U = EPL >= 8 ? 2 : 8 / EPL;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[j][t] = 0.0;
    for (int kb = k0; kb < k1; kb += U) {
        float wv[U][EPL];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int j = 0; j < EPL; ++j) {
                const int e = lane + 32 * j;
                wv[u][j] = (kb + u < k1 && e < E) ? __ldg(wt + (size_t)(kb + u) * E + e) : 0.0f;
            }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (kb + u >= k1) break;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const double xv = (double)xn[t * H + kb + u];
#pragma unroll
                for (int j = 0; j < EPL; ++j) acc[j][t] += xv * (double)wv[u][j];
            }
        }
    }
}

// One CTA = one chunk of kRouteTokens tokens x one K-slice.  With ksplit > 1
// the last CTA of a chunk to finish (arrival counter) reduces the partial sums
// in fixed slice order and runs top-k, so the result does not depend on timing.
template <int EPL>
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(RouteParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int H = p.H, E = p.E;
    float *xn = reinterpret_cast<float *>(smem);                                  // [8][H]
    double *part = reinterpret_cast<double *>(xn + kRouteTokens * H);             // [warps][8][E]
    int *hist_s = reinterpret_cast<int *>(part + kRouteWarps * kRouteTokens * E); // [E]
    __shared__ int is_last;

    const int chunk = blockIdx.x, ks = blockIdx.y;
    const int t0 = chunk * kRouteTokens;
    const int nt = min(kRouteTokens, p.T - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // 1. RMSNorm (primitives.go:61-70).  All threads sweep the chunk's rows with
    //    float4 loads (every token's loads in flight together); float64 sums of
    //    squares per token, reduced per warp and then across warps.
    __shared__ double ssq[kRouteWarps][kRouteTokens];
    __shared__ double inv_s[kRouteTokens];
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
        __syncthreads();
        if (threadIdx.x < kRouteTokens) {
            double sum = 0.0;
            for (int w = 0; w < kRouteWarps; ++w) sum += ssq[w][threadIdx.x];
            inv_s[threadIdx.x] = 1.0 / sqrt(sum / (double)H + (double)p.eps);
        }
        __syncthreads();
        const float4 *g4 = reinterpret_cast<const float4 *>(p.gain);
        const bool write_split = ks == 0;
        for (int i = threadIdx.x; i < H4; i += blockDim.x) {
            const float4 g = __ldg(g4 + i);
#pragma unroll
            for (int t = 0; t < kRouteTokens; ++t) {
                float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (t < nt) {
                    const float4 x = __ldg(res4 + (size_t)t * H4 + i);
                    const double inv = inv_s[t];
                    // float32(float64(x) * inverseRMS * float64(g)), evaluated left to right
                    o.x = (float)((double)x.x * inv * (double)g.x);
                    o.y = (float)((double)x.y * inv * (double)g.y);
                    o.z = (float)((double)x.z * inv * (double)g.z);
                    o.w = (float)((double)x.w * inv * (double)g.w);
                    if (write_split) {
                        const __half2 h01 = __floats2half2_rn(o.x, o.y), h23 = __floats2half2_rn(o.z, o.w);
                        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                        const __half2 l01 = __floats2half2_rn(o.x - f01.x, o.y - f01.y);
                        const __half2 l23 = __floats2half2_rn(o.z - f23.x, o.w - f23.y);
                        __half2 *dh = reinterpret_cast<__half2 *>(p.o.x_hi + (size_t)(t0 + t) * H + 4 * i);
                        __half2 *dl = reinterpret_cast<__half2 *>(p.o.x_lo + (size_t)(t0 + t) * H + 4 * i);
                        dh[0] = h01;
                        dh[1] = h23;
                        dl[0] = l01;
                        dl[1] = l23;
                    }
                }
                reinterpret_cast<float4 *>(xn + t * H)[i] = o;
            }
        }
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist_s[e] = 0;
    __syncthreads();

    // 2. partial router logits over this CTA's K-slice, split across warps
    const int kslice = (H + p.ksplit - 1) / p.ksplit;
    const int kbeg = ks * kslice, kend = min(H, kbeg + kslice);
    const int wslice = (kend - kbeg + kRouteWarps - 1) / kRouteWarps;
    const int k0 = min(kend, kbeg + warp * wslice), k1 = min(kend, k0 + wslice);
    {
        double acc[EPL][kRouteTokens];
        if (nt == 1) {
            double a1[EPL][1];
            partial_logits<1, EPL>(xn, H, p.wt, E, k0, k1, lane, a1);
#pragma unroll
            for (int j = 0; j < EPL; ++j) {
                acc[j][0] = a1[j][0];
#pragma unroll
                for (int t = 1; t < kRouteTokens; ++t) acc[j][t] = 0.0;
            }
        } else if (nt <= 4) {
            double a4[EPL][4];
            partial_logits<4, EPL>(xn, H, p.wt, E, k0, k1, lane, a4);
#pragma unroll
            for (int j = 0; j < EPL; ++j)
#pragma unroll
                for (int t = 0; t < kRouteTokens; ++t) acc[j][t] = t < 4 ? a4[j][t] : 0.0;
        } else {
            partial_logits<kRouteTokens, EPL>(xn, H, p.wt, E, k0, k1, lane, acc);
        }
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            int e = lane + 32 * j;
            if (e < E)
#pragma unroll
                for (int t = 0; t < kRouteTokens; ++t) part[(warp * kRouteTokens + t) * E + e] = acc[j][t];
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
        float lg[EPL];
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            int e = lane + 32 * j;
            lg[j] = 0.0f;
            if (e < E) {
                double s = 0.0;
                if (p.ksplit > 1) {
                    for (int q = 0; q < p.ksplit; ++q)
                        s += __ldcg(p.partial + ((size_t)q * p.T + t) * E + e);
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
                p.o.chunk_base[e] = acc;
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

// K2: one CTA.  Column scan of the per-chunk expert histograms, then every pair
// (t, s) gets position offsets[e] + (#pairs of expert e in earlier chunks) +
// (#earlier pairs of expert e in its own chunk): a stable sort by (e, t, s).
__global__ void __launch_bounds__(1024) permute_kernel(int T, int E, int k, RouteOut o) {
    extern __shared__ int sm[];
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    const int groups = max(1, (int)blockDim.x / E);
    int *gsum = sm;                    // [groups][E]
    int *tot = gsum + groups * E;      // [E]
    int *eoff = tot + E;               // [E+1]
    const int tid = threadIdx.x;
    const int e = tid % E, g = tid / E;
    const int per = (nchunk + groups - 1) / groups;
    const int c0 = min(nchunk, g * per), c1 = min(nchunk, c0 + per);
    if (g < groups) {
        int s = 0;
        for (int c = c0; c < c1; ++c) s += o.hist[(size_t)c * E + e];
        gsum[g * E + e] = s;
    }
    __syncthreads();
    if (tid < E) {
        int s = 0;
        for (int gg = 0; gg < groups; ++gg) {
            int v = gsum[gg * E + tid];
            gsum[gg * E + tid] = s;
            s += v;
        }
        tot[tid] = s;
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0, na = 0;
        for (int x = 0; x < E; ++x) {
            eoff[x] = s;
            o.offsets[x] = s;
            o.counts[x] = tot[x];
            if (tot[x] > 0) o.active[na++] = x;
            s += tot[x];
        }
        eoff[E] = s;
        o.offsets[E] = s;
        o.active[E] = na;
    }
    __syncthreads();
    if (g < groups) {
        int s = eoff[e] + gsum[g * E + e];
        for (int c = c0; c < c1; ++c) {
            o.chunk_base[(size_t)c * E + e] = s;
            s += o.hist[(size_t)c * E + e];
        }
    }
    __syncthreads();
    const int npairs = T * k;
    for (int pidx = tid; pidx < npairs; pidx += blockDim.x) {
        const int ex = o.topk_idx[pidx];
        const int c = (pidx / k) / kRouteTokens;
        const int first = c * kRouteTokens * k;
        int rank = 0;
        for (int q = first; q < pidx; ++q) rank += o.topk_idx[q] == ex;
        const int pos = o.chunk_base[(size_t)c * E + ex] + rank;
        o.perm_pair[pos] = pidx;
        o.inv[pidx] = pos;
    }
}

}  // namespace

static int route_ksplit(int H, int nchunk) {
    int ksplit = (2 * 148 + nchunk - 1) / nchunk;
    ksplit = ksplit < 1 ? 1 : (ksplit > kMaxKSplit ? kMaxKSplit : ksplit);
    // every K-slice must be non-empty
    while (ksplit > 1 && (H + ksplit - 1) / ksplit * (ksplit - 1) >= H) --ksplit;
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
    p.wt = L.router_wt;
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
    const size_t smem = (size_t)kRouteTokens * d.H * sizeof(float) +
                        (size_t)kRouteWarps * kRouteTokens * d.E * sizeof(double) + d.E * sizeof(int);
    dim3 grid(nchunk, ksplit);
    cudaError_t err;
#define AMOE_ROUTE(EPL)                                                                         \
    do {                                                                                        \
        err = cudaFuncSetAttribute(route_kernel<EPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem);                                                  \
        if (err != cudaSuccess) return err;                                                     \
        route_kernel<EPL><<<grid, kRouteWarps * 32, smem, st>>>(p);                             \
    } while (0)
    if (d.E <= 32) AMOE_ROUTE(1);
    else if (d.E <= 64) AMOE_ROUTE(2);
    else if (d.E <= 128) AMOE_ROUTE(4);
    else AMOE_ROUTE(8);
#undef AMOE_ROUTE
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    if (hook) hook(hook_arg, 0);
    if (nchunk == 1) return cudaSuccess;  // permutation written by route_kernel
    const int threads = 1024;
    const int groups = threads / d.E > 0 ? threads / d.E : 1;
    const size_t psmem = (size_t)(groups * d.E + d.E + d.E + 1) * sizeof(int);
    permute_kernel<<<1, threads, psmem, st>>>(T, d.E, d.k, o);
    err = cudaGetLastError();
    if (hook) hook(hook_arg, 1);
    return err;
}

}  // namespace amoe
