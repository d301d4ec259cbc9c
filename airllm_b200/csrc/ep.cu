// ep.cu -- expert parallelism: experts sharded over the GPUs of one box, rows
// exchanged by stores into peer memory over NVLink (no counterpart in the
// reference, which is single-threaded CPU code; the single-GPU path is its
// oracle: the per-row arithmetic is the same, so outputs match bit for bit).
//
// Per forward, on every rank, in stream order:
//   ep_counts_kernel    (1 CTA)  counts -> every rank's table, wait for all rows,
//                                derive the exchange layout
//   ep_dispatch_kernel  (grid)   rows -> owners' receive buffers (expert-major);
//                                return targets of the rows this rank receives;
//                                last CTA publishes the dispatch flags
//   ep_wait_kernel      (1 warp) all dispatch flags of this epoch are in
//   gate_up, down GEMMs          down stores outputs into the sources' windows,
//                                last CTA publishes the return flags
//   ep_wait_kernel      (1 warp) all return flags are in; then the combine
// Flags hold the epoch (forward count), which grows monotonically, so none is
// ever reset.  A rank writes into a peer's buffers only after the peer has
// finished reading them for the previous epoch: a peer's receive buffer is
// consumed before the peer returns outputs, and a rank dispatches epoch f+1 only
// after every peer's epoch-f returns reached it.  Every wait is bounded (global
// timer); a failed wait records an error code, empties the expert ranges and
// withholds this rank's later flags, so peers time out instead of reading
// incomplete data.
#include "amoe_internal.cuh"

#include <dlfcn.h>

#include <mutex>

namespace amoe {

// ---- NCCL (setup only: IPC handle exchange), resolved at run time ----------------
NcclApi g_nccl;

bool nccl_load(std::string *err) {
    static std::once_flag once;
    static bool ok = false;
    static std::string why;
    std::call_once(once, []() {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            why = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
#define AMOE_SYM(name)                                                        \
    g_nccl.name = reinterpret_cast<decltype(g_nccl.name)>(dlsym(h, #name));   \
    if (!g_nccl.name) {                                                       \
        why = "libnccl.so.2 lacks " #name;                                     \
        return;                                                               \
    }
        AMOE_SYM(ncclGetUniqueId)
        AMOE_SYM(ncclCommInitRank)
        AMOE_SYM(ncclCommDestroy)
        AMOE_SYM(ncclAllGather)
        AMOE_SYM(ncclGetErrorString)
#undef AMOE_SYM
        ok = true;
    });
    if (!ok && err) *err = why;
    return ok;
}

namespace {
inline size_t up256(size_t v) { return (v + 255) & ~size_t(255); }
}  // namespace

EpWindow ep_window(int N, int E, int H, int p_cap, int r_cap) {
    EpWindow w{};
    size_t off = 0;
    w.flags = off;
    off = up256(off + 3 * kMaxEpRanks * 4);
    w.table = off;
    off = up256(off + (size_t)N * E * 4);
    w.recv_hi = off;
    off = up256(off + (size_t)r_cap * H * 2);
    w.recv_lo = off;
    off = up256(off + (size_t)r_cap * H * 2);
    // the token records of the tcgen05 path share the two row buffers' space
    const size_t rec = (size_t)r_cap * ((H + 127) / 128) * 4 * (5 * 16 + 8);
    if (w.recv_hi + rec > off) off = up256(w.recv_hi + rec);
    w.y = off;
    off = up256(off + (size_t)p_cap * H * 4);
    w.bytes = off;
    return w;
}

// ---- layout of one exchange ------------------------------------------------------
// table[s][e]: pairs source s routes to global expert e; colsum(e) = sum_s table[s][e].
//   send_base[e]       = sum_{owner(e)*El <= e' < e} colsum(e') + sum_{s < me} table[s][e]
//   offsets_loc[el]    = sum_{me*El <= e' < me*El + el} colsum(e')
//   seg_start[el][s]   = offsets_loc[el] + sum_{s' < s} table[s'][me*El + el]
//   src_pos[el][s]     = sum_{e' < me*El + el} table[s][e']
// so the owner's receive buffer holds expert el's rows source by source, each
// source's rows in its own (token, slot) order -- the order the single-GPU path
// gives them when the ranks' tokens are concatenated.
int ep_layout(int N, int El, int me, const int32_t *table, int32_t *send_base, int32_t *offsets_loc,
              int32_t *seg_start, int32_t *src_pos) {
    if (N < 1 || N > kMaxEpRanks || El < 1 || me < 0 || me >= N || !table) return -1;
    const int E = N * El;
    for (int i = 0; i < N * E; ++i)
        if (table[i] < 0) return -1;
    std::vector<long long> col(E, 0);
    for (int s = 0; s < N; ++s)
        for (int e = 0; e < E; ++e) col[e] += table[s * E + e];
    for (int q = 0; q < N; ++q) {
        long long acc = 0;
        for (int el = 0; el < El; ++el) {
            const int e = q * El + el;
            long long lower = 0;
            for (int s = 0; s < me; ++s) lower += table[s * E + e];
            if (send_base) send_base[e] = (int32_t)(acc + lower);
            if (q == me && offsets_loc) offsets_loc[el] = (int32_t)acc;
            acc += col[e];
        }
        if (q == me && offsets_loc) offsets_loc[El] = (int32_t)acc;
    }
    for (int s = 0; s < N; ++s) {
        long long pre = 0;
        for (int e = 0; e < me * El; ++e) pre += table[s * E + e];
        for (int el = 0; el < El; ++el) {
            const int e = me * El + el;
            if (src_pos) src_pos[el * N + s] = (int32_t)pre;
            pre += table[s * E + e];
        }
    }
    if (seg_start) {
        long long acc = 0;
        for (int el = 0; el < El; ++el) {
            const int e = me * El + el;
            for (int s = 0; s < N; ++s) {
                seg_start[el * N + s] = (int32_t)acc;
                acc += table[s * E + e];
            }
        }
    }
    return 0;
}

namespace {

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for *flag >= epoch (system scope); false once limit_ns passed.
__device__ bool wait_epoch(const int32_t *flag, int epoch, long long limit_ns) {
    const unsigned long long t0 = global_ns();
    while (ld_acquire_sys(flag) - epoch < 0) {
        if ((long long)(global_ns() - t0) > limit_ns) return false;
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ int32_t *win_flag(uint8_t *win, const EpWindow &w, int which, int src) {
    return reinterpret_cast<int32_t *>(win + w.flags) + which * kMaxEpRanks + src;
}

// Empties this rank's expert ranges so that the GEMMs do nothing (failed wait).
__device__ void empty_ranges(const EpArgs &a) {
    for (int i = threadIdx.x; i <= a.El; i += blockDim.x) {
        a.m.offsets_loc[i] = 0;
        a.m.active_loc[i] = 0;
    }
    if (threadIdx.x == 0) *a.m.status = 0;
}

constexpr int kCountThreads = 256;

// One CTA.  E <= 256 (validated at create), N <= kMaxEpRanks.
__global__ void __launch_bounds__(kCountThreads) ep_counts_kernel(EpArgs a) {
    __shared__ int32_t tab[kMaxEpRanks * 256];
    __shared__ int32_t col[256], lower[256], inblock[256];
    __shared__ int32_t total_loc;
    __shared__ uint8_t *win[kMaxEpRanks];
    __shared__ int ok;
    const int tid = threadIdx.x, N = a.N, E = a.E, El = a.El, me = a.me;
    if (tid < N) win[tid] = a.m.win[tid];
    if (tid == 0) ok = 1;
    __syncthreads();
    // 1. this rank's counts into row `me` of every rank's table, then its count flags
    for (int i = tid; i < N * E; i += kCountThreads) {
        const int q = i / E, e = i - q * E;
        reinterpret_cast<int32_t *>(win[q] + a.w.table)[me * E + e] = a.counts[e];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < N) st_release_sys(win_flag(win[tid], a.w, kEpFlagCount, me), a.epoch);
    // 2. every rank's row of this epoch
    if (tid < N && !wait_epoch(win_flag(win[me], a.w, kEpFlagCount, tid), a.epoch, a.count_limit_ns)) {
        ok = 0;
        atomicCAS(a.err, 0, 30);
    }
    __syncthreads();
    if (!ok) {
        empty_ranges(a);
        return;
    }
    const int32_t *tg = reinterpret_cast<const int32_t *>(win[me] + a.w.table);
    for (int i = tid; i < N * E; i += kCountThreads) tab[i] = __ldcv(tg + i);
    __syncthreads();
    // 3. column sums and the rows of lower ranks, per expert
    if (tid < E) {
        int s = 0, lo = 0;
        for (int q = 0; q < N; ++q) {
            const int v = tab[q * E + tid];
            if (q < me) lo += v;
            s += v;
        }
        col[tid] = s;
        lower[tid] = lo;
    }
    __syncthreads();
    // 4. exclusive prefix of the column sums inside each owner's expert block
    if (tid < N) {
        int acc = 0;
        for (int el = 0; el < El; ++el) {
            inblock[tid * El + el] = acc;
            acc += col[tid * El + el];
        }
        if (tid == me) total_loc = acc;
    } else if (tid >= 32 && tid - 32 < N) {
        // 5. src_pos: source s's sorted position of its first pair for each local expert
        const int s = tid - 32;
        int pre = 0;
        for (int e = 0; e < me * El; ++e) pre += tab[s * E + e];
        for (int el = 0; el < El; ++el) {
            a.m.src_pos[el * N + s] = pre;
            pre += tab[s * E + me * El + el];
        }
    }
    __syncthreads();
    if (tid < E) a.m.send_base[tid] = inblock[tid] + lower[tid];
    for (int el = tid; el <= El; el += kCountThreads) a.m.offsets_loc[el] = el < El ? inblock[me * El + el] : total_loc;
    for (int el = tid; el < El; el += kCountThreads) {
        int acc = inblock[me * El + el];
        for (int s = 0; s < N; ++s) {
            a.m.seg_start[el * N + s] = acc;
            acc += tab[s * E + me * El + el];
        }
    }
    if (tid == 0) {
        int na = 0;
        for (int el = 0; el < El; ++el)
            if (col[me * El + el] > 0) a.m.active_loc[na++] = el;
        a.m.active_loc[El] = na;
        // expert path: every rank reaches the same choice from the same table,
        // and it is the single-GPU rule applied to the group's tokens
        long long pairs = 0;
        for (int e = 0; e < E; ++e) pairs += col[e];
        *a.m.mode = a.path == 2 || (a.path == 0 && pairs >= 32LL * E) ? 1 : 0;
        *a.m.status = 1;
    }
}

constexpr int kDispatchThreads = 256;
constexpr int kDispatchUnroll = 4;

// Grid-stride over this rank's expert-sorted pairs, one warp per row: the pair's
// token goes into the owner's receive buffer, as its five-term token records when
// the group takes the tcgen05 path (2.75 bytes an element, quantized once at the
// source), else as the fp16 hi and lo rows the GEMV reads.  Then the return
// targets of the rows this rank receives.
__global__ void __launch_bounds__(kDispatchThreads) ep_dispatch_kernel(EpArgs a) {
    __shared__ uint8_t *win[kMaxEpRanks];
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < a.N) win[tid] = a.m.win[tid];
    __syncthreads();
    const bool ok = *reinterpret_cast<const volatile int32_t *>(a.m.status) == 1;
    const bool records = a.tq && *a.m.mode == 1;
    if (ok) {
        const int P = a.offsets[a.E];
        const int H8 = a.H / 8;
        const int warps = kDispatchThreads / 32;
        const int rq = a.nkb * 4 * 5, rs = a.nkb * 4;  // a token's record words (uint4, uint2)
        for (int q = blockIdx.x * warps + (tid >> 5); q < P; q += gridDim.x * warps) {
            const int pair = a.perm_pair[q];
            const int e = a.topk_idx[pair];
            const int t = pair / a.k;
            const int dst = e / a.El;
            const int row = a.m.send_base[e] + (q - a.offsets[e]);
            if (row < 0 || row >= a.r_cap || dst >= a.N) {  // inconsistent counts: skip the store
                if (lane == 0) atomicCAS(a.err, 0, 33);
                continue;
            }
            if (records) {
                uint4 *dq;
                uint2 *ds;
                ep_recv_records(win[dst], a.w, a.r_cap, a.H, &dq, &ds);
                const uint4 *sq = a.tq + (size_t)t * rq;
                const uint2 *ss = a.ts + (size_t)t * rs;
                dq += (size_t)row * rq;
                ds += (size_t)row * rs;
                for (int i = lane; i < rq; i += 32) dq[i] = __ldg(sq + i);
                for (int i = lane; i < rs; i += 32) ds[i] = __ldg(ss + i);
                continue;
            }
            const uint4 *sh = reinterpret_cast<const uint4 *>(a.x_hi + (size_t)t * a.H);
            const uint4 *sl = reinterpret_cast<const uint4 *>(a.x_lo + (size_t)t * a.H);
            uint4 *dh = reinterpret_cast<uint4 *>(win[dst] + a.w.recv_hi + (size_t)row * a.H * 2);
            uint4 *dl = reinterpret_cast<uint4 *>(win[dst] + a.w.recv_lo + (size_t)row * a.H * 2);
            for (int i0 = 0; i0 < H8; i0 += 32 * kDispatchUnroll) {
                uint4 vh[kDispatchUnroll], vl[kDispatchUnroll];
#pragma unroll
                for (int u = 0; u < kDispatchUnroll; ++u) {
                    const int i = i0 + u * 32 + lane;
                    if (i < H8) {
                        vh[u] = __ldg(sh + i);
                        vl[u] = __ldg(sl + i);
                    }
                }
#pragma unroll
                for (int u = 0; u < kDispatchUnroll; ++u) {
                    const int i = i0 + u * 32 + lane;
                    if (i < H8) {
                        dh[i] = vh[u];
                        dl[i] = vl[u];
                    }
                }
            }
        }
        // return targets: received row p of local expert el came from source s
        const int N = a.N, El = a.El;
        const int R = min(a.m.offsets_loc[El], a.r_cap);
        for (int p = blockIdx.x * kDispatchThreads + tid; p < R; p += gridDim.x * kDispatchThreads) {
            int lo = 0, hi = El;  // last el with offsets_loc[el] <= p
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (a.m.offsets_loc[mid] <= p) lo = mid;
                else hi = mid;
            }
            const int32_t *ss = a.m.seg_start + lo * N;
            int s = 0;
            while (s + 1 < N && ss[s + 1] <= p) ++s;
            int pos = a.m.src_pos[lo * N + s] + p - ss[s];
            if (pos < 0 || pos >= a.p_cap) {  // inconsistent counts: keep the store in bounds
                atomicCAS(a.err, 0, 33);
                pos = 0;
            }
            a.m.y_rows[p] = (int32_t)(((uint32_t)s << kEpRowShift) | (uint32_t)pos);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        const unsigned total = gridDim.x;
        if (atomicInc(a.m.arrive, total - 1) == total - 1 && ok) {
            __threadfence_system();
            for (int q = 0; q < a.N; ++q) st_release_sys(win_flag(win[q], a.w, kEpFlagDispatch, a.me), a.epoch);
        }
    }
}

// One warp: lane s < N waits for this rank's flag `which` from source s.  After
// an earlier failed wait of this exchange (status 0) it returns at once: the
// error is recorded and this rank's flags are withheld, so its peers fail too.
__global__ void ep_wait_kernel(EpArgs a, int which, int code) {
    const int lane = threadIdx.x;
    if (*reinterpret_cast<const volatile int32_t *>(a.m.status) != 1) return;
    uint8_t *own = a.m.win[a.me];
    bool good = true;
    if (lane < a.N) good = wait_epoch(win_flag(own, a.w, which, lane), a.epoch, a.limit_ns);
    if (__any_sync(0xffffffffu, !good)) {
        if (lane == 0) atomicCAS(a.err, 0, code);
        if (which == kEpFlagDispatch) empty_ranges(a);
        else if (lane == 0) *a.m.status = 0;
    }
}

}  // namespace

cudaError_t launch_ep_counts(const EpArgs &a, cudaStream_t st) {
    if (a.E > 256 || a.N > kMaxEpRanks) return cudaErrorInvalidValue;
    ep_counts_kernel<<<1, kCountThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpArgs &a, int grid, cudaStream_t st) {
    ep_dispatch_kernel<<<grid, kDispatchThreads, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait(const EpArgs &a, int which, int code, cudaStream_t st) {
    ep_wait_kernel<<<1, 32, 0, st>>>(a, which, code);
    return cudaGetLastError();
}

}  // namespace amoe
