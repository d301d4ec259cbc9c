// ep.cu -- expert parallelism: experts sharded over the GPUs of one box, with
// NCCL all-to-all dispatch of token rows to the expert's GPU and return of the
// expert outputs (no counterpart in the reference, which is single-threaded
// CPU code; the single-GPU path is its oracle).
//
// Rank r owns experts [r*E_loc, (r+1)*E_loc).  Its locally routed pairs are
// already sorted by expert, hence by destination rank.  The exchange:
//   1. per-expert pair counts -> every rank (grouped ncclSend/ncclRecv);
//   2. ep_plan() turns them into send/receive row ranges and the segments that
//      reorder received rows (source-major) into expert-major order;
//   3. the fp16 hi/lo rows go out, the expert GEMMs run on the received rows,
//      their f32 outputs go back in the order they came.
#include "amoe_internal.cuh"

#include <dlfcn.h>

#include <mutex>

namespace amoe {

// ---- NCCL, resolved at run time (same soname torch loads; no link dependency) ----
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
        AMOE_SYM(ncclCommAbort)
        AMOE_SYM(ncclGroupStart)
        AMOE_SYM(ncclGroupEnd)
        AMOE_SYM(ncclSend)
        AMOE_SYM(ncclRecv)
        AMOE_SYM(ncclGetErrorString)
        AMOE_SYM(ncclCommGetAsyncError)
#undef AMOE_SYM
        ok = true;
    });
    if (!ok && err) *err = why;
    return ok;
}

// ---- exchange plan (host only) --------------------------------------------------
int ep_plan(int N, int E_loc, int rank, const int32_t *local_offsets, const int32_t *recv_counts, EpPlan *p) {
    if (N < 1 || E_loc < 1 || rank < 0 || rank >= N) return -1;
    p->N = N;
    p->E_loc = E_loc;
    p->send_off.assign(N, 0);
    p->send_rows.assign(N, 0);
    p->recv_off.assign(N, 0);
    p->recv_rows.assign(N, 0);
    p->offsets_loc.assign(E_loc + 1, 0);
    p->seg.assign((size_t)N * E_loc * 3, 0);
    for (int d = 0; d < N; ++d) {
        p->send_off[d] = local_offsets[d * E_loc];
        p->send_rows[d] = local_offsets[(d + 1) * E_loc] - local_offsets[d * E_loc];
        if (p->send_rows[d] < 0) return -1;
    }
    int acc = 0;
    for (int s = 0; s < N; ++s) {
        int rows = 0;
        for (int e = 0; e < E_loc; ++e) {
            const int v = recv_counts[s * E_loc + e];
            if (v < 0) return -1;
            rows += v;
        }
        p->recv_off[s] = acc;
        p->recv_rows[s] = rows;
        acc += rows;
    }
    p->R = acc;
    // expert-major order: expert e's rows from source 0, then source 1, ...
    for (int e = 0; e < E_loc; ++e) {
        int c = 0;
        for (int s = 0; s < N; ++s) c += recv_counts[s * E_loc + e];
        p->offsets_loc[e + 1] = p->offsets_loc[e] + c;
    }
    std::vector<int> dst_cursor(p->offsets_loc.begin(), p->offsets_loc.end() - 1);
    for (int s = 0; s < N; ++s) {
        int src = p->recv_off[s];
        for (int e = 0; e < E_loc; ++e) {
            const int len = recv_counts[s * E_loc + e];
            int *g = &p->seg[((size_t)s * E_loc + e) * 3];
            g[0] = src;
            g[1] = dst_cursor[e];
            g[2] = len;
            src += len;
            dst_cursor[e] += len;
        }
    }
    return 0;
}

namespace {

// One CTA per (source, expert) segment: copy `len` received rows (fp16 hi/lo)
// to their expert-major positions and record where each came from.
__global__ void __launch_bounds__(256) ep_reorder_kernel(const int32_t *__restrict__ seg, int H,
                                                         const __half *__restrict__ src_hi,
                                                         const __half *__restrict__ src_lo,
                                                         __half *__restrict__ dst_hi, __half *__restrict__ dst_lo,
                                                         int32_t *__restrict__ ret_map) {
    const int src = seg[blockIdx.x * 3], dst = seg[blockIdx.x * 3 + 1], len = seg[blockIdx.x * 3 + 2];
    const int H8 = H / 8;
    const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < len; j += warps) {
        const uint4 *sh = reinterpret_cast<const uint4 *>(src_hi + (size_t)(src + j) * H);
        const uint4 *sl = reinterpret_cast<const uint4 *>(src_lo + (size_t)(src + j) * H);
        uint4 *dh = reinterpret_cast<uint4 *>(dst_hi + (size_t)(dst + j) * H);
        uint4 *dl = reinterpret_cast<uint4 *>(dst_lo + (size_t)(dst + j) * H);
        for (int i = lane; i < H8; i += 32) {
            dh[i] = sh[i];
            dl[i] = sl[i];
        }
        if (lane == 0) ret_map[dst + j] = src + j;
    }
}

// Experts with rows, ascending, then their count at [E_loc] (the GEMV's list).
__global__ void ep_active_kernel(const int32_t *__restrict__ offsets, int E_loc, int32_t *__restrict__ active) {
    if (threadIdx.x != 0) return;
    int na = 0;
    for (int e = 0; e < E_loc; ++e)
        if (offsets[e + 1] > offsets[e]) active[na++] = e;
    active[E_loc] = na;
}

}  // namespace

cudaError_t launch_ep_reorder(const int32_t *seg_dev, int nseg, int H, const __half *src_hi, const __half *src_lo,
                              __half *dst_hi, __half *dst_lo, int32_t *ret_map, cudaStream_t st) {
    if (nseg <= 0) return cudaSuccess;
    ep_reorder_kernel<<<nseg, 256, 0, st>>>(seg_dev, H, src_hi, src_lo, dst_hi, dst_lo, ret_map);
    return cudaGetLastError();
}

cudaError_t launch_ep_active(const int32_t *offsets, int E_loc, int32_t *active, cudaStream_t st) {
    ep_active_kernel<<<1, 32, 0, st>>>(offsets, E_loc, active);
    return cudaGetLastError();
}

}  // namespace amoe
