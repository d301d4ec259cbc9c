// ctx.cu -- the C ABI (include/amoe.h): context, weight upload, forward.
//
// Host-side orchestration only; the arithmetic lives in route.cu, decode.cu,
// gemv.cu, gemm_bs.cu, combine.cu and ep.cu.  Error behaviour mirrors the reference's Go
// error returns (e.g. internal/model/gptoss/layer.go:35-39, tensor.go:95-97,
// moe.go:13-18): every failure is a negative status plus a message, never an
// abort.
#include "../../include/amoe.h"
#include "amoe_internal.cuh"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace amoe {


namespace {

thread_local std::string g_create_error;

struct Status {
    int code;
    std::string msg;
};

struct LayerBlock {
    // byte offsets inside one layer's device-format block (256-B aligned parts)
    size_t norm, router_w, router_b, gu_b, dn_b, gu_s, dn_s, gu_q, dn_q, gu_tq, dn_tq, total;
    bool frag;  // GEMV fragment tiles stored
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Dims d: router over d.E experts; experts E_x of them stored (E_x < d.E in EP mode).
// The parts the tcgen05 kernels read come first; the GEMV fragment tiles (frag)
// follow, and are left out of streamed layers (only the TMA-plane kernels run there).
LayerBlock layer_block(const Dims &d, int E_x, bool frag) {
    LayerBlock b{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o = align256(o + bytes);
        return at;
    };
    const size_t H = d.H, I = d.I, E = E_x;
    b.norm = take(H * 4);
    b.router_w = take(H * (size_t)d.E * 4);
    b.router_b = take((size_t)d.E * 4);
    b.gu_b = take(E * 2 * I * 4);
    b.dn_b = take(E * H * 4);
    b.gu_tq = take(box_plane_bytes((int)E, (int)(2 * I), (int)H));
    b.dn_tq = take(box_plane_bytes((int)E, (int)H, (int)I));
    b.frag = frag;
    if (frag) {
        b.gu_s = take(E * 2 * I * (H / 32));
        b.dn_s = take(E * H * (I / 32));
        b.gu_q = take(E * 2 * I * (H / 2));
        b.dn_q = take(E * H * (I / 2));
    }
    b.total = o;
    return b;
}

LayerDev layer_view(uint8_t *base, const LayerBlock &b) {
    LayerDev L;
    L.norm_gain = reinterpret_cast<float *>(base + b.norm);
    L.router_w = reinterpret_cast<float *>(base + b.router_w);
    L.router_b = reinterpret_cast<float *>(base + b.router_b);
    L.gu_b = reinterpret_cast<float *>(base + b.gu_b);
    L.dn_b = reinterpret_cast<float *>(base + b.dn_b);
    if (b.frag) {
        L.gu_s = base + b.gu_s;
        L.dn_s = base + b.dn_s;
        L.gu_q = base + b.gu_q;
        L.dn_q = base + b.dn_q;
    }
    L.gu_tq = base + b.gu_tq;
    L.dn_tq = base + b.dn_tq;
    return L;
}

}  // namespace

void set_thread_error(const std::string &msg) { g_create_error = msg; }

}  // namespace amoe

using namespace amoe;

// amoe_forward splits large calls into at most this many token slices, so that
// host copies overlap the compute of neighbouring slices.
constexpr int kMaxIoChunks = 8;

struct amoe_ctx {
    amoe_config cfg{};
    Dims d{};       // routing (all experts)
    Dims dx{};      // expert stage (this rank's experts)
    LayerBlock blk{};
    cudaStream_t stream = nullptr;       // compute
    cudaStream_t copy_stream = nullptr;  // layer streaming
    std::string err;

    // resident mode: one device block per layer; streaming: pinned host blocks + slots
    std::vector<uint8_t *> layer_dev;    // [layers] (resident) device block or null
    std::vector<uint8_t *> layer_host;   // [layers] (streaming) pinned block or null
    std::vector<bool> uploaded;
    std::vector<uint8_t *> slot_dev;     // [stream_slots]
    // stream_experts: every layer's norm and router stay resident; the routed
    // experts of a call are copied into one compact slot
    float *router_res = nullptr;         // [layers][H + E*H + E]: norm gain, router weight, router bias
    uint8_t *xslot = nullptr;            // expert slot: xblk layout for xs experts
    LayerBlock xblk{};
    int xs = 0;
    int32_t *h_sel = nullptr;            // pinned: offsets [E+1], then compact offsets and active [2 (xs+1)]
    int32_t *sel_dev = nullptr;          // compact offsets [xs+1], active [xs+1]
    std::vector<int> slot_layer;
    std::vector<cudaEvent_t> slot_ready, slot_free;
    std::vector<long long> slot_used;    // LRU stamp
    long long tick = 0;

    // scratch
    int max_tokens = 0, nchunk_max = 0;
    void *scratch = nullptr;
    RouteOut r{};
    double *partial = nullptr;
    int32_t *arrivals = nullptr;
    __half *act_hi = nullptr, *act_lo = nullptr;
    float *y = nullptr;
    int32_t *err_flag = nullptr;  // set by a kernel whose bounded wait gave up (0 = fine)
    void *bs_scratch = nullptr;  // token tiles and the five-term E2M1 operands of the block-scaled GEMMs
    DecodeBarrier *dec_bar = nullptr;  // launch counts of the fused decode kernel's CTAs
    void *dec_scratch = nullptr;       // its activation operand, partial tiles and tile counters
    float *io_in = nullptr, *io_out = nullptr;
    int32_t *io_idx = nullptr;
    float *io_w = nullptr;
    int last_T = 0;
    std::vector<int> last_chunks;           // token counts of the last call's passes (routing slices)
    cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;  // host-buffer forward pipeline
    int32_t *h_flag = nullptr;              // pinned copy of the device error flag
    cudaEvent_t io_in_ready[kMaxIoChunks] = {}, io_out_ready[kMaxIoChunks] = {};

    // expert parallelism (ep_size > 1)
    int ep_n = 1, ep_rank = 0, e_loc = 0;
    ncclComm_t comm = nullptr;                 // setup only (IPC handle exchange)
    size_t r_max = 0;                          // rows this rank can receive (every source's pairs)
    uint8_t *ep_win = nullptr;                 // this rank's exported window
    std::vector<uint8_t *> ep_peer;            // every rank's window as mapped here (self: ep_win)
    EpWindow ep_w{};
    EpMeta ep_m{};
    int ep_epoch = 0;                          // forwards so far (the exchange's flag value)
    bool ep_broken = false;                    // a wait failed: the group is out of step
    long long ep_count_wait_ns = 0;            // bound on the count exchange's wait
    long long ep_data_wait_ns = 0;             // bound on the dispatch and return waits
    int sms = 0;

    // diagnostics
    bool profiling = false;
    amoe_stats stats{};
    struct PendingTiming {
        cudaEvent_t ev[AMOE_STAGES + 1];
        int stage_of[AMOE_STAGES + 1];
        int n;
    };
    std::vector<PendingTiming> pending;
    std::vector<cudaEvent_t> event_pool;
};

namespace {

int fail(amoe_ctx *c, int code, const std::string &msg) {
    if (c) c->err = msg;
    return code;
}

int cuda_fail(amoe_ctx *c, cudaError_t e, const char *what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    return fail(c, e == cudaErrorMemoryAllocation ? AMOE_ERR_NOMEM : AMOE_ERR_CUDA, m);
}

#define AMOE_CUDA(ctx, call)                                  \
    do {                                                      \
        cudaError_t e_ = (call);                              \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
    } while (0)

// Fault injection for the allocation error paths (host side; off unless the
// environment sets it): AMOE_FAIL_ALLOC_ABOVE=<bytes> makes every device or
// pinned-host allocation of more than <bytes> fail as out of memory, so that
// tests can check that amoe_create and amoe_upload_layer report AMOE_ERR_NOMEM
// and leave the context usable.
bool injected_alloc_failure(size_t bytes) {
    const char *v = std::getenv("AMOE_FAIL_ALLOC_ABOVE");
    if (!v || !*v) return false;
    char *end = nullptr;
    const unsigned long long limit = std::strtoull(v, &end, 10);
    return end != v && bytes > limit;
}

template <class T>
cudaError_t dev_alloc(T **p, size_t bytes) {
    if (injected_alloc_failure(bytes)) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMalloc(reinterpret_cast<void **>(p), bytes);
}

template <class T>
cudaError_t host_alloc(T **p, size_t bytes, unsigned flags) {
    if (injected_alloc_failure(bytes)) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaHostAlloc(reinterpret_cast<void **>(p), bytes, flags);
}

std::string validate(const amoe_config *c) {
    if (!c) return "config must not be NULL";
    if (c->hidden <= 0 || c->hidden % 64) return "hidden must be a positive multiple of 64";
    if (c->intermediate <= 0 || c->intermediate % 64)
        return "intermediate must be a positive multiple of 64";
    if (c->experts < 1 || c->experts > 256) return "experts must be in [1, 256]";
    if (c->top_k < 1 || c->top_k > c->experts || c->top_k > 32)
        return "moe router top-k " + std::to_string(c->top_k) + " outside [1, " +
               std::to_string(c->experts < 32 ? c->experts : 32) + "]";
    if (c->layers < 1) return "layers must be positive";
    if (!(c->rms_eps > 0.0f) || !std::isfinite(c->rms_eps))
        return "rmsnorm epsilon must be positive";
    if (c->swiglu_alpha != 1.702f || c->swiglu_limit != 7.0f)
        return "gpt-oss swiglu constants are fixed at alpha 1.702, limit 7";
    if (c->max_tokens < 1) return "max_tokens must be positive";
    if (c->stream_slots != 0 && c->stream_slots < 2) return "stream_slots must be 0 or >= 2";
    if (c->stream_slots >= 2 && c->path == AMOE_PATH_GEMV)
        return "streamed layers run on the tensor-core kernels: stream_slots needs path AUTO or TENSOR";
    if (c->stream_experts != 0 && c->stream_experts != 1) return "stream_experts must be 0 or 1";
    if (c->stream_experts && c->stream_slots < 2) return "stream_experts needs stream_slots >= 2";
    if (c->ep_size < 1 || c->ep_rank < 0 || c->ep_rank >= c->ep_size)
        return "ep_rank must be in [0, ep_size)";
    if (c->ep_size > 1) {
        if (c->ep_size > kMaxEpRanks) return "ep_size must be at most 8 (the GPUs of one box)";
        if (c->experts % c->ep_size) return "experts must divide evenly over ep_size";
        if ((long long)c->max_tokens * c->top_k * c->ep_size >= (1LL << kEpRowShift))
            return "max_tokens * top_k * ep_size must stay below 2^28";
        if (!c->nccl_id) return "nccl_id must be set when ep_size > 1";
        if (c->stream_slots) return "expert parallelism keeps every layer resident (stream_slots 0)";
    }
    if (c->path < AMOE_PATH_AUTO || c->path > AMOE_PATH_TENSOR) return "unknown path";
    return "";
}

int alloc_scratch(amoe_ctx *c) {
    const Dims &d = c->d;
    const size_t T = c->cfg.max_tokens, P = T * d.k;
    c->max_tokens = (int)T;
    c->nchunk_max = (int)((T + kRouteTokens - 1) / kRouteTokens);
    const size_t partial = route_partial_elems((int)T, d.H, d.E);
    const size_t R = c->ep_n > 1 ? (size_t)c->ep_n * P : 0;  // worst case: every source sends all pairs here
    c->r_max = R;
    const size_t A = R > P ? R : P;  // rows of the expert stage
    const size_t nseg = (size_t)c->ep_n * (c->e_loc > 0 ? c->e_loc : 1);
    size_t off = 0;
    struct Part {
        void **dst;
        size_t bytes;
    };
    std::vector<Part> parts = {
        {(void **)&c->r.x_hi, T * d.H * 2},
        {(void **)&c->r.x_lo, T * d.H * 2},
        {(void **)&c->r.logits, T * d.E * 4},
        {(void **)&c->r.topk_idx, P * 4},
        {(void **)&c->r.topk_w, P * 4},
        {(void **)&c->r.hist, (size_t)c->nchunk_max * d.E * 4},
        {(void **)&c->r.chunk_base, (size_t)c->nchunk_max * d.E * 4},
        {(void **)&c->r.counts, (size_t)kMaxIoChunks * d.E * 4},
        {(void **)&c->r.offsets, (size_t)kMaxIoChunks * (d.E + 1) * 4},
        {(void **)&c->r.active, (size_t)kMaxIoChunks * (d.E + 1) * 4},
        {(void **)&c->r.perm_pair, P * 4},
        {(void **)&c->r.inv, P * 4},
        {(void **)&c->partial, partial * 8},
        {(void **)&c->arrivals, (size_t)c->nchunk_max * 4},
        {(void **)&c->act_hi, A * d.I * 2},
        {(void **)&c->act_lo, A * d.I * 2},
        {(void **)&c->y, P * d.H * 4},
        {(void **)&c->err_flag, 16},
        {(void **)&c->bs_scratch, bs_scratch_bytes((int)A, (int)T, c->dx.E, d.H, d.I)},
        {(void **)&c->dec_bar, sizeof(DecodeBarrier)},
        {(void **)&c->dec_scratch, decode_scratch_bytes(d, c->cfg.device)},
        {(void **)&c->io_in, T * d.H * 4},
        {(void **)&c->io_out, T * d.H * 4},
        {(void **)&c->io_idx, P * 4},
        {(void **)&c->io_w, P * 4},
        {(void **)&c->ep_m.send_base, R ? (size_t)d.E * 4 : 0},
        {(void **)&c->ep_m.offsets_loc, R ? (size_t)(c->e_loc + 1) * 4 : 0},
        {(void **)&c->ep_m.active_loc, R ? (size_t)(c->e_loc + 1) * 4 : 0},
        {(void **)&c->ep_m.seg_start, R ? nseg * 4 : 0},
        {(void **)&c->ep_m.src_pos, R ? nseg * 4 : 0},
        {(void **)&c->ep_m.y_rows, R * 4},
        {(void **)&c->ep_m.status, R ? size_t(16) : 0},
        {(void **)&c->ep_m.arrive, R ? size_t(16) : 0},
        {(void **)&c->ep_m.win, R ? size_t(kMaxEpRanks * 8) : 0},
        {(void **)&c->ep_m.ret_y, R ? size_t(kMaxEpRanks * 8) : 0},
        {(void **)&c->ep_m.ret_flag, R ? size_t(kMaxEpRanks * 8) : 0},
    };
    std::vector<size_t> at(parts.size());
    for (size_t i = 0; i < parts.size(); ++i) {
        at[i] = off;
        off = align256(off + parts[i].bytes);
    }
    AMOE_CUDA(c, dev_alloc(&c->scratch, off));
    uint8_t *base = static_cast<uint8_t *>(c->scratch);
    for (size_t i = 0; i < parts.size(); ++i) *parts[i].dst = parts[i].bytes ? base + at[i] : nullptr;
    AMOE_CUDA(c, cudaMemset(c->arrivals, 0, (size_t)c->nchunk_max * 4));
    AMOE_CUDA(c, cudaMemset(c->dec_bar, 0, sizeof(DecodeBarrier)));
    AMOE_CUDA(c, init_decode_scratch(d, c->cfg.device, c->dec_scratch, nullptr));
    AMOE_CUDA(c, init_bs_scratch(c->bs_scratch, (int)A, (int)T, c->dx.E, d.H, d.I));
    AMOE_CUDA(c, cudaDeviceSynchronize());
    AMOE_CUDA(c, cudaMemset(c->err_flag, 0, sizeof(int32_t)));
    if (R) {
        AMOE_CUDA(c, cudaMemset(c->ep_m.status, 0, 16));
        c->ep_m.mode = c->ep_m.status + 1;
        AMOE_CUDA(c, cudaMemset(c->ep_m.arrive, 0, 16));
    }
    return AMOE_OK;
}

cudaEvent_t pool_event(amoe_ctx *c) {
    if (!c->event_pool.empty()) {
        cudaEvent_t e = c->event_pool.back();
        c->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Stage timer for one forward: records an event before the first stage and
// after every stage on the launch stream (profiling only).
struct StageTimer {
    amoe_ctx *c;
    cudaStream_t st;
    amoe_ctx::PendingTiming t{};
    StageTimer(amoe_ctx *c_, cudaStream_t st_) : c(c_), st(st_) {
        if (c->profiling) {
            t.ev[0] = pool_event(c);
            t.stage_of[0] = -1;
            t.n = 1;
            cudaEventRecord(t.ev[0], st);
        }
    }
    void mark(int stage) {
        if (!c->profiling || t.n > AMOE_STAGES) return;
        t.ev[t.n] = pool_event(c);
        t.stage_of[t.n] = stage;
        cudaEventRecord(t.ev[t.n], st);
        ++t.n;
    }
    void finish() {
        if (c->profiling && t.n > 1) {
            c->pending.push_back(t);
            c->stats.timed_forwards++;
        } else if (c->profiling) {
            c->event_pool.push_back(t.ev[0]);
        }
    }
};

void fold_timings(amoe_ctx *c) {
    for (auto &t : c->pending) {
        for (int i = 1; i < t.n; ++i) {
            float ms = 0.0f;
            if (cudaEventElapsedTime(&ms, t.ev[i - 1], t.ev[i]) == cudaSuccess)
                c->stats.stage_ms[t.stage_of[i]] += ms;
        }
        for (int i = 0; i < t.n; ++i) c->event_pool.push_back(t.ev[i]);
    }
    c->pending.clear();
}

void release(amoe_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    if (c->h2d_stream) cudaStreamSynchronize(c->h2d_stream);
    if (c->d2h_stream) cudaStreamSynchronize(c->d2h_stream);
    for (auto p : c->layer_dev) if (p) cudaFree(p);
    for (auto p : c->layer_host) if (p) cudaFreeHost(p);
    for (auto p : c->slot_dev) if (p) cudaFree(p);
    if (c->router_res) cudaFree(c->router_res);
    if (c->xslot) cudaFree(c->xslot);
    if (c->sel_dev) cudaFree(c->sel_dev);
    if (c->h_sel) cudaFreeHost(c->h_sel);
    for (auto e : c->slot_ready) if (e) cudaEventDestroy(e);
    for (auto e : c->slot_free) if (e) cudaEventDestroy(e);
    if (c->scratch) cudaFree(c->scratch);
    for (size_t q = 0; q < c->ep_peer.size(); ++q)
        if (c->ep_peer[q] && c->ep_peer[q] != c->ep_win) cudaIpcCloseMemHandle(c->ep_peer[q]);
    if (c->ep_win) cudaFree(c->ep_win);
    if (c->comm) g_nccl.ncclCommDestroy(c->comm);
    for (auto &t : c->pending)
        for (int i = 0; i < t.n; ++i) cudaEventDestroy(t.ev[i]);
    for (auto e : c->event_pool) cudaEventDestroy(e);
    for (int i = 0; i < kMaxIoChunks; ++i) {
        if (c->io_in_ready[i]) cudaEventDestroy(c->io_in_ready[i]);
        if (c->io_out_ready[i]) cudaEventDestroy(c->io_out_ready[i]);
    }
    if (c->h_flag) cudaFreeHost(c->h_flag);
    if (c->h2d_stream) cudaStreamDestroy(c->h2d_stream);
    if (c->d2h_stream) cudaStreamDestroy(c->d2h_stream);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
}

bool streaming(const amoe_ctx *c) { return c->cfg.stream_slots >= 2; }

// Makes `layer` available in a device slot and returns its view; the compute
// stream `st` is made to wait for the copy.  Streaming mode only.
int acquire_slot(amoe_ctx *c, int layer, cudaStream_t st, int *slot_out) {
    const int n = (int)c->slot_dev.size();
    int slot = -1;
    for (int i = 0; i < n; ++i)
        if (c->slot_layer[i] == layer) slot = i;
    if (slot < 0) {
        // least recently used slot
        slot = 0;
        for (int i = 1; i < n; ++i)
            if (c->slot_used[i] < c->slot_used[slot]) slot = i;
        AMOE_CUDA(c, cudaStreamWaitEvent(c->copy_stream, c->slot_free[slot], 0));
        AMOE_CUDA(c, cudaMemcpyAsync(c->slot_dev[slot], c->layer_host[layer], c->blk.total,
                                     cudaMemcpyHostToDevice, c->copy_stream));
        AMOE_CUDA(c, cudaEventRecord(c->slot_ready[slot], c->copy_stream));
        c->slot_layer[slot] = layer;
    }
    c->slot_used[slot] = ++c->tick;
    if (st) AMOE_CUDA(c, cudaStreamWaitEvent(st, c->slot_ready[slot], 0));
    *slot_out = slot;
    return AMOE_OK;
}

void timer_hook(void *timer, int stage) { static_cast<StageTimer *>(timer)->mark(stage); }

// A tcgen05 kernel that gave up on a bounded wait leaves a code in its flag.
// `known`: the flag's value already copied to the host behind the call's work
// (-1: read it now).
int check_device_flag(amoe_ctx *c, int32_t known = -1) {
    int32_t *flag = c->err_flag;
    int32_t v = known;
    if (v < 0) {
        cudaError_t e = cudaMemcpy(&v, flag, sizeof(v), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(c, e, "read device error flag");
    }
    if (v != 0) {
        cudaMemset(flag, 0, sizeof(int32_t));
        if (v == 21) return fail(c, AMOE_ERR_STATE, "expert GEMV: an expert received more rows than the launch bound");
        if (v >= 30 && v <= 33) {
            // the ranks are out of step (a peer failed, left or never called):
            // the group cannot be resumed
            c->ep_broken = true;
            static const char *what[] = {"count exchange", "row dispatch", "output return",
                                         "row dispatch (inconsistent counts)"};
            return fail(c, v == 33 ? AMOE_ERR_STATE : AMOE_ERR_TIMEOUT,
                        std::string("expert-parallel ") + what[v - 30] + " failed (code " + std::to_string(v) + ")");
        }
        if (v >= 50 && v <= 54) {
            static const char *what[] = {"ring slot release", "weight box arrival", "expert activation",
                                         "router logits", "copy drain"};
            return fail(c, AMOE_ERR_TIMEOUT, std::string("decode kernel: wait for the ") + what[v - 50] +
                                                 " timed out (code " + std::to_string(v) + ")");
        }
        return fail(c, AMOE_ERR_TIMEOUT, "device pipeline wait timed out (code " + std::to_string(v) + ")");
    }
    return AMOE_OK;
}

int check_ctx(amoe_ctx *c) {
    if (!c) return AMOE_ERR_INVALID;
    cudaError_t e = cudaSetDevice(c->cfg.device);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
    return AMOE_OK;
}

int use_tensor_path(const amoe_ctx *c, int T) {
    if (c->cfg.path == AMOE_PATH_GEMV) return 0;
    if (c->cfg.path == AMOE_PATH_TENSOR) return 1;
    // AUTO: the GEMV streams each selected weight tile once per 32 tokens of
    // an expert; past ~32 tokens per expert the tcgen05 GEMM wins.
    const long long pairs_per_expert = (long long)T * c->d.k / c->d.E;
    return tc_supported() && pairs_per_expert >= 32;
}

// Bounds on the exchange's waits (AMOE_EP_WAIT_MS overrides both).  The count
// exchange at the start of a forward also absorbs the ranks' host-side skew (a
// rank reaching the forward later than its peers), hence seconds; the dispatch
// and return waits only wait for the peers' kernels that are already running
// (the longest is a peer's expert GEMMs, milliseconds), hence one second.
constexpr long long kEpCountWaitNs = 5000000000LL;
constexpr long long kEpDataWaitNs = 1000000000LL;

long long ep_wait_override_ns() {
    const char *v = std::getenv("AMOE_EP_WAIT_MS");
    if (!v || !*v) return 0;
    const long long ms = std::atoll(v);
    return ms > 0 ? ms * 1000000LL : 0;
}

// Maps every rank's window into this process: the windows' IPC handles and the
// block shape go round once through an NCCL all-gather (the only NCCL use).
int ep_setup(amoe_ctx *c) {
    const Dims &d = c->d;
    const int N = c->ep_n, me = c->ep_rank;
    c->ep_w = ep_window(N, d.E, d.H, c->max_tokens * d.k, (int)c->r_max);
    AMOE_CUDA(c, dev_alloc(&c->ep_win, c->ep_w.bytes));
    AMOE_CUDA(c, cudaMemset(c->ep_win, 0, c->ep_w.table));  // the flags
    AMOE_CUDA(c, cudaDeviceSynchronize());
    struct Hello {
        cudaIpcMemHandle_t handle;
        int64_t shape[8];
    };
    Hello mine{};
    AMOE_CUDA(c, cudaIpcGetMemHandle(&mine.handle, c->ep_win));
    const int64_t shape[8] = {N, d.H, d.I, d.E, d.k, c->max_tokens, (int64_t)c->ep_w.bytes, c->cfg.path};
    std::memcpy(mine.shape, shape, sizeof(shape));
    std::vector<Hello> all(N);
    uint8_t *buf = nullptr;
    AMOE_CUDA(c, dev_alloc(&buf, sizeof(Hello) * (N + 1)));
    cudaError_t e = cudaMemcpy(buf, &mine, sizeof(Hello), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        const ncclResult_t r = g_nccl.ncclAllGather(buf, buf + sizeof(Hello), sizeof(Hello), ncclUint8, c->comm,
                                                    c->stream);
        if (r != ncclSuccess) {
            cudaFree(buf);
            return fail(c, AMOE_ERR_NCCL, std::string("ncclAllGather: ") + g_nccl.ncclGetErrorString(r));
        }
        e = cudaStreamSynchronize(c->stream);
        if (e == cudaSuccess) e = cudaMemcpy(all.data(), buf + sizeof(Hello), sizeof(Hello) * N, cudaMemcpyDeviceToHost);
    }
    cudaFree(buf);
    AMOE_CUDA(c, e);
    for (int q = 0; q < N; ++q)
        if (std::memcmp(all[q].shape, shape, sizeof(shape)) != 0)
            return fail(c, AMOE_ERR_INVALID, "expert-parallel rank " + std::to_string(q) +
                                                 " has another block shape, max_tokens or path");
    c->ep_peer.assign(N, nullptr);
    for (int q = 0; q < N; ++q) {
        if (q == me) {
            c->ep_peer[q] = c->ep_win;
            continue;
        }
        void *p = nullptr;
        e = cudaIpcOpenMemHandle(&p, all[q].handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return cuda_fail(c, e, ("cudaIpcOpenMemHandle(rank " + std::to_string(q) + ")").c_str());
        c->ep_peer[q] = static_cast<uint8_t *>(p);
    }
    uint8_t *win[kMaxEpRanks] = {};
    float *ret_y[kMaxEpRanks] = {};
    int32_t *ret_flag[kMaxEpRanks] = {};
    for (int q = 0; q < N; ++q) {
        win[q] = c->ep_peer[q];
        ret_y[q] = reinterpret_cast<float *>(win[q] + c->ep_w.y);
        ret_flag[q] = reinterpret_cast<int32_t *>(win[q] + c->ep_w.flags) + kEpFlagReturn * kMaxEpRanks + me;
    }
    AMOE_CUDA(c, cudaMemcpy(c->ep_m.win, win, sizeof(win), cudaMemcpyHostToDevice));
    AMOE_CUDA(c, cudaMemcpy(c->ep_m.ret_y, ret_y, sizeof(ret_y), cudaMemcpyHostToDevice));
    AMOE_CUDA(c, cudaMemcpy(c->ep_m.ret_flag, ret_flag, sizeof(ret_flag), cudaMemcpyHostToDevice));
    return AMOE_OK;
}

// Expert-parallel expert stage: each routed row goes to the rank that owns its
// expert, this rank's experts run on what arrives, and their outputs land in
// the source ranks' windows at the rows' local sorted positions (where the
// combine reads them).  Device-side throughout: no host synchronisation.
int ep_experts(amoe_ctx *c, const LayerDev &L, const RouteOut &r, int T, int nchunk, cudaStream_t st,
               StageTimer &timer, bool *used_tc) {
    const Dims &d = c->d;
    const int N = c->ep_n, El = c->e_loc;
    int32_t *flag = c->err_flag;
    if (nchunk > 1) {  // the stable permutation (one routing chunk writes it itself)
        AMOE_CUDA(c, launch_scatter(d, T, r, false, nullptr, nullptr, st));
        c->stats.launches += 1;
    }
    EpArgs a{};
    a.N = N;
    a.me = c->ep_rank;
    a.E = d.E;
    a.El = El;
    a.H = d.H;
    a.k = d.k;
    a.r_cap = (int)c->r_max;
    a.p_cap = c->max_tokens * d.k;
    a.epoch = ++c->ep_epoch;
    a.count_limit_ns = c->ep_count_wait_ns;
    a.limit_ns = c->ep_data_wait_ns;
    a.w = c->ep_w;
    a.m = c->ep_m;
    a.counts = r.counts;
    a.offsets = r.offsets;
    a.topk_idx = r.topk_idx;
    a.perm_pair = r.perm_pair;
    a.x_hi = r.x_hi;
    a.x_lo = r.x_lo;
    a.err = flag;
    a.path = c->cfg.path == AMOE_PATH_GEMV ? 1 : c->cfg.path == AMOE_PATH_TENSOR ? 2 : 0;
    if (a.path == 0 && !tc_supported()) a.path = 1;
    // Expert path: AUTO is decided on the device by the count kernel from the
    // whole group's pairs (the single-GPU rule on the group's tokens), so every
    // rank agrees and the result equals one GPU's; both paths are launched and
    // the one not chosen returns at once.
    const bool run_tc = tc_supported() && a.path != 1;
    const bool run_gemv = a.path != 2;
    const int32_t *gate = run_tc && run_gemv ? c->ep_m.mode : nullptr;
    AMOE_CUDA(c, launch_ep_counts(a, st));
    a.tq = nullptr;
    a.ts = nullptr;
    a.nkb = (d.H + 127) / 128;
    if (run_tc) {  // the tcgen05 path sends token records: this rank's tokens, quantized once
        AMOE_CUDA(c, launch_tok_quant(r.x_hi, r.x_lo, T, d.H, d.I, c->bs_scratch, (int)c->r_max, c->max_tokens,
                                      c->dx.E, c->ep_m.mode, st, &a.tq, &a.ts));
        c->stats.launches += 1;
    }
    AMOE_CUDA(c, launch_ep_dispatch(a, 2 * c->sms, st));
    timer.mark(5);
    AMOE_CUDA(c, launch_ep_wait(a, kEpFlagDispatch, 31, st));
    c->stats.launches += 3;
    // this rank's experts on the receive buffer; down stores into the sources' windows
    __half *rh = reinterpret_cast<__half *>(c->ep_win + c->ep_w.recv_hi);
    __half *rl = reinterpret_cast<__half *>(c->ep_win + c->ep_w.recv_lo);
    float *y_own = reinterpret_cast<float *>(c->ep_win + c->ep_w.y);
    EpReturn ret;
    ret.y = c->ep_m.ret_y;
    ret.flag = c->ep_m.ret_flag;
    ret.arrive = c->ep_m.arrive + 1;
    ret.status = c->ep_m.status;
    ret.n = N;
    ret.epoch = a.epoch;
    *used_tc = run_tc && (a.path == 2 || (long long)N * T * d.k >= 32LL * d.E);  // stats guess
    if (run_tc) {
        int n = 0;
        uint4 *rq;
        uint2 *rs;
        ep_recv_records(c->ep_win, c->ep_w, (int)c->r_max, d.H, &rq, &rs);
        AMOE_CUDA(c, launch_bs_experts(c->dx, L, c->ep_m.offsets_loc, rh, rl, nullptr, 0, (int)c->r_max,
                                       c->max_tokens, c->bs_scratch, c->dx.E, y_own, c->ep_m.y_rows, flag, st,
                                       &timer_hook, &timer, &n, &ret, gate, 1, rq, rs));
        c->stats.launches += n;
    }
    if (run_gemv) {
        // any expert's rows: at most one per token of the group
        const int bound = N * c->max_tokens;
        GemvRows rows{rh, rl, nullptr, c->ep_m.offsets_loc, c->ep_m.active_loc, c->ep_m.y_rows, El, gate, 0};
        AMOE_CUDA(c, launch_gemv_gate_up(c->dx, L, rows, bound, c->act_hi, c->act_lo, flag, st));
        timer.mark(2);
        AMOE_CUDA(c, launch_gemv_down(c->dx, L, rows, bound, c->act_hi, c->act_lo, y_own, flag, st, &ret));
        timer.mark(3);
        c->stats.launches += 2;
    }
    AMOE_CUDA(c, launch_ep_wait(a, kEpFlagReturn, 32, st));
    c->stats.launches += 1;
    return AMOE_OK;
}

// Routing arrays of the pass over tokens [t0, t0 + T) of a call: token- and
// pair-indexed arrays are offset into the call's arrays; the per-expert ones
// (counts, offsets, active) are the pass's own copy.
RouteOut route_view(const amoe_ctx *c, int t0, int pass) {
    const Dims &d = c->d;
    RouteOut r = c->r;
    r.x_hi += (size_t)t0 * d.H;
    r.x_lo += (size_t)t0 * d.H;
    r.logits += (size_t)t0 * d.E;
    r.topk_idx += (size_t)t0 * d.k;
    r.topk_w += (size_t)t0 * d.k;
    r.perm_pair += (size_t)t0 * d.k;
    r.inv += (size_t)t0 * d.k;
    r.hist += (size_t)(t0 / kRouteTokens) * d.E;
    r.chunk_base += (size_t)(t0 / kRouteTokens) * d.E;
    r.counts += (size_t)pass * d.E;
    r.offsets += (size_t)pass * (d.E + 1);
    r.active += (size_t)pass * (d.E + 1);
    return r;
}

// Expert streaming (stream_experts): route on the device with the layer's resident
// norm and router, read back which experts received rows, copy only those experts
// (box planes, scale chunks, biases) from the pinned host layer into the compact
// slot, and run the block-scaled expert stage on them.  The compact ids keep the
// experts' order, so the permutation and every row's arithmetic are those of the
// whole layer.  The host waits once per call, for the routing.
int forward_selected(amoe_ctx *c, int32_t layer, const float *residual, int32_t T, float *out, int32_t *topk_idx,
                     float *topk_w, cudaStream_t st, const RouteOut &r) {
    const Dims &d = c->d;
    const size_t H = d.H, E = d.E;
    StageTimer timer(c, st);
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    LayerDev Lr{};
    float *res = c->router_res + (size_t)layer * (H + E * H + E);
    Lr.norm_gain = res;
    Lr.router_w = res + H;
    Lr.router_b = res + H + E * H;
    AMOE_CUDA(c, launch_route_impl(d, Lr, residual, T, r, c->partial, c->arrivals, st, &timer_hook, &timer));
    c->stats.launches += nchunk > 1 ? 3 : 1;  // route, then the two scan kernels
    if (nchunk > 1) {
        AMOE_CUDA(c, launch_scatter(d, T, r, false, nullptr, nullptr, st));
        c->stats.launches += 1;
    }
    int32_t *h_off = c->h_sel, *h_cmp = c->h_sel + E + 1;
    AMOE_CUDA(c, cudaMemcpyAsync(h_off, r.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost, st));
    AMOE_CUDA(c, cudaStreamSynchronize(st));
    timer.mark(1);
    // the routed experts, ascending, into slot positions 0..n-1
    const LayerBlock &b = c->blk, &x = c->xblk;
    const size_t gq = box_plane_bytes(1, 2 * d.I, d.H), dq = box_plane_bytes(1, d.H, d.I);
    const size_t gb = (size_t)2 * d.I * 4, db = H * 4;
    const uint8_t *host = c->layer_host[layer];
    const int P = h_off[E];
    int n = 0;
    for (size_t e = 0; e < E; ++e) {
        if (h_off[e + 1] == h_off[e]) continue;
        const size_t j = (size_t)n;
        struct Part {
            size_t src, dst, bytes;
        } parts[] = {{b.gu_tq + e * gq, x.gu_tq + j * gq, gq}, {b.dn_tq + e * dq, x.dn_tq + j * dq, dq},
                     {b.gu_b + e * gb, x.gu_b + j * gb, gb},    {b.dn_b + e * db, x.dn_b + j * db, db}};
        for (const Part &q : parts)
            AMOE_CUDA(c, cudaMemcpyAsync(c->xslot + q.dst, host + q.src, q.bytes, cudaMemcpyHostToDevice, st));
        h_cmp[n] = h_off[e];
        h_cmp[c->xs + 1 + n] = n;
        ++n;
    }
    for (int j = n; j <= c->xs; ++j) h_cmp[j] = P;  // empty ranges past the routed experts
    h_cmp[c->xs + 1 + c->xs] = n;
    AMOE_CUDA(c, cudaMemcpyAsync(c->sel_dev, h_cmp, (size_t)2 * (c->xs + 1) * 4, cudaMemcpyHostToDevice, st));
    timer.mark(5);
    RouteOut rs = r;
    rs.offsets = c->sel_dev;
    rs.active = c->sel_dev + c->xs + 1;
    const Dims dx{d.H, d.I, c->xs, d.k, d.eps};
    LayerDev Lx = layer_view(c->xslot, x);
    int launches = 0;
    AMOE_CUDA(c, launch_bs_experts(dx, Lx, rs.offsets, r.x_hi, r.x_lo, r.perm_pair, T, c->max_tokens * d.k,
                                   c->max_tokens, c->bs_scratch, c->dx.E, c->y, nullptr, c->err_flag, st, &timer_hook,
                                   &timer, &launches));
    c->stats.launches += launches;
    AMOE_CUDA(c, launch_combine(d, residual, r, c->y, T, out, st));
    timer.mark(4);
    c->stats.launches += 1;
    timer.finish();
    c->stats.forwards += 1;
    c->stats.last_path = AMOE_PATH_TENSOR;
    if (topk_idx)
        AMOE_CUDA(c, cudaMemcpyAsync(topk_idx, r.topk_idx, (size_t)T * d.k * 4, cudaMemcpyDeviceToDevice, st));
    if (topk_w)
        AMOE_CUDA(c, cudaMemcpyAsync(topk_w, r.topk_w, (size_t)T * d.k * 4, cudaMemcpyDeviceToDevice, st));
    return AMOE_OK;
}

// One forward pass (arguments already validated) on stream st with routing view r.
int forward_impl(amoe_ctx *c, int32_t layer, const float *residual, int32_t T, float *out, int32_t *topk_idx,
                 float *topk_w, cudaStream_t st, const RouteOut &r) {
    if (c->router_res) return forward_selected(c, layer, residual, T, out, topk_idx, topk_w, st, r);
    int rc = AMOE_OK;
    LayerDev L;
    int slot = -1;
    if (streaming(c)) {
        rc = acquire_slot(c, layer, st, &slot);
        if (rc) return rc;
        L = layer_view(c->slot_dev[slot], c->blk);
    } else {
        L = layer_view(c->layer_dev[layer], c->blk);
    }
    const Dims &d = c->d;
    StageTimer timer(c, st);
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;
    bool tc = use_tensor_path(c, T);
    // decode: routing, gate_up, down and the combine in one cooperative launch
    // (the fused kernel reads the residual rows as float4)
    const bool fused_decode = c->ep_n == 1 && !tc && decode_supported(d, T, c->cfg.device) &&
                              reinterpret_cast<uintptr_t>(residual) % 16 == 0;
    if (!c->blk.frag && !fused_decode) tc = true;  // streamed layers carry no GEMV tiles
    if (!fused_decode) {
        AMOE_CUDA(c, launch_route_impl(d, L, residual, T, r, c->partial, c->arrivals, st, &timer_hook, &timer));
        c->stats.launches += nchunk > 1 ? 3 : 1;  // route, then the two scan kernels
    }
    if (c->ep_n > 1) {
        if (c->ep_broken)
            return fail(c, AMOE_ERR_STATE, "expert-parallel group is out of step after a failed exchange; "
                                           "recreate the contexts");
        timer.mark(1);
        rc = ep_experts(c, L, r, T, nchunk, st, timer, &tc);
        if (rc) return rc;
    } else if (!tc && nchunk > 1 && !fused_decode) {
        AMOE_CUDA(c, launch_scatter(d, T, r, false, nullptr, nullptr, st));
        c->stats.launches += 1;
    }
    bool fused = false;
    if (c->ep_n > 1) {
    } else if (fused_decode) {
        timer.mark(1);
        int32_t *flag = c->err_flag;
        AMOE_CUDA(c, launch_decode(d, L, r, residual, T, c->dec_scratch, out, c->dec_bar, flag, c->cfg.device,
                                   st));
        timer.mark(6);
        c->stats.launches += 1;
        fused = true;
    } else if (tc) {
        timer.mark(1);
        if (nchunk > 1) {  // the stable permutation (one routing chunk writes it itself)
            AMOE_CUDA(c, launch_scatter(d, T, r, false, nullptr, nullptr, st));
            c->stats.launches += 1;
        }
        int n = 0;
        int32_t *flag = c->err_flag;
        AMOE_CUDA(c, launch_bs_experts(d, L, r.offsets, r.x_hi, r.x_lo, r.perm_pair, T, c->max_tokens * d.k,
                                       c->max_tokens, c->bs_scratch, c->dx.E, c->y, nullptr, flag, st, &timer_hook,
                                       &timer, &n));
        c->stats.launches += n;
    } else {
        timer.mark(1);
        int32_t *flag = c->err_flag;
        GemvRows rows{r.x_hi, r.x_lo, r.perm_pair, r.offsets, r.active, nullptr,
                      std::min(T * d.k, d.E)};
        AMOE_CUDA(c, launch_gemv_gate_up(d, L, rows, T, c->act_hi, c->act_lo, flag, st));
        timer.mark(2);
        AMOE_CUDA(c, launch_gemv_down(d, L, rows, T, c->act_hi, c->act_lo, c->y, flag, st));
        timer.mark(3);
        c->stats.launches += 2;
    }
    if (!fused) {
        const float *y = c->ep_n > 1 ? reinterpret_cast<const float *>(c->ep_win + c->ep_w.y) : c->y;
        AMOE_CUDA(c, launch_combine(d, residual, r, y, T, out, st));
        timer.mark(4);
        c->stats.launches += 1;
    }
    timer.finish();
    c->stats.forwards += 1;
    c->stats.last_path = tc ? AMOE_PATH_TENSOR : AMOE_PATH_GEMV;
    if (slot >= 0) {
        AMOE_CUDA(c, cudaEventRecord(c->slot_free[slot], st));
        // AirLLM-style streaming: start copying the next layer into the least
        // recently used slot while this layer computes.
        if (c->cfg.layers > (int)c->slot_dev.size()) {
            const int next = (layer + 1) % c->cfg.layers;
            int next_slot;
            if (c->uploaded[next]) {
                rc = acquire_slot(c, next, nullptr, &next_slot);
                if (rc) return rc;
            }
        }
    }
    if (topk_idx)
        AMOE_CUDA(c, cudaMemcpyAsync(topk_idx, r.topk_idx, (size_t)T * d.k * 4,
                                     cudaMemcpyDeviceToDevice, st));
    if (topk_w)
        AMOE_CUDA(c, cudaMemcpyAsync(topk_w, r.topk_w, (size_t)T * d.k * 4,
                                     cudaMemcpyDeviceToDevice, st));
    return AMOE_OK;
}

int check_forward_args(amoe_ctx *c, int32_t layer, const float *residual, int32_t T, const float *out) {
    if (layer < 0 || layer >= c->cfg.layers || !c->uploaded[layer])
        return fail(c, AMOE_ERR_STATE, "layer " + std::to_string(layer) + " is not uploaded");
    if (T <= 0) return fail(c, AMOE_ERR_INVALID, "gptoss: prefill sequence length must be positive");
    if (T > c->max_tokens)
        return fail(c, AMOE_ERR_INVALID, "T " + std::to_string(T) + " exceeds max_tokens " +
                                             std::to_string(c->max_tokens));
    if (!residual || !out) return fail(c, AMOE_ERR_INVALID, "residual and out must not be NULL");
    return AMOE_OK;
}

// Token slices of a host-buffer call: one pass unless the call is large enough
// that overlapping its host copies with compute pays (>= 2048 tokens; n passes of
// the size below become n + 1 with half-length ends), and only
// when every slice takes the same expert path as the whole call (so the output
// is bit-identical to one pass: tokens are independent).  Expert-parallel calls
// stay whole: every rank must make the same sequence of exchanges.
std::vector<int> plan_passes(const amoe_ctx *c, int T) {
    std::vector<int> one{T};
    if (T < 2048 || c->ep_n > 1) return one;
    // a pass keeps at least 64 pairs per expert on average, so that the tensor-core GEMM's
    // 48-token tiles stay mostly full (128 experts: 2048-token passes)
    const int per_expert = (int)std::min<long long>(1 << 20, (64LL * c->d.E + c->d.k - 1) / c->d.k);
    const int target = std::max({1024, per_expert, (T + kMaxIoChunks - 1) / kMaxIoChunks});
    const int n = std::min((T + target - 1) / target, kMaxIoChunks - 1);  // n + 1 passes with the split end
    int len = (T + n - 1) / n;
    len = (len + kRouteTokens - 1) / kRouteTokens * kRouteTokens;  // slices start on routing-chunk bounds
    // the first and last passes are half as long: the first pass's upload and the
    // last pass's download are the two copies no compute overlaps
    std::vector<int> passes;
    if (n >= 2) {  // every pass but the last starts and ends on a routing-chunk bound
        const int edge = (len / 2 + kRouteTokens - 1) / kRouteTokens * kRouteTokens;
        const int last0 = (T - edge) / kRouteTokens * kRouteTokens;  // the last pass's first token
        const int nm = n - 1, mid = last0 - edge;
        const int ml = ((mid + nm - 1) / nm + kRouteTokens - 1) / kRouteTokens * kRouteTokens;
        passes.push_back(edge);
        for (int t0 = edge; t0 < last0; t0 += ml) passes.push_back(std::min(ml, last0 - t0));
        passes.push_back(T - last0);
    }
    if (passes.size() < 2 || (int)passes.size() > kMaxIoChunks) return one;
    const int smallest = *std::min_element(passes.begin(), passes.end());
    if (use_tensor_path(c, smallest) != use_tensor_path(c, T)) return one;
    if (decode_supported(c->d, smallest, c->cfg.device) && !use_tensor_path(c, smallest)) return one;
    return passes;
}

}  // namespace

extern "C" {

int amoe_abi_version(void) { return AMOE_ABI_VERSION; }

const char *amoe_last_error(const amoe_ctx *ctx) {
    return ctx ? ctx->err.c_str() : g_create_error.c_str();
}

int amoe_create(const amoe_config *cfg, amoe_ctx **out) {
    g_create_error.clear();
    if (!out) {
        g_create_error = "out must not be NULL";
        return AMOE_ERR_INVALID;
    }
    *out = nullptr;
    std::string v = validate(cfg);
    if (!v.empty()) {
        g_create_error = v;
        return AMOE_ERR_INVALID;
    }
    amoe_ctx *c = new (std::nothrow) amoe_ctx();
    if (!c) {
        g_create_error = "out of host memory";
        return AMOE_ERR_NOMEM;
    }
    c->cfg = *cfg;
    c->cfg.nccl_id = nullptr;
    c->d = Dims{cfg->hidden, cfg->intermediate, cfg->experts, cfg->top_k, cfg->rms_eps};
    c->ep_n = cfg->ep_size;
    c->ep_rank = cfg->ep_rank;
    c->e_loc = cfg->experts / cfg->ep_size;
    c->dx = Dims{cfg->hidden, cfg->intermediate, c->e_loc, cfg->top_k, cfg->rms_eps};
    c->blk = layer_block(c->d, c->e_loc, cfg->stream_slots < 2);
    int rc = AMOE_OK;
    do {
        cudaError_t e = cudaSetDevice(cfg->device);
        if (e != cudaSuccess) { rc = cuda_fail(c, e, "cudaSetDevice"); break; }
        e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { rc = cuda_fail(c, e, "cudaStreamCreate"); break; }
        e = cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { rc = cuda_fail(c, e, "cudaStreamCreate"); break; }
        e = cudaStreamCreateWithFlags(&c->h2d_stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->d2h_stream, cudaStreamNonBlocking);
        for (int i = 0; i < kMaxIoChunks && e == cudaSuccess; ++i) {
            e = cudaEventCreateWithFlags(&c->io_in_ready[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->io_out_ready[i], cudaEventDisableTiming);
        }
        if (e == cudaSuccess) e = host_alloc(&c->h_flag, sizeof(int32_t), cudaHostAllocDefault);
        if (e != cudaSuccess) { rc = cuda_fail(c, e, "cudaStreamCreate/cudaEventCreate/cudaHostAlloc"); break; }
        if (c->ep_n > 1) {
            std::string why;
            if (!nccl_load(&why)) { rc = fail(c, AMOE_ERR_NCCL, why); break; }
            ncclUniqueId id;
            std::memcpy(&id, cfg->nccl_id, sizeof(id));
            const ncclResult_t nr = g_nccl.ncclCommInitRank(&c->comm, c->ep_n, id, c->ep_rank);
            if (nr != ncclSuccess) {
                c->comm = nullptr;
                rc = fail(c, AMOE_ERR_NCCL, std::string("ncclCommInitRank: ") + g_nccl.ncclGetErrorString(nr));
                break;
            }
        }
        c->layer_dev.assign(cfg->layers, nullptr);
        c->layer_host.assign(cfg->layers, nullptr);
        c->uploaded.assign(cfg->layers, false);
        if (cfg->stream_slots >= 2 && cfg->stream_experts) {
            const Dims &d = c->d;
            c->xs = std::min(d.E, cfg->max_tokens * d.k);
            c->xblk = layer_block(Dims{d.H, d.I, c->xs, d.k, d.eps}, c->xs, false);
            const size_t per_layer = ((size_t)d.H + (size_t)d.E * d.H + d.E) * 4;
            e = dev_alloc(&c->router_res, per_layer * cfg->layers);
            if (e == cudaSuccess) e = dev_alloc(&c->xslot, c->xblk.total);
            if (e == cudaSuccess) e = dev_alloc(&c->sel_dev, (size_t)2 * (c->xs + 1) * 4);
            if (e == cudaSuccess) e = host_alloc(&c->h_sel, ((size_t)d.E + 1 + 2 * (c->xs + 1)) * 4, 0);
            if (e != cudaSuccess) { rc = cuda_fail(c, e, "expert-streaming buffers"); break; }
        } else if (cfg->stream_slots >= 2) {
            for (int i = 0; i < cfg->stream_slots && rc == AMOE_OK; ++i) {
                uint8_t *p = nullptr;
                e = dev_alloc(&p, c->blk.total);
                if (e != cudaSuccess) { rc = cuda_fail(c, e, "cudaMalloc(stream slot)"); break; }
                c->slot_dev.push_back(p);
                c->slot_layer.push_back(-1);
                c->slot_used.push_back(0);
                cudaEvent_t a = nullptr, b = nullptr;
                e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
                if (a) c->slot_ready.push_back(a);
                if (b) c->slot_free.push_back(b);
                if (e == cudaSuccess) e = cudaEventRecord(b, c->stream);
                if (e != cudaSuccess) { rc = cuda_fail(c, e, "stream slot events"); break; }
            }
            if (rc != AMOE_OK) break;
        }
        rc = alloc_scratch(c);
        if (rc == AMOE_OK) {
            int sms = 0;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device);
            c->sms = sms > 0 ? sms : 148;
        }
        const long long ov = ep_wait_override_ns();
        c->ep_count_wait_ns = ov ? ov : kEpCountWaitNs;
        c->ep_data_wait_ns = ov ? ov : kEpDataWaitNs;
        if (rc == AMOE_OK && c->ep_n > 1) rc = ep_setup(c);
    } while (0);
    if (rc != AMOE_OK) {
        g_create_error = c->err;
        release(c);
        delete c;
        return rc;
    }
    *out = c;
    return AMOE_OK;
}

void amoe_destroy(amoe_ctx *ctx) {
    if (!ctx) return;
    release(ctx);
    delete ctx;
}

int amoe_upload_layer(amoe_ctx *c, int32_t layer, const float *norm_gain, const float *router_w,
                      const float *router_b, const uint8_t *gate_up, const float *gate_up_b,
                      const uint8_t *down, const float *down_b) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (layer < 0 || layer >= c->cfg.layers)
        return fail(c, AMOE_ERR_INVALID, "layer " + std::to_string(layer) + " outside [0, " +
                                             std::to_string(c->cfg.layers) + ")");
    if (!norm_gain || !router_w || !router_b || !gate_up || !gate_up_b || !down || !down_b)
        return fail(c, AMOE_ERR_INVALID, "layer tensors must not be NULL");
    const Dims &d = c->d;
    const size_t H = d.H, I = d.I, E_all = d.E;
    // this context stores experts [e0, e0 + E) (all of them unless expert-parallel)
    const size_t E = (size_t)c->e_loc, e0 = (size_t)c->ep_rank * c->e_loc;
    const size_t gu_expert = 2 * I * (H / 32) * 17, dn_expert = H * (I / 32) * 17;
    const size_t gu_bytes = E * gu_expert, dn_bytes = E * dn_expert;
    // Device-format block: built in a temporary device buffer, then kept there
    // (resident) or copied to pinned host memory (streaming).
    uint8_t *blockp = nullptr, *staging = nullptr;
    const size_t stage_bytes = gu_bytes > dn_bytes ? gu_bytes : dn_bytes;
    auto cleanup = [&]() {
        if (staging) cudaFree(staging);
        if (streaming(c) && blockp) cudaFree(blockp);
    };
    cudaError_t e;
#define UP_CUDA(call)                                       \
    do {                                                    \
        e = (call);                                         \
        if (e != cudaSuccess) {                             \
            cleanup();                                      \
            return cuda_fail(c, e, #call);                  \
        }                                                   \
    } while (0)
    if (!streaming(c)) {
        if (!c->layer_dev[layer]) {
            e = dev_alloc(&c->layer_dev[layer], c->blk.total);
            if (e != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(layer)");
        }
        blockp = c->layer_dev[layer];
    } else {
        if (!c->layer_host[layer]) {
            e = host_alloc(&c->layer_host[layer], c->blk.total, cudaHostAllocDefault);
            if (e != cudaSuccess) return cuda_fail(c, e, "cudaHostAlloc(layer)");
        }
        UP_CUDA(dev_alloc(&blockp, c->blk.total));
    }
    UP_CUDA(dev_alloc(&staging, stage_bytes));
    const LayerDev L = layer_view(blockp, c->blk);
    cudaStream_t st = c->stream;
    UP_CUDA(cudaMemcpyAsync(L.norm_gain, norm_gain, H * 4, cudaMemcpyHostToDevice, st));
    UP_CUDA(cudaMemcpyAsync(L.router_w, router_w, E_all * H * 4, cudaMemcpyHostToDevice, st));
    UP_CUDA(cudaMemcpyAsync(L.router_b, router_b, E_all * 4, cudaMemcpyHostToDevice, st));
    UP_CUDA(cudaMemcpyAsync(L.gu_b, gate_up_b + e0 * 2 * I, E * 2 * I * 4, cudaMemcpyHostToDevice, st));
    UP_CUDA(cudaMemcpyAsync(L.dn_b, down_b + e0 * H, E * H * 4, cudaMemcpyHostToDevice, st));
    UP_CUDA(cudaMemcpyAsync(staging, gate_up + e0 * gu_expert, gu_bytes, cudaMemcpyHostToDevice, st));
    if (c->blk.frag) UP_CUDA(launch_repack(staging, (int)E, (int)(2 * I), (int)H, true, L.gu_q, L.gu_s, st));
    UP_CUDA(launch_repack_tma(staging, (int)E, (int)(2 * I), (int)H, true, L.gu_tq, st));
    UP_CUDA(cudaStreamSynchronize(st));  // staging is reused for down
    UP_CUDA(cudaMemcpyAsync(staging, down + e0 * dn_expert, dn_bytes, cudaMemcpyHostToDevice, st));
    if (c->blk.frag) UP_CUDA(launch_repack(staging, (int)E, (int)H, (int)I, false, L.dn_q, L.dn_s, st));
    UP_CUDA(launch_repack_tma(staging, (int)E, (int)H, (int)I, false, L.dn_tq, st));
    if (streaming(c)) {
        if (c->router_res) {  // expert streaming: the layer's norm and router stay on the device
            float *dst = c->router_res + (size_t)layer * (H + E_all * H + E_all);
            UP_CUDA(cudaMemcpyAsync(dst, L.norm_gain, H * 4, cudaMemcpyDeviceToDevice, st));
            UP_CUDA(cudaMemcpyAsync(dst + H, L.router_w, E_all * H * 4, cudaMemcpyDeviceToDevice, st));
            UP_CUDA(cudaMemcpyAsync(dst + H + E_all * H, L.router_b, E_all * 4, cudaMemcpyDeviceToDevice, st));
        }
        UP_CUDA(cudaMemcpyAsync(c->layer_host[layer], blockp, c->blk.total, cudaMemcpyDeviceToHost, st));
        // a slot holding a stale copy of this layer must be refilled
        for (size_t i = 0; i < c->slot_layer.size(); ++i)
            if (c->slot_layer[i] == layer) c->slot_layer[i] = -1;
    }
    UP_CUDA(cudaStreamSynchronize(st));
#undef UP_CUDA
    cleanup();
    c->uploaded[layer] = true;
    return AMOE_OK;
}

int amoe_upload_layer_gguf(amoe_ctx *c, const amoe_gguf *g, int32_t layer) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!g) return fail(c, AMOE_ERR_INVALID, "gguf must not be NULL");
    if (layer < 0 || layer >= c->cfg.layers)
        return fail(c, AMOE_ERR_INVALID, "layer " + std::to_string(layer) + " outside [0, " +
                                             std::to_string(c->cfg.layers) + ")");
    GgufLayer t;
    std::string err;
    if (gguf_layer(g, layer, c->d.H, c->d.I, c->d.E, &t, &err))
        return fail(c, AMOE_ERR_INVALID, "gptoss: load layer " + std::to_string(layer) + ": " + err);
    return amoe_upload_layer(c, layer, t.norm, t.router_w, t.router_b, t.gu, t.gu_b, t.dn, t.dn_b);
}

int amoe_prefetch_layer(amoe_ctx *c, int32_t layer) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!streaming(c)) return fail(c, AMOE_ERR_STATE, "prefetch needs stream_slots >= 2");
    if (c->cfg.stream_experts) return AMOE_OK;  // which experts a layer needs is known only after routing
    if (layer < 0 || layer >= c->cfg.layers || !c->uploaded[layer])
        return fail(c, AMOE_ERR_STATE, "layer " + std::to_string(layer) + " is not uploaded");
    int slot;
    return acquire_slot(c, layer, nullptr, &slot);
}

int amoe_forward_device(amoe_ctx *c, int32_t layer, const float *residual, int32_t T, float *out,
                        int32_t *topk_idx, float *topk_w, void *stream) {
    int rc = check_ctx(c);
    if (rc) return rc;
    rc = check_forward_args(c, layer, residual, T, out);
    if (rc) return rc;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    rc = forward_impl(c, layer, residual, T, out, topk_idx, topk_w, st, route_view(c, 0, 0));
    if (rc) return rc;
    c->last_T = T;
    c->last_chunks.assign(1, T);
    return AMOE_OK;
}

int amoe_forward(amoe_ctx *c, int32_t layer, const float *residual, int32_t T, float *out,
                 int32_t *topk_idx, float *topk_w) {
    int rc = check_ctx(c);
    if (rc) return rc;
    rc = check_forward_args(c, layer, residual, T, out);
    if (rc) return rc;
    const Dims &d = c->d;
    const size_t H = d.H, k = d.k;
    const std::vector<int> passes = plan_passes(c, T);
    cudaStream_t st = c->stream;
    if (passes.size() == 1) {
        auto one_pass = [&]() -> int {
            AMOE_CUDA(c, cudaMemcpyAsync(c->io_in, residual, (size_t)T * H * 4, cudaMemcpyHostToDevice, st));
            const int prc = forward_impl(c, layer, c->io_in, T, c->io_out, nullptr, nullptr, st, route_view(c, 0, 0));
            if (prc) return prc;
            AMOE_CUDA(c, cudaMemcpyAsync(out, c->io_out, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st));
            if (topk_idx)
                AMOE_CUDA(c, cudaMemcpyAsync(topk_idx, c->r.topk_idx, (size_t)T * k * 4, cudaMemcpyDeviceToHost, st));
            if (topk_w)
                AMOE_CUDA(c, cudaMemcpyAsync(topk_w, c->r.topk_w, (size_t)T * k * 4, cudaMemcpyDeviceToHost, st));
            AMOE_CUDA(c, cudaMemcpyAsync(c->h_flag, c->err_flag, 4, cudaMemcpyDeviceToHost, st));
            return AMOE_OK;
        };
        rc = one_pass();
        if (rc) {
            cudaStreamSynchronize(st);  // nothing still reads or writes the caller's buffers
            return rc;
        }
    } else {
        // Pipeline: every slice's rows go up on the H2D stream at once; slice i
        // computes once its rows are in, and its outputs come down on the D2H
        // stream while slice i+1 computes (two copy engines, both directions).
        // On any failure all three streams are drained before returning, so no
        // copy into the caller's buffers is still in flight after the call.
        auto passes_run = [&]() -> int {
            AMOE_CUDA(c, cudaEventRecord(c->io_out_ready[0], st));  // earlier work on the compute stream
            AMOE_CUDA(c, cudaStreamWaitEvent(c->h2d_stream, c->io_out_ready[0], 0));
            int t0 = 0;
            for (size_t i = 0; i < passes.size(); ++i) {
                AMOE_CUDA(c, cudaMemcpyAsync(c->io_in + (size_t)t0 * H, residual + (size_t)t0 * H,
                                             (size_t)passes[i] * H * 4, cudaMemcpyHostToDevice, c->h2d_stream));
                AMOE_CUDA(c, cudaEventRecord(c->io_in_ready[i], c->h2d_stream));
                t0 += passes[i];
            }
            t0 = 0;
            for (size_t i = 0; i < passes.size(); ++i) {
                const int Tp = passes[i];
                AMOE_CUDA(c, cudaStreamWaitEvent(st, c->io_in_ready[i], 0));
                const RouteOut r = route_view(c, t0, (int)i);
                const int prc = forward_impl(c, layer, c->io_in + (size_t)t0 * H, Tp, c->io_out + (size_t)t0 * H,
                                             nullptr, nullptr, st, r);
                if (prc) return prc;
                AMOE_CUDA(c, cudaEventRecord(c->io_out_ready[i], st));
                AMOE_CUDA(c, cudaStreamWaitEvent(c->d2h_stream, c->io_out_ready[i], 0));
                AMOE_CUDA(c, cudaMemcpyAsync(out + (size_t)t0 * H, c->io_out + (size_t)t0 * H, (size_t)Tp * H * 4,
                                             cudaMemcpyDeviceToHost, c->d2h_stream));
                if (topk_idx)
                    AMOE_CUDA(c, cudaMemcpyAsync(topk_idx + (size_t)t0 * k, r.topk_idx, (size_t)Tp * k * 4,
                                                 cudaMemcpyDeviceToHost, c->d2h_stream));
                if (topk_w)
                    AMOE_CUDA(c, cudaMemcpyAsync(topk_w + (size_t)t0 * k, r.topk_w, (size_t)Tp * k * 4,
                                                 cudaMemcpyDeviceToHost, c->d2h_stream));
                t0 += Tp;
            }
            AMOE_CUDA(c, cudaMemcpyAsync(c->h_flag, c->err_flag, 4,
                                         cudaMemcpyDeviceToHost, c->d2h_stream));  // after the last pass
            AMOE_CUDA(c, cudaStreamSynchronize(c->d2h_stream));
            return AMOE_OK;
        };
        rc = passes_run();
        if (rc) {
            cudaStreamSynchronize(c->h2d_stream);
            cudaStreamSynchronize(st);
            cudaStreamSynchronize(c->d2h_stream);
            return rc;
        }
    }
    AMOE_CUDA(c, cudaStreamSynchronize(st));
    c->last_T = T;
    c->last_chunks = passes;
    return check_device_flag(c, *c->h_flag);
}

int amoe_synchronize(amoe_ctx *c) {
    int rc = check_ctx(c);
    if (rc) return rc;
    AMOE_CUDA(c, cudaStreamSynchronize(c->stream));
    AMOE_CUDA(c, cudaStreamSynchronize(c->copy_stream));
    AMOE_CUDA(c, cudaDeviceSynchronize());
    return check_device_flag(c);
}

int amoe_last_routing(amoe_ctx *c, float *logits, int32_t *perm_pair, int32_t *counts,
                      int32_t *offsets) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (c->last_T <= 0) return fail(c, AMOE_ERR_STATE, "no forward has run yet");
    const Dims &d = c->d;
    const size_t T = c->last_T, E = d.E, k = d.k;
    AMOE_CUDA(c, cudaStreamSynchronize(c->stream));
    if (logits) AMOE_CUDA(c, cudaMemcpy(logits, c->r.logits, T * E * 4, cudaMemcpyDeviceToHost));
    const size_t np = c->last_chunks.size();
    if (np <= 1) {
        if (perm_pair) AMOE_CUDA(c, cudaMemcpy(perm_pair, c->r.perm_pair, T * k * 4, cudaMemcpyDeviceToHost));
        if (counts) AMOE_CUDA(c, cudaMemcpy(counts, c->r.counts, E * 4, cudaMemcpyDeviceToHost));
        if (offsets) AMOE_CUDA(c, cudaMemcpy(offsets, c->r.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost));
        return AMOE_OK;
    }
    // A call made in several passes: each pass sorted its own pairs; the call's
    // stable (expert, token, slot) order is, per expert, the passes' runs in
    // token order, with pass-local pair ids shifted by the pass's first pair.
    std::vector<int32_t> cnt(np * E), off(np * (E + 1)), perm(T * k);
    AMOE_CUDA(c, cudaMemcpy(cnt.data(), c->r.counts, np * E * 4, cudaMemcpyDeviceToHost));
    AMOE_CUDA(c, cudaMemcpy(off.data(), c->r.offsets, np * (E + 1) * 4, cudaMemcpyDeviceToHost));
    AMOE_CUDA(c, cudaMemcpy(perm.data(), c->r.perm_pair, T * k * 4, cudaMemcpyDeviceToHost));
    std::vector<int32_t> total(E + 1, 0);
    for (size_t e = 0; e < E; ++e) {
        int32_t s = 0;
        for (size_t i = 0; i < np; ++i) s += cnt[i * E + e];
        total[e + 1] = total[e] + s;
    }
    if (counts)
        for (size_t e = 0; e < E; ++e) counts[e] = total[e + 1] - total[e];
    if (offsets) std::memcpy(offsets, total.data(), (E + 1) * 4);
    if (perm_pair) {
        size_t pos = 0;
        for (size_t e = 0; e < E; ++e) {
            size_t t0 = 0;
            for (size_t i = 0; i < np; ++i) {
                const int32_t *o = &off[i * (E + 1)];
                for (int32_t j = o[e]; j < o[e + 1]; ++j) perm_pair[pos++] = perm[t0 * k + j] + (int32_t)(t0 * k);
                t0 += c->last_chunks[i];
            }
        }
    }
    return AMOE_OK;
}

int amoe_ep_unique_id(void *out) {
    if (!out) {
        set_thread_error("out must not be NULL");
        return AMOE_ERR_INVALID;
    }
    std::string why;
    if (!nccl_load(&why)) {
        set_thread_error(why);
        return AMOE_ERR_NCCL;
    }
    ncclUniqueId id;
    const ncclResult_t r = g_nccl.ncclGetUniqueId(&id);
    if (r != ncclSuccess) {
        set_thread_error(std::string("ncclGetUniqueId: ") + g_nccl.ncclGetErrorString(r));
        return AMOE_ERR_NCCL;
    }
    std::memcpy(out, &id, sizeof(id));
    return AMOE_OK;
}

int amoe_ep_layout(int32_t n_ranks, int32_t experts_per_rank, int32_t rank, const int32_t *table,
                   int32_t *send_base, int32_t *offsets_loc, int32_t *seg_start, int32_t *src_pos) {
    if (ep_layout(n_ranks, experts_per_rank, rank, table, send_base, offsets_loc, seg_start, src_pos)) {
        set_thread_error("expert-parallel layout needs 1 <= n_ranks <= 8, experts_per_rank >= 1, "
                         "0 <= rank < n_ranks and a non-negative count table");
        return AMOE_ERR_INVALID;
    }
    return AMOE_OK;
}

int amoe_set_profiling(amoe_ctx *c, int32_t on) {
    int rc = check_ctx(c);
    if (rc) return rc;
    c->profiling = on != 0;
    return AMOE_OK;
}

int amoe_get_stats(amoe_ctx *c, amoe_stats *out, int32_t reset) {
    int rc = check_ctx(c);
    if (rc) return rc;
    if (!out) return fail(c, AMOE_ERR_INVALID, "stats must not be NULL");
    AMOE_CUDA(c, cudaStreamSynchronize(c->stream));
    AMOE_CUDA(c, cudaDeviceSynchronize());
    fold_timings(c);
    c->stats.layer_bytes = (int64_t)c->blk.total;
    *out = c->stats;
    if (reset) {
        const int32_t last = c->stats.last_path;
        c->stats = amoe_stats{};
        c->stats.last_path = last;
    }
    return AMOE_OK;
}

}  // extern "C"
