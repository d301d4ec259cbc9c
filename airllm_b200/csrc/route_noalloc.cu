// route_noalloc.cu -- the routing step (RMSNorm + router + top-k + softmax)
// for callers that cannot allocate device memory.
//
// Some callers cannot let a library call cudaMalloc: a host runtime that plans
// its device memory up front and hands every region out itself (the reference
// budgets memory ahead of time, pkg/memory/memory.go:91-138), or a process in
// which another allocator (for example PyTorch's caching allocator) has already
// reserved the GPU, so a fresh cudaMalloc can fail or synchronise the device.
// amoe_route_noalloc takes only caller-owned inputs and outputs and keeps its
// scratch (split-K partial sums, arrival counters, the fp16 split of the
// normalized rows, the per-chunk histograms and the permutation) in one file-scope device array
// of fixed size, kNoAllocScratchBytes.  It calls no cudaMalloc/cudaFree.
//
// The array is shared by every call on a device and keeps the last call's
// contents; the arrival counters are cleared (cudaMemsetAsync) at the start of
// each call.  Calls that overlap on the GPU (different streams, or threads
// calling concurrently) race on the array.
#include "../../include/amoe.h"
#include "amoe_internal.cuh"

#include <mutex>
#include <string>

namespace amoe {

namespace {

constexpr int kNoAllocMaxTokens = 64;
constexpr int kNoAllocMaxHidden = 4096;
constexpr int kNoAllocMaxExperts = 128;
constexpr int kNoAllocMaxTopK = 32;
constexpr int kNoAllocMaxChunks = (kNoAllocMaxTokens + kRouteTokens - 1) / kRouteTokens;
constexpr int kNoAllocMaxDevices = 64;

// Byte layout of the scratch array (each part 256-B aligned).
constexpr size_t al(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kOffXhi = 0;
constexpr size_t kOffXlo = kOffXhi + al((size_t)kNoAllocMaxTokens * kNoAllocMaxHidden * 2);
constexpr size_t kOffPartial = kOffXlo + al((size_t)kNoAllocMaxTokens * kNoAllocMaxHidden * 2);
constexpr size_t kPartialElems = (size_t)16 * kNoAllocMaxTokens * kNoAllocMaxExperts;  // ksplit <= 16
constexpr size_t kOffHist = kOffPartial + al(kPartialElems * 8);
constexpr size_t kOffBase = kOffHist + al((size_t)kNoAllocMaxChunks * kNoAllocMaxExperts * 4);
constexpr size_t kOffCounts = kOffBase + al((size_t)kNoAllocMaxChunks * kNoAllocMaxExperts * 4);
constexpr size_t kOffOffsets = kOffCounts + al((size_t)kNoAllocMaxExperts * 4);
constexpr size_t kOffActive = kOffOffsets + al((size_t)(kNoAllocMaxExperts + 1) * 4);
constexpr size_t kOffPerm = kOffActive + al((size_t)(kNoAllocMaxExperts + 1) * 4);
constexpr size_t kOffInv = kOffPerm + al((size_t)kNoAllocMaxTokens * kNoAllocMaxTopK * 4);
constexpr size_t kOffArrivals = kOffInv + al((size_t)kNoAllocMaxTokens * kNoAllocMaxTopK * 4);
constexpr size_t kNoAllocScratchBytes = kOffArrivals + al((size_t)kNoAllocMaxChunks * 4);

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_route_scratch on `device` (which must be current).  The
// host-side name g_route_scratch is only a stand-in; kernels need this address.
int scratch_address(int device, unsigned char **out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess) {
            set_thread_error(std::string("cudaGetSymbolAddress(route scratch): ") + cudaGetErrorString(e));
            return AMOE_ERR_CUDA;
        }
        g_scratch_addr[device] = p;
    }
    *out = static_cast<unsigned char *>(g_scratch_addr[device]);
    return AMOE_OK;
}

// Makes `device` current for the call and gives the calling thread back the
// device it had: a host whose GPU work another runtime manages keeps its
// current device across this call.
struct DeviceScope {
    int prev = -1;
    cudaError_t enter(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        return cudaSetDevice(device);
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int reject(const std::string &msg) {
    set_thread_error(msg);
    return AMOE_ERR_INVALID;
}

}  // namespace

}  // namespace amoe

using namespace amoe;

extern "C" AMOE_API int amoe_route_noalloc(int32_t device, int32_t hidden, int32_t experts, int32_t top_k,
                                           float rms_eps, const float *residual, int32_t T,
                                           const float *norm_gain, const float *router_w,
                                           const float *router_b, float *logits, int32_t *topk_idx,
                                           float *topk_w, void *stream) {
    if (device < 0 || device >= kNoAllocMaxDevices) return reject("device ordinal out of range");
    if (T < 1 || T > kNoAllocMaxTokens)
        return reject("T " + std::to_string(T) + " outside [1, " + std::to_string(kNoAllocMaxTokens) +
                      "] (fixed scratch limit)");
    if (hidden < 64 || hidden % 64 || hidden > kNoAllocMaxHidden)
        return reject("hidden must be a multiple of 64 in [64, " + std::to_string(kNoAllocMaxHidden) +
                      "] (fixed scratch limit)");
    if (experts < 1 || experts > kNoAllocMaxExperts)
        return reject("experts outside [1, " + std::to_string(kNoAllocMaxExperts) + "] (fixed scratch limit)");
    if (top_k < 1 || top_k > experts || top_k > kNoAllocMaxTopK)
        return reject("moe router top-k " + std::to_string(top_k) + " outside [1, " +
                      std::to_string(experts < kNoAllocMaxTopK ? experts : kNoAllocMaxTopK) + "]");
    if (!(rms_eps > 0.0f)) return reject("rmsnorm epsilon must be positive");
    if (!residual || !norm_gain || !router_w || !router_b || !logits || !topk_idx || !topk_w)
        return reject("inputs and outputs must not be NULL");

    DeviceScope scope;
    cudaError_t e = scope.enter(device);
    if (e != cudaSuccess) {
        set_thread_error(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
        return AMOE_ERR_CUDA;
    }
    unsigned char *base = nullptr;
    int rc = scratch_address(device, &base);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nchunk = (T + kRouteTokens - 1) / kRouteTokens;

    RouteOut o{};
    o.x_hi = reinterpret_cast<__half *>(base + kOffXhi);
    o.x_lo = reinterpret_cast<__half *>(base + kOffXlo);
    o.logits = logits;
    o.topk_idx = topk_idx;
    o.topk_w = topk_w;
    o.hist = reinterpret_cast<int32_t *>(base + kOffHist);
    o.chunk_base = reinterpret_cast<int32_t *>(base + kOffBase);
    o.counts = reinterpret_cast<int32_t *>(base + kOffCounts);
    o.offsets = reinterpret_cast<int32_t *>(base + kOffOffsets);
    o.active = reinterpret_cast<int32_t *>(base + kOffActive);
    o.perm_pair = reinterpret_cast<int32_t *>(base + kOffPerm);
    o.inv = reinterpret_cast<int32_t *>(base + kOffInv);
    double *partial = reinterpret_cast<double *>(base + kOffPartial);
    int32_t *arrivals = reinterpret_cast<int32_t *>(base + kOffArrivals);

    LayerDev L;
    L.norm_gain = const_cast<float *>(norm_gain);
    L.router_w = const_cast<float *>(router_w);
    L.router_b = const_cast<float *>(router_b);

    // the split-K arrival counters must start at zero
    e = cudaMemsetAsync(arrivals, 0, (size_t)nchunk * sizeof(int32_t), st);
    const Dims d{hidden, 0, experts, top_k, rms_eps};
    if (e == cudaSuccess) e = launch_route_impl(d, L, residual, T, o, partial, arrivals, st);
    if (e != cudaSuccess) {
        set_thread_error(std::string("amoe_route_noalloc: ") + cudaGetErrorString(e));
        return AMOE_ERR_CUDA;
    }
    return AMOE_OK;
}
