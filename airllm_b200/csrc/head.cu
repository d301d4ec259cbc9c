// head.cu -- the model head of the GPT-OSS runtime: final RMSNorm, lm_head and
// greedy token choice (Runtime.nextToken, internal/model/gptoss/runtime.go:234-250).
//
//   normalized = RMSNorm(hidden, output_norm, eps)        (primitives.go:50-72)
//   logits[v]  = f32(sum_k f64(normalized[k]) * f64(W[v][k]))   (primitives.go:11-32, no bias)
//   token      = the first index of the largest logit     (runtime.go:243-248)
//
// One launch streams the whole lm_head (V x H, stored as F32, F16 or BF16 exactly as
// the GGUF holds it) once for up to kHeadMaxTokens rows: a GEMV bound by HBM
// bandwidth (the 201,088 x 2880 bf16 head of GPT-OSS is 1.16 GB per call).  Each
// warp takes whole vocabulary rows, each lane a strided slice of 16-byte weight
// vectors, and accumulates every token's dot product in f64 (the products of two
// f32 values are exact there, so only the summation order differs from the
// reference's sequential sum, far below the f32 rounding of the logit).  The
// argmax is a max over 64-bit keys (order-preserving bits of the logit, then the
// complemented index, so equal logits resolve to the lowest index) combined per
// CTA in shared memory and across CTAs with atomicMax; a NaN logit never wins,
// and, as in the reference's loop, a NaN at index 0 leaves token 0.
#include "../../include/amoe.h"
#include "amoe_internal.cuh"

#include <cuda_bf16.h>

#include <cmath>
#include <string>

namespace amoe {
namespace {

constexpr int kHeadMaxTokens = 16;
constexpr int kHeadThreads = 256;
constexpr size_t kHeadMaxSmem = 200 * 1024;  // normalized rows staged in shared memory
constexpr size_t kHeadRowsAt = 512;          // after the reduction slots and the per-row best keys
static_assert(33 * 8 + kHeadMaxTokens * 8 <= kHeadRowsAt, "shared-memory layout");

// Order-preserving 32-bit image of a non-NaN float.
__device__ __forceinline__ uint32_t ordered(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long key_of(float v, int index) {
    return ((unsigned long long)ordered(v) << 32) | (unsigned long long)(~(uint32_t)index);
}

// Eight weights (16 bytes of the row, BF16 or F16) as doubles.
template <int TYPE>
__device__ __forceinline__ void widen8(const uint4 u, double (&w)[8]) {
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
    if (TYPE == AMOE_GGUF_BF16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[2 * i] = (double)__uint_as_float(v[i] << 16);
            w[2 * i + 1] = (double)__uint_as_float(v[i] & 0xffff0000u);
        }
    } else {  // F16
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&v[i]));
            w[2 * i] = (double)f.x;
            w[2 * i + 1] = (double)f.y;
        }
    }
}

// acc[t] += sum over the 8 elements from k of xs[t][k..] * w (every product exact in f64).
template <int T>
__device__ __forceinline__ void dot8(const float *xs, int H, int k, const double (&w)[8], double (&acc)[T]) {
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const float4 a = *reinterpret_cast<const float4 *>(xs + (size_t)t * H + k);
        const float4 b = *reinterpret_cast<const float4 *>(xs + (size_t)t * H + k + 4);
        acc[t] += (double)a.x * w[0] + (double)a.y * w[1] + (double)a.z * w[2] + (double)a.w * w[3] +
                  (double)b.x * w[4] + (double)b.y * w[5] + (double)b.z * w[6] + (double)b.w * w[7];
    }
}

template <int TYPE>
__device__ __forceinline__ double load1(const uint8_t *row, int k) {
    if (TYPE == AMOE_GGUF_F32) return (double)__ldg(reinterpret_cast<const float *>(row) + k);
    const uint16_t h = __ldg(reinterpret_cast<const unsigned short *>(row) + k);
    if (TYPE == AMOE_GGUF_BF16) return (double)__uint_as_float((uint32_t)h << 16);
    return (double)__half2float(__ushort_as_half(h));
}

// normalized rows [T][H] f32 in shared memory, computed by every CTA (T*H is small).
__device__ void stage_rows(const float *__restrict__ hidden, const float *__restrict__ gain, int T, int H,
                           float eps, float *xs, double *red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    for (int t = 0; t < T; ++t) {
        double ss = 0.0;
        for (int i = tid; i < H; i += blockDim.x) {
            const double v = (double)hidden[(size_t)t * H + i];
            ss += v * v;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            double s = 0.0;
            for (int w = 0; w < nw; ++w) s += red[w];  // fixed order: every CTA gets the same value
            red[32] = 1.0 / sqrt(s / (double)H + (double)eps);
        }
        __syncthreads();
        const double inv = red[32];
        for (int i = tid; i < H; i += blockDim.x)
            xs[(size_t)t * H + i] = (float)((double)hidden[(size_t)t * H + i] * inv * (double)gain[i]);
        __syncthreads();
    }
}

template <int TYPE, int T>
__global__ void __launch_bounds__(kHeadThreads) head_kernel(const float *__restrict__ hidden,
                                                            const float *__restrict__ gain,
                                                            const uint8_t *__restrict__ W, int H, int V, float eps,
                                                            float *__restrict__ logits,
                                                            unsigned long long *__restrict__ keys,
                                                            int32_t *__restrict__ nan0) {
    extern __shared__ __align__(16) uint8_t smem[];
    double *red = reinterpret_cast<double *>(smem);  // [33]
    unsigned long long *best_s = reinterpret_cast<unsigned long long *>(smem + 33 * 8);  // [T]
    float *xs = reinterpret_cast<float *>(smem + kHeadRowsAt);  // [T][H], 16-byte aligned
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < T) best_s[tid] = 0ull;
    stage_rows(hidden, gain, T, H, eps, xs, red);
    const size_t esz = TYPE == AMOE_GGUF_F32 ? 4 : 2;
    const size_t row_bytes = (size_t)H * esz;
    // 16-byte vectors cover the row when it is 16-byte aligned (the rows follow each other)
    const bool vec = TYPE != AMOE_GGUF_F32 && (row_bytes % 16) == 0;
    const int nvec = vec ? (int)(row_bytes / 16) : 0;
    unsigned long long best[T];
#pragma unroll
    for (int t = 0; t < T; ++t) best[t] = 0ull;
    const int gw = blockIdx.x * (blockDim.x >> 5) + warp, nwarps = gridDim.x * (blockDim.x >> 5);
    for (int v = gw; v < V; v += nwarps) {
        const uint8_t *row = W + (size_t)v * row_bytes;
        double acc[T];
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = 0.0;
        if (vec) {
            // U independent 16-byte loads per lane in flight before their arithmetic: a row is
            // only a few KB, so without them a warp waits out one memory latency per load
            constexpr int U = T <= 2 ? 8 : (T <= 4 ? 4 : 2);
            int j = lane;
            for (; j + 32 * (U - 1) < nvec; j += 32 * U) {
                uint4 raw[U];
#pragma unroll
                for (int q = 0; q < U; ++q) raw[q] = __ldg(reinterpret_cast<const uint4 *>(row + (size_t)(j + 32 * q) * 16));
#pragma unroll
                for (int q = 0; q < U; ++q) {
                    double w[8];
                    widen8<TYPE>(raw[q], w);
                    dot8<T>(xs, H, 8 * (j + 32 * q), w, acc);
                }
            }
            for (; j < nvec; j += 32) {
                double w[8];
                widen8<TYPE>(__ldg(reinterpret_cast<const uint4 *>(row + (size_t)j * 16)), w);
                dot8<T>(xs, H, 8 * j, w, acc);
            }
        } else {
            for (int k = lane; k < H; k += 32) {
                const double w = load1<TYPE>(row, k);
#pragma unroll
                for (int t = 0; t < T; ++t) acc[t] += (double)xs[(size_t)t * H + k] * w;
            }
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            double s = acc[t];
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            const float lg = (float)s;
            if (lane == 0) {
                if (logits) logits[(size_t)t * V + v] = lg;
                if (isnan(lg)) {
                    if (v == 0) nan0[t] = 1;
                } else {
                    const unsigned long long k = key_of(lg, v);
                    best[t] = k > best[t] ? k : best[t];
                }
            }
        }
    }
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < T; ++t) atomicMax(best_s + t, best[t]);
    __syncthreads();
    if (tid < T && best_s[tid]) atomicMax(keys + tid, best_s[tid]);
}

__global__ void head_finish_kernel(const unsigned long long *keys, const int32_t *nan0, int T, int32_t *tokens) {
    const int t = threadIdx.x;
    if (t >= T) return;
    // no finite logit, or a NaN at index 0 (the reference's loop never replaces it): token 0
    tokens[t] = (nan0[t] || keys[t] == 0ull) ? 0 : (int32_t)(~(uint32_t)(keys[t] & 0xffffffffull));
}

template <int TYPE>
cudaError_t launch_head_t(const float *hidden, const float *gain, const uint8_t *W, int T, int H, int V, float eps,
                          float *logits, unsigned long long *keys, int32_t *nan0, int grid, size_t smem,
                          cudaStream_t st) {
#define AMOE_HEAD_CASE(n)                                                                                     \
    case n: {                                                                                                 \
        cudaError_t e = cudaFuncSetAttribute(head_kernel<TYPE, n>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                             (int)smem);                                                       \
        if (e != cudaSuccess) return e;                                                                       \
        head_kernel<TYPE, n><<<grid, kHeadThreads, smem, st>>>(hidden, gain, W, H, V, eps, logits, keys, nan0); \
        return cudaGetLastError();                                                                            \
    }
    switch (T) {
        AMOE_HEAD_CASE(1)
        AMOE_HEAD_CASE(2)
        AMOE_HEAD_CASE(4)
        AMOE_HEAD_CASE(8)
        AMOE_HEAD_CASE(16)
        default: return cudaErrorInvalidValue;
    }
#undef AMOE_HEAD_CASE
}

}  // namespace
}  // namespace amoe

using namespace amoe;

struct amoe_head {
    int32_t hidden = 0, vocab = 0, device = 0, type = AMOE_GGUF_F32;
    float eps = 0.0f;
    bool uploaded = false;
    float *gain = nullptr;          // [H]
    uint8_t *W = nullptr;           // [V][H] as uploaded (F32, F16 or BF16)
    float *io_hidden = nullptr;     // [kHeadMaxTokens][H] staging of host rows (padded tokens read zeros)
    unsigned long long *keys = nullptr;  // [kHeadMaxTokens]
    int32_t *nan0 = nullptr;        // [kHeadMaxTokens]
    int32_t *tokens = nullptr;      // [kHeadMaxTokens]
    float *io_logits = nullptr;     // [kHeadMaxTokens][V] for host calls that want the logits
    cudaStream_t stream = nullptr;
    int sms = 148;
    std::string err;
};

namespace {

int head_fail(amoe_head *h, int code, const std::string &msg) {
    if (h) h->err = msg;
    else set_thread_error(msg);
    return code;
}

int head_cuda(amoe_head *h, cudaError_t e, const char *what) {
    return head_fail(h, e == cudaErrorMemoryAllocation ? AMOE_ERR_NOMEM : AMOE_ERR_CUDA,
                     std::string(what) + ": " + cudaGetErrorString(e));
}

#define HEAD_CUDA(h, call)                                        \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return head_cuda(h, e_, #call);    \
    } while (0)

size_t elem_bytes(int type) { return type == AMOE_GGUF_F32 ? 4 : 2; }

// Rows are launched in groups of 1, 2, 4, 8 or 16 (the compiled kernels).
int group_of(int T) { return T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : T <= 8 ? 8 : 16; }

size_t head_smem(int T, int H) { return kHeadRowsAt + (size_t)group_of(T) * H * 4; }

int head_run(amoe_head *h, const float *hidden, int T, int32_t *tokens, float *logits, cudaStream_t st) {
    const int G = group_of(T);
    // rows past T of the launch group read the zeroed tail of the staging buffer
    const float *src = hidden;
    if (G != T) {
        if (hidden != h->io_hidden)
            HEAD_CUDA(h, cudaMemcpyAsync(h->io_hidden, hidden, (size_t)T * h->hidden * 4, cudaMemcpyDeviceToDevice, st));
        HEAD_CUDA(h, cudaMemsetAsync(h->io_hidden + (size_t)T * h->hidden, 0, (size_t)(G - T) * h->hidden * 4, st));
        src = h->io_hidden;
    }
    float *lg = logits;
    if (logits && G != T) lg = h->io_logits;
    HEAD_CUDA(h, cudaMemsetAsync(h->keys, 0, kHeadMaxTokens * 8, st));
    HEAD_CUDA(h, cudaMemsetAsync(h->nan0, 0, kHeadMaxTokens * 4, st));
    const int grid = 4 * h->sms;  // four CTAs of eight warps per SM keep enough loads in flight
    const size_t smem = head_smem(T, h->hidden);
    cudaError_t e = cudaErrorInvalidValue;
    if (h->type == AMOE_GGUF_BF16)
        e = launch_head_t<AMOE_GGUF_BF16>(src, h->gain, h->W, G, h->hidden, h->vocab, h->eps, lg, h->keys, h->nan0,
                                          grid, smem, st);
    else if (h->type == AMOE_GGUF_F16)
        e = launch_head_t<AMOE_GGUF_F16>(src, h->gain, h->W, G, h->hidden, h->vocab, h->eps, lg, h->keys, h->nan0,
                                         grid, smem, st);
    else
        e = launch_head_t<AMOE_GGUF_F32>(src, h->gain, h->W, G, h->hidden, h->vocab, h->eps, lg, h->keys, h->nan0,
                                         grid, smem, st);
    HEAD_CUDA(h, e);
    head_finish_kernel<<<1, kHeadMaxTokens, 0, st>>>(h->keys, h->nan0, T, tokens);
    HEAD_CUDA(h, cudaGetLastError());
    if (logits && lg != logits)
        HEAD_CUDA(h, cudaMemcpyAsync(logits, lg, (size_t)T * h->vocab * 4, cudaMemcpyDeviceToDevice, st));
    return AMOE_OK;
}

int head_check(amoe_head *h) {
    if (!h) return head_fail(nullptr, AMOE_ERR_INVALID, "head must not be NULL");
    cudaError_t e = cudaSetDevice(h->device);
    if (e != cudaSuccess) return head_cuda(h, e, "cudaSetDevice");
    return AMOE_OK;
}

int head_args(amoe_head *h, const float *hidden, int32_t T, const int32_t *tokens) {
    if (!h->uploaded) return head_fail(h, AMOE_ERR_STATE, "gptoss: final norm and lm head are not uploaded");
    if (T < 1 || T > kHeadMaxTokens)
        return head_fail(h, AMOE_ERR_INVALID, "T " + std::to_string(T) + " outside [1, " +
                                                  std::to_string(kHeadMaxTokens) + "]");
    if (!hidden || !tokens) return head_fail(h, AMOE_ERR_INVALID, "hidden and tokens must not be NULL");
    return AMOE_OK;
}

}  // namespace

extern "C" {

int amoe_head_create(int32_t hidden, int32_t vocab, float rms_eps, int32_t device, amoe_head **out) {
    set_thread_error("");
    if (!out) return head_fail(nullptr, AMOE_ERR_INVALID, "out must not be NULL");
    *out = nullptr;
    if (hidden < 1 || vocab < 1) return head_fail(nullptr, AMOE_ERR_INVALID, "hidden and vocab must be positive");
    if (!(rms_eps > 0.0f) || !std::isfinite(rms_eps))
        return head_fail(nullptr, AMOE_ERR_INVALID, "rmsnorm epsilon must be positive");
    if (head_smem(kHeadMaxTokens, hidden) > kHeadMaxSmem)
        return head_fail(nullptr, AMOE_ERR_INVALID, "hidden " + std::to_string(hidden) + " too large for the head kernel");
    amoe_head *h = new (std::nothrow) amoe_head();
    if (!h) return head_fail(nullptr, AMOE_ERR_NOMEM, "out of host memory");
    h->hidden = hidden;
    h->vocab = vocab;
    h->eps = rms_eps;
    h->device = device;
    int rc = AMOE_OK;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&h->gain, (size_t)hidden * 4);
    if (e == cudaSuccess) e = cudaMalloc(&h->io_hidden, (size_t)kHeadMaxTokens * hidden * 4);
    if (e == cudaSuccess) e = cudaMalloc(&h->keys, kHeadMaxTokens * 8);
    if (e == cudaSuccess) e = cudaMalloc(&h->nan0, kHeadMaxTokens * 4);
    if (e == cudaSuccess) e = cudaMalloc(&h->tokens, kHeadMaxTokens * 4);
    if (e == cudaSuccess) e = cudaMalloc(&h->io_logits, (size_t)kHeadMaxTokens * vocab * 4);
    if (e == cudaSuccess) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        h->sms = sms > 0 ? sms : 148;
    }
    if (e != cudaSuccess) rc = head_cuda(h, e, "amoe_head_create");
    if (rc != AMOE_OK) {
        set_thread_error(h->err);
        amoe_head_destroy(h);
        return rc;
    }
    *out = h;
    return AMOE_OK;
}

void amoe_head_destroy(amoe_head *h) {
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    cudaFree(h->gain);
    cudaFree(h->W);
    cudaFree(h->io_hidden);
    cudaFree(h->keys);
    cudaFree(h->nan0);
    cudaFree(h->tokens);
    cudaFree(h->io_logits);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

const char *amoe_head_last_error(const amoe_head *h) { return h ? h->err.c_str() : amoe_last_error(nullptr); }

int amoe_head_upload(amoe_head *h, const float *final_norm, const void *lm_head, int32_t type) {
    int rc = head_check(h);
    if (rc) return rc;
    if (!final_norm || !lm_head) return head_fail(h, AMOE_ERR_INVALID, "final norm and lm head must not be NULL");
    if (type != AMOE_GGUF_F32 && type != AMOE_GGUF_F16 && type != AMOE_GGUF_BF16)
        return head_fail(h, AMOE_ERR_INVALID, "unsupported lm head type " + std::to_string(type) +
                                                  " (F32, F16 or BF16)");
    const size_t bytes = (size_t)h->vocab * h->hidden * elem_bytes(type);
    if (h->W && h->type != type) {
        cudaFree(h->W);
        h->W = nullptr;
    }
    if (!h->W) {
        cudaError_t e = cudaMalloc(&h->W, bytes);
        if (e != cudaSuccess) {
            h->W = nullptr;
            h->uploaded = false;
            return head_cuda(h, e, "cudaMalloc(lm head)");
        }
    }
    h->type = type;
    HEAD_CUDA(h, cudaMemcpyAsync(h->gain, final_norm, (size_t)h->hidden * 4, cudaMemcpyHostToDevice, h->stream));
    HEAD_CUDA(h, cudaMemcpyAsync(h->W, lm_head, bytes, cudaMemcpyHostToDevice, h->stream));
    HEAD_CUDA(h, cudaStreamSynchronize(h->stream));
    h->uploaded = true;
    return AMOE_OK;
}

int amoe_head_upload_gguf(amoe_head *h, const amoe_gguf *g) {
    int rc = head_check(h);
    if (rc) return rc;
    if (!g) return head_fail(h, AMOE_ERR_INVALID, "gguf must not be NULL");
    GgufHead t;
    std::string err;
    if (gguf_head(g, h->hidden, h->vocab, &t, &err)) return head_fail(h, AMOE_ERR_INVALID, "gptoss: " + err);
    return amoe_head_upload(h, t.norm, t.lm_head, t.type);
}

int amoe_head_next_token_device(amoe_head *h, const float *hidden, int32_t T, int32_t *tokens, float *logits,
                                void *stream) {
    int rc = head_check(h);
    if (rc) return rc;
    rc = head_args(h, hidden, T, tokens);
    if (rc) return rc;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    return head_run(h, hidden, T, tokens, logits, st);
}

int amoe_head_next_token(amoe_head *h, const float *hidden, int32_t T, int32_t *tokens, float *logits) {
    int rc = head_check(h);
    if (rc) return rc;
    rc = head_args(h, hidden, T, tokens);
    if (rc) return rc;
    cudaStream_t st = h->stream;
    auto run = [&]() -> int {
        HEAD_CUDA(h, cudaMemcpyAsync(h->io_hidden, hidden, (size_t)T * h->hidden * 4, cudaMemcpyHostToDevice, st));
        // the staged rows are already on the device; head_run pads them in place
        const int r = head_run(h, h->io_hidden, T, h->tokens, logits ? h->io_logits : nullptr, st);
        if (r) return r;
        HEAD_CUDA(h, cudaMemcpyAsync(tokens, h->tokens, (size_t)T * 4, cudaMemcpyDeviceToHost, st));
        if (logits)
            HEAD_CUDA(h, cudaMemcpyAsync(logits, h->io_logits, (size_t)T * h->vocab * 4, cudaMemcpyDeviceToHost, st));
        HEAD_CUDA(h, cudaStreamSynchronize(st));
        return AMOE_OK;
    };
    rc = run();
    if (rc) cudaStreamSynchronize(st);
    return rc;
}

}  // extern "C"
