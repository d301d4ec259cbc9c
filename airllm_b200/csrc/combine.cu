// combine.cu -- K6: routing-weighted combine and residual add, and the K8
// upload-time MXFP4 repack.
#include "amoe_internal.cuh"

namespace amoe {

namespace {

// out[t] = residual[t] + f32( sum_s f64(w[t,s]) * f64(y[inv[t,s]]) ), slot order
// s = 0..k-1 (layer.go:109-121: float64 mixture, float32 add of the pre-norm row).
__global__ void __launch_bounds__(256) combine_kernel(const float *__restrict__ residual,
                                                      const float *__restrict__ y,
                                                      const int32_t *__restrict__ inv,
                                                      const float *__restrict__ w, int H, int k,
                                                      float *__restrict__ out) {
    const int t = blockIdx.x;
    __shared__ int pos_s[32];
    __shared__ double w_s[32];
    if (threadIdx.x < k) {
        pos_s[threadIdx.x] = inv[(size_t)t * k + threadIdx.x];
        w_s[threadIdx.x] = (double)w[(size_t)t * k + threadIdx.x];
    }
    __syncthreads();
    const float4 *res4 = reinterpret_cast<const float4 *>(residual + (size_t)t * H);
    float4 *out4 = reinterpret_cast<float4 *>(out + (size_t)t * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        double m0 = 0.0, m1 = 0.0, m2 = 0.0, m3 = 0.0;
        for (int s = 0; s < k; ++s) {
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(y + (size_t)pos_s[s] * H) + i);
            const double ws = w_s[s];
            m0 += ws * (double)v.x;
            m1 += ws * (double)v.y;
            m2 += ws * (double)v.z;
            m3 += ws * (double)v.w;
        }
        const float4 r = res4[i];
        out4[i] = make_float4(r.x + (float)m0, r.y + (float)m1, r.z + (float)m2, r.w + (float)m3);
    }
}

// K8: GGUF MXFP4 (17-byte blocks, tensor.go:150-160) -> tiled nibble/scale
// planes (amoe_internal.cuh).  Lossless byte shuffle; one thread per 16-byte
// lane chunk of a 16x64 tile.
__global__ void repack_kernel(const uint8_t *__restrict__ gguf, int E, int R, int K,
                              int pair_rows, uint8_t *__restrict__ q, uint8_t *__restrict__ s) {
    const int nkt = K / kTileK, nrt = R / kTileRows, nblk = K / 32;
    const long long total = (long long)E * nrt * nkt * 32;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= total) return;
    const int lane = (int)(tid % 32);
    long long t = tid / 32;
    const int kt = (int)(t % nkt);
    t /= nkt;
    const int rt = (int)(t % nrt);
    const int e = (int)(t / nrt);
    const int g = lane >> 2, c = lane & 3;
    const int row_g = pair_rows ? 2 * (8 * rt + g) : kTileRows * rt + g;
    const int row_g8 = pair_rows ? 2 * (8 * rt + g) + 1 : kTileRows * rt + g + 8;
    const uint8_t *src_g = gguf + ((size_t)e * R + row_g) * nblk * 17;
    const uint8_t *src_g8 = gguf + ((size_t)e * R + row_g8) * nblk * 17;
    uint32_t w[4];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int blk = 2 * kt + b;
        const uint8_t *a = src_g + blk * 17 + 1 + 4 * c;
        const uint8_t *bb = src_g8 + blk * 17 + 1 + 4 * c;
        w[2 * b] = a[0] | (a[1] << 8) | (a[2] << 16) | ((uint32_t)a[3] << 24);
        w[2 * b + 1] = bb[0] | (bb[1] << 8) | (bb[2] << 16) | ((uint32_t)bb[3] << 24);
    }
    const size_t tile = ((size_t)e * nrt + rt) * nkt + kt;
    *reinterpret_cast<uint4 *>(q + tile * kTileQBytes + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    if (c == 0) {
        uint8_t *sd = s + tile * kTileSBytes + 4 * g;
        sd[0] = src_g[(2 * kt) * 17];
        sd[1] = src_g[(2 * kt + 1) * 17];
        sd[2] = src_g8[(2 * kt) * 17];
        sd[3] = src_g8[(2 * kt + 1) * 17];
    }
}

// K8b: GGUF MXFP4 -> box planes (amoe_internal.cuh).  One thread per
// (expert, padded row, 32-element block) of the padded K range; lossless.
__global__ void repack_tma_kernel(const uint8_t *__restrict__ gguf, int E, int R, int K, int pair_rows,
                                  uint8_t *__restrict__ tq) {
    const int Kp = (K + kTmaBoxK - 1) / kTmaBoxK * kTmaBoxK;
    const int nblk = K / 32, nblkp = Kp / 32, nmt = (R + 127) / 128, Rp = nmt * 128;
    const long long total = (long long)E * Rp * nblkp;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= total) return;
    const int kb = (int)(tid % nblkp);
    const long long er = tid / nblkp;
    const int r = (int)(er % Rp), e = (int)(er / Rp);
    int grow = r;
    if (pair_rows) {
        const int t = r / 16, j = r % 16;
        grow = j < 8 ? 2 * (8 * t + j) : 2 * (8 * t + j - 8) + 1;
    }
    uint4 q = make_uint4(0, 0, 0, 0);
    uint8_t scale = 127;
    if (kb < nblk && r < R) {
        const uint8_t *src = gguf + (((size_t)e * R + grow) * nblk + kb) * 17;
        scale = src[0];
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            w[i] = src[1 + 4 * i] | (src[2 + 4 * i] << 8) | (src[3 + 4 * i] << 16) | ((uint32_t)src[4 + 4 * i] << 24);
        q = make_uint4(w[0], w[1], w[2], w[3]);
    }
    const int mt = r / 128, rr = r % 128, kc = kb / 4, j = kb % 4;
    const size_t box = ((size_t)e * nmt + mt) * (Kp / kTmaBoxK) + kc;
    // 16-byte chunk j of row rr sits at chunk j ^ ((rr / 2) % 4): the 64-byte swizzle the
    // tensor core and the decode kernel read, applied here so that a box (rows, then
    // its scale chunk) moves as one plain copy
    uint8_t *bx = tq + box * kBoxStride;
    *reinterpret_cast<uint4 *>(bx + (size_t)rr * 64 + (size_t)((j ^ ((rr >> 1) & 3)) * 16)) = q;
    bx[kBoxData + (rr % 32) * 16 + (rr / 32) * 4 + j] = scale;
}

}  // namespace

cudaError_t launch_repack_tma(const uint8_t *gguf, int E, int R, int K, bool pair_rows, uint8_t *tq, cudaStream_t st) {
    const long long total = (long long)E * ((R + 127) / 128) * 128 * (kpad128(K) / 32);
    const int threads = 256;
    repack_tma_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(gguf, E, R, K,
                                                                                       pair_rows ? 1 : 0, tq);
    return cudaGetLastError();
}

cudaError_t launch_combine(const Dims &d, const float *residual, const RouteOut &r,
                           const float *y, int T, float *out, cudaStream_t st) {
    combine_kernel<<<T, 256, 0, st>>>(residual, y, r.inv, r.topk_w, d.H, d.k, out);
    return cudaGetLastError();
}

cudaError_t launch_repack(const uint8_t *gguf, int E, int R, int K, bool pair_rows, uint8_t *q,
                          uint8_t *s, cudaStream_t st) {
    const long long total = (long long)E * (R / kTileRows) * (K / kTileK) * 32;
    const int threads = 256;
    const long long blocks = (total + threads - 1) / threads;
    repack_kernel<<<(unsigned)blocks, threads, 0, st>>>(gguf, E, R, K, pair_rows ? 1 : 0, q, s);
    return cudaGetLastError();
}

}  // namespace amoe
