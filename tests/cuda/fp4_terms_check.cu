// Runs the device quantizer of airllm_b200/csrc/fp4_terms.cuh (5 block-scaled
// E2M1 terms) over a file of float32 values with L = 1, 2, 4 and 16 lanes per
// 32-element block (the layouts the kernels use), and writes the codes
// [terms][n/2] and scale bytes [terms][n/32] of each mode in the layout of
// oracle_e2m1_terms.  Usage: fp4_terms_check in.f32 out_l1 out_l2 out_l4 out_l16
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "fp4_terms.cuh"

using namespace amoe;

template <int L>
__global__ void run(const float *x, long long nb, uint8_t *codes, uint8_t *scales) {
    constexpr int N = 32 / L;
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long blk = gid / L;
    const int part = (int)(gid % L);
    const bool live = blk < nb;  // every lane of the warp runs quantize (shuffles)
    float r[N];
    for (int i = 0; i < N; ++i) r[i] = live ? x[blk * 32 + part * N + i] : 0.0f;
    uint32_t c[fp4::kTerms][(N + 7) / 8], s[fp4::kTerms];
    fp4::quantize<N, L>(r, c, s);
    if (!live) return;
    const long long n = nb * 32;
    for (int j = 0; j < fp4::kTerms; ++j) {
        uint8_t *dst = codes + j * (n / 2) + blk * 16 + part * (N / 2);
        for (int b = 0; b < N / 2; ++b) dst[b] = (uint8_t)(c[j][b / 4] >> (8 * (b % 4)));
        if (part == 0) scales[j * nb + blk] = (uint8_t)s[j];
    }
}

#define CK(x)                                                                              \
    do {                                                                                   \
        cudaError_t e = (x);                                                               \
        if (e != cudaSuccess) {                                                            \
            printf("CUDA %s: %s\n", #x, cudaGetErrorString(e));                             \
            return 1;                                                                      \
        }                                                                                  \
    } while (0)

int main(int argc, char **argv) {
    if (argc != 6) {
        printf("usage: fp4_terms_check in.f32 out_l1 out_l2 out_l4 out_l16\n");
        return 1;
    }
    FILE *f = fopen(argv[1], "rb");
    if (!f) return 1;
    fseek(f, 0, SEEK_END);
    const long long n = ftell(f) / 4;
    fseek(f, 0, SEEK_SET);
    if (n <= 0 || n % 32) return 1;
    std::vector<float> x(n);
    if (fread(x.data(), 4, n, f) != (size_t)n) return 1;
    fclose(f);
    const long long nb = n / 32, cbytes = fp4::kTerms * (n / 2), sbytes = fp4::kTerms * nb;
    float *dx;
    uint8_t *dc, *ds;
    CK(cudaMalloc(&dx, n * 4));
    CK(cudaMalloc(&dc, cbytes));
    CK(cudaMalloc(&ds, sbytes));
    CK(cudaMemcpy(dx, x.data(), n * 4, cudaMemcpyHostToDevice));
    std::vector<uint8_t> out(cbytes + sbytes);
    const int lanes[4] = {1, 2, 4, 16};
    for (int mode = 1; mode <= 4; ++mode) {
        CK(cudaMemset(dc, 0xAA, cbytes));
        CK(cudaMemset(ds, 0xAA, sbytes));
        const int L = lanes[mode - 1];
        const long long threads = nb * L;
        const int grid = (int)((threads + 127) / 128);
        if (L == 1) run<1><<<grid, 128>>>(dx, nb, dc, ds);
        else if (L == 2) run<2><<<grid, 128>>>(dx, nb, dc, ds);
        else if (L == 4) run<4><<<grid, 128>>>(dx, nb, dc, ds);
        else run<16><<<grid, 128>>>(dx, nb, dc, ds);
        CK(cudaGetLastError());
        CK(cudaDeviceSynchronize());
        CK(cudaMemcpy(out.data(), dc, cbytes, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(out.data() + cbytes, ds, sbytes, cudaMemcpyDeviceToHost));
        FILE *o = fopen(argv[1 + mode], "wb");
        if (!o) return 1;
        fwrite(out.data(), 1, out.size(), o);
        fclose(o);
    }
    printf("ok %lld blocks\n", nb);
    return 0;
}
