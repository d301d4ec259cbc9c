// fp4_terms.cuh -- activations as a sum of block-scaled E2M1 (FP4) terms, the
// B operand of the kind::mxf4 expert GEMMs (gemm_bs.cu).
//
// Per block of 32 elements, term j rounds the remainder r_j left by the
// previous terms (r_0 = x, f32) onto the E2M1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}
// at the smallest power-of-two scale 2^e with max|r_j| <= 6 * 2^e (E8M0 byte
// e + 127; 127 for an all-zero remainder; e >= -127), round to nearest with
// ties to the even code, and r_{j+1} = r_j - q_j 2^e, which is exact in f32.
// A value that rounds to zero gets code 0 whatever its sign (the hardware
// conversion keeps the sign of zero; it is cleared).  Five terms carry the
// activation to about 2^-12 of its block maximum, inside the parity tolerance
// against the float64 reference.  These are exactly the bytes the CPU
// definition produces (oracle_e2m1_terms, tested byte for byte).
//
// A block whose remainder holds a NaN or an infinity gets the E8M0 NaN scale
// (0xFF) on its first term, so the products of that block are NaN and the
// reference's NaN propagation (tensor.go:152-155) carries through the GEMM.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace amoe {
namespace fp4 {

constexpr int kTerms = 5;

// Smallest e with amax <= 6 * 2^e, clamped to [-127, 126]; 0 for amax == 0.
// amax = 1.f * 2^(E-127): 6 * 2^e = 1.5 * 2^(e+2), so e = E - 129 when the
// mantissa 1.f <= 1.5 and E - 128 above.  Subnormal amax gives -127.
__device__ __forceinline__ int scale_exp(float amax) {
    const uint32_t b = __float_as_uint(amax);
    const int E = (int)((b >> 23) & 0xffu);
    if ((b & 0x7fffffffu) == 0u) return 0;
    if (E == 0) return -127;
    const int e = E - 129 + ((b & 0x7fffffu) > 0x400000u ? 1 : 0);
    return e < -127 ? -127 : e;
}

// 2^e as f32 for e in [-127, 127] (2^-127 is subnormal).
__device__ __forceinline__ float pow2(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// Two values -> one byte of E2M1 codes (lo in the low nibble), round to
// nearest even, saturated at +-6.
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
    uint32_t r;
    asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n cvt.u32.u8 %0, t;\n}"
        : "=r"(r)
        : "f"(hi), "f"(lo));
    return r;
}

// One byte of E2M1 codes -> the two values (low nibble first).
__device__ __forceinline__ float2 e2m1x2_value(uint32_t byte) {
    uint32_t h;
    asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(h) : "r"(byte));
    return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

// Clears the sign of every zero code (0x8 -> 0x0) in a word of eight codes.
__device__ __forceinline__ uint32_t clear_negative_zero(uint32_t w) {
    const uint32_t zero = ((~w & 0x77777777u) + 0x11111111u) & 0x88888888u;
    return w & ~zero;
}

// The terms of one block of 32 elements held as N elements by each of L
// consecutive lanes (N * L == 32; lanes xor-reducible, all 32 lanes of the warp
// call it).  codes[j][w]: term j, elements 8w..8w+7 of this lane's part (low
// nibble first; with N < 8 the word holds the lane's N codes); sbyte[j]: term j's
// E8M0 byte.  r is consumed (left holding the final remainder).  The terms form one
// dependent chain, so fewer elements per lane (more lanes per block) shorten it.
template <int N, int L>
__device__ __forceinline__ void quantize(float (&r)[N], uint32_t (&codes)[kTerms][(N + 7) / 8],
                                         uint32_t (&sbyte)[kTerms]) {
    static_assert(N * L == 32 && N % 2 == 0 && (N & (N - 1)) == 0, "a block is 32 elements, two codes a byte");
    constexpr int kWords = (N + 7) / 8, kPairs = N < 8 ? N / 2 : 4;  // code words, byte pairs per word
    bool bad = false;
#pragma unroll
    for (int i = 0; i < N; ++i) bad |= !isfinite(r[i]);
#pragma unroll
    for (int o = 1; o < L; o <<= 1) bad |= __shfl_xor_sync(0xffffffffu, (int)bad, o) != 0;
#pragma unroll
    for (int j = 0; j < kTerms; ++j) {
        float m[N];
#pragma unroll
        for (int i = 0; i < N; ++i) m[i] = fabsf(r[i]);
#pragma unroll
        for (int w = N / 2; w >= 1; w >>= 1)  // tree: log2(N) dependent steps
#pragma unroll
            for (int i = 0; i < w; ++i) m[i] = fmaxf(m[i], m[i + w]);
        float amax = m[0];
#pragma unroll
        for (int o = 1; o < L; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int e = bad ? 0 : scale_exp(amax);
        sbyte[j] = (bad && j == 0) ? 0xffu : (uint32_t)(e + 127);
        const float inv = pow2(-e), s = pow2(e);
#pragma unroll
        for (int w = 0; w < kWords; ++w) {
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < kPairs; ++b) {
                float &x0 = r[8 * w + 2 * b], &x1 = r[8 * w + 2 * b + 1];
                const uint32_t byte = bad ? 0u : e2m1x2(x0 * inv, x1 * inv);
                const float2 q = e2m1x2_value(byte);
                x0 = fmaf(-q.x, s, x0);  // q * 2^e is exact, so this is the exact remainder
                x1 = fmaf(-q.y, s, x1);
                word |= byte << (8 * b);
            }
            codes[j][w] = clear_negative_zero(word);
        }
    }
}

}  // namespace fp4
}  // namespace amoe
