// Shared device helpers for the Shieldstral scoring kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ops.h"

namespace shield {

__host__ __device__ constexpr int block_bytes(int type) {
    return type == T_Q4_0 ? 18 : type == T_Q4_1 ? 20 : type == T_Q5_0 ? 22 : type == T_Q5_1 ? 24 : type == T_Q8_0 ? 34 : 0;
}
// What the unsigned payload sits above the signed weight (IntegerGemm.cs:75-81).
__host__ __device__ constexpr int zero_point(int type) {
    return type == T_Q4_0 ? 8 : type == T_Q5_0 ? 16 : type == T_Q8_0 ? 128 : 0;
}
__host__ __device__ constexpr bool has_offset(int type) { return type == T_Q4_1 || type == T_Q5_1; }

// Exact f16 bit pattern -> f32 (hardware conversion is exact for every pattern).
__device__ __forceinline__ float h2f(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Byte offsets of a block's fields: payload (qs or the 32 Q8 bytes), qh, offset.
__host__ __device__ constexpr int qs_offset(int type) {
    return type == T_Q4_0 ? 2 : type == T_Q4_1 ? 4 : type == T_Q5_0 ? 6 : type == T_Q5_1 ? 8 : 2;
}
__host__ __device__ constexpr int qh_offset(int type) { return type == T_Q5_0 ? 2 : 4; }

// Weight j (0..31) of a block as its signed value w = u - z (or u for the
// offset types), IntegerGemm.cs:258-329 / Dequantizer.cs:127-213.
template <int TYPE>
__device__ __forceinline__ int weight_at(const uint8_t *blk, int j) {
    if (TYPE == T_Q8_0) return (int)(int8_t)blk[2 + j];
    const uint8_t *qs = blk + qs_offset(TYPE);
    int u = j < 16 ? (qs[j] & 0x0F) : (qs[j - 16] >> 4);
    if (TYPE == T_Q5_0 || TYPE == T_Q5_1) u |= (int)((ld_u32_unaligned(blk + qh_offset(TYPE)) >> j) & 1u) << 4;
    return u - zero_point(TYPE);
}

// exp(x) evaluated exactly as the CPU oracle does: Cody-Waite reduction
// x = k·ln2 + r (ln2 as a 16-bit head, so k·head is exact, plus a tail), the
// degree-7 Taylor polynomial of e^r by Horner's rule with fused
// multiply-adds, then scaling by 2^k. Every step is one IEEE operation, so the
// bits match the host's. k > 127 gives +inf, k < -126 gives 0.
__device__ __forceinline__ float shield_expf(float x) {
    if (x != x) return x;
    float k = rintf(__fmul_rn(x, __uint_as_float(0x3FB8AA3Bu)));
    if (k > 127.0f) return __int_as_float(0x7F800000);
    if (k < -126.0f) return 0.0f;
    float r = __fmaf_rn(k, -__uint_as_float(0x3F317200u), x);
    r = __fmaf_rn(k, -__uint_as_float(0x35BFBE8Eu), r);
    float p = __uint_as_float(0x39500D01u);
    p = __fmaf_rn(p, r, __uint_as_float(0x3AB60B61u));
    p = __fmaf_rn(p, r, __uint_as_float(0x3C088889u));
    p = __fmaf_rn(p, r, __uint_as_float(0x3D2AAAABu));
    p = __fmaf_rn(p, r, __uint_as_float(0x3E2AAAABu));
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __uint_as_float((uint32_t)((int)k + 127) << 23));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Vector<float>.Sum of 8 lanes in the order the oracle states:
// ((e0+e4)+(e1+e5)) + ((e2+e6)+(e3+e7)).
// Two independent IEEE f32 operations per instruction (sm_100 packed f32x2):
// each lane rounds exactly as the scalar __fmul_rn / __fmaf_rn would.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ uint64_t pack2u(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ float lo_f(uint64_t p) { return __uint_as_float((uint32_t)p); }
__device__ __forceinline__ float hi_f(uint64_t p) { return __uint_as_float((uint32_t)(p >> 32)); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ float vsum8(const float e[8]) {
    float s0 = __fadd_rn(e[0], e[4]), s1 = __fadd_rn(e[1], e[5]);
    float s2 = __fadd_rn(e[2], e[6]), s3 = __fadd_rn(e[3], e[7]);
    return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// Quantizes one 32-value block held one value per lane (IntegerGemm.cs:97-138):
// d = max|x|/127, inverse = 1/d (0 for an all-zero block), q = rne(x*inverse).
// Returns q; d and the block sum come back in every lane.
__device__ __forceinline__ int quantize_lane(float x, float &d, int &sum) {
    float m = warp_max(fabsf(x));
    d = __fdiv_rn(m, 127.0f);
    float inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = __float2int_rn(__fmul_rn(x, inv));
    sum = warp_sum_i(q);
    return q;
}

}  // namespace shield
