// Activation quantization, fused RMSNorm + quantization, embedding gather,
// and the one-time derived scale planes of an uploaded weight.
#include "common.cuh"
#include "ops.h"

namespace shield {

// One warp per 32-block: lane j owns element j (IntegerGemm.cs:97-138).
__global__ void k_quantize(const float *__restrict__ x, int64_t M, int64_t K, int64_t ldx, QAct q) {
    int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    int64_t nb = K / 32;
    if (warp >= M * nb) return;
    int64_t t = warp / nb, b = warp % nb;
    float v = x[t * ldx + b * 32 + lane];
    float d;
    int sum;
    int qv = quantize_lane(v, d, sum);
    int64_t o = t * K + b * 32 + lane;
    if (q.a8) q.a8[o] = (int8_t)qv;
    if (q.a16) q.a16[o] = __int2half_rn(qv);
    if (lane == 0) {
        int64_t so = t * nb + b;
        q.da[so] = d;
        if (q.ds) q.ds[so] = __fmul_rn(d, (float)sum);
        if (q.sums) q.sums[so] = sum;
    }
}

// IntegerGemm.Quantize (IntegerGemm.cs:97-138) of block b of row t, the 32
// values in registers: scale, int8 and f16 integers (16-byte stores), d·Σq, Σq.
__device__ __forceinline__ void store_quantized_block(const float (&v)[32], int64_t t, int64_t b, int64_t K,
                                                      const QAct &q) {
    const int64_t nb = K / 32;
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) m = fmaxf(m, fabsf(v[i]));
    const float d = __fdiv_rn(m, 127.0f);
    const float inv = d != 0.0f ? __frcp_rn(d) : 0.0f;
    int qv[32], sum = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        qv[i] = __float2int_rn(__fmul_rn(v[i], inv));
        sum += qv[i];
    }
    const int64_t o = t * K + b * 32;
    if (q.a8) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            w[i] = (uint32_t)(qv[4 * i] & 0xFF) | ((uint32_t)(qv[4 * i + 1] & 0xFF) << 8) |
                   ((uint32_t)(qv[4 * i + 2] & 0xFF) << 16) | ((uint32_t)(qv[4 * i + 3] & 0xFF) << 24);
        uint4 *dst = reinterpret_cast<uint4 *>(q.a8 + o);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
    if (q.a16) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const __half2 h = __halves2half2(__int2half_rn(qv[2 * i]), __int2half_rn(qv[2 * i + 1]));
            w[i] = *reinterpret_cast<const uint32_t *>(&h);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(q.a16 + o);
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
    const int64_t so = t * nb + b;
    q.da[so] = d;
    if (q.ds) q.ds[so] = __fmul_rn(d, (float)sum);
    if (q.sums) q.sums[so] = sum;
}

// Four lanes per 32-block (lane sub of a quad owns elements 8sub..8sub+7):
// the same operations as k_quantize (max |x|, d = max/127, inv = 1/d or 0,
// q = rne(x*inv), sum q; the maximum and the integer sum are exact in any
// order, folded over the quad by shuffles). A warp reads 8 whole blocks, 1 KB
// contiguous, and stores 8 int8 and 8 f16 integers per lane. With u, the
// values are first SwiGLU(g = x, u) as Kernels.SwiGlu (Kernels.cs:83-90)
// computes it: u = g*u, then sigmoid(g)*u with sigmoid = 1/(1 + exp(-g)); the
// f32 product never reaches memory.
__global__ void __launch_bounds__(256) k_quantize_quads(const float *__restrict__ x, const float *__restrict__ u,
                                                        int64_t M, int64_t K, int64_t ldx, QAct q) {
    const int64_t nb = K / 32;
    const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 2;
    const int sub = threadIdx.x & 3;
    const bool live = blk < M * nb;  // the same for the 4 lanes of a quad
    const int64_t t = live ? blk / nb : 0, b = live ? blk % nb : 0;
    float v[8];
    if (live) {
        const float4 *src = reinterpret_cast<const float4 *>(x + t * ldx + b * 32 + 8 * sub);
        const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
        v[0] = f0.x, v[1] = f0.y, v[2] = f0.z, v[3] = f0.w, v[4] = f1.x, v[5] = f1.y, v[6] = f1.z, v[7] = f1.w;
        if (u) {
            const float4 *us = reinterpret_cast<const float4 *>(u + t * ldx + b * 32 + 8 * sub);
            const float4 u0 = __ldg(us), u1 = __ldg(us + 1);
            const float uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float gv = v[e];
                const float uv = __fmul_rn(gv, uu[e]);
                const float sg = __frcp_rn(__fadd_rn(1.0f, shield_expf(-gv)));  // == 1/(1+e), correctly rounded
                v[e] = __fmul_rn(sg, uv);
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = 0.0f;
    }
    float m = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) m = fmaxf(m, fabsf(v[e]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float d = __fdiv_rn(m, 127.0f);
    const float inv = d != 0.0f ? __frcp_rn(d) : 0.0f;
    int qv[8], sum = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        qv[e] = __float2int_rn(__fmul_rn(v[e], inv));
        sum += qv[e];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (!live) return;
    const int64_t o = t * K + b * 32 + 8 * sub;
    if (q.a8) {
        uint32_t w[2];
#pragma unroll
        for (int i = 0; i < 2; i++)
            w[i] = (uint32_t)(qv[4 * i] & 0xFF) | ((uint32_t)(qv[4 * i + 1] & 0xFF) << 8) |
                   ((uint32_t)(qv[4 * i + 2] & 0xFF) << 16) | ((uint32_t)(qv[4 * i + 3] & 0xFF) << 24);
        *reinterpret_cast<uint2 *>(q.a8 + o) = make_uint2(w[0], w[1]);
    }
    if (q.a16) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const __half2 h = __halves2half2(__int2half_rn(qv[2 * i]), __int2half_rn(qv[2 * i + 1]));
            w[i] = *reinterpret_cast<const uint32_t *>(&h);
        }
        *reinterpret_cast<uint4 *>(q.a16 + o) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (sub == 0) {
        const int64_t so = t * nb + b;
        q.da[so] = d;
        if (q.ds) q.ds[so] = __fmul_rn(d, (float)sum);
        if (q.sums) q.sums[so] = sum;
    }
}

static bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

cudaError_t launch_quantize(const float *x, int64_t M, int64_t K, int64_t ldx, const QAct &q, cudaStream_t s) {
    const int64_t nblk = M * (K / 32);
    if (nblk == 0) return cudaSuccess;
    const int threads = 256;
    if (aligned16(x) && ldx % 4 == 0 && aligned16(q.a8) && aligned16(q.a16)) {
        k_quantize_quads<<<(unsigned)((4 * nblk + threads - 1) / threads), threads, 0, s>>>(x, nullptr, M, K, ldx, q);
    } else {
        const int64_t blocks = (nblk * 32 + threads - 1) / threads;
        k_quantize<<<(unsigned)blocks, threads, 0, s>>>(x, M, K, ldx, q);
    }
    return cudaGetLastError();
}

cudaError_t launch_swiglu_quantize(const float *g, const float *u, int64_t M, int64_t K, const QAct &q,
                                   cudaStream_t s) {
    const int64_t nblk = M * (K / 32);
    if (nblk == 0) return cudaSuccess;
    if (!aligned16(g) || !aligned16(u) || K % 32 || !aligned16(q.a8) || !aligned16(q.a16)) return cudaErrorInvalidValue;
    const int threads = 256;
    k_quantize_quads<<<(unsigned)((4 * nblk + threads - 1) / threads), threads, 0, s>>>(g, u, M, K, K, q);
    return cudaGetLastError();
}

// Kernels.RmsNorm (Kernels.cs:26-61) in the oracle's operation order:
// 16 lanes (two 8-wide vectors) of x*x then +, each a sequential chain over
// the row; Vector.Sum of each vector; the sum widened to double; the tail in
// double; scale = 1/sqrt((float)(sum/n) + eps); y = (x*scale)*w. Then every
// 32-block of y is quantized like k_quantize. One CTA of 128 threads per row.
__global__ void k_rmsnorm_quant(const float *__restrict__ x, const int32_t *__restrict__ row_idx, int K,
                                const float *__restrict__ w, float eps, float *__restrict__ y, QAct q) {
    int64_t t = blockIdx.x;
    int64_t src = row_idx ? row_idx[t] : t;
    const float *xr = x + src * (int64_t)K;
    __shared__ float partial[16];
    __shared__ float s_scale;
    int tid = threadIdx.x;
    int vec_end = K >= 16 ? (K / 16) * 16 : 0;
    if (tid < 16) {
        float acc = 0.0f;
        for (int i = tid; i < vec_end; i += 16) acc = __fadd_rn(acc, __fmul_rn(xr[i], xr[i]));
        partial[tid] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        double sum = 0.0;
        if (vec_end > 0) sum = __dadd_rn((double)vsum8(partial), (double)vsum8(partial + 8));
        for (int i = vec_end; i < K; i++) sum = __dadd_rn(sum, __dmul_rn((double)xr[i], (double)xr[i]));
        float ms = __double2float_rn(__ddiv_rn(sum, (double)K));
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    }
    __syncthreads();
    float scale = s_scale;
    int lane = tid & 31, wid = tid >> 5;
    int nb = K / 32;
    for (int b = wid; b < nb; b += blockDim.x / 32) {
        int i = b * 32 + lane;
        float v = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
        if (y) y[t * K + i] = v;
        float d;
        int sum;
        int qv = quantize_lane(v, d, sum);
        int64_t o = t * K + i;
        if (q.a8) q.a8[o] = (int8_t)qv;
        if (q.a16) q.a16[o] = __int2half_rn(qv);
        if (lane == 0) {
            int64_t so = t * nb + b;
            q.da[so] = d;
            if (q.ds) q.ds[so] = __fmul_rn(d, (float)sum);
            if (q.sums) q.sums[so] = sum;
        }
    }
}

// The same RMSNorm + quantization with two rows per warp: lanes 0-15 and
// 16-31 each run one row's 16 partial chains (coalesced 64-byte reads), fold
// them in Vector.Sum order with shuffles, then each lane normalizes and
// quantizes whole 32-blocks (blocks lane%16, +16, ...) from registers.
// Needs K % 32 == 0 and 16-byte aligned rows.
__global__ void __launch_bounds__(256) k_rmsnorm_quant_rows(const float *__restrict__ x,
                                                            const int32_t *__restrict__ row_idx, int64_t M, int K,
                                                            const float *__restrict__ w, float eps,
                                                            float *__restrict__ y, QAct q) {
    const int lane = threadIdx.x & 31, c = lane & 15;
    const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;  // row of this half-warp
    const bool live = t < M;
    const int64_t src = live ? (row_idx ? row_idx[t] : t) : 0;
    const float *xr = x + src * (int64_t)K;
    const int vec_end = K >= 16 ? (K / 16) * 16 : 0;
    float acc = 0.0f;
    if (live)
        for (int i = c; i < vec_end; i += 16) acc = __fadd_rn(acc, __fmul_rn(xr[i], xr[i]));
    // Vector.Sum of partials 0-7 (in lane 0 of the half) and 8-15 (in lane 8):
    // ((e0+e4)+(e1+e5)) + ((e2+e6)+(e3+e7))
    float v = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2));
    const float hi = __shfl_down_sync(0xffffffffu, v, 8);
    float scale = 0.0f;
    if (c == 0 && live) {
        double sum = 0.0;
        if (vec_end > 0) sum = __dadd_rn((double)v, (double)hi);
        for (int i = vec_end; i < K; i++) sum = __dadd_rn(sum, __dmul_rn((double)xr[i], (double)xr[i]));
        const float ms = __double2float_rn(__ddiv_rn(sum, (double)K));
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    }
    scale = __shfl_sync(0xffffffffu, scale, lane & 16);
    if (!live) return;
    const int nb = K / 32;
    for (int b = c; b < nb; b += 16) {
        float vals[32];
        const float4 *xs = reinterpret_cast<const float4 *>(xr + b * 32);
        const float4 *ws = reinterpret_cast<const float4 *>(w + b * 32);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 xv = __ldg(xs + i), wv = __ldg(ws + i);
            vals[4 * i + 0] = __fmul_rn(__fmul_rn(xv.x, scale), wv.x);
            vals[4 * i + 1] = __fmul_rn(__fmul_rn(xv.y, scale), wv.y);
            vals[4 * i + 2] = __fmul_rn(__fmul_rn(xv.z, scale), wv.z);
            vals[4 * i + 3] = __fmul_rn(__fmul_rn(xv.w, scale), wv.w);
        }
        if (y) {
            float4 *ys = reinterpret_cast<float4 *>(y + t * (int64_t)K + b * 32);
#pragma unroll
            for (int i = 0; i < 8; i++) ys[i] = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
        }
        store_quantized_block(vals, t, b, K, q);
    }
}

// The same RMSNorm + quantization for few rows (a single short request, the
// final norm of the last positions), where 16 lanes per row leave most SMs
// idle and each lane's strided walk waits on one load per step. One CTA of
// 128 threads per row: the row is staged in shared memory with every load in
// flight; lanes 0-15 of warp 0 (16-31 as copies) run the 16 chains from
// shared memory in the same order, eight squares formed ahead of their adds;
// then every thread normalizes and quantizes whole 32-blocks (block tid,
// tid + 128, ..).
constexpr int RMS_CTA_THREADS = 128;

__global__ void __launch_bounds__(RMS_CTA_THREADS) k_rmsnorm_quant_cta(const float *__restrict__ x,
                                                                       const int32_t *__restrict__ row_idx, int K,
                                                                       const float *__restrict__ w, float eps,
                                                                       float *__restrict__ y, QAct q) {
    extern __shared__ float4 s_row4[];
    __shared__ float s_scale;
    const int tid = threadIdx.x, lane = tid & 31, c = lane & 15;
    const int64_t t = blockIdx.x;
    const int64_t src = row_idx ? row_idx[t] : t;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + src * (int64_t)K);
    const int n4 = K / 4;
    {
        int i = tid;
        for (; i + 5 * RMS_CTA_THREADS < n4; i += 6 * RMS_CTA_THREADS) {
            float4 v[6];
#pragma unroll
            for (int u = 0; u < 6; u++) v[u] = __ldg(x4 + i + RMS_CTA_THREADS * u);
#pragma unroll
            for (int u = 0; u < 6; u++) s_row4[i + RMS_CTA_THREADS * u] = v[u];
        }
        for (; i < n4; i += RMS_CTA_THREADS) s_row4[i] = __ldg(x4 + i);
    }
    __syncthreads();
    const float *row = reinterpret_cast<const float *>(s_row4);
    if (tid < 32) {
        float acc = 0.0f;
        int i = c;
        for (; i + 7 * 16 < K; i += 8 * 16) {
            float sq[8];
#pragma unroll
            for (int u = 0; u < 8; u++) sq[u] = __fmul_rn(row[i + 16 * u], row[i + 16 * u]);
#pragma unroll
            for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, sq[u]);
        }
        for (; i < K; i += 16) acc = __fadd_rn(acc, __fmul_rn(row[i], row[i]));
        // Vector.Sum of partials 0-7 and 8-15, then the two halves in double
        float v = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
        v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1));
        v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2));
        const float hi = __shfl_down_sync(0xffffffffu, v, 8);
        if (lane == 0) {
            const double sum = __dadd_rn((double)v, (double)hi);
            const float ms = __double2float_rn(__ddiv_rn(sum, (double)K));
            s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
        }
    }
    __syncthreads();
    const float scale = s_scale;
    const int nb = K / 32;
    for (int b = tid; b < nb; b += RMS_CTA_THREADS) {
        float vals[32];
        const float4 *xs = s_row4 + b * 8;
        const float4 *ws = reinterpret_cast<const float4 *>(w + b * 32);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 xv = xs[i], wv = __ldg(ws + i);
            vals[4 * i + 0] = __fmul_rn(__fmul_rn(xv.x, scale), wv.x);
            vals[4 * i + 1] = __fmul_rn(__fmul_rn(xv.y, scale), wv.y);
            vals[4 * i + 2] = __fmul_rn(__fmul_rn(xv.z, scale), wv.z);
            vals[4 * i + 3] = __fmul_rn(__fmul_rn(xv.w, scale), wv.w);
        }
        if (y) {
            float4 *ys = reinterpret_cast<float4 *>(y + t * (int64_t)K + b * 32);
#pragma unroll
            for (int i = 0; i < 8; i++) ys[i] = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
        }
        store_quantized_block(vals, t, b, K, q);
    }
}

cudaError_t launch_rmsnorm_quant(const float *x, const int32_t *row_idx, int64_t M, int K, const float *w,
                                 float eps, float *y, const QAct &q, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (K % 32 == 0 && aligned16(x) && aligned16(w) && aligned16(y) && aligned16(q.a8) && aligned16(q.a16)) {
        const int64_t threads = M * 16;
        const size_t smem = (size_t)K * 4;
        if ((threads + 255) / 256 < 2 * sm_count_of_device() && smem <= 200 * 1024 && M <= 0x7fffffff) {
            // fewer than two waves of the 16-lane kernel
            if (smem > 48 * 1024) {
                const cudaError_t e =
                    cudaFuncSetAttribute(k_rmsnorm_quant_cta, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                if (e != cudaSuccess) return e;
            }
            k_rmsnorm_quant_cta<<<(unsigned)M, RMS_CTA_THREADS, smem, s>>>(x, row_idx, K, w, eps, y, q);
        } else {
            k_rmsnorm_quant_rows<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, row_idx, M, K, w, eps, y, q);
        }
    } else {
        k_rmsnorm_quant<<<(unsigned)M, 128, 0, s>>>(x, row_idx, K, w, eps, y, q);
    }
    return cudaGetLastError();
}

// QuantMatMul.GatherRows + Dequantizer legacy decode (QuantMatMul.cs:534-545,
// Dequantizer.cs:127-213): one warp per (token, block), lane j -> element j.
template <int TYPE>
__global__ void k_embed(const uint8_t *__restrict__ table, int64_t rows, int64_t row_bytes, int64_t K,
                        const int32_t *__restrict__ ids, int64_t M, float *__restrict__ h, int32_t *err) {
    int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    int64_t nb = K / 32;
    if (warp >= M * nb) return;
    int64_t t = warp / nb, b = warp % nb;
    int id = ids[t];
    if (id < 0 || id >= rows) {
        if (lane == 0 && b == 0) atomicExch(err, 2);
        h[t * K + b * 32 + lane] = 0.0f;
        return;
    }
    const uint8_t *row = table + (int64_t)id * row_bytes;
    float v;
    if (TYPE == T_F32) {
        v = reinterpret_cast<const float *>(row)[b * 32 + lane];
    } else if (TYPE == T_F16) {
        v = h2f(ld_u16(row + (b * 32 + lane) * 2));
    } else {
        const uint8_t *blk = row + b * block_bytes(TYPE);
        float d = h2f(ld_u16(blk));
        int wv = weight_at<TYPE>(blk, lane);
        if (has_offset(TYPE))
            v = __fadd_rn(__fmul_rn(d, (float)wv), h2f(ld_u16(blk + 2)));
        else
            v = __fmul_rn(d, (float)wv);
    }
    h[t * K + b * 32 + lane] = v;
}

cudaError_t launch_embed(const DevWeight &emb, const int32_t *ids, int64_t M, float *h, int32_t *err,
                         cudaStream_t s) {
    int64_t warps = M * (emb.cols / 32);
    if (warps == 0) return cudaSuccess;
    int threads = 256;
    unsigned blocks = (unsigned)((warps * 32 + threads - 1) / threads);
#define EMB(T) k_embed<T><<<blocks, threads, 0, s>>>(emb.data, emb.rows, emb.row_bytes, emb.cols, ids, M, h, err)
    switch (emb.type) {
    case T_F32: EMB(T_F32); break;
    case T_F16: EMB(T_F16); break;
    case T_Q4_0: EMB(T_Q4_0); break;
    case T_Q4_1: EMB(T_Q4_1); break;
    case T_Q5_0: EMB(T_Q5_0); break;
    case T_Q5_1: EMB(T_Q5_1); break;
    case T_Q8_0: EMB(T_Q8_0); break;
    default: return cudaErrorInvalidValue;
    }
#undef EMB
    return cudaGetLastError();
}

// Scale (and offset) planes [K/32][rows] in f32, read once at upload.
__global__ void k_build_planes(const uint8_t *__restrict__ data, int64_t rows, int64_t row_bytes, int64_t nb,
                               int bb, int with_offset, float *__restrict__ scale, float *__restrict__ offset) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    int64_t b = i / rows, r = i % rows;
    const uint8_t *blk = data + r * row_bytes + b * bb;
    scale[i] = h2f(ld_u16(blk));
    if (with_offset) offset[i] = h2f(ld_u16(blk + 2));
}

cudaError_t launch_build_planes(const DevWeight &w, cudaStream_t s) {
    int bb = block_bytes(w.type);
    if (!bb || !w.scale_plane) return cudaSuccess;
    int64_t n = w.rows * (w.cols / 32);
    k_build_planes<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, bb,
                                                                has_offset(w.type) ? 1 : 0, w.scale_plane,
                                                                w.offset_plane);
    return cudaGetLastError();
}

// One thread per (row, block): the block's 32 weights as f16 integers w = u - z
// (Q4_1/Q5_1: u), exact in f16, in weight order.
template <int TYPE>
__global__ void k_unpack_f16(const uint8_t *__restrict__ data, int64_t rows, int64_t row_bytes, int64_t nb,
                             __half *__restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    int64_t r = i / nb, b = i % nb;
    const uint8_t *blk = data + r * row_bytes + b * block_bytes(TYPE);
    __half *dst = out + r * nb * 32 + b * 32;
#pragma unroll
    for (int j = 0; j < 32; j += 2)
        *reinterpret_cast<__half2 *>(dst + j) =
            __halves2half2(__int2half_rn(weight_at<TYPE>(blk, j)), __int2half_rn(weight_at<TYPE>(blk, j + 1)));
}

cudaError_t launch_unpack_f16(const DevWeight &w, cudaStream_t s) {
    int64_t n = w.rows * (w.cols / 32);
    if (!w.w16 || n == 0) return cudaSuccess;
    unsigned g = (unsigned)((n + 255) / 256);
    switch (w.type) {
    case T_Q4_0: k_unpack_f16<T_Q4_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, w.w16); break;
    case T_Q4_1: k_unpack_f16<T_Q4_1><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, w.w16); break;
    case T_Q5_0: k_unpack_f16<T_Q5_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, w.w16); break;
    case T_Q5_1: k_unpack_f16<T_Q5_1><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, w.w16); break;
    case T_Q8_0: k_unpack_f16<T_Q8_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols / 32, w.w16); break;
    default: return cudaErrorNotSupported;
    }
    return cudaGetLastError();
}

}  // namespace shield
