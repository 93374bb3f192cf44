// Elementwise and attention kernels of the Ministral forward
// (MinistralModel.cs:282-482): RoPE, causal GQA attention over a ragged batch
// of requests, SwiGLU.
#include "common.cuh"
#include "ops.h"

namespace shield {

// Rope.Apply (Rope.cs:112-135) on adjacent pairs, with cos/sin taken from the
// per-position table the host computed (cos(pos·freq)·mscale), and the
// attention temperature of MinistralModel.ApplyPositionScale (:476-482) as a
// per-position factor (nullptr = none). Products and sums are rounded
// separately, as the reference writes them.
__global__ void k_rope(float *__restrict__ x, int64_t M, int heads, int head_dim, int64_t ld,
                       const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                       const float *__restrict__ sin_t, int half, const float *__restrict__ temp) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t per_tok = (int64_t)heads * half;
    if (i >= M * per_tok) return;
    int64_t t = i / per_tok;
    int h = (int)((i % per_tok) / half), p = (int)(i % half);
    int ps = pos[t];
    float c = cos_t[(int64_t)ps * half + p], s = sin_t[(int64_t)ps * half + p];
    float *hd = x + t * ld + (int64_t)h * head_dim;
    float x0 = hd[2 * p], x1 = hd[2 * p + 1];
    float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    if (temp) {
        float f = temp[ps];
        y0 = __fmul_rn(y0, f);
        y1 = __fmul_rn(y1, f);
    }
    hd[2 * p] = y0;
    hd[2 * p + 1] = y1;
}

cudaError_t launch_rope(float *x, int64_t M, int heads, int head_dim, int64_t ld, const int32_t *pos,
                        const float *cos_t, const float *sin_t, int half, const float *temp, cudaStream_t s) {
    int64_t n = M * heads * half;
    if (n == 0) return cudaSuccess;
    k_rope<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, M, heads, head_dim, ld, pos, cos_t, sin_t, half, temp);
    return cudaGetLastError();
}

// Causal grouped-query attention (AttendGroup, MinistralModel.cs:372-440) for
// one query token and one KV head: warp g handles query head kvh*group + g.
// Scores follow Kernels.Dot4's order (8 lanes of fused multiply-adds, then
// Vector.Sum), the softmax sums 32 lane-strided partials folded by a butterfly
// and uses shield_expf (the oracle's order and exp), the context follows
// AddScaled4 (a fused multiply-add chain over positions in order), so the
// result is bit-identical to the oracle.
// q: M x (H*hd), k/v: M x (KVH*hd), tok_start[t] = index of t's request start.
__global__ void k_attention(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                            float *__restrict__ ctx, const int32_t *__restrict__ tok_start, int n_heads,
                            int n_kv_heads, int head_dim, float scale) {
    extern __shared__ float smem[];
    const int group = n_heads / n_kv_heads;
    const int64_t t = blockIdx.x;
    const int kvh = blockIdx.y;
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t start = tok_start[t];
    const int limit = (int)(t - start + 1);
    const int head = kvh * group + g;
    const int64_t qdim = (int64_t)n_heads * head_dim, kvdim = (int64_t)n_kv_heads * head_dim;
    float *qs = smem + g * head_dim;                        // this head's query
    float *sc = smem + group * head_dim + (int64_t)g * limit;  // this head's scores
    for (int d = lane; d < head_dim; d += 32) qs[d] = q[t * qdim + (int64_t)head * head_dim + d];
    __syncwarp();
    float mx = -INFINITY;
    for (int p = lane; p < limit; p += 32) {
        const float *kp = k + (start + p) * kvdim + (int64_t)kvh * head_dim;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i + 8 <= head_dim; i += 8) {
            float4 k0 = *reinterpret_cast<const float4 *>(kp + i);
            float4 k1 = *reinterpret_cast<const float4 *>(kp + i + 4);
            acc[0] = __fmaf_rn(qs[i + 0], k0.x, acc[0]);
            acc[1] = __fmaf_rn(qs[i + 1], k0.y, acc[1]);
            acc[2] = __fmaf_rn(qs[i + 2], k0.z, acc[2]);
            acc[3] = __fmaf_rn(qs[i + 3], k0.w, acc[3]);
            acc[4] = __fmaf_rn(qs[i + 4], k1.x, acc[4]);
            acc[5] = __fmaf_rn(qs[i + 5], k1.y, acc[5]);
            acc[6] = __fmaf_rn(qs[i + 6], k1.z, acc[6]);
            acc[7] = __fmaf_rn(qs[i + 7], k1.w, acc[7]);
        }
        float s = __fmul_rn(vsum8(acc), scale);
        sc[p] = s;
        mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int p = lane; p < limit; p += 32) {
        float e = shield_expf(__fsub_rn(sc[p], mx));
        sc[p] = e;
        sum = __fadd_rn(sum, e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    __syncwarp();
    for (int p = lane; p < limit; p += 32) sc[p] = __fdiv_rn(sc[p], sum);
    __syncwarp();
    for (int d = lane; d < head_dim; d += 32) {
        float c = 0.0f;
        const float *vp = v + start * kvdim + (int64_t)kvh * head_dim + d;
        for (int p = 0; p < limit; p++) {
            float w = sc[p];
            if (w != 0.0f) c = __fmaf_rn(vp[(int64_t)p * kvdim], w, c);
        }
        ctx[t * qdim + (int64_t)head * head_dim + d] = c;
    }
}

cudaError_t launch_attention(const float *q, const float *k, const float *v, float *ctx, const int32_t *tok_start,
                             int64_t M, int n_heads, int n_kv_heads, int head_dim, float scale, int max_len,
                             cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    int group = n_heads / n_kv_heads;
    size_t smem = (size_t)group * head_dim * 4 + (size_t)group * max_len * 4;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((unsigned)M, (unsigned)n_kv_heads);
    k_attention<<<grid, group * 32, smem, s>>>(q, k, v, ctx, tok_start, n_heads, n_kv_heads, head_dim, scale);
    return cudaGetLastError();
}

// Kernels.SwiGlu (Kernels.cs:83-90): u = g*u; g = sigmoid(g)*u, in place in g.
__global__ void k_swiglu(float *__restrict__ g, float *__restrict__ u, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float gv = g[i];
    float uv = __fmul_rn(gv, u[i]);
    float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, shield_expf(-gv)));
    g[i] = __fmul_rn(sg, uv);
}

cudaError_t launch_swiglu(float *g, float *u, int64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, u, n);
    return cudaGetLastError();
}

}  // namespace shield
