// Elementwise and attention kernels of the Ministral forward
// (MinistralModel.cs:282-482): RoPE, causal GQA attention over a ragged batch
// of requests, SwiGLU.
#include <algorithm>

#include "common.cuh"
#include "ops.h"

namespace shield {

namespace att {
constexpr int R = 128;       // query rows per CTA
constexpr int HD = 128;      // head_dim this kernel is written for
constexpr int KT = 32;       // keys per tile
constexpr int LD = HD + 4;   // padded row of a Q/K/V tile in shared memory
constexpr int THREADS = 256;  // threads of a 128-row CTA (2 per row)
constexpr int PKT = 32;      // keys per PV tile
constexpr int LDP = PKT + 4; // padded row of a PV weight tile
}  // namespace att


// Scratch row stride of a CTA whose rows attend to kend keys: a multiple of 4
// floats, so every row starts on a 16-byte boundary.
__device__ __forceinline__ int64_t att_ld(int64_t kend) { return (kend + 3) & ~int64_t(3); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Where dim d of a head is stored for the attention ("chain-major"): the
// score's 8 FMA chains (chain j: dims j, j+8, .., j+120) are taken in pairs
// (j, j+4), j < 4, and pair j's 32 floats are its two chains interleaved step
// by step: dims j, j+4, j+8, j+12, .., so one 64-bit load holds the operands of
// both chains at one step, for one packed f32x2 FMA.
__device__ __forceinline__ int chain_pos(int d) { return (d & 3) * 32 + (d >> 3) * 2 + ((d >> 2) & 1); }

// Rope.Apply (Rope.cs:112-135) on adjacent pairs, with cos/sin taken from the
// per-position table the host computed (cos(pos·freq)·mscale), and the
// attention temperature of MinistralModel.ApplyPositionScale (:476-482) as a
// per-position factor (nullptr = none). Products and sums are rounded
// separately, as the reference writes them. With perm, the rotated heads are
// also written in the attention's chain-major order (see chain_pos).
__global__ void k_rope(float *__restrict__ x, int64_t M, int heads, int head_dim, int64_t ld,
                       const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                       const float *__restrict__ sin_t, int half, const float *__restrict__ temp,
                       float *__restrict__ perm) {
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
    if (perm) {
        float *ph = perm + t * ld + (int64_t)h * head_dim;
        ph[chain_pos(2 * p)] = y0;
        ph[chain_pos(2 * p + 1)] = y1;
    }
}

// The same rotation for the attention's layout: one warp per (token, head)
// row of 128 dims, lane l taking dims 4l..4l+3 (pairs 2l, 2l+1; pairs from
// `half` on are not rotated, as in Rope.Apply). The rotated row goes to perm
// in chain-major order through a shared-memory transpose (16-byte stores),
// and back to x in place only when natural is set. One launch covers two
// tensors (the queries, then the keys): rows below rows0 belong to set 0.
struct RopeSet {
    float *x, *perm;
    const float *temp;  // attention temperature per position, or null
    int64_t ld;
    int heads;
    bool natural;
};

__global__ void __launch_bounds__(256) k_rope_rows(const RopeSet s0, const RopeSet s1, int64_t rows0, int64_t rows,
                                                   const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                                                   const float *__restrict__ sin_t, int half) {
    __shared__ float srow[8][att::HD];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = (int64_t)blockIdx.x * 8 + wid;
    if (row >= rows) return;  // whole warp
    const bool first = row < rows0;  // warp-uniform
    if (!first) row -= rows0;
    float *const x = first ? s0.x : s1.x;
    float *const perm = first ? s0.perm : s1.perm;
    const float *const temp = first ? s0.temp : s1.temp;
    const int64_t ld = first ? s0.ld : s1.ld;
    const int heads = first ? s0.heads : s1.heads;
    const bool natural = first ? s0.natural : s1.natural;
    const int64_t t = row / heads;
    const int h = (int)(row % heads);
    const int ps = pos[t];
    float *hd = x + t * ld + (int64_t)h * att::HD;
    float4 v = *reinterpret_cast<const float4 *>(hd + 4 * lane);
    float y[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int p = 2 * lane + k;
        if (p >= half) continue;
        const float c = cos_t[(int64_t)ps * half + p], sn = sin_t[(int64_t)ps * half + p];
        const float x0 = y[2 * k], x1 = y[2 * k + 1];
        float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        if (temp) {
            const float f = temp[ps];
            y0 = __fmul_rn(y0, f);
            y1 = __fmul_rn(y1, f);
        }
        y[2 * k] = y0;
        y[2 * k + 1] = y1;
    }
    if (natural) *reinterpret_cast<float4 *>(hd + 4 * lane) = make_float4(y[0], y[1], y[2], y[3]);
#pragma unroll
    for (int e = 0; e < 4; e++) srow[wid][chain_pos(4 * lane + e)] = y[e];
    __syncwarp();
    *reinterpret_cast<float4 *>(perm + t * ld + (int64_t)h * att::HD + 4 * lane) =
        *reinterpret_cast<const float4 *>(&srow[wid][4 * lane]);
}

static bool rope_rows_ok(const float *x, int head_dim, int64_t ld, const float *perm) {
    return head_dim == att::HD && ld % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(perm) % 16 == 0;
}

cudaError_t launch_rope(float *x, int64_t M, int heads, int head_dim, int64_t ld, const int32_t *pos,
                        const float *cos_t, const float *sin_t, int half, const float *temp, float *perm,
                        cudaStream_t s, bool natural) {
    if (M == 0) return cudaSuccess;
    if (perm) {
        if (!rope_rows_ok(x, head_dim, ld, perm)) return cudaErrorInvalidValue;
        const int64_t rows = M * heads;
        const RopeSet rs{x, perm, temp, ld, heads, natural};
        k_rope_rows<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(rs, rs, rows, rows, pos, cos_t, sin_t, half);
        return cudaGetLastError();
    }
    int64_t n = M * heads * half;
    if (n == 0) return cudaSuccess;
    k_rope<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, M, heads, head_dim, ld, pos, cos_t, sin_t, half, temp,
                                                        nullptr);
    return cudaGetLastError();
}

cudaError_t launch_rope_qk(float *q, int q_heads, float *k, int k_heads, int64_t M, int head_dim, const int32_t *pos,
                           const float *cos_t, const float *sin_t, int half, const float *q_temp, float *q_perm,
                           float *k_perm, bool q_natural, bool k_natural, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    const int64_t q_ld = (int64_t)q_heads * head_dim, k_ld = (int64_t)k_heads * head_dim;
    if (!rope_rows_ok(q, head_dim, q_ld, q_perm) || !rope_rows_ok(k, head_dim, k_ld, k_perm))
        return cudaErrorInvalidValue;
    const RopeSet qs{q, q_perm, q_temp, q_ld, q_heads, q_natural}, ks{k, k_perm, nullptr, k_ld, k_heads, k_natural};
    const int64_t rows0 = M * q_heads, rows = rows0 + M * k_heads;
    k_rope_rows<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(qs, ks, rows0, rows, pos, cos_t, sin_t, half);
    return cudaGetLastError();
}

// Causal grouped-query attention over a ragged batch (AttendGroup,
// MinistralModel.cs:372-440) in one kernel that keeps the oracle's exact
// operation order, so the context is bit-identical to it. One CTA owns 128
// query rows (64 for small batches, which then get twice the CTAs, each with
// as many threads as a 128-row one) of one request and one KV head: rows/G
// tokens x the G query heads
// sharing that KV head, so each key and value row is read once per CTA for all
// of them. A request's queries are its tokens in the batch; its keys are the
// first pre positions of its cache (the system-prompt cache of
// SystemPromptCache.cs:51-75, or the request's own sequence, as
// MinistralModel.ForwardAsync attends to KvCache, MinistralModel.cs:183-271)
// followed by its own tokens, so query token t sits at position pre + t.
//
//   phase 1  s = (Σ over 8 FMA chains, folded as Vector.Sum) * scale, chain j
//            = fma over dims j, j+8, .., j+120 in order (Kernels.Dot4); every
//            score goes to the CTA's scratch rows and its row maximum is kept
//   phase 2  per row: e = shield_expf(s - max) in place, summed as 32
//            lane-strided partials folded pairwise (Kernels.Softmax), then
//            w = e / sum in place
//   phase 3  ctx[d] = fma(v[p][d], w[p], ctx[d]) over p in order (AddScaled4)
//
// The scratch rows of a CTA (rows x round_up(kend, 4) floats) are written and
// read back within its lifetime, so short requests' scores never leave L2.
// Work items arrive longest first (host side), so the long CTAs of a ragged
// batch start early instead of forming a tail.

// Per-work-item view.
struct AttView {
    int len, pre, q0, qend, kend;  // queries, cached keys, this CTA's query range, keys it needs
    int64_t start, ld;             // first batch row, scratch row stride
    float *sc;                     // this CTA's 128 scratch rows
    const float *ck, *cv;          // this layer's cached keys and values (pre > 0)
};

// Thread layout of a CTA: RR query rows, TPR threads per row. TPR = 2 (RR/16
// warps): a phase-1 key tile is 32 keys, a phase-3 thread owns 4 rows.
// TPR = 4 (twice the warps for the same rows, for small batches where one
// CTA per SM is all there is): the phase-1 tile is 64 keys, warps w and
// w + RR/16 taking its two 32-key halves, and a phase-3 thread owns 2 rows.
template <int RR, int TPR>
struct AttShape {
    static constexpr int THREADS = TPR * RR;
    static constexpr int KH = TPR / 2;           // key halves of a phase-1 tile
    static constexpr int KTE = att::KT * KH;     // keys of a phase-1 tile
    static constexpr int NA = 8 * RR / THREADS;  // rows per phase-3 thread
    static constexpr int RSTEP = THREADS / 8;    // phase-3 row stride
    static_assert(TPR == 2 || TPR == 4, "2 or 4 threads per row");
};

template <int RR>
__device__ __forceinline__ AttView att_view(const AttArgs &A, int QT) {
    const int2 wk = A.work[blockIdx.x];
    AttView w;
    const int r = wk.x;
    w.q0 = wk.y;
    w.len = A.req_len[r];
    w.pre = A.req_pre ? A.req_pre[r] : 0;
    w.start = A.req_start[r];
    w.qend = min(w.q0 + QT, w.len);
    w.kend = w.pre + w.qend;
    w.ld = att_ld(w.kend);
    w.sc = A.scores + A.work_base[blockIdx.x] + (int64_t)blockIdx.y * RR * w.ld;
    w.ck = w.cv = nullptr;
    if (w.pre > 0) {
        const int64_t off = (int64_t)A.layer * A.cache_stride[r];
        w.ck = A.cache_k[r] + off;
        w.cv = A.cache_v[r] + off;
    }
    return w;
}

// Row p of a request's keys or values: cached row p, or its own token p - pre.
__device__ __forceinline__ const float *kv_row(const float *own, const float *cached, const AttView &w, int p,
                                               int64_t kvdim) {
    return p < w.pre ? cached + (int64_t)p * kvdim : own + (w.start + p - w.pre) * kvdim;
}

// Phase 1: the CTA's RR x kend scores into its scratch rows, and each row's
// maximum over each key half into rowmax[half][row] (shared). Keys and the
// CTA's query rows arrive in chain-major order (see chain_pos) by cp.async,
// key tiles double-buffered. Thread (warp = wr + (RR/16) kh, rl, kl) owns rows
// wr*16 + rl + 4a and keys 32 kh + kl + 8b of a tile.
template <int RR, int TPR>
__device__ __forceinline__ void attn_scores(const AttArgs &A, const AttView &w, float *sm, float *rowmax) {
    using namespace att;
    using S = AttShape<RR, TPR>;
    constexpr int R = RR, THREADS = S::THREADS, KTE = S::KTE;
    float *Qs = sm;  // R x LD, then two KTE x LD key tiles
    const int G = A.n_heads / A.n_kv_heads;
    const int h = blockIdx.y;
    const int64_t qdim = (int64_t)A.n_heads * HD, kvdim = (int64_t)A.n_kv_heads * HD;
    const int tid = threadIdx.x;
    const uint32_t kbase = (uint32_t)__cvta_generic_to_shared(sm + R * LD);
    auto load = [&](int st, int kt0) {
#pragma unroll
        for (int it = 0; it < KTE * (HD / 4) / THREADS; it++) {
            const int idx = tid + it * THREADS, kk = idx / (HD / 4), c4 = idx % (HD / 4), p = kt0 + kk;
            const bool ok = p < w.kend;
            cp_async16(kbase + (uint32_t)(st * KTE * LD + kk * LD + c4 * 4) * 4,
                       ok ? kv_row(A.kc, w.ck, w, p, kvdim) + (int64_t)h * HD + c4 * 4 : A.kc, ok);
        }
    };
    const uint32_t qbase = (uint32_t)__cvta_generic_to_shared(Qs);
#pragma unroll 4
    for (int it = 0; it < R * (HD / 4) / THREADS; it++) {
        const int idx = tid + it * THREADS, row = idx / (HD / 4), c4 = idx % (HD / 4);
        const int i = row / G, g = row % G, tok = w.q0 + i;
        const bool ok = tok < w.len;
        cp_async16(qbase + (uint32_t)(row * LD + c4 * 4) * 4,
                   ok ? A.qc + (w.start + tok) * qdim + (int64_t)(h * G + g) * HD + c4 * 4 : A.qc, ok);
    }
    load(0, 0);
    cp_async_commit();
    const int warp = tid >> 5, lane = tid & 31;
    const int wr = warp % (R / 16), kh = warp / (R / 16);  // row group, key half
    const int rl = lane >> 3, kl = lane & 7;
    int limit[4];  // keys each of the thread's rows attends to
    float mx[4];
#pragma unroll
    for (int a = 0; a < 4; a++) {
        const int row = wr * 16 + rl + 4 * a, tok = w.q0 + row / G;
        limit[a] = tok < w.len ? w.pre + tok + 1 : 0;
        mx[a] = -INFINITY;
    }
    for (int kt0 = 0, st = 0; kt0 < w.kend; kt0 += KTE, st ^= 1) {
        if (kt0 + KTE < w.kend) load(st ^ 1, kt0 + KTE);
        cp_async_commit();
        cp_async_wait1();
        __syncthreads();
        const float *Ks = sm + R * LD + (st * KTE + kh * KT) * LD;
        // chains j and j+4 of each of the 4 x 4 (row, key) scores as one f32
        // pair: each lane of a packed fma is the scalar fma of its chain
        float T[16], U[16];
        auto chain_pair = [&](int j, uint64_t (&c)[16]) {
#pragma unroll
            for (int o = 0; o < 16; o++) c[o] = 0;
#pragma unroll
            for (int s = 0; s < 32; s += 4) {  // two steps of the pair per 16 bytes
                float4 qa[4], kb[4];
#pragma unroll
                for (int a = 0; a < 4; a++)
                    qa[a] = *reinterpret_cast<const float4 *>(&Qs[(wr * 16 + rl + 4 * a) * LD + j * 32 + s]);
#pragma unroll
                for (int b = 0; b < 4; b++)
                    kb[b] = *reinterpret_cast<const float4 *>(&Ks[(kl + 8 * b) * LD + j * 32 + s]);
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        uint64_t &acc = c[a * 4 + b];
                        acc = fma2(pack2(qa[a].x, qa[a].y), pack2(kb[b].x, kb[b].y), acc);
                        acc = fma2(pack2(qa[a].z, qa[a].w), pack2(kb[b].z, kb[b].w), acc);
                    }
            }
        };
        // Vector.Sum order: ((e0+e4)+(e1+e5)) + ((e2+e6)+(e3+e7)); pair j holds (ej, ej+4)
        uint64_t c2[16];
        chain_pair(0, c2);
#pragma unroll
        for (int o = 0; o < 16; o++) T[o] = __fadd_rn(lo_f(c2[o]), hi_f(c2[o]));
        chain_pair(1, c2);
#pragma unroll
        for (int o = 0; o < 16; o++) T[o] = __fadd_rn(T[o], __fadd_rn(lo_f(c2[o]), hi_f(c2[o])));
        chain_pair(2, c2);
#pragma unroll
        for (int o = 0; o < 16; o++) U[o] = __fadd_rn(lo_f(c2[o]), hi_f(c2[o]));
        chain_pair(3, c2);
#pragma unroll
        for (int o = 0; o < 16; o++) U[o] = __fadd_rn(U[o], __fadd_rn(lo_f(c2[o]), hi_f(c2[o])));
#pragma unroll
        for (int a = 0; a < 4; a++) {
            float *dst = w.sc + (int64_t)(wr * 16 + rl + 4 * a) * w.ld;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int p = kt0 + kh * KT + kl + 8 * b;
                if (p < limit[a]) {
                    const float s = __fmul_rn(__fadd_rn(T[a * 4 + b], U[a * 4 + b]), A.scale);
                    dst[p] = s;
                    mx[a] = fmaxf(mx[a], s);
                }
            }
        }
        __syncthreads();
    }
    // the 8 lanes sharing a row (kl) hold its maxima over disjoint keys
#pragma unroll
    for (int a = 0; a < 4; a++) {
        float m = mx[a];
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        if (kl == 0) rowmax[kh * R + wr * 16 + rl + 4 * a] = m;
    }
}

// Phase 2: one warp per row, rows warp, warp + 8, ..: e = exp(s - max) in
// place summed as 32 lane-strided partials, then w = e / sum in place; a row
// whose maximum is not finite becomes uniform (Kernels.Softmax).
template <int RR, int TPR>
__device__ __forceinline__ void attn_softmax(const AttArgs &A, const AttView &w, const float *rowmax) {
    using namespace att;
    using S = AttShape<RR, TPR>;
    constexpr int R = RR, THREADS = S::THREADS;
    const int G = A.n_heads / A.n_kv_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = warp; row < R; row += THREADS / 32) {
        const int tok = w.q0 + row / G;
        if (tok >= w.len) continue;
        const int limit = w.pre + tok + 1;
        // the maximum is exact in any order: over the key halves, then the two
        const float mx = S::KH == 1 ? rowmax[row] : fmaxf(rowmax[row], rowmax[R + row]);
        float *s = w.sc + (int64_t)row * w.ld;
        // phase 3 loads weights in 4-key granules: the keys after the row's own
        // position in its last granule must read as 0
        if (lane < ((limit + 3) & ~3) - limit) s[limit + lane] = 0.0f;
        if (!isfinite(mx)) {
            const float u = __fdiv_rn(1.0f, (float)limit);
            for (int p = lane; p < limit; p += 32) s[p] = u;
            continue;
        }
        // lane j sums keys j, j + 32, .. in order; eight of its keys are
        // loaded together so the pass is not one round trip per key
        float sum = 0.0f;
        int p = lane;
        for (; p + 7 * 32 < limit; p += 8 * 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = s[p + 32 * u];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float e = shield_expf(__fsub_rn(v[u], mx));
                s[p + 32 * u] = e;
                sum = __fadd_rn(sum, e);
            }
        }
        for (; p < limit; p += 32) {
            const float e = shield_expf(__fsub_rn(s[p], mx));
            s[p] = e;
            sum = __fadd_rn(sum, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        for (p = lane; p + 7 * 32 < limit; p += 8 * 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = s[p + 32 * u];
#pragma unroll
            for (int u = 0; u < 8; u++) s[p + 32 * u] = __fdiv_rn(v[u], sum);
        }
        for (; p < limit; p += 32) s[p] = __fdiv_rn(s[p], sum);
    }
}

// Phase 3: ctx[row][d] = sum over keys p in order of fma(v[p][d], w[row][p], .)
// with w = e / sum (MinistralModel.cs:372-440). Key tiles of V and of the
// weights (masked keys read as 0) are double-buffered in shared memory by
// cp.async. Thread (tr, td) owns rows tr + RSTEP*a (a < NA) and dims
// td*4 + 32e (e < 4).
template <int RR, int TPR>
__device__ __forceinline__ void attn_pv(const AttArgs &A, const AttView &w, float *sm) {
    using namespace att;
    using S = AttShape<RR, TPR>;
    constexpr int R = RR, THREADS = S::THREADS, RSTEP = S::RSTEP, NA = S::NA;
    constexpr int V_FLOATS = PKT * LD, W_FLOATS = R * LDP;
    const int G = A.n_heads / A.n_kv_heads;
    const int h = blockIdx.y;
    const int64_t qdim = (int64_t)A.n_heads * HD, kvdim = (int64_t)A.n_kv_heads * HD;
    const int tid = threadIdx.x, tr = tid >> 3, td = tid & 7;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);
    auto Ws = [&](int st) { return sm + st * (V_FLOATS + W_FLOATS) + V_FLOATS; };
    auto load = [&](int st, int kt0) {
        const uint32_t vb = sbase + (uint32_t)(st * (V_FLOATS + W_FLOATS)) * 4, wb = vb + V_FLOATS * 4;
#pragma unroll
        for (int it = 0; it < PKT * (HD / 4) / THREADS; it++) {
            const int idx = tid + it * THREADS, kk = idx / (HD / 4), c4 = idx % (HD / 4), p = kt0 + kk;
            const bool ok = p < w.kend;
            cp_async16(vb + (uint32_t)(kk * LD + c4 * 4) * 4,
                       ok ? kv_row(A.v, w.cv, w, p, kvdim) + (int64_t)h * HD + c4 * 4 : A.v, ok);
        }
#pragma unroll
        for (int it = 0; it < R * (PKT / 4) / THREADS; it++) {
            const int idx = tid + it * THREADS, row = idx / (PKT / 4), c4 = idx % (PKT / 4);
            const int tok = w.q0 + row / G, p = kt0 + c4 * 4;
            const bool ok = tok < w.len && p <= w.pre + tok;
            cp_async16(wb + (uint32_t)(row * LDP + c4 * 4) * 4, ok ? w.sc + (int64_t)row * w.ld + p : w.sc, ok);
        }
    };
    // c2[a][2e + h]: dims td*4 + 32e + 2h + {0, 1} of row tr + RSTEP*a, as f32
    // pairs; each lane of a packed fma is the scalar fma(v[d], w, c[d])
    uint64_t c2[NA][8];
#pragma unroll
    for (int a = 0; a < NA; a++)
#pragma unroll
        for (int e = 0; e < 8; e++) c2[a][e] = 0;
    auto key = [&](uint32_t vrow, const float (&wa)[NA]) {
        uint64_t wd[NA];
#pragma unroll
        for (int a = 0; a < NA; a++) wd[a] = pack2u(__float_as_uint(wa[a]), __float_as_uint(wa[a]));
#pragma unroll
        for (int e = 0; e < 4; e++) {
            uint64_t v0, v1;
            asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "r"(vrow + (td * 4 + 32 * e) * 4));
#pragma unroll
            for (int a = 0; a < NA; a++) {
                c2[a][2 * e] = fma2(v0, wd[a], c2[a][2 * e]);
                c2[a][2 * e + 1] = fma2(v1, wd[a], c2[a][2 * e + 1]);
            }
        }
    };
    load(0, 0);
    cp_async_commit();
    for (int kt0 = 0, st = 0; kt0 < w.kend; kt0 += PKT, st ^= 1) {
        if (kt0 + PKT < w.kend) load(st ^ 1, kt0 + PKT);
        cp_async_commit();
        cp_async_wait1();
        __syncthreads();
        const float *W = Ws(st);
        const uint32_t vs = sbase + (uint32_t)(st * (V_FLOATS + W_FLOATS)) * 4;
        const int kn = min(PKT, w.kend - kt0);
        int kk = 0;
        for (; kk + 4 <= kn; kk += 4) {
            float4 wt[NA];
#pragma unroll
            for (int a = 0; a < NA; a++) wt[a] = *reinterpret_cast<const float4 *>(&W[(tr + RSTEP * a) * LDP + kk]);
            float wx[NA], wy[NA], wz[NA], ww[NA];
#pragma unroll
            for (int a = 0; a < NA; a++) wx[a] = wt[a].x, wy[a] = wt[a].y, wz[a] = wt[a].z, ww[a] = wt[a].w;
            key(vs + (uint32_t)((kk + 0) * LD) * 4, wx);
            key(vs + (uint32_t)((kk + 1) * LD) * 4, wy);
            key(vs + (uint32_t)((kk + 2) * LD) * 4, wz);
            key(vs + (uint32_t)((kk + 3) * LD) * 4, ww);
        }
        for (; kk < kn; kk++) {
            float wa[NA];
#pragma unroll
            for (int a = 0; a < NA; a++) wa[a] = W[(tr + RSTEP * a) * LDP + kk];
            key(vs + (uint32_t)(kk * LD) * 4, wa);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < NA; a++) {
        const int row = tr + RSTEP * a, i = row / G, g = row % G, tok = w.q0 + i;
        if (tok >= w.len) continue;
        float *dst = A.ctx + (w.start + tok) * qdim + (int64_t)(h * G + g) * HD;
#pragma unroll
        for (int e = 0; e < 4; e++)
            *reinterpret_cast<float4 *>(dst + td * 4 + 32 * e) =
                make_float4(lo_f(c2[a][2 * e]), hi_f(c2[a][2 * e]), lo_f(c2[a][2 * e + 1]), hi_f(c2[a][2 * e + 1]));
    }
}

// RR query rows per CTA, TPR threads per row: 128 rows x 2 for large
// batches (two CTAs per SM); 64 rows for small or sparsely filled ones (twice
// the CTAs when few work items would leave SMs idle; half the idle rows when
// items hold few tokens), x 4 when every CTA has an SM to itself, so a lone
// CTA still has 8 warps to hide its latencies, else x 2 (two CTAs per SM).
// One 128-row CTA per SM with more registers lost 3% on config 5 and 11% on
// config 4.
template <int RR, int TPR>
__global__ void __launch_bounds__(TPR * RR, RR == 128 ? 2 : 1) k_attn(const AttArgs A) {
    extern __shared__ float sm[];
    __shared__ float rowmax[AttShape<RR, TPR>::KH * RR];
    const AttView w = att_view<RR>(A, RR / (A.n_heads / A.n_kv_heads));
    attn_scores<RR, TPR>(A, w, sm, rowmax);
    __syncthreads();
    attn_softmax<RR, TPR>(A, w, rowmax);
    __syncthreads();
    attn_pv<RR, TPR>(A, w, sm);
}

template <int RR, int TPR>
static cudaError_t launch_attn_rows(const AttArgs &A, int n_work, cudaStream_t s) {
    using namespace att;
    using S = AttShape<RR, TPR>;
    if (RR % (A.n_heads / A.n_kv_heads)) return cudaErrorInvalidValue;
    const size_t smem = std::max((size_t)(RR + 2 * S::KTE) * LD * 4, (size_t)2 * (PKT * LD + RR * LDP) * 4);
    cudaError_t e = cudaFuncSetAttribute(k_attn<RR, TPR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_attn<RR, TPR><<<dim3((unsigned)n_work, (unsigned)A.n_kv_heads), S::THREADS, smem, s>>>(A);
    return cudaGetLastError();
}

cudaError_t launch_attention(const AttArgs &A, int n_work, int head_dim, int rows, cudaStream_t s) {
    using namespace att;
    if (n_work == 0) return cudaSuccess;
    if (head_dim != HD || A.n_heads % A.n_kv_heads) return cudaErrorInvalidValue;
    if (rows == 128) return launch_attn_rows<128, 2>(A, n_work, s);
    if (rows == 64) {
        // measured: a single 256-token request (128 CTAs) 9.8 -> 9.1 ms with
        // x 4; 64 one-token decode sequences (512 CTAs) 31.1 -> 32.7 ms
        if ((int64_t)n_work * A.n_kv_heads <= sm_count_of_device()) return launch_attn_rows<64, 4>(A, n_work, s);
        return launch_attn_rows<64, 2>(A, n_work, s);
    }
    return cudaErrorInvalidValue;
}

int attention_rows_per_cta() { return att::R; }

// One thread per 4 floats of a new key or value row; the row's request by
// binary search over the requests' first rows.
__global__ void k_append_kv(const AttArgs A, const uint8_t *__restrict__ append, int n_req, int64_t M, int kvdim) {
    const int64_t per_row = kvdim / 4;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * per_row) return;
    const int64_t t = idx / per_row;
    const int c4 = (int)(idx % per_row);
    int lo = 0, hi = n_req - 1;  // last request whose first row <= t
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (A.req_start[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    const int r = lo;
    if (!append[r]) return;
    const int64_t pos = A.req_pre[r] + (t - A.req_start[r]);
    const int64_t off = (int64_t)A.layer * A.cache_stride[r] + pos * kvdim + c4 * 4;
    const int64_t src = t * kvdim + c4 * 4;
    *reinterpret_cast<float4 *>(const_cast<float *>(A.cache_k[r]) + off) = *reinterpret_cast<const float4 *>(A.kc + src);
    *reinterpret_cast<float4 *>(const_cast<float *>(A.cache_v[r]) + off) = *reinterpret_cast<const float4 *>(A.v + src);
}

cudaError_t launch_append_kv(const AttArgs &A, const uint8_t *append, int n_req, int64_t M, int kvdim,
                             cudaStream_t s) {
    const int64_t n = M * (kvdim / 4);
    if (n == 0 || n_req == 0) return cudaSuccess;
    if (kvdim % 4) return cudaErrorInvalidValue;
    k_append_kv<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(A, append, n_req, M, kvdim);
    return cudaGetLastError();
}

// One thread per (position, head, stored dim c) of the device layout. Chain
// position c holds dim 4·(c % 32) + c / 32 (the inverse of chain_pos), so the
// snapshot's natural-order key row is read through that map; values are
// stored in natural order on both sides.
__global__ void k_prefix_state(float *__restrict__ dev_k, float *__restrict__ dev_v, float *__restrict__ snap_k,
                               float *__restrict__ snap_v, int64_t P, int kv_heads, bool to_device) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P * kv_heads * att::HD) return;
    const int c = (int)(i % att::HD);
    const int h = (int)((i / att::HD) % kv_heads);
    const int64_t pos = i / ((int64_t)kv_heads * att::HD);
    const int64_t row = ((int64_t)h * P + pos) * att::HD;
    const int d = 4 * (c & 31) + (c >> 5);
    if (to_device) {
        dev_k[i] = snap_k[row + d];
        dev_v[i] = snap_v[row + c];
    } else {
        snap_k[row + d] = dev_k[i];
        snap_v[row + c] = dev_v[i];
    }
}

cudaError_t launch_prefix_state(float *dev_k, float *dev_v, float *snap_k, float *snap_v, int64_t P, int kv_heads,
                                int head_dim, bool to_device, cudaStream_t s) {
    if (head_dim != att::HD || kv_heads <= 0 || P < 0) return cudaErrorInvalidValue;
    const int64_t n = P * kv_heads * att::HD;
    if (n == 0) return cudaSuccess;
    k_prefix_state<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dev_k, dev_v, snap_k, snap_v, P, kv_heads, to_device);
    return cudaGetLastError();
}

}  // namespace shield
