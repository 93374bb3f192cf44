// Exact integer GEMM on CUDA cores: y[t, n] over weight rows n (or a subset),
// with the reference's per-output arithmetic (IntegerGemm.cs:371-457):
//   i = Σ_k w_k·a_k                      (= -z·Σa + Σ u·a, exact int32)
//   f = fma(float(i), d_w·d_a, f)         block by block, in order
//   f = fma(m_w, d_a·float(Σa), f)        Q4_1 / Q5_1 only
// Used for small token counts, row subsets (the verdict head) and any K that
// the tensor-core kernel does not take. Bit-identical to that kernel.
#include "common.cuh"
#include "ops.h"

namespace shield {

constexpr int SIMT_ROWS = 64;    // weight rows per CTA
constexpr int SIMT_TOKENS = 32;  // tokens per CTA
constexpr int SIMT_THREADS = 128;

template <int TYPE, int EPI>
__global__ void __launch_bounds__(SIMT_THREADS)
k_gemm_simt(const uint8_t *__restrict__ W, int64_t w_rows, int64_t row_bytes, const int32_t *__restrict__ row_ids,
            int64_t n_out, int64_t K, const int8_t *__restrict__ A, const float *__restrict__ da,
            const float *__restrict__ ds, int64_t M, float *__restrict__ Y, int64_t ldy) {
    constexpr int BB = block_bytes(TYPE);
    constexpr bool OFF = has_offset(TYPE);
    __shared__ int32_t ws[SIMT_ROWS][9];     // 32 signed weights as 8 packed words (+1 pad)
    __shared__ float wsc[SIMT_ROWS], woff[SIMT_ROWS];
    __shared__ int32_t as_[SIMT_TOKENS][9];
    __shared__ float ad[SIMT_TOKENS], ads[SIMT_TOKENS];

    const int tid = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * SIMT_ROWS;
    const int64_t t0 = (int64_t)blockIdx.y * SIMT_TOKENS;
    const int tr = tid % 16, tt = tid / 16;  // 4 rows x 4 tokens per thread
    const int64_t nb = K / 32;

    // the weight row this thread unpacks half of
    const int lr = tid / 2, half = tid % 2;
    const int64_t out_row = n0 + lr;
    const bool row_ok = out_row < n_out;
    const int64_t src_row = row_ok ? (row_ids ? (int64_t)row_ids[out_row] : out_row) : 0;
    const uint8_t *wrow = W + src_row * row_bytes;
    const int lt = tid / 4, part = tid % 4;  // token this thread loads a quarter of
    const bool tok_ok = t0 + lt < M;

    float f[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) f[i][j] = 0.0f;

    for (int64_t b = 0; b < nb; b++) {
        // -- weights: 16 signed values per thread, packed 4 per word
        {
            const uint8_t *blk = wrow + b * BB;
            int32_t words[4];
#pragma unroll
            for (int wi = 0; wi < 4; wi++) {
                uint32_t packed = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    int j = half * 16 + wi * 4 + k;
                    int v = row_ok ? weight_at<TYPE>(blk, j) : 0;
                    packed |= (uint32_t)(v & 0xFF) << (8 * k);
                }
                words[wi] = (int32_t)packed;
            }
#pragma unroll
            for (int wi = 0; wi < 4; wi++) ws[lr][half * 4 + wi] = words[wi];
            if (half == 0) {
                wsc[lr] = row_ok ? h2f(ld_u16(blk)) : 0.0f;
                if (OFF) woff[lr] = row_ok ? h2f(ld_u16(blk + 2)) : 0.0f;
            }
        }
        // -- activations: 8 bytes per thread
        {
            int2 v = make_int2(0, 0);
            if (tok_ok) v = *reinterpret_cast<const int2 *>(A + (t0 + lt) * K + b * 32 + part * 8);
            as_[lt][part * 2] = v.x;
            as_[lt][part * 2 + 1] = v.y;
            if (part == 0) {
                ad[lt] = tok_ok ? da[(t0 + lt) * nb + b] : 0.0f;
                if (OFF) ads[lt] = tok_ok ? ds[(t0 + lt) * nb + b] : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = tr * 4 + i;
            const float sw = wsc[r];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int t = tt * 4 + j;
                int acc = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) acc = __dp4a(ws[r][k], as_[t][k], acc);
                f[i][j] = __fmaf_rn((float)acc, __fmul_rn(sw, ad[t]), f[i][j]);
                if (OFF) f[i][j] = __fmaf_rn(woff[r], ads[t], f[i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t n = n0 + tr * 4 + i;
        if (n >= n_out) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t t = t0 + tt * 4 + j;
            if (t >= M) continue;
            float *dst = Y + t * ldy + n;
            if (EPI == EPI_ADD)
                *dst = __fadd_rn(*dst, f[i][j]);
            else
                *dst = f[i][j];
        }
    }
}

template <int TYPE>
static void gemm_simt_t(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                        int64_t ldy, int epi, cudaStream_t s) {
    dim3 grid((unsigned)((n_out + SIMT_ROWS - 1) / SIMT_ROWS), (unsigned)((q.M + SIMT_TOKENS - 1) / SIMT_TOKENS));
    if (epi == EPI_ADD)
        k_gemm_simt<TYPE, EPI_ADD><<<grid, SIMT_THREADS, 0, s>>>(w.data, w.rows, w.row_bytes, row_ids, n_out,
                                                                  w.cols, q.a8, q.da, q.ds, q.M, y, ldy);
    else
        k_gemm_simt<TYPE, EPI_STORE><<<grid, SIMT_THREADS, 0, s>>>(w.data, w.rows, w.row_bytes, row_ids, n_out,
                                                                    w.cols, q.a8, q.da, q.ds, q.M, y, ldy);
}

cudaError_t launch_gemm_simt(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                             int64_t ldy, int epi, cudaStream_t s) {
    if (n_out == 0 || q.M == 0) return cudaSuccess;
    if (w.cols % 32 || !q.a8) return cudaErrorInvalidValue;
    if (q.M > 65535LL * SIMT_TOKENS) return cudaErrorInvalidValue;
    switch (w.type) {
    case T_Q4_0: gemm_simt_t<T_Q4_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q4_1: gemm_simt_t<T_Q4_1>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q5_0: gemm_simt_t<T_Q5_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q5_1: gemm_simt_t<T_Q5_1>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q8_0: gemm_simt_t<T_Q8_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    default: return cudaErrorNotSupported;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- few tokens
//
// A handful of tokens (decode steps, the last rows of a batch): every weight
// byte is read once and the whole GPU works on one launch. The per-block work
// (unpack a block to signed int8 weights, each token's exact dot with dp4a,
// the scale product dw·da) runs in parallel over blocks; the results go
// through shared memory so that one thread per output then runs its chain in
// block order,
//   f = fma(float(i), dw·da, f)   (then f = fma(m_w, d_a·Σa, f) for Q4_1/Q5_1)
// the same operations, in the same order, as every other GEMM here.
constexpr int GEMV_WARPS = 4;
constexpr int GEMV_MAX_TOKENS = 16;

// bit i of the 4-bit x -> bit 4 of byte i (the Q5 fifth bits as 0x10 per byte)
__device__ __forceinline__ uint32_t spread4_bits(uint32_t x) { return ((x * 0x00204081u) & 0x01010101u) << 4; }

// One block to 8 words of 4 signed int8 weights w = u - z (element order),
// read with 16-bit loads (blocks are 2-byte aligned).
template <int TYPE>
__device__ __forceinline__ void block_to_i8x4(const uint8_t *blk, int (&wq)[8]) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
    if (TYPE == T_Q8_0) {
#pragma unroll
        for (int g = 0; g < 8; g++) wq[g] = (int)((uint32_t)h[1 + 2 * g] | ((uint32_t)h[2 + 2 * g] << 16));
        return;
    }
    const uint16_t *qs = h + qs_offset(TYPE) / 2;
    uint32_t qh = 0;
    if (TYPE == T_Q5_0 || TYPE == T_Q5_1)
        qh = (uint32_t)h[qh_offset(TYPE) / 2] | ((uint32_t)h[qh_offset(TYPE) / 2 + 1] << 16);
    const uint32_t z = (uint32_t)zero_point(TYPE) * 0x01010101u;
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const uint32_t q = (uint32_t)qs[2 * g] | ((uint32_t)qs[2 * g + 1] << 16);
        uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;  // elements 4g.. and 16+4g..
        if (TYPE == T_Q5_0 || TYPE == T_Q5_1) {
            lo |= spread4_bits((qh >> (4 * g)) & 0xFu);
            hi |= spread4_bits((qh >> (16 + 4 * g)) & 0xFu);
        }
        wq[g] = (int)__vsub4(lo, z);
        wq[4 + g] = (int)__vsub4(hi, z);
    }
}

// 2..16 tokens: one warp per output row. Per chunk of 32 blocks each lane
// unpacks one block and forms its dp4a dots and scale products for every
// token into shared memory; then lane m runs token m's chain over the chunk
// in block order, f = fma(float(dot), dw·da, f) (+ fma(m, Σa·da, f)), the
// reference's order (IntegerGemm.cs:371-457).
// A whole block as 32-bit words (w[j] = block bytes 4j..4j+3), read with
// 8-byte loads from the 8-byte boundary at or below it: blocks are only
// 2-byte aligned, and three 8-byte loads of a Q4_0 block touch a third of the
// cache sectors nine 2-byte loads do. The loads end at most 13 bytes past the
// block, inside the 64 bytes of slack every uploaded weight buffer carries.
template <int TYPE>
struct BlockWords {
    static constexpr int BB = block_bytes(TYPE);
    static constexpr int NW = (BB + 3) / 4;      // words of the block
    static constexpr int NL = (BB + 6 + 7) / 8;  // 8-byte loads that cover it at any even misalignment
};

template <int TYPE>
__device__ __forceinline__ void load_block_words(const uint8_t *blk, uint32_t (&w)[BlockWords<TYPE>::NW]) {
    using B = BlockWords<TYPE>;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
    const uint2 *p = reinterpret_cast<const uint2 *>(addr & ~uintptr_t(7));
    const uint32_t sh = (uint32_t)(addr & 7);  // 0, 2, 4 or 6
    uint32_t raw[2 * B::NL + 2];
#pragma unroll
    for (int i = 0; i < B::NL; i++) {
        const uint2 v = __ldg(p + i);
        raw[2 * i] = v.x;
        raw[2 * i + 1] = v.y;
    }
    raw[2 * B::NL] = 0u;  // only ever shifted in beyond the block's last byte
    raw[2 * B::NL + 1] = 0u;
    const bool skip = sh >= 4;
    const uint32_t bits = (sh & 3u) * 8u;
#pragma unroll
    for (int j = 0; j < B::NW; j++) {
        const uint32_t lo = skip ? raw[j + 1] : raw[j];
        const uint32_t hi = skip ? raw[j + 2] : raw[j + 1];
        w[j] = __funnelshift_r(lo, hi, bits);
    }
}

// The 4 bytes of a block at even byte offset OFF, from its words.
template <int OFF, int N>
__device__ __forceinline__ uint32_t word_at(const uint32_t (&w)[N]) {
    static_assert(OFF % 2 == 0 && OFF / 4 < N, "offset outside the block");
    if constexpr (OFF % 4 == 0) return w[OFF / 4];
    else return __funnelshift_r(w[OFF / 4], w[OFF / 4 + 1], 16);
}

// block_to_i8x4 from the block's words; also the f16 scale (and offset).
template <int TYPE>
__device__ __forceinline__ void words_to_i8x4(const uint32_t (&w)[BlockWords<TYPE>::NW], int (&wq)[8], float &dw,
                                              float &mw) {
    constexpr int QS = qs_offset(TYPE);
    dw = h2f((uint16_t)(w[0] & 0xFFFFu));
    mw = has_offset(TYPE) ? h2f((uint16_t)(w[0] >> 16)) : 0.0f;
    if constexpr (TYPE == T_Q8_0) {
        wq[0] = (int)word_at<QS + 0>(w);
        wq[1] = (int)word_at<QS + 4>(w);
        wq[2] = (int)word_at<QS + 8>(w);
        wq[3] = (int)word_at<QS + 12>(w);
        wq[4] = (int)word_at<QS + 16>(w);
        wq[5] = (int)word_at<QS + 20>(w);
        wq[6] = (int)word_at<QS + 24>(w);
        wq[7] = (int)word_at<QS + 28>(w);
        return;
    } else {
        uint32_t qh = 0;
        if constexpr (TYPE == T_Q5_0 || TYPE == T_Q5_1) qh = word_at<qh_offset(TYPE)>(w);
        const uint32_t z = (uint32_t)zero_point(TYPE) * 0x01010101u;
        const uint32_t q[4] = {word_at<QS>(w), word_at<QS + 4>(w), word_at<QS + 8>(w), word_at<QS + 12>(w)};
#pragma unroll
        for (int g = 0; g < 4; g++) {
            uint32_t lo = q[g] & 0x0F0F0F0Fu, hi = (q[g] >> 4) & 0x0F0F0F0Fu;  // elements 4g.. and 16+4g..
            if (TYPE == T_Q5_0 || TYPE == T_Q5_1) {
                lo |= spread4_bits((qh >> (4 * g)) & 0xFu);
                hi |= spread4_bits((qh >> (16 + 4 * g)) & 0xFu);
            }
            wq[g] = (int)__vsub4(lo, z);
            wq[4 + g] = (int)__vsub4(hi, z);
        }
    }
}

template <int TYPE, int EPI>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
k_gemv_small(const uint8_t *__restrict__ W, const int32_t *__restrict__ row_ids, int64_t rows, int64_t row_bytes,
             int64_t K, const int8_t *__restrict__ A, const float *__restrict__ da, const float *__restrict__ ds, int M,
             float *__restrict__ y, int64_t ldy) {
    constexpr bool OFF = has_offset(TYPE);
    __shared__ int32_t s_dot[GEMV_WARPS][32][GEMV_MAX_TOKENS + 1];
    __shared__ float s_p[GEMV_WARPS][32][GEMV_MAX_TOKENS + 1];
    __shared__ float s_off[GEMV_WARPS][32];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * GEMV_WARPS + wid;
    if (n >= rows) return;  // whole warp
    const int64_t nb = K / 32;
    const uint8_t *row = W + (row_ids ? (int64_t)row_ids[n] : n) * row_bytes;
    float f = 0.0f;  // lane m < M: token m's output
    for (int64_t c0 = 0; c0 < nb; c0 += 32) {
        const int64_t b = c0 + lane;
        if (b < nb) {
            const uint8_t *blk = row + b * block_bytes(TYPE);
            int wq[8];
            block_to_i8x4<TYPE>(blk, wq);
            const float dw = h2f(*reinterpret_cast<const uint16_t *>(blk));
            if (OFF) s_off[wid][lane] = h2f(*reinterpret_cast<const uint16_t *>(blk + 2));
            for (int m = 0; m < M; m++) {
                const int4 *a4 = reinterpret_cast<const int4 *>(A + (int64_t)m * K + b * 32);
                const int4 x0 = a4[0], x1 = a4[1];
                int acc = 0;
                acc = __dp4a(wq[0], x0.x, acc);
                acc = __dp4a(wq[1], x0.y, acc);
                acc = __dp4a(wq[2], x0.z, acc);
                acc = __dp4a(wq[3], x0.w, acc);
                acc = __dp4a(wq[4], x1.x, acc);
                acc = __dp4a(wq[5], x1.y, acc);
                acc = __dp4a(wq[6], x1.z, acc);
                acc = __dp4a(wq[7], x1.w, acc);
                s_dot[wid][lane][m] = acc;
                s_p[wid][lane][m] = __fmul_rn(dw, da[(int64_t)m * nb + b]);
            }
        }
        __syncwarp();
        if (lane < M) {
            const int nblk = nb - c0 < 32 ? (int)(nb - c0) : 32;
            for (int l = 0; l < nblk; l++) {
                f = __fmaf_rn((float)s_dot[wid][l][lane], s_p[wid][l][lane], f);
                if (OFF) f = __fmaf_rn(s_off[wid][l], ds[(int64_t)lane * nb + c0 + l], f);
            }
        }
        __syncwarp();
    }
    if (lane < M) {
        float *dst = y + (int64_t)lane * ldy + n;
        *dst = EPI == EPI_ADD ? __fadd_rn(*dst, f) : f;
    }
}

// One token (a decode step at batch 1, the M = 1 sweep shape): GEMV1_ROWS
// rows per CTA, their blocks in chunks of GEMV1_CHUNK. Phase 1: every thread
// forms (row, block) dots and scale products, GEMV1_UNROLL pairs at a time so
// their loads are in flight together; consecutive threads take consecutive
// blocks of a row. Phase 2: thread r runs row r's chain over the chunk in
// block order from shared memory, the same fma sequence as k_gemv_small.
constexpr int GEMV1_ROWS = 16, GEMV1_THREADS = 256, GEMV1_CHUNK = 96, GEMV1_UNROLL = 2;

template <int TYPE, int EPI>
__global__ void __launch_bounds__(GEMV1_THREADS)
k_gemv_one(const uint8_t *__restrict__ W, const int32_t *__restrict__ row_ids, int64_t rows, int64_t row_bytes,
           int64_t K, const int8_t *__restrict__ A, const float *__restrict__ da, const float *__restrict__ ds,
           float *__restrict__ y) {
    constexpr bool OFF = has_offset(TYPE);
    constexpr int LD = GEMV1_CHUNK + 1;  // odd row stride: phase 2's threads read distinct banks
    __shared__ int32_t s_dot[GEMV1_ROWS * LD];
    __shared__ float s_p[GEMV1_ROWS * LD];
    __shared__ float s_m[OFF ? GEMV1_ROWS * LD : 1];
    __shared__ int64_t s_src[GEMV1_ROWS];  // weight row of each output row
    const int64_t n0 = (int64_t)blockIdx.x * GEMV1_ROWS;
    const int nrow = rows - n0 < GEMV1_ROWS ? (int)(rows - n0) : GEMV1_ROWS;
    const int64_t nb = K / 32;
    if (threadIdx.x < nrow) s_src[threadIdx.x] = row_ids ? (int64_t)row_ids[n0 + threadIdx.x] : n0 + threadIdx.x;
    __syncthreads();
    float f = 0.0f;  // thread r < nrow: row n0 + r
    for (int64_t c0 = 0; c0 < nb; c0 += GEMV1_CHUNK) {
        const int nc = nb - c0 < GEMV1_CHUNK ? (int)(nb - c0) : GEMV1_CHUNK;
        const int pairs = nrow * nc;
        for (int base = threadIdx.x; base < pairs; base += GEMV1_THREADS * GEMV1_UNROLL) {
#pragma unroll
            for (int u = 0; u < GEMV1_UNROLL; u++) {
                const int i = base + u * GEMV1_THREADS;
                if (i < pairs) {
                    const int r = i / nc, bl = i - r * nc;
                    const int64_t b = c0 + bl;
                    uint32_t bw[BlockWords<TYPE>::NW];
                    load_block_words<TYPE>(W + s_src[r] * row_bytes + b * block_bytes(TYPE), bw);
                    int wq[8];
                    float dw, mw;
                    words_to_i8x4<TYPE>(bw, wq, dw, mw);
                    const int4 *a4 = reinterpret_cast<const int4 *>(A + b * 32);
                    const int4 x0 = a4[0], x1 = a4[1];
                    int acc = 0;
                    acc = __dp4a(wq[0], x0.x, acc);
                    acc = __dp4a(wq[1], x0.y, acc);
                    acc = __dp4a(wq[2], x0.z, acc);
                    acc = __dp4a(wq[3], x0.w, acc);
                    acc = __dp4a(wq[4], x1.x, acc);
                    acc = __dp4a(wq[5], x1.y, acc);
                    acc = __dp4a(wq[6], x1.z, acc);
                    acc = __dp4a(wq[7], x1.w, acc);
                    s_dot[r * LD + bl] = acc;
                    s_p[r * LD + bl] = __fmul_rn(dw, da[b]);
                    if (OFF) s_m[r * LD + bl] = mw;
                }
            }
        }
        __syncthreads();
        if (threadIdx.x < nrow) {
            const int r = threadIdx.x;
            for (int bl = 0; bl < nc; bl++) {
                f = __fmaf_rn((float)s_dot[r * LD + bl], s_p[r * LD + bl], f);
                if (OFF) f = __fmaf_rn(s_m[r * LD + bl], ds[c0 + bl], f);
            }
        }
        __syncthreads();  // the next chunk overwrites the arrays
    }
    if (threadIdx.x < nrow) {
        float *dst = y + n0 + threadIdx.x;
        *dst = EPI == EPI_ADD ? __fadd_rn(*dst, f) : f;
    }
}

// n_out outputs per token: weight rows row_ids[0..n_out) (all rows in order
// when row_ids is null).
template <int TYPE>
static void gemv_small_t(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                         int64_t ldy, int epi, cudaStream_t s) {
    if (q.M == 1) {
        const unsigned g1 = (unsigned)((n_out + GEMV1_ROWS - 1) / GEMV1_ROWS);
        if (epi == EPI_ADD)
            k_gemv_one<TYPE, EPI_ADD><<<g1, GEMV1_THREADS, 0, s>>>(w.data, row_ids, n_out, w.row_bytes, w.cols, q.a8,
                                                                   q.da, q.ds, y);
        else
            k_gemv_one<TYPE, EPI_STORE><<<g1, GEMV1_THREADS, 0, s>>>(w.data, row_ids, n_out, w.row_bytes, w.cols,
                                                                     q.a8, q.da, q.ds, y);
        return;
    }
    const unsigned grid = (unsigned)((n_out + GEMV_WARPS - 1) / GEMV_WARPS);
    if (epi == EPI_ADD)
        k_gemv_small<TYPE, EPI_ADD><<<grid, GEMV_WARPS * 32, 0, s>>>(w.data, row_ids, n_out, w.row_bytes, w.cols, q.a8,
                                                                     q.da, q.ds, (int)q.M, y, ldy);
    else
        k_gemv_small<TYPE, EPI_STORE><<<grid, GEMV_WARPS * 32, 0, s>>>(w.data, row_ids, n_out, w.row_bytes, w.cols,
                                                                       q.a8, q.da, q.ds, (int)q.M, y, ldy);
}

bool gemv_small_supports(const DevWeight &w, int64_t M) {
    return M >= 1 && M <= GEMV_MAX_TOKENS && w.cols % 32 == 0 && block_bytes(w.type) != 0;
}

cudaError_t launch_gemv_small(const DevWeight &w, const QAct &q, float *y, int64_t ldy, int epi, cudaStream_t s) {
    return launch_gemv_rows(w, nullptr, w.rows, q, y, ldy, epi, s);
}

cudaError_t launch_gemv_rows(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                             int64_t ldy, int epi, cudaStream_t s) {
    if (!gemv_small_supports(w, q.M) || !q.a8 || reinterpret_cast<uintptr_t>(q.a8) % 16 || w.cols % 16)
        return cudaErrorNotSupported;
    if (n_out == 0) return cudaSuccess;
    switch (w.type) {
    case T_Q4_0: gemv_small_t<T_Q4_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q4_1: gemv_small_t<T_Q4_1>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q5_0: gemv_small_t<T_Q5_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q5_1: gemv_small_t<T_Q5_1>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    case T_Q8_0: gemv_small_t<T_Q8_0>(w, row_ids, n_out, q, y, ldy, epi, s); break;
    default: return cudaErrorNotSupported;
    }
    return cudaGetLastError();
}

// Raw per-block dots: one thread per (t, n, b).
template <int TYPE>
__global__ void k_block_dots(const uint8_t *__restrict__ W, int64_t rows, int64_t row_bytes, int64_t K,
                             const int8_t *__restrict__ A, int64_t M, int32_t *__restrict__ dots) {
    int64_t nb = K / 32;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * rows * nb) return;
    int64_t b = i % nb, n = (i / nb) % rows, t = i / (nb * rows);
    const uint8_t *blk = W + n * row_bytes + b * block_bytes(TYPE);
    const int8_t *a = A + t * K + b * 32;
    int acc = 0;
    for (int j = 0; j < 32; j++) acc += weight_at<TYPE>(blk, j) * (int)a[j];
    dots[i] = acc;
}

cudaError_t launch_block_dots(const DevWeight &w, const QAct &q, int32_t *dots, cudaStream_t s) {
    int64_t n = q.M * w.rows * (w.cols / 32);
    if (n == 0) return cudaSuccess;
    unsigned g = (unsigned)((n + 255) / 256);
    switch (w.type) {
    case T_Q4_0: k_block_dots<T_Q4_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols, q.a8, q.M, dots); break;
    case T_Q4_1: k_block_dots<T_Q4_1><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols, q.a8, q.M, dots); break;
    case T_Q5_0: k_block_dots<T_Q5_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols, q.a8, q.M, dots); break;
    case T_Q5_1: k_block_dots<T_Q5_1><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols, q.a8, q.M, dots); break;
    case T_Q8_0: k_block_dots<T_Q8_0><<<g, 256, 0, s>>>(w.data, w.rows, w.row_bytes, w.cols, q.a8, q.M, dots); break;
    default: return cudaErrorNotSupported;
    }
    return cudaGetLastError();
}

}  // namespace shield
