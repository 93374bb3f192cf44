/*
 * CPU oracle for the Shieldstral scoring prefill — TEST INFRASTRUCTURE ONLY.
 * See shield_oracle.h for what it restates and how it is pinned.
 *
 * Build flags matter: -ffp-contract=off keeps every a*b+c the reference writes
 * as two operations from being fused, and every fused multiply-add the
 * reference does issue (Fma.MultiplyAdd, Vector.FusedMultiplyAdd) is spelled
 * fmaf() or _mm256_fmadd_ps here.
 */
#define _GNU_SOURCE
#include "shield_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ type table */

int orc_block_bytes(int type) {
    switch (type) {
    case ORC_Q4_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q5_1: return 24;
    case ORC_Q8_0: return 34;
    default: return 0;
    }
}

int64_t orc_row_bytes(int type, int64_t cols) {
    if (type == ORC_F32) return cols * 4;
    if (type == ORC_F16) return cols * 2;
    int bb = orc_block_bytes(type);
    if (!bb || cols % 32) return -1;
    return cols / 32 * bb;
}

/* IEEE binary16 -> binary32, exact for every bit pattern, NaNs quieted
 * (the semantics IntegerGemm.HalfToSingle matches, IntegerGemm.cs:222-245). */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13) | (man ? 0x00400000u : 0);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal half: value = man * 2^-24, exactly representable */
            float v = (float)man * 0x1p-24f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* -------------------------------------------------------- thread fan-out */

typedef void (*orc_task_fn)(void *ctx, int64_t item);
typedef struct {
    orc_task_fn fn;
    void *ctx;
    int64_t n;
    atomic_llong next;
} orc_pool;

static void *orc_worker(void *arg) {
    orc_pool *p = (orc_pool *)arg;
    for (;;) {
        int64_t i = atomic_fetch_add(&p->next, 1);
        if (i >= p->n) break;
        p->fn(p->ctx, i);
    }
    return NULL;
}

/* Parallel.ForAsync over items; results never depend on the thread count
 * because items write disjoint outputs (QuantMatMul.cs:315-321). */
static void orc_parallel_for(int64_t n, int threads, orc_task_fn fn, void *ctx) {
    if (threads <= 1 || n <= 1) {
        for (int64_t i = 0; i < n; i++) fn(ctx, i);
        return;
    }
    if (threads > n) threads = (int)n;
    orc_pool pool = {fn, ctx, n, 0};
    pthread_t tid[256];
    if (threads > 256) threads = 256;
    for (int t = 1; t < threads; t++) pthread_create(&tid[t], NULL, orc_worker, &pool);
    orc_worker(&pool);
    for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------ activations */

/* IntegerGemm.QuantizeActivations (IntegerGemm.cs:97-138): per 32-block,
 * d = max|x| / 127f (kept float32), inverse = 1/d (0 for an all-zero block),
 * q = round-to-nearest-even(x * inverse) (vcvtps2dq), and the block's Σq. */
void orc_quantize_activations(const float *x, int count, int8_t *values, float *scales, int32_t *sums) {
    int blocks = count / 32;
    for (int b = 0; b < blocks; b++, x += 32, values += 32) {
        float max = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(x[i]);
            max = a > max ? a : max;
        }
        float d = max / 127.0f;
        float inverse = d != 0.0f ? 1.0f / d : 0.0f;
        int32_t s = 0;
        for (int i = 0; i < 32; i++) {
            float p = x[i] * inverse;
            int32_t q = (int32_t)lrintf(p); /* default MXCSR rounding: nearest-even */
            values[i] = (int8_t)q;
            s += q;
        }
        scales[b] = d;
        sums[b] = s;
    }
}

/* ---------------------------------------------------------------- blocks */

int orc_zero_point(int type) {
    switch (type) {
    case ORC_Q4_0: return 8;
    case ORC_Q5_0: return 16;
    case ORC_Q8_0: return 128;
    default: return 0;
    }
}

int orc_has_offset(int type) { return type == ORC_Q4_1 || type == ORC_Q5_1; }

/* Nibbles(): 16 bytes -> every low nibble, then every high one (IntegerGemm.cs:302-311). */
static void orc_nibbles(const uint8_t *qs, uint8_t u[32]) {
    for (int j = 0; j < 16; j++) {
        u[j] = qs[j] & 0x0F;
        u[j + 16] = qs[j] >> 4;
    }
}

/* FifthBits(): bit j of qh -> 0x10 in byte j (IntegerGemm.cs:313-329). */
static void orc_fifth_bits(uint32_t qh, uint8_t u[32]) {
    for (int j = 0; j < 32; j++) u[j] |= (uint8_t)(((qh >> j) & 1u) << 4);
}

void orc_unpack_block(int type, const uint8_t *b, uint8_t u[32], float *scale, float *offset) {
    *scale = orc_half_to_float(rd16(b));
    if (offset) *offset = 0.0f;
    switch (type) {
    case ORC_Q4_0: orc_nibbles(b + 2, u); break;
    case ORC_Q4_1:
        if (offset) *offset = orc_half_to_float(rd16(b + 2));
        orc_nibbles(b + 4, u);
        break;
    case ORC_Q5_0:
        orc_nibbles(b + 6, u);
        orc_fifth_bits(rd32(b + 2), u);
        break;
    case ORC_Q5_1:
        if (offset) *offset = orc_half_to_float(rd16(b + 2));
        orc_nibbles(b + 8, u);
        orc_fifth_bits(rd32(b + 4), u);
        break;
    case ORC_Q8_0:
        /* w + 128 as an unsigned byte is w with its sign bit flipped (IntegerGemm.cs:296-299) */
        for (int j = 0; j < 32; j++) u[j] = b[2 + j] ^ 0x80;
        break;
    default: memset(u, 0, 32); break;
    }
}

/* -------------------------------------------------------------- dequant */

int orc_dequantize(int type, const uint8_t *src, float *dst, int64_t n) {
    switch (type) {
    case ORC_F32: memcpy(dst, src, (size_t)n * 4); return 0;
    case ORC_F16:
        for (int64_t i = 0; i < n; i++) dst[i] = orc_half_to_float(rd16(src + 2 * i));
        return 0;
    default: break;
    }
    if (n % 32) return -1;
    for (int64_t blk = 0; blk < n / 32; blk++, dst += 32) {
        const uint8_t *s = src + blk * orc_block_bytes(type);
        float d = orc_half_to_float(rd16(s));
        switch (type) {
        case ORC_Q4_0: /* Dequantizer.cs:127-139 */
            for (int j = 0; j < 16; j++) {
                const uint8_t *qs = s + 2;
                dst[j] = d * (float)((qs[j] & 0x0F) - 8);
                dst[16 + j] = d * (float)((qs[j] >> 4) - 8);
            }
            break;
        case ORC_Q4_1: { /* Dequantizer.cs:141-154 */
            float m = orc_half_to_float(rd16(s + 2));
            const uint8_t *qs = s + 4;
            for (int j = 0; j < 16; j++) {
                dst[j] = d * (float)(qs[j] & 0x0F) + m;
                dst[16 + j] = d * (float)(qs[j] >> 4) + m;
            }
            break;
        }
        case ORC_Q5_0: { /* Dequantizer.cs:156-171 */
            uint32_t qh = rd32(s + 2);
            const uint8_t *qs = s + 6;
            for (int j = 0; j < 16; j++) {
                int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1u) << 4);
                int hi = (qs[j] >> 4) | (int)(((qh >> (j + 16)) & 1u) << 4);
                dst[j] = d * (float)(lo - 16);
                dst[16 + j] = d * (float)(hi - 16);
            }
            break;
        }
        case ORC_Q5_1: { /* Dequantizer.cs:173-189 */
            float m = orc_half_to_float(rd16(s + 2));
            uint32_t qh = rd32(s + 4);
            const uint8_t *qs = s + 8;
            for (int j = 0; j < 16; j++) {
                int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1u) << 4);
                int hi = (qs[j] >> 4) | (int)(((qh >> (j + 16)) & 1u) << 4);
                dst[j] = d * (float)lo + m;
                dst[16 + j] = d * (float)hi + m;
            }
            break;
        }
        case ORC_Q8_0: /* Dequantizer.cs:191-213 */
            for (int j = 0; j < 32; j++) dst[j] = d * (float)(int8_t)s[2 + j];
            break;
        default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------- integer GEMM */

/*
 * Scalar statement of one output of the integer GEMM, the sequence every lane
 * of Multiply4 and Multiply1 runs (IntegerGemm.cs:376-412, 438-454):
 *   i  = -z·Σa + Σ_k u_k·a_k                     exact int32
 *   f  = fma(float(i), scale·d_a, f)              scale·d_a rounded first
 *   f  = fma(offset, d_a·float(Σa), f)            offset types only
 * over blocks b = 0 .. blocks-1 in order.
 */
int orc_qmatmul_scalar(int type, const uint8_t *w, int64_t rows, int64_t cols,
                       const float *x, int64_t tokens, float *y) {
    int bb = orc_block_bytes(type);
    if (!bb || cols % 32) return -1;
    int64_t blocks = cols / 32;
    int z = orc_zero_point(type), has_off = orc_has_offset(type);
    int8_t *a = (int8_t *)malloc((size_t)(tokens * cols));
    float *ad = (float *)malloc((size_t)(tokens * blocks) * 4);
    int32_t *as = (int32_t *)malloc((size_t)(tokens * blocks) * 4);
    for (int64_t t = 0; t < tokens; t++)
        orc_quantize_activations(x + t * cols, (int)cols, a + t * cols, ad + t * blocks, as + t * blocks);
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *row = w + r * blocks * bb;
        for (int64_t t = 0; t < tokens; t++) {
            float f = 0.0f;
            for (int64_t b = 0; b < blocks; b++) {
                uint8_t u[32];
                float sc, off;
                orc_unpack_block(type, row + b * bb, u, &sc, &off);
                const int8_t *at = a + t * cols + b * 32;
                int32_t s = as[t * blocks + b];
                int32_t i = -z * s;
                for (int k = 0; k < 32; k++) i += (int32_t)u[k] * (int32_t)at[k];
                float da = ad[t * blocks + b];
                f = fmaf((float)i, sc * da, f);
                if (has_off) f = fmaf(off, da * (float)s, f);
            }
            y[t * rows + r] = f;
        }
    }
    free(a);
    free(ad);
    free(as);
    return 0;
}

static int g_simd = -1;

int orc_simd_level(void) {
    if (g_simd < 0) {
        __builtin_cpu_init();
        if (__builtin_cpu_supports("avxvnni"))
            g_simd = 3;
        else if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl"))
            g_simd = 2;
        else if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"))
            g_simd = 1;
        else
            g_simd = 0;
    }
    return g_simd;
}

int orc_set_simd_level(int level) {
    int best = (g_simd = -1, orc_simd_level());
    g_simd = level < best ? (level < 0 ? 0 : level) : best;
    return g_simd;
}

/* PackGroup (IntegerGemm.cs:173-212): for block b, eight 32-byte vectors;
 * vector k holds weights 4k..4k+3 of each of the 8 rows in turn. Missing rows
 * pack as an all-zero block. */
static void orc_pack_group(int type, const uint8_t *const *rowp, int count, int64_t blocks,
                           uint8_t *packed, float *scales, float *offsets) {
    int bb = orc_block_bytes(type);
    static const uint8_t zero_block[64] = {0};
    for (int64_t b = 0; b < blocks; b++, packed += 256) {
        for (int r = 0; r < 8; r++) {
            uint8_t u[32];
            float sc, off;
            const uint8_t *blk = r < count ? rowp[r] + b * bb : zero_block;
            orc_unpack_block(type, blk, u, &sc, &off);
            for (int k = 0; k < 8; k++)
                for (int i = 0; i < 4; i++) packed[k * 32 + r * 4 + i] = u[4 * k + i];
            scales[b * 8 + r] = sc;
            if (offsets) offsets[b * 8 + r] = off;
        }
    }
}

/* acc[j] += Σ_{i<4} w[4j+i]·a[4j+i] (unsigned by signed), the MultiplyAdd step
 * (IntegerGemm.cs:463-473), in whichever exact form the host has. */
__attribute__((target("avxvnni"))) static inline __m256i orc_madd_vnni(__m256i acc, __m256i w, __m256i a) {
    return _mm256_dpbusd_avx_epi32(acc, w, a);
}

__attribute__((target("avx512vnni,avx512vl"))) static inline __m256i orc_madd_vnni512(__m256i acc, __m256i w, __m256i a) {
    return _mm256_dpbusd_epi32(acc, w, a);
}

__attribute__((target("avx2"))) static inline __m256i orc_madd_avx2(__m256i acc, __m256i w, __m256i a) {
    /* exact for any u8 weight: widen both operands to 16 bits before multiplying */
    __m256i wl = _mm256_unpacklo_epi8(w, _mm256_setzero_si256());
    __m256i wh = _mm256_unpackhi_epi8(w, _mm256_setzero_si256());
    __m256i al = _mm256_srai_epi16(_mm256_unpacklo_epi8(_mm256_setzero_si256(), a), 8);
    __m256i ah = _mm256_srai_epi16(_mm256_unpackhi_epi8(_mm256_setzero_si256(), a), 8);
    /* unpacklo/hi interleave within 128-bit lanes: bytes 0-7 and 8-15 of each lane;
     * each 32-bit group of 4 bytes stays inside one half, so pair sums land in
     * the right dword after one more horizontal pair add */
    __m256i pl = _mm256_madd_epi16(wl, al); /* dwords: bytes (0,1),(2,3),(4,5),(6,7) of each lane */
    __m256i ph = _mm256_madd_epi16(wh, ah);
    /* pl dword k = w[2k]a[2k]+w[2k+1]a[2k+1] for bytes 0..7 of the lane; group sums
     * of 4 bytes are adjacent dword pairs: hadd gives (d0+d1, d2+d3) */
    __m256i s = _mm256_hadd_epi32(pl, ph); /* lane: [l0+l1, l2+l3, h0+h1, h2+h3] = dwords 0..3 of the lane */
    return _mm256_add_epi32(acc, s);
}

typedef struct {
    int type;
    const uint8_t *w;
    int64_t rows, cols, blocks, out_rows, tokens;
    const int32_t *row_ids;
    const int8_t *a;
    const float *ad;
    const int32_t *as;
    float *y;
    int simd;
} orc_gemm_job;

/* Multiply4 / Multiply1 against one packed group (IntegerGemm.cs:371-457);
 * every lane runs the same sequence, so tiles and tails agree bit for bit. */
__attribute__((target("avx2,fma,avxvnni,avx512vnni,avx512vl")))
static void orc_multiply(const orc_gemm_job *J, const uint8_t *packed, const float *scales,
                         const float *offsets, int64_t t0, int nt, float out[4][8]) {
    int z = orc_zero_point(J->type);
    int64_t blocks = J->blocks, cols = J->cols;
    __m256 f[4];
    for (int j = 0; j < nt; j++) f[j] = _mm256_setzero_ps();
    for (int64_t b = 0; b < blocks; b++) {
        const uint8_t *pk = packed + b * 256;
        __m256i acc[4];
        for (int j = 0; j < nt; j++) acc[j] = _mm256_set1_epi32(-z * J->as[(t0 + j) * blocks + b]);
        for (int k = 0; k < 8; k++) {
            __m256i wv = _mm256_loadu_si256((const __m256i *)(pk + k * 32));
            for (int j = 0; j < nt; j++) {
                int32_t a4;
                memcpy(&a4, J->a + (t0 + j) * cols + b * 32 + 4 * k, 4);
                __m256i av = _mm256_set1_epi32(a4);
                acc[j] = J->simd == 3   ? orc_madd_vnni(acc[j], wv, av)
                         : J->simd == 2 ? orc_madd_vnni512(acc[j], wv, av)
                                        : orc_madd_avx2(acc[j], wv, av);
            }
        }
        __m256 sc = _mm256_loadu_ps(scales + b * 8);
        for (int j = 0; j < nt; j++) {
            float da = J->ad[(t0 + j) * blocks + b];
            f[j] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(acc[j]), _mm256_mul_ps(sc, _mm256_set1_ps(da)), f[j]);
            if (offsets) {
                __m256 off = _mm256_loadu_ps(offsets + b * 8);
                float ds = da * (float)J->as[(t0 + j) * blocks + b];
                f[j] = _mm256_fmadd_ps(off, _mm256_set1_ps(ds), f[j]);
            }
        }
    }
    for (int j = 0; j < nt; j++) _mm256_storeu_ps(out[j], f[j]);
}

/* Scalar fallback with the same arithmetic, for hosts without AVX2+FMA. */
static void orc_multiply_scalar(const orc_gemm_job *J, const uint8_t *packed, const float *scales,
                                const float *offsets, int64_t t0, int nt, float out[4][8]) {
    int z = orc_zero_point(J->type);
    for (int j = 0; j < nt; j++) {
        for (int r = 0; r < 8; r++) {
            float f = 0.0f;
            for (int64_t b = 0; b < J->blocks; b++) {
                int32_t s = J->as[(t0 + j) * J->blocks + b];
                int32_t i = -z * s;
                const int8_t *at = J->a + (t0 + j) * J->cols + b * 32;
                for (int k = 0; k < 8; k++)
                    for (int q = 0; q < 4; q++)
                        i += (int32_t)packed[b * 256 + k * 32 + r * 4 + q] * (int32_t)at[4 * k + q];
                float da = J->ad[(t0 + j) * J->blocks + b];
                f = fmaf((float)i, scales[b * 8 + r] * da, f);
                if (offsets) f = fmaf(offsets[b * 8 + r], da * (float)s, f);
            }
            out[j][r] = f;
        }
    }
}

/* RunGroups for one 64-row chunk (QuantMatMul.cs:345-410). */
static void orc_gemm_chunk(void *ctx, int64_t chunk) {
    const orc_gemm_job *J = (const orc_gemm_job *)ctx;
    int bb = orc_block_bytes(J->type);
    int64_t groups = (J->out_rows + 7) / 8;
    int64_t g0 = chunk * 8, g1 = g0 + 8 < groups ? g0 + 8 : groups;
    uint8_t *packed = (uint8_t *)aligned_alloc(64, (size_t)(J->blocks * 256));
    float *scales = (float *)malloc((size_t)J->blocks * 8 * 4);
    float *offsets = orc_has_offset(J->type) ? (float *)malloc((size_t)J->blocks * 8 * 4) : NULL;
    for (int64_t g = g0; g < g1; g++) {
        int64_t r0 = g * 8;
        int count = (int)(J->out_rows - r0 < 8 ? J->out_rows - r0 : 8);
        const uint8_t *rowp[8];
        for (int i = 0; i < count; i++) {
            int64_t src = J->row_ids ? J->row_ids[r0 + i] : r0 + i;
            rowp[i] = J->w + src * J->blocks * bb;
        }
        orc_pack_group(J->type, rowp, count, J->blocks, packed, scales, offsets);
        float out[4][8];
        int64_t t = 0;
        while (t < J->tokens) {
            int nt = J->tokens - t >= 4 ? 4 : 1;
            if (J->simd >= 1)
                orc_multiply(J, packed, scales, offsets, t, nt, out);
            else
                orc_multiply_scalar(J, packed, scales, offsets, t, nt, out);
            for (int j = 0; j < nt; j++)
                for (int i = 0; i < count; i++) J->y[(t + j) * J->out_rows + r0 + i] = out[j][i];
            t += nt;
        }
    }
    free(packed);
    free(scales);
    free(offsets);
}

int orc_qmatmul(int type, const uint8_t *w, int64_t rows, int64_t cols,
                const float *x, int64_t tokens, float *y,
                const int32_t *row_ids, int64_t n_rows, int threads) {
    if (!orc_block_bytes(type) || cols % 32 || rows <= 0) return -1;
    int64_t out_rows = row_ids ? n_rows : rows;
    if (row_ids)
        for (int64_t i = 0; i < n_rows; i++)
            if (row_ids[i] < 0 || row_ids[i] >= rows) return -2;
    if (out_rows == 0 || tokens == 0) return 0;
    int64_t blocks = cols / 32;
    orc_gemm_job J;
    J.type = type;
    J.w = w;
    J.rows = rows;
    J.cols = cols;
    J.blocks = blocks;
    J.out_rows = out_rows;
    J.tokens = tokens;
    J.row_ids = row_ids;
    J.y = y;
    J.simd = orc_simd_level();
    int8_t *a = (int8_t *)malloc((size_t)(tokens * cols));
    float *ad = (float *)malloc((size_t)(tokens * blocks) * 4);
    int32_t *as = (int32_t *)malloc((size_t)(tokens * blocks) * 4);
    /* quantized once for the whole call (QuantMatMul.cs:309) */
    for (int64_t t = 0; t < tokens; t++)
        orc_quantize_activations(x + t * cols, (int)cols, a + t * cols, ad + t * blocks, as + t * blocks);
    J.a = a;
    J.ad = ad;
    J.as = as;
    int64_t groups = (out_rows + 7) / 8;
    int64_t chunks = (groups + 7) / 8;
    orc_parallel_for(chunks, threads, orc_gemm_chunk, &J);
    free(a);
    free(ad);
    free(as);
    return 0;
}

int orc_block_dots(int type, const uint8_t *w, int64_t rows, int64_t cols,
                   const float *x, int64_t tokens, int32_t *dots) {
    int bb = orc_block_bytes(type);
    if (!bb || cols % 32) return -1;
    int64_t blocks = cols / 32;
    int z = orc_zero_point(type);
    int8_t a[32];
    float ad;
    int32_t as;
    for (int64_t t = 0; t < tokens; t++) {
        for (int64_t b = 0; b < blocks; b++) {
            orc_quantize_activations(x + t * cols + b * 32, 32, a, &ad, &as);
            for (int64_t r = 0; r < rows; r++) {
                uint8_t u[32];
                float sc, off;
                orc_unpack_block(type, w + (r * blocks + b) * bb, u, &sc, &off);
                int32_t i = -z * as;
                for (int k = 0; k < 32; k++) i += (int32_t)u[k] * (int32_t)a[k];
                dots[(t * rows + r) * blocks + b] = i;
            }
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- kernels */

/* Vector<float>.Sum of an 8-lane vector. Assumed order (the JIT's
 * lower+upper halves, then two horizontal adds):
 * ((e0+e4)+(e1+e5)) + ((e2+e6)+(e3+e7)). */
static inline float orc_vsum8(const float e[8]) {
    float s0 = e[0] + e[4], s1 = e[1] + e[5], s2 = e[2] + e[6], s3 = e[3] + e[7];
    return (s0 + s1) + (s2 + s3);
}

/* Kernels.RmsNorm (Kernels.cs:26-61) with Vector<float>.Count = 8. */
void orc_rmsnorm(const float *x, const float *w, int n, float eps, float *y) {
    double sum = 0.0;
    int i = 0;
    const int width = 8;
    if (n >= 2 * width) {
        float even[8] = {0}, odd[8] = {0};
        for (; i + 2 * width <= n; i += 2 * width) {
            for (int j = 0; j < 8; j++) {
                float a = x[i + j], b = x[i + width + j];
                float aa = a * a, bb = b * b;
                even[j] = even[j] + aa;
                odd[j] = odd[j] + bb;
            }
        }
        sum = (double)orc_vsum8(even) + (double)orc_vsum8(odd);
    }
    for (; i < n; i++) sum += (double)x[i] * (double)x[i];
    float scale = 1.0f / sqrtf((float)(sum / n) + eps);
    for (i = 0; i < n; i++) {
        float v = x[i] * scale;
        y[i] = v * w[i];
    }
}

static inline float orc_f32_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/*
 * exp(x) as both this oracle and the CUDA library evaluate it (the reference's
 * TensorPrimitives.Exp is a .NET library kernel whose bits are not
 * reproducible here): Cody-Waite reduction x = k·ln2 + r with ln2 split in a
 * 16-bit head and a tail (k·head is exact), then the degree-7 Taylor
 * polynomial of e^r on |r| <= ln2/2 by Horner's rule with fused
 * multiply-adds, then scaling by 2^k.  Every step is one IEEE operation, so
 * host and device produce the same bits.  k > 127 gives +inf and k < -126
 * gives 0 (the result would be subnormal).
 */
float orc_expf(float x) {
    if (x != x) return x;
    float k = rintf(x * orc_f32_bits(0x3FB8AA3Bu)); /* log2(e) */
    if (k > 127.0f) return INFINITY;
    if (k < -126.0f) return 0.0f;
    float r = fmaf(k, -orc_f32_bits(0x3F317200u), x); /* ln2 head: exact product */
    r = fmaf(k, -orc_f32_bits(0x35BFBE8Eu), r);       /* ln2 tail */
    float p = orc_f32_bits(0x39500D01u);              /* 1/7! */
    p = fmaf(p, r, orc_f32_bits(0x3AB60B61u));         /* 1/6! */
    p = fmaf(p, r, orc_f32_bits(0x3C088889u));         /* 1/5! */
    p = fmaf(p, r, orc_f32_bits(0x3D2AAAABu));         /* 1/4! */
    p = fmaf(p, r, orc_f32_bits(0x3E2AAAABu));         /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * orc_f32_bits((uint32_t)((int)k + 127) << 23);
}

/* Kernels.Softmax (Kernels.cs:103-122): max shift, exp, sum, divide; an
 * all-masked row becomes uniform. TensorPrimitives.Sum's order is a .NET
 * library detail; the sum here is 32 strided partial sums (element i goes to
 * partial i % 32, in order) folded pairwise (j += j+16, j += j+8, ... ),
 * the order one GPU warp computes it in. */
void orc_softmax(float *x, int n) {
    if (n == 0) return;
    float max = x[0];
    for (int i = 1; i < n; i++) max = x[i] > max ? x[i] : max;
    if (!isfinite(max)) {
        for (int i = 0; i < n; i++) x[i] = 1.0f / (float)n;
        return;
    }
    float part[32] = {0};
    for (int i = 0; i < n; i++) {
        x[i] = orc_expf(x[i] - max);
        part[i % 32] = part[i % 32] + x[i];
    }
    for (int off = 16; off >= 1; off >>= 1)
        for (int j = 0; j < off; j++) part[j] = part[j] + part[j + off];
    float sum = part[0];
    for (int i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* Kernels.SwiGlu (Kernels.cs:83-90); Sigmoid = 1/(1+exp(-v)) (Kernels.cs:226). */
void orc_swiglu(const float *gate, float *up, float *dst, int n) {
    for (int i = 0; i < n; i++) up[i] = gate[i] * up[i];
    for (int i = 0; i < n; i++) {
        float s = 1.0f / (1.0f + orc_expf(-gate[i]));
        dst[i] = s * up[i];
    }
}

/* ------------------------------------------------------------------- rope */

static float orc_mscale_term(float scale, float m) {
    return scale <= 1.0f ? 1.0f : 0.1f * m * logf(scale) + 1.0f;
}

/* Rope ctor (Rope.cs:33-66), YarnCorrectionDims (Rope.cs:91-106),
 * ComputeMagnitudeScale (Rope.cs:78-88). */
void orc_rope_freqs(const orc_rope_params *p, float *freqs, float *mscale) {
    int dim = p->rope_dim, half = dim / 2;
    float freq_scale = 1.0f / p->scale_factor;
    if (!p->yarn) {
        for (int i = 0; i < half; i++) freqs[i] = freq_scale / powf(p->freq_base, 2.0f * (float)i / (float)dim);
        *mscale = p->attn_factor;
        return;
    }
    float low, high;
    if (p->beta_fast == 0.0f && p->beta_slow == 0.0f) {
        low = 3.4028235e38f;
        high = (float)dim / 2.0f - 1.0f;
    } else {
        const float PI = 3.14159265358979323846f;
        float cf = (float)dim * logf((float)p->orig_ctx / (p->beta_fast * 2.0f * PI)) / (2.0f * logf(p->freq_base));
        float cs = (float)dim * logf((float)p->orig_ctx / (p->beta_slow * 2.0f * PI)) / (2.0f * logf(p->freq_base));
        low = fmaxf(0.0f, floorf(cf));
        high = fminf((float)dim / 2.0f - 1.0f, ceilf(cs));
    }
    for (int i = 0; i < half; i++) {
        float extrapolated = 1.0f / powf(p->freq_base, 2.0f * (float)i / (float)dim);
        float interpolated = freq_scale * extrapolated;
        float y = ((float)i - low) / fmaxf(0.001f, high - low);
        float c = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
        float mix = (1.0f - c) * p->ext_factor;
        float a = interpolated * (1.0f - mix);
        float b = extrapolated * mix;
        freqs[i] = a + b;
    }
    float factor = p->scale_factor;
    float m = p->mscale != 0.0f ? p->mscale : 1.0f;
    float ratio = p->mscale_all_dim != 0.0f ? orc_mscale_term(factor, m) / orc_mscale_term(factor, p->mscale_all_dim)
                                            : orc_mscale_term(factor, 1.0f);
    *mscale = ratio * p->attn_factor;
}

/* Rope.Apply (Rope.cs:112-135): adjacent pairs (x[2i], x[2i+1]). */
void orc_rope_apply(float *data, int heads, int head_dim, int position, const float *freqs, int half, float mscale) {
    float cs[128], sn[128];
    for (int i = 0; i < half; i++) {
        float theta = (float)position * freqs[i];
        cs[i] = cosf(theta) * mscale;
        sn[i] = sinf(theta) * mscale;
    }
    for (int h = 0; h < heads; h++) {
        float *hd = data + (int64_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float x0 = hd[2 * i], x1 = hd[2 * i + 1];
            float a = x0 * cs[i], b = x1 * sn[i];
            float c = x0 * sn[i], d = x1 * cs[i];
            hd[2 * i] = a - b;
            hd[2 * i + 1] = c + d;
        }
    }
}

/* ------------------------------------------------------------------ model */

typedef struct {
    int type;
    int64_t rows, cols;
    const uint8_t *data;
} orc_tensor;

typedef struct {
    float *attn_norm, *ffn_norm;
    orc_tensor q, k, v, o, gate, up, down;
} orc_layer;

struct orc_model {
    orc_config cfg;
    orc_tensor tok_embd;
    float *output_norm;
    orc_layer *layers;
};

orc_model *orc_model_create(const orc_config *cfg) {
    if (cfg->n_layers <= 0 || cfg->hidden % 32 || cfg->n_kv_heads <= 0 || cfg->n_heads % cfg->n_kv_heads ||
        cfg->head_dim > 256 || cfg->rope_half * 2 > cfg->head_dim)
        return NULL;
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    m->layers = (orc_layer *)calloc((size_t)cfg->n_layers, sizeof(orc_layer));
    return m;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    for (int l = 0; l < m->cfg.n_layers; l++) {
        free(m->layers[l].attn_norm);
        free(m->layers[l].ffn_norm);
    }
    free(m->layers);
    free(m->output_norm);
    free(m);
}

/* VectorParameter.From: 1-D parameters widened to float once (WeightMatrix.cs:76-90). */
static float *orc_vector(int type, int64_t n, const void *data) {
    float *v = (float *)malloc((size_t)n * 4);
    if (orc_dequantize(type, (const uint8_t *)data, v, n) != 0) {
        free(v);
        return NULL;
    }
    return v;
}

int orc_model_set_tensor(orc_model *m, const char *name, int type, int64_t rows, int64_t cols, const void *data) {
    const orc_config *c = &m->cfg;
    orc_tensor t = {type, rows, cols, (const uint8_t *)data};
    if (!strcmp(name, "token_embd.weight")) {
        if (cols != c->hidden) return -1;
        m->tok_embd = t;
        return 0;
    }
    if (!strcmp(name, "output_norm.weight")) {
        free(m->output_norm);
        m->output_norm = orc_vector(type, rows * cols, data);
        return m->output_norm ? 0 : -1;
    }
    int l = -1, off = 0;
    if (sscanf(name, "blk.%d.%n", &l, &off) != 1 || l < 0 || l >= c->n_layers) return -1;
    const char *rest = name + off;
    orc_layer *L = &m->layers[l];
    if (!strcmp(rest, "attn_norm.weight")) {
        free(L->attn_norm);
        L->attn_norm = orc_vector(type, rows * cols, data);
        return L->attn_norm ? 0 : -1;
    }
    if (!strcmp(rest, "ffn_norm.weight")) {
        free(L->ffn_norm);
        L->ffn_norm = orc_vector(type, rows * cols, data);
        return L->ffn_norm ? 0 : -1;
    }
    struct { const char *n; orc_tensor *dst; int64_t r, k; } map[] = {
        {"attn_q.weight", &L->q, (int64_t)c->n_heads * c->head_dim, c->hidden},
        {"attn_k.weight", &L->k, (int64_t)c->n_kv_heads * c->head_dim, c->hidden},
        {"attn_v.weight", &L->v, (int64_t)c->n_kv_heads * c->head_dim, c->hidden},
        {"attn_output.weight", &L->o, c->hidden, (int64_t)c->n_heads * c->head_dim},
        {"ffn_gate.weight", &L->gate, c->ffn, c->hidden},
        {"ffn_up.weight", &L->up, c->ffn, c->hidden},
        {"ffn_down.weight", &L->down, c->hidden, c->ffn},
    };
    for (size_t i = 0; i < sizeof(map) / sizeof(map[0]); i++) {
        if (!strcmp(rest, map[i].n)) {
            if (rows != map[i].r || cols != map[i].k) return -1;
            *map[i].dst = t;
            return 0;
        }
    }
    return -1;
}

typedef struct {
    const orc_config *c;
    const float *q, *keys, *values;
    float *ctx;
    int seq;
    float scale;
} orc_attn_job;

/* x rounded to nearest-even with `bits` explicit mantissa bits (finite x). */
static inline float orc_round_mantissa(float x, int bits) {
    uint32_t u;
    memcpy(&u, &x, 4);
    const int drop = 23 - bits;
    const uint32_t lsb = (u >> drop) & 1u;
    u += (1u << (drop - 1)) - 1u + lsb;
    u &= ~((1u << drop) - 1u);
    memcpy(&x, &u, 4);
    return x;
}

/* AttendGroup (MinistralModel.cs:372-440) for one (kv head, query token):
 * every query head sharing the KV head, on an empty cache (startPos = 0). */
static void orc_attend(void *vctx, int64_t item) {
    const orc_attn_job *J = (const orc_attn_job *)vctx;
    const orc_config *c = J->c;
    int hd = c->head_dim, group = c->n_heads / c->n_kv_heads;
    int qdim = c->n_heads * hd, kvdim = c->n_kv_heads * hd;
    int kvh = (int)(item / J->seq), t = (int)(item % J->seq);
    int limit = t + 1;
    const int rb = c->attn_operand_bits;
    float *s = (float *)malloc((size_t)limit * 4);
    float qr[512], kr[512], vr[512];
    for (int g = 0; g < group; g++) {
        int head = kvh * group + g;
        const float *qh = J->q + (int64_t)t * qdim + (int64_t)head * hd;
        if (rb > 0 && hd <= 512) {
            for (int d = 0; d < hd; d++) qr[d] = orc_round_mantissa(qh[d], rb);
            qh = qr;
        }
        for (int p = 0; p < limit; p++) {
            const float *kp = J->keys + (int64_t)p * kvdim + (int64_t)kvh * hd;
            if (rb > 0 && hd <= 512) {
                for (int d = 0; d < hd; d++) kr[d] = orc_round_mantissa(kp[d], rb);
                kp = kr;
            }
            /* Kernels.Dot4: 8 lanes of fused multiply-adds, then Vector.Sum */
            float acc[8] = {0};
            int i = 0;
            for (; i + 8 <= hd; i += 8)
                for (int j = 0; j < 8; j++) acc[j] = fmaf(qh[i + j], kp[i + j], acc[j]);
            float r = orc_vsum8(acc);
            for (; i < hd; i++) r = r + qh[i] * kp[i];
            s[p] = r * J->scale;
        }
        orc_softmax(s, limit);
        float *ch = J->ctx + (int64_t)t * qdim + (int64_t)head * hd;
        for (int d = 0; d < hd; d++) ch[d] = 0.0f;
        /* AddScaled4 for every position. The reference skips a position only when
         * all four heads' weights are exactly zero (MinistralModel.cs:422);
         * fma(v, 0, c) == c for finite v except that it may turn a -0 context
         * into +0, so the skip changes no value beyond the sign of a zero. */
        for (int p = 0; p < limit; p++) {
            float w = rb > 0 ? orc_round_mantissa(s[p], rb) : s[p];
            const float *vp = J->values + (int64_t)p * kvdim + (int64_t)kvh * hd;
            if (rb > 0 && hd <= 512) {
                for (int d = 0; d < hd; d++) vr[d] = orc_round_mantissa(vp[d], rb);
                vp = vr;
            }
            for (int d = 0; d < hd; d++) ch[d] = fmaf(vp[d], w, ch[d]); /* Kernels.AddScaled4 */
        }
    }
    free(s);
}

int orc_model_forward(const orc_model *m, const int32_t *ids, int n, const int32_t *vocab_ids,
                      int n_vocab_ids, float *out, int threads, int capture_layer, int capture_what,
                      float *capture) {
    const orc_config *c = &m->cfg;
    if (n <= 0 || !m->tok_embd.data || !m->output_norm) return -1;
    int hid = c->hidden, ff = c->ffn, hd = c->head_dim;
    int qdim = c->n_heads * hd, kvdim = c->n_kv_heads * hd;
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= m->tok_embd.rows) return -2;
    float *h = (float *)malloc((size_t)n * hid * 4);
    float *norm = (float *)malloc((size_t)n * hid * 4);
    float *scratch = (float *)malloc((size_t)n * hid * 4);
    float *q = (float *)malloc((size_t)n * qdim * 4);
    float *kc = (float *)malloc((size_t)n * kvdim * 4);
    float *vc = (float *)malloc((size_t)n * kvdim * 4);
    float *ctx = (float *)malloc((size_t)n * qdim * 4);
    float *g = (float *)malloc((size_t)n * ff * 4);
    float *u = (float *)malloc((size_t)n * ff * 4);
    int64_t erb = orc_row_bytes(m->tok_embd.type, hid);
    /* QuantMatMul.GatherRows (QuantMatMul.cs:534-545) */
    for (int i = 0; i < n; i++)
        orc_dequantize(m->tok_embd.type, m->tok_embd.data + (int64_t)ids[i] * erb, h + (int64_t)i * hid, hid);
    float scale = 1.0f / sqrtf((float)hd);
    int rc = 0;
#define ORC_CAPTURE(what, src, width)                                                   \
    do {                                                                             \
        if (l == capture_layer && capture && capture_what == (what))                  \
            memcpy(capture, (src), (size_t)n * (size_t)(width) * sizeof(float));      \
    } while (0)
    for (int l = 0; l < c->n_layers && rc == 0; l++) {
        const orc_layer *L = &m->layers[l];
        if (!L->attn_norm || !L->ffn_norm || !L->q.data || !L->down.data) { rc = -1; break; }
        for (int t = 0; t < n; t++)
            orc_rmsnorm(h + (int64_t)t * hid, L->attn_norm, hid, c->rms_eps, norm + (int64_t)t * hid);
        ORC_CAPTURE(ORC_CAP_ATTN_NORM, norm, hid);
        /* AttentionAsync (MinistralModel.cs:282-354) */
        orc_qmatmul(L->q.type, L->q.data, L->q.rows, L->q.cols, norm, n, q, NULL, 0, threads);
        for (int t = 0; t < n; t++) {
            float *row = q + (int64_t)t * qdim;
            orc_rope_apply(row, c->n_heads, hd, t, c->rope_freqs, c->rope_half, c->rope_mscale);
            /* ApplyPositionScale (MinistralModel.cs:476-482) */
            if (c->rope_orig_ctx > 0 && c->attn_temperature_beta != 0.0f) {
                float interval = floorf((float)t / (float)c->rope_orig_ctx);
                if (interval != 0.0f) {
                    float f = 1.0f + c->attn_temperature_beta * logf(1.0f + interval);
                    for (int i = 0; i < qdim; i++) row[i] = row[i] * f;
                }
            }
        }
        orc_qmatmul(L->k.type, L->k.data, L->k.rows, L->k.cols, norm, n, kc, NULL, 0, threads);
        for (int t = 0; t < n; t++)
            orc_rope_apply(kc + (int64_t)t * kvdim, c->n_kv_heads, hd, t, c->rope_freqs, c->rope_half, c->rope_mscale);
        orc_qmatmul(L->v.type, L->v.data, L->v.rows, L->v.cols, norm, n, vc, NULL, 0, threads);
        ORC_CAPTURE(ORC_CAP_Q_ROPE, q, qdim);
        ORC_CAPTURE(ORC_CAP_K_ROPE, kc, kvdim);
        ORC_CAPTURE(ORC_CAP_V, vc, kvdim);
        orc_attn_job AJ = {c, q, kc, vc, ctx, n, scale};
        orc_parallel_for((int64_t)c->n_kv_heads * n, threads, orc_attend, &AJ);
        ORC_CAPTURE(ORC_CAP_ATTN_WEIGHTED, ctx, qdim);
        orc_qmatmul(L->o.type, L->o.data, L->o.rows, L->o.cols, ctx, n, scratch, NULL, 0, threads);
        for (int64_t i = 0; i < (int64_t)n * hid; i++) h[i] = h[i] + scratch[i]; /* Kernels.Add */
        ORC_CAPTURE(ORC_CAP_POST_ATTN, h, hid);
        for (int t = 0; t < n; t++)
            orc_rmsnorm(h + (int64_t)t * hid, L->ffn_norm, hid, c->rms_eps, norm + (int64_t)t * hid);
        orc_qmatmul(L->gate.type, L->gate.data, L->gate.rows, L->gate.cols, norm, n, g, NULL, 0, threads);
        orc_qmatmul(L->up.type, L->up.data, L->up.rows, L->up.cols, norm, n, u, NULL, 0, threads);
        orc_swiglu(g, u, g, n * ff);
        orc_qmatmul(L->down.type, L->down.data, L->down.rows, L->down.cols, g, n, scratch, NULL, 0, threads);
        for (int64_t i = 0; i < (int64_t)n * hid; i++) h[i] = h[i] + scratch[i];
        ORC_CAPTURE(ORC_CAP_OUTPUT, h, hid);
    }
    if (rc == 0) {
        /* last position only, tied head, verdict rows only (MinistralModel.cs:246-255) */
        orc_rmsnorm(h + (int64_t)(n - 1) * hid, m->output_norm, hid, c->rms_eps, norm);
        rc = orc_qmatmul(m->tok_embd.type, m->tok_embd.data, m->tok_embd.rows, hid, norm, 1, out,
                         vocab_ids, n_vocab_ids, threads);
    }
    free(h); free(norm); free(scratch); free(q); free(kc); free(vc); free(ctx); free(g); free(u);
    return rc;
}

void orc_score(const float *v, int n_yes, int n_no, float *score, float *yes, float *no) {
    float y = -INFINITY, nn = -INFINITY;
    for (int i = 0; i < n_yes; i++) if (v[i] > y) y = v[i];
    for (int i = 0; i < n_no; i++) if (v[n_yes + i] > nn) nn = v[n_yes + i];
    float mx = fmaxf(y, nn);
    float ey = expf(y - mx), en = expf(nn - mx);
    *score = ey / (ey + en);
    *yes = y;
    *no = nn;
}
