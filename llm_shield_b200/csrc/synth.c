/*
 * Synthetic checkpoint generator: seeded N(mean, std) tensors quantized to
 * GGML legacy blocks with the semantics of gguf-py's quantizers (gguf 0.19,
 * gguf/quants.py Q4_0/Q4_1/Q5_0/Q5_1/Q8_0.quantize_blocks), which is what the
 * reference's converter writes (tools/convert_shieldstral_to_gguf.py:265-272).
 *
 * Host-side input generation for tests and benchmarks; it is not on the
 * scoring path. Every value depends only on (seed, stream, index), so the
 * thread count never changes the bytes.
 */
#define _GNU_SOURCE
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8 };

static int block_bytes(int type) {
    switch (type) {
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_Q8_0: return 34;
    default: return 0;
    }
}

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Box-Muller on two 24-bit uniforms drawn from one counter hash. */
static inline float normal_at(uint64_t seed, uint64_t stream, uint64_t i, float mean, float std) {
    uint64_t h = splitmix64(splitmix64(seed * 0xD1B54A32D192ED03ull + stream) + (i >> 1));
    double u1 = ((double)(h >> 40) + 0.5) * (1.0 / 16777216.0);
    double u2 = ((double)(h & 0xFFFFFFull) + 0.5) * (1.0 / 16777216.0);
    double r = sqrt(-2.0 * log(u1));
    double z = (i & 1) ? r * sin(6.283185307179586 * u2) : r * cos(6.283185307179586 * u2);
    return mean + std * (float)z;
}

static inline uint16_t f32_to_f16(float x) { return _cvtss_sh(x, 0); /* round to nearest even */ }

static inline void wr16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* numpy's abs(blocks).argmax(): the first index of the largest magnitude. */
static int argmax_abs(const float *x) {
    int best = 0;
    float m = fabsf(x[0]);
    for (int i = 1; i < 32; i++)
        if (fabsf(x[i]) > m) { m = fabsf(x[i]); best = i; }
    return best;
}

static uint8_t trunc_clip(float v, int hi) {
    float t = truncf(v);
    int q = t < 0.0f ? 0 : (int)t;
    return (uint8_t)(q > hi ? hi : q);
}

/* gguf np_roundf: sign(n) * (floor(|n|) + floor(2*(|n| - floor(|n|)))) */
static float np_roundf(float n) {
    float a = fabsf(n), fl = floorf(a);
    float b = fl + floorf(2.0f * (a - fl));
    return n > 0.0f ? b : (n < 0.0f ? -b : 0.0f);
}

static void quantize_block(int type, const float *x, uint8_t *out) {
    uint8_t q[32];
    switch (type) {
    case T_Q4_0:
    case T_Q5_0: {
        float max = x[argmax_abs(x)];
        float d = type == T_Q4_0 ? max / -8.0f : max / -16.0f;
        float id = d == 0.0f ? 0.0f : 1.0f / d;
        float bias = type == T_Q4_0 ? 8.5f : 16.5f;
        int hi = type == T_Q4_0 ? 15 : 31;
        for (int j = 0; j < 32; j++) {
            float v = x[j] * id;
            q[j] = trunc_clip(v + bias, hi);
        }
        wr16(out, f32_to_f16(d));
        if (type == T_Q4_0) {
            for (int j = 0; j < 16; j++) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
        } else {
            uint32_t qh = 0;
            for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
            memcpy(out + 2, &qh, 4);
            for (int j = 0; j < 16; j++) out[6 + j] = (uint8_t)((q[j] & 0x0F) | (uint8_t)(q[j + 16] << 4));
        }
        break;
    }
    case T_Q4_1:
    case T_Q5_1: {
        float max = x[0], min = x[0];
        for (int j = 1; j < 32; j++) {
            if (x[j] > max) max = x[j];
            if (x[j] < min) min = x[j];
        }
        float d = (max - min) / (type == T_Q4_1 ? 15.0f : 31.0f);
        float id = d == 0.0f ? 0.0f : 1.0f / d;
        int hi = type == T_Q4_1 ? 15 : 31;
        for (int j = 0; j < 32; j++) {
            float v = (x[j] - min) * id;
            q[j] = trunc_clip(v + 0.5f, hi);
        }
        wr16(out, f32_to_f16(d));
        wr16(out + 2, f32_to_f16(min));
        if (type == T_Q4_1) {
            for (int j = 0; j < 16; j++) out[4 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
        } else {
            uint32_t qh = 0;
            for (int j = 0; j < 32; j++) qh |= (uint32_t)((q[j] >> 4) & 1) << j;
            memcpy(out + 4, &qh, 4);
            for (int j = 0; j < 16; j++) out[8 + j] = (uint8_t)((q[j] & 0x0F) | (uint8_t)(q[j + 16] << 4));
        }
        break;
    }
    case T_Q8_0: {
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fabsf(x[j]) > amax ? fabsf(x[j]) : amax;
        float d = amax / 127.0f;
        float id = d == 0.0f ? 0.0f : 1.0f / d;
        wr16(out, f32_to_f16(d));
        for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)np_roundf(x[j] * id);
        break;
    }
    }
}

/* Quantizes n floats (n % 32 == 0) into GGML blocks; F32/F16 are plain casts. */
int synth_quantize(int type, const float *x, int64_t n, uint8_t *out) {
    if (type == T_F32) { memcpy(out, x, (size_t)n * 4); return 0; }
    if (type == T_F16) {
        for (int64_t i = 0; i < n; i++) wr16(out + 2 * i, f32_to_f16(x[i]));
        return 0;
    }
    int bb = block_bytes(type);
    if (!bb || n % 32) return -1;
    for (int64_t b = 0; b < n / 32; b++) quantize_block(type, x + b * 32, out + b * bb);
    return 0;
}

typedef struct {
    int type;
    int64_t rows, cols;
    uint64_t seed, stream;
    float mean, std;
    uint8_t *out;
    float *fout;
    atomic_llong next;
} job_t;

static void *worker(void *arg) {
    job_t *J = (job_t *)arg;
    float *buf = (float *)malloc((size_t)J->cols * 4);
    int64_t rb = J->type == T_F32 ? J->cols * 4 : J->type == T_F16 ? J->cols * 2 : J->cols / 32 * block_bytes(J->type);
    for (;;) {
        int64_t r0 = atomic_fetch_add(&J->next, 64);
        if (r0 >= J->rows) break;
        int64_t r1 = r0 + 64 < J->rows ? r0 + 64 : J->rows;
        for (int64_t r = r0; r < r1; r++) {
            float *dst = J->fout ? J->fout + r * J->cols : buf;
            for (int64_t c = 0; c < J->cols; c++)
                dst[c] = normal_at(J->seed, J->stream, (uint64_t)(r * J->cols + c), J->mean, J->std);
            if (J->out) synth_quantize(J->type, dst, J->cols, J->out + r * rb);
        }
    }
    free(buf);
    return NULL;
}

/*
 * Fills a rows x cols tensor with N(mean, std) values from (seed, stream) and
 * quantizes each row to `type` into out (may be NULL); fout (may be NULL)
 * receives the float values before quantization.
 */
int synth_tensor(int type, int64_t rows, int64_t cols, uint64_t seed, uint64_t stream, float mean, float std,
                 uint8_t *out, float *fout, int threads) {
    if (type != T_F32 && type != T_F16 && (!block_bytes(type) || cols % 32)) return -1;
    job_t J;
    J.type = type;
    J.rows = rows;
    J.cols = cols;
    J.seed = seed;
    J.stream = stream;
    J.mean = mean;
    J.std = std;
    J.out = out;
    J.fout = fout;
    atomic_init(&J.next, 0);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    for (int t = 1; t < threads; t++) pthread_create(&tid[t], NULL, worker, &J);
    worker(&J);
    for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
    return 0;
}
