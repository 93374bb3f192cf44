// The quantized GEMM without any device allocation, for callers that cannot
// allocate GPU memory while they run (see shield_qmatmul_noalloc in
// include/shield_b200.h).
//
// The per-call scratch the GEMM needs — the activations quantized to int8
// (and the same integers as f16 for the tensor cores), their per-block
// scales and sums, and an error word — lives in one file-scope device array
// of fixed size. Host code must not use the array's name as a pointer (on the
// host it is only a stand-in for the symbol): its device address is looked up
// once per GPU with cudaGetSymbolAddress, with that GPU current.
#include <mutex>

#include "common.cuh"
#include "ops.h"

namespace shield {

// Largest M * K (activation elements) one call may quantize.
constexpr int64_t NOALLOC_MAX_ELEMENTS = int64_t(1) << 21;
// int8 values, f16 values, then d, d*Σq and Σq per 32-block, then the error word.
constexpr size_t NOALLOC_A8 = 0;
constexpr size_t NOALLOC_A16 = NOALLOC_A8 + NOALLOC_MAX_ELEMENTS;
constexpr size_t NOALLOC_DA = NOALLOC_A16 + 2 * NOALLOC_MAX_ELEMENTS;
constexpr size_t NOALLOC_DS = NOALLOC_DA + 4 * (NOALLOC_MAX_ELEMENTS / 32);
constexpr size_t NOALLOC_SUMS = NOALLOC_DS + 4 * (NOALLOC_MAX_ELEMENTS / 32);
constexpr size_t NOALLOC_ERR = NOALLOC_SUMS + 4 * (NOALLOC_MAX_ELEMENTS / 32);
constexpr size_t NOALLOC_BYTES = NOALLOC_ERR + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

int64_t noalloc_max_elements() { return NOALLOC_MAX_ELEMENTS; }

// Device address of the scratch array on the current GPU, looked up once per GPU.
static cudaError_t noalloc_scratch_ptr(unsigned char **out) {
    static std::mutex mu;
    static unsigned char *ptrs[128] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        ptrs[dev] = static_cast<unsigned char *>(p);
    }
    *out = ptrs[dev];
    return cudaSuccess;
}

cudaError_t launch_qmatmul_noalloc(const DevWeight &w, const float *x, int64_t M, float *y, int path,
                                   int32_t *err_out, cudaStream_t s) {
    *err_out = 0;
    if (M * w.cols > NOALLOC_MAX_ELEMENTS) return cudaErrorInvalidValue;
    unsigned char *base = nullptr;
    cudaError_t e = noalloc_scratch_ptr(&base);
    if (e != cudaSuccess) return e;
    QAct q;
    q.a8 = reinterpret_cast<int8_t *>(base + NOALLOC_A8);
    q.a16 = reinterpret_cast<__half *>(base + NOALLOC_A16);
    q.da = reinterpret_cast<float *>(base + NOALLOC_DA);
    q.ds = reinterpret_cast<float *>(base + NOALLOC_DS);
    q.sums = reinterpret_cast<int32_t *>(base + NOALLOC_SUMS);
    q.M = M;
    q.K = w.cols;
    int32_t *err = reinterpret_cast<int32_t *>(base + NOALLOC_ERR);
    // the error word keeps the previous call's value: clear it first
    if ((e = cudaMemsetAsync(err, 0, sizeof(int32_t), s)) != cudaSuccess) return e;
    if ((e = launch_quantize(x, M, w.cols, w.cols, q, s)) != cudaSuccess) return e;
    // the kernel choice of every other GEMM entry point (shield_set_gemm_path):
    // 0 the few-token kernel, then tensor cores, then CUDA cores; 1 CUDA cores;
    // 2/3 tensor cores only; 4 the few-token kernel only
    bool done = false;
    if ((path == 0 || path == 4) && gemv_small_supports(w, M)) {
        e = launch_gemv_small(w, q, y, w.rows, EPI_STORE, s);
        if (e == cudaSuccess)
            done = true;
        else if (e != cudaErrorNotSupported)
            return e;
    }
    if (!done && path != 1 && path != 4 && gemm_tc_supports(w, M)) {
        e = launch_gemm_tc(w, q, y, w.rows, EPI_STORE, err, s);
        if (e == cudaSuccess)
            done = true;
        else if (e != cudaErrorNotSupported)
            return e;
    }
    if (!done) {
        if (path >= 2) return cudaErrorNotSupported;
        if ((e = launch_gemm_simt(w, nullptr, w.rows, q, y, w.rows, EPI_STORE, s)) != cudaSuccess) return e;
    }
    if ((e = cudaMemcpyAsync(err_out, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s)) != cudaSuccess) return e;
    return cudaStreamSynchronize(s);
}

}  // namespace shield
