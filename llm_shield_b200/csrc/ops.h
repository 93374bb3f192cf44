// Host-side launchers of the Shieldstral kernels. Every launcher is
// asynchronous on the given stream and does no allocation.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace shield {

// GGML type ids (reference Gguf/GgmlType.cs:10-44).
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8 };

// Bytes per 32-weight block (GgmlType.cs:78-82); 0 when the type has no integer kernel.
inline constexpr int block_bytes_host(int type) {
    return type == T_Q4_0 ? 18 : type == T_Q4_1 ? 20 : type == T_Q5_0 ? 22 : type == T_Q5_1 ? 24 : type == T_Q8_0 ? 34 : 0;
}

// Quantized activations, row-major M x K (IntegerGemm.QuantizeActivations
// output, IntegerGemm.cs:97-138): int8 values (and the same integers as f16
// for the tensor-core path), one f32 scale d per 32-block, the block's Σq,
// and ds = d * float(Σq), the multiplier of the Q4_1/Q5_1 offsets
// (IntegerGemm.cs:405-411).
struct QAct {
    int8_t *a8 = nullptr;
    __half *a16 = nullptr;
    float *da = nullptr;
    float *ds = nullptr;
    int32_t *sums = nullptr;
    int64_t M = 0, K = 0;
};

// A weight matrix resident on one device: the GGUF bytes unchanged, rows =
// output features, each row K/32 contiguous blocks (WeightMatrix.cs:16-40),
// plus planes derived once at upload: the f16 block scales (and offsets)
// widened to f32, stored block-major [K/32][rows].
struct DevWeight {
    int type = 0;
    int64_t rows = 0, cols = 0, row_bytes = 0;
    const uint8_t *data = nullptr;
    float *scale_plane = nullptr;
    float *offset_plane = nullptr;
    // the weights unpacked once to f16 integers (u - z), row-major [rows][cols],
    // for the tensor-core GEMM on long token batches (null when not built)
    __half *w16 = nullptr;
};

enum Epilogue : int { EPI_STORE = 0, EPI_ADD = 1 };

cudaError_t launch_quantize(const float *x, int64_t M, int64_t K, int64_t ldx, const QAct &q, cudaStream_t s);
// SwiGLU(g, u) of [M][K] rows (K % 32 == 0) quantized like launch_quantize.
cudaError_t launch_swiglu_quantize(const float *g, const float *u, int64_t M, int64_t K, const QAct &q,
                                   cudaStream_t s);
// RMSNorm (Kernels.cs:26-61) fused with the activation quantizer; rows are
// optionally gathered (row_idx) and the normalized floats optionally kept (y).
cudaError_t launch_rmsnorm_quant(const float *x, const int32_t *row_idx, int64_t M, int K, const float *w,
                                 float eps, float *y, const QAct &q, cudaStream_t s);
cudaError_t launch_embed(const DevWeight &emb, const int32_t *ids, int64_t M, float *h, int32_t *err,
                         cudaStream_t s);
cudaError_t launch_build_planes(const DevWeight &w, cudaStream_t s);
cudaError_t launch_unpack_f16(const DevWeight &w, cudaStream_t s);

// SMs of the current device, cached per device.
int sm_count_of_device();

// Exact integer GEMM on CUDA cores; any K % 32 == 0, optional row subset.
// A few tokens (1..16): one token 16 rows per CTA, 2..16 one warp per output
// row; the same arithmetic as the other GEMMs.
bool gemv_small_supports(const DevWeight &w, int64_t M);
cudaError_t launch_gemv_small(const DevWeight &w, const QAct &q, float *y, int64_t ldy, int epi, cudaStream_t s);
// The same for weight rows row_ids[0..n_out) (the verdict head, row subsets).
cudaError_t launch_gemv_rows(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                             int64_t ldy, int epi, cudaStream_t s);
cudaError_t launch_gemm_simt(const DevWeight &w, const int32_t *row_ids, int64_t n_out, const QAct &q, float *y,
                             int64_t ldy, int epi, cudaStream_t s);
// tcgen05 tensor-core GEMM; K % 256 == 0, full row range. Returns
// cudaErrorNotSupported for shapes it does not take.
cudaError_t launch_gemm_tc(const DevWeight &w, const QAct &q, float *y, int64_t ldy, int epi, int32_t *err,
                           cudaStream_t s);
bool gemm_tc_supports(const DevWeight &w, int64_t M);
// One launch over up to 3 weights sharing the activations, the weight type and
// K (the Q/K/V projections): weight g's outputs go to ys[g] with row stride
// ldys[g]; every output equals the single-weight launch's.
cudaError_t launch_gemm_tc_group(const DevWeight *const *ws, float *const *ys, const int64_t *ldys, int count,
                                 const QAct &q, int epi, int32_t *err, cudaStream_t s);
void gemm_tc_set_pre_min_tokens(int64_t m);
void gemm_tc_set_tile_width(int w);
// Per-block int32 dots (t, n, b) for the bit-exactness check.
cudaError_t launch_block_dots(const DevWeight &w, const QAct &q, int32_t *dots, cudaStream_t s);
cudaError_t launch_block_dots_tc(const DevWeight &w, const QAct &q, int32_t *dots, int32_t *err, cudaStream_t s);

// The GEMM with its activation scratch in a fixed device array (noalloc.cu);
// synchronizes s and returns the kernel's error word in *err_out.
cudaError_t launch_qmatmul_noalloc(const DevWeight &w, const float *x, int64_t M, float *y, int path,
                                   int32_t *err_out, cudaStream_t s);
int64_t noalloc_max_elements();

// In place on x, or, with perm (head_dim 128 only), into perm in the
// chain-major order the attention reads — and into x as well only when
// natural is set (the rotated x is then needed only to inspect it).
cudaError_t launch_rope(float *x, int64_t M, int heads, int head_dim, int64_t ld, const int32_t *pos,
                        const float *cos_t, const float *sin_t, int half, const float *temp, float *perm,
                        cudaStream_t s, bool natural = true);
// RoPE of the queries (with the attention temperature, when given) and the
// keys in one launch, both to the attention's chain-major copies (and back in
// place where *_natural is set); rows of q_heads and k_heads heads, packed.
cudaError_t launch_rope_qk(float *q, int q_heads, float *k, int k_heads, int64_t M, int head_dim, const int32_t *pos,
                           const float *cos_t, const float *sin_t, int half, const float *q_temp, float *q_perm,
                           float *k_perm, bool q_natural, bool k_natural, cudaStream_t s);
// Causal GQA attention of a group of work items (one fused kernel, see
// forward_ops.cu). work[i] = {request, first query token}; one CTA per (work
// item, KV head) covers `rows` query rows (rows / G tokens x the G heads of a
// group; rows is attention_rows_per_cta(), or half of it for small batches).
// Its scores live in the scratch while it runs: attention_scratch_floats(kend,
// n_kv_heads, rows) floats per work item from work_base[i], kend = pre + the
// last query token + 1, the KV heads' rows one after another.
struct AttArgs {
    const float *qc = nullptr;      // queries after RoPE, chain-major (launch_rope's perm output)
    const float *kc = nullptr;      // keys after RoPE, chain-major
    const float *v = nullptr;
    float *ctx = nullptr;
    float *scores = nullptr;        // the scratch
    const int2 *work = nullptr;
    const int64_t *work_base = nullptr;  // scratch offset (floats, a multiple of 4) per work item
    const int32_t *req_start = nullptr, *req_len = nullptr;
    const int32_t *req_pre = nullptr;   // cached positions in front of each request (nullptr: none)
    // per request with pre > 0: its cache (the system-prompt prefix or its own
    // sequence), layer 0 row 0 of the keys (chain-major) and values, and the
    // floats from one layer's rows to the next
    const float *const *cache_k = nullptr, *const *cache_v = nullptr;
    const int64_t *cache_stride = nullptr;
    int layer = 0;
    int n_heads = 0, n_kv_heads = 0;
    float scale = 0.0f;
};
// rows: query rows per CTA, 128 or 64 (the work list's tokens per item are
// rows / the GQA group).
cudaError_t launch_attention(const AttArgs &args, int n_work, int head_dim, int rows, cudaStream_t s);
// Appends the batch's new keys (chain-major) and values of one layer to the
// caches of the requests with a non-null append[r]: rows req_start[r] + t go
// to position req_pre[r] + t of that cache (KvCache.Append, KvCache.cs).
cudaError_t launch_append_kv(const AttArgs &args, const uint8_t *append, int n_req, int64_t M, int kvdim,
                             cudaStream_t s);
// One layer of cached keys and values between the device layout ([position]
// [kv head][head_dim], keys chain-major) and KvCache.Snapshot's ([kv head]
// [position][head_dim], natural order; KvCache.cs:102-118), for P positions.
// to_device: snap_k/snap_v -> dev_k/dev_v; else the reverse.
cudaError_t launch_prefix_state(float *dev_k, float *dev_v, float *snap_k, float *snap_v, int64_t P, int kv_heads,
                                int head_dim, bool to_device, cudaStream_t s);
int attention_rows_per_cta();
// Scratch floats of one work item of `rows` query rows attending to kend keys,
// all KV heads.
inline int64_t attention_scratch_floats(int64_t kend, int n_kv_heads, int rows) {
    return (int64_t)n_kv_heads * rows * ((kend + 3) & ~int64_t(3));
}

}  // namespace shield
