/*
 * shield_b200 — C ABI of the B200-native Shieldstral scoring prefill.
 *
 * This is the drop-in boundary for the hot path of curiosity-ai/llm-shield:
 * everything under MinistralModel.ForwardSelectedAsync (token ids -> yes/no
 * logits) and QuantMatMul.ForwardAsync/ForwardRowsAsync (the quantized GEMM)
 * runs on sm_100a behind these entry points.  The .NET surface
 * (ShieldstralModerator, ModerationResult, GgufFile, TekkenTokenizer,
 * ModelConfig) stays where it is and calls in through P/Invoke.
 *
 * Conventions (mirroring the reference):
 *  - Weights are uploaded once, byte-for-byte in their GGUF block layout
 *    (GgufFile.GetTensorPointer, Gguf/GgufFile.cs:195-199); the caller keeps
 *    ownership of the bytes it passes.
 *  - Errors are status codes; shield_last_error() gives the message of the
 *    calling thread's last failure.  Codes map to the reference's exceptions:
 *    ARG -> ArgumentException, RANGE -> ArgumentOutOfRangeException,
 *    UNSUPPORTED -> NotSupportedException, CANCELLED -> OperationCanceledException,
 *    SHAPE -> InvalidDataException (MinistralModel.cs:110-123).
 *  - A context is not re-entrant: one call at a time, as one MinistralModel
 *    instance is not thread-safe (MinistralModel.cs:21-22).  Internally a
 *    context drives one host thread and one CUDA stream per selected GPU.
 *  - Results do not depend on how requests are batched or on how many GPUs
 *    the context spans (the reference's MatMulTilingTests.cs:42-95 invariants).
 *
 * Citations are path:line within the reference project.
 */
#ifndef SHIELD_B200_H
#define SHIELD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct shield_ctx shield_ctx;
typedef int32_t shield_status;

enum {
    SHIELD_OK = 0,
    SHIELD_ERR_ARG = 1,          /* ArgumentException */
    SHIELD_ERR_RANGE = 2,        /* ArgumentOutOfRangeException */
    SHIELD_ERR_UNSUPPORTED = 3,  /* NotSupportedException */
    SHIELD_ERR_CANCELLED = 4,    /* OperationCanceledException */
    SHIELD_ERR_CUDA = 5,         /* a CUDA runtime or launch failure */
    SHIELD_ERR_TIMEOUT = 6,      /* a device-side wait gave up (bounded spin) */
    SHIELD_ERR_SHAPE = 7,        /* InvalidDataException: tensors disagree with the config */
    SHIELD_ERR_STATE = 8,        /* called before configuration / upload */
    SHIELD_ERR_NOMEM = 9         /* device or pinned host memory exhausted */
};

/* GGML type ids (Gguf/GgmlType.cs:10-44); the legacy 32-blocks are the ones
 * with an integer kernel (IntegerGemm.Supports, Quantization/IntegerGemm.cs:58-65). */
enum {
    SHIELD_TYPE_F32 = 0,
    SHIELD_TYPE_F16 = 1,
    SHIELD_TYPE_Q4_0 = 2,
    SHIELD_TYPE_Q4_1 = 3,
    SHIELD_TYPE_Q5_0 = 6,
    SHIELD_TYPE_Q5_1 = 7,
    SHIELD_TYPE_Q8_0 = 8
};

/*
 * Model hyperparameters, the fields of ModelConfig (Model/ModelConfig.cs:12-60)
 * the forward pass uses.  RoPE frequencies are computed from the YaRN fields
 * exactly as the Rope constructor does (Model/Rope.cs:33-106) unless the caller
 * passes its own table (n_rope_freqs > 0: Rope.Frequencies and
 * Rope.MagnitudeScale as computed by the unchanged C# code).
 */
typedef struct shield_config {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float rms_eps;
    float rope_freq_base;
    int32_t rope_dim;
    float rope_scale_factor;
    int32_t rope_yarn; /* ModelConfig.YarnActive */
    int32_t rope_orig_ctx;
    float yarn_beta_fast, yarn_beta_slow, yarn_ext_factor, yarn_mscale, yarn_mscale_all_dim, rope_attn_factor;
    float attn_temperature_beta; /* ModelConfig.AttentionTemperatureScale */
    int32_t n_rope_freqs;        /* 0, or rope_dim/2 with rope_freqs set */
    const float *rope_freqs;
    float rope_mscale;
    int32_t max_positions;    /* longest request accepted; 0 = 8192 */
    int32_t max_batch_tokens; /* tokens per device micro-batch; 0 = 16384 */
} shield_config;

/* Opens one context over the GPUs whose bits are set in device_mask
 * (bit i = CUDA device i); 0 selects device 0.  Each selected GPU will hold a
 * full replica of the uploaded weights. */
shield_status shield_open(int32_t device_mask, shield_ctx **out);
void shield_close(shield_ctx *ctx);
/* Number of GPUs the context spans. */
int32_t shield_device_count(const shield_ctx *ctx);

/* ModelConfig.FromGguf's result (ModelConfig.cs:62-112), set once before upload. */
shield_status shield_set_config(shield_ctx *ctx, const shield_config *cfg);

/*
 * Copies one GGUF tensor's bytes, unchanged, to every GPU of the context
 * (WeightMatrix.From / VectorParameter.From, Numerics/WeightMatrix.cs:53-90).
 * name: the GGUF name ("token_embd.weight", "blk.3.attn_q.weight", ...);
 * rows = output features (ne[1]), cols = input features (ne[0]).
 * Quantized matrices must be Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 with cols % 32 == 0;
 * norm vectors may be F32 or F16.  nbytes must equal rows * row bytes.
 */
shield_status shield_upload_tensor(shield_ctx *ctx, const char *name, uint32_t ggml_type, int64_t rows,
                                   int64_t cols, const void *bytes, size_t nbytes);

/*
 * Scores a ragged batch of independent requests: ShieldstralModerator's
 * ModerateAsync from the prompt's token ids on (ShieldstralModerator.cs:246-263),
 * i.e. MinistralModel.ForwardSelectedAsync on an empty cache followed by
 * Score (ShieldstralModerator.cs:348-364).
 *   ids[offsets[r] .. offsets[r+1])   token ids of request r (n_req + 1 offsets)
 *   verdict_ids[0 .. n_yes)           "yes" vocabulary rows; then n_no "no" rows
 *   yes[r], no[r], score[r]           best yes logit, best no logit, 2-way softmax
 *   logits (optional)                 n_req x (n_yes + n_no) verdict logits
 *   cancel (optional)                 polled between layers; non-zero cancels
 * Requests are sharded across the context's GPUs; results do not depend on
 * the sharding.  The verdict is score > 0.5 (ModerationResult.IsUnsafe).
 */
shield_status shield_score_batch(shield_ctx *ctx, const int32_t *ids, const int64_t *offsets, int32_t n_req,
                                 const int32_t *verdict_ids, int32_t n_yes, int32_t n_no, float *yes, float *no,
                                 float *score, float *logits, const volatile int32_t *cancel);

/*
 * The whole tied head at every request's last position: logits[r * vocab + v]
 * for token v of request r (ShieldstralModerator.VerdictLogitsAsync /
 * TopVerdictTokenAsync, ShieldstralModerator.cs:269-277,370-378).  Every
 * entry is bit-identical to the same vocabulary row's logit from
 * shield_score_batch (the row-subset head, MatMulTilingTests.cs:67-87).
 * Requests, sharding and the cached prefix are handled as in
 * shield_score_batch.
 */
shield_status shield_last_logits(shield_ctx *ctx, const int32_t *ids, const int64_t *offsets, int32_t n_req,
                                 float *logits, const volatile int32_t *cancel);

/*
 * SystemPromptCache.CaptureAsync / Restore (SystemPromptCache.cs:51-75,
 * KvCache.Snapshot/Restore, KvCache.cs:94-136) on the GPUs: forwards ids[0..n)
 * once on every GPU of the context and keeps each layer's keys (after RoPE)
 * and values there.  Afterwards, a request to shield_score_batch or
 * shield_last_logits whose ids begin with these n ids and go beyond them
 * forwards only the rest, attending to the cached prefix; its results are
 * bit-identical to forwarding it whole (SystemPromptCacheTests.cs:41-74).
 * Other requests are forwarded whole.  n = 0 drops the cache; so do
 * shield_set_config and shield_upload_tensor (the weights changed).
 * SHIELD_ERR_RANGE if n >= max_positions.
 */
shield_status shield_set_prefix(shield_ctx *ctx, const int32_t *ids, int32_t n);

/*
 * The cached prefix's keys and values in the layout of KvCache.Snapshot
 * (KvCache.cs:102-118), i.e. SystemPromptCache.State, the payload of its SHKV
 * file (SystemPromptCache.cs:29-30,110-127): for P = the prefix's length,
 * floats [layer][kv head][position][head_dim] of the keys after RoPE, then
 * the values the same way, 2 * n_layers * n_kv_heads * P * head_dim floats.
 * shield_get_prefix_state reads them from the context's first GPU;
 * SHIELD_ERR_STATE if no prefix is cached, SHIELD_ERR_ARG if n_floats is not
 * that count.
 */
shield_status shield_get_prefix_state(shield_ctx *ctx, float *state, int64_t n_floats);

/* The number of token ids in the cached prefix, 0 when none
 * (SystemPromptCache.TokenCount, SystemPromptCache.cs:35). */
shield_status shield_prefix_length(shield_ctx *ctx, int32_t *n);

/*
 * SystemPromptCache.RestoreInto (SystemPromptCache.cs:66-74, KvCache.Restore
 * KvCache.cs:121-136) without the prefill: copies a snapshot in the layout
 * above to every GPU of the context as the cached prefix for ids[0..n), in
 * place of the forward shield_set_prefix makes.  The caller vouches that the
 * snapshot belongs to these weights and ids (the reference's fingerprint
 * check, SystemPromptCache.cs:88-104, stays on the host).  A snapshot taken
 * by shield_get_prefix_state, or by the reference from the same weights,
 * restores bit-identical results.  SHIELD_ERR_ARG if n_floats does not
 * match n (the message of KvCache.Restore), SHIELD_ERR_RANGE as for
 * shield_set_prefix.  n = 0 drops the cache.
 */
shield_status shield_set_prefix_state(shield_ctx *ctx, const int32_t *ids, int32_t n, const float *state,
                                      int64_t n_floats);

/*
 * Incremental forwards on a KV cache, as MinistralModel.ForwardAsync appends
 * to its KvCache (MinistralModel.cs:179-271, KvCache.cs) — the prefill-then-
 * decode loop of Benchmark.cs:399-410.  A sequence is an empty cache for up
 * to `capacity` positions (<= max_positions) on one GPU of the context.
 * shield_seq_forward appends ids[offsets[i] .. offsets[i+1]) to sequence
 * seqs[i] for i < n, all sequences in one batched forward per GPU (a decode
 * step is one token per sequence), and writes each sequence's whole tied head
 * at its new last position to logits[i * vocab ..] when logits is non-null.
 * Every logit is bit-identical to forwarding the sequence's whole history in
 * one call (shield_last_logits).  A sequence may appear once per call;
 * SHIELD_ERR_RANGE when a sequence would exceed its capacity (nothing is
 * appended then).  shield_upload_tensor empties every sequence (its keys and
 * values came from the old weights); shield_set_config frees them all.
 */
shield_status shield_seq_create(shield_ctx *ctx, int32_t device, int32_t capacity, int64_t *seq);
shield_status shield_seq_forward(shield_ctx *ctx, const int64_t *seqs, const int32_t *ids, const int64_t *offsets,
                                 int32_t n, float *logits, const volatile int32_t *cancel);
/* Positions the sequence holds (MinistralModel.CachedTokenCount). */
shield_status shield_seq_length(shield_ctx *ctx, int64_t seq, int32_t *length);
/* Empties the cache, keeping its memory (MinistralModel.ResetKvCache). */
shield_status shield_seq_reset(shield_ctx *ctx, int64_t seq);
/* Frees the sequence's device memory. */
shield_status shield_seq_release(shield_ctx *ctx, int64_t seq);

/*
 * QuantMatMul.ForwardAsync / ForwardRowsAsync (Numerics/QuantMatMul.cs:71-110)
 * on one GPU of the context, host buffers in and out:
 *   y[t, i] = dot(x[t, :], W[row(i), :]),  x: M x cols, y: M x n_out
 * with row(i) = row_ids[i] when row_ids is non-null (n_out = n_rows), else i
 * (n_out = rows).  Activations are quantized once per call
 * (IntegerGemm.QuantizeActivations) and every output is bit-identical to the
 * reference's integer GEMM arithmetic.
 */
shield_status shield_qmatmul(shield_ctx *ctx, int32_t device, const char *weight, const float *x, int64_t M,
                             float *y, const int32_t *row_ids, int32_t n_rows);

/* As shield_qmatmul with device-resident x and y (full row range), enqueued on
 * the context's stream for that GPU without synchronizing. */
shield_status shield_qmatmul_device(shield_ctx *ctx, int32_t device, const char *weight, const float *d_x,
                                    int64_t M, float *d_y);

/*
 * shield_qmatmul_device for callers that cannot allocate GPU memory while they
 * run: hosts that hand the GPU's memory to their own pool or arena up front,
 * real-time services that forbid allocation on the request path, and
 * embedders whose allocator is not CUDA's.  The other GEMM entry points
 * allocate their activation scratch on first use and grow it with the
 * problem size; this one allocates nothing, ever.  It has no counterpart in
 * the reference, whose managed code rents its buffers from an ArrayPool.
 *
 * The scratch (the activations quantized to int8 and f16, their block
 * scales and sums, an error word) is one fixed device array of about 6.8 MB
 * that every GPU loading the library holds until the process exits, so
 *   M * cols <= SHIELD_NOALLOC_MAX_ELEMENTS (2^21)
 * and larger calls fail with SHIELD_ERR_ARG before touching the GPU.
 * d_x (M x cols f32) and d_y (M x rows f32) are the caller's device buffers.
 * The first call on a GPU looks up the array's device address for that GPU;
 * make that first call before any stream capture.  The address is kept for
 * the life of the process: do not go on using the library on a device after
 * cudaDeviceReset (or anything else that destroys its primary context).
 * All calls on a GPU share the one array and it keeps the last call's
 * contents: calls that may overlap on the GPU (other host threads, other
 * contexts) race and must be serialized by the caller.  The kernel is chosen
 * as for the other GEMM entry points (shield_set_gemm_path).  The call returns
 * after its work completes.
 */
#define SHIELD_NOALLOC_MAX_ELEMENTS (1 << 21)
shield_status shield_qmatmul_noalloc(shield_ctx *ctx, int32_t device, const char *weight, const float *d_x,
                                     int64_t M, float *d_y);

/* The raw per-block int32 dot products i = -z*Σa + Σ u*a of the integer GEMM
 * (IntegerGemm.cs:384-397): dots[(t*rows + n)*(cols/32) + b], for checking
 * bit-exactness.  path: 0 = the GEMM path shield_qmatmul would take,
 * 1 = CUDA-core kernel, 2 = tensor-core kernel. */
shield_status shield_debug_block_dots(shield_ctx *ctx, int32_t device, const char *weight, const float *x,
                                      int64_t M, int32_t *dots, int32_t path);

/* Which GEMM kernel the context uses: 0 = automatic (1..16 tokens: one warp
 * per output row; otherwise tensor cores where the shape allows, reading the
 * once-unpacked f16 copy of a layer weight, or unpacking the GGUF blocks on
 * the fly for a matrix without one), 1 = CUDA-core tiled kernel only,
 * 2 = tensor cores unpacking GGUF blocks only, 3 = tensor cores on the
 * unpacked copy only, 4 = the few-token kernels only. 2, 3 and 4 fail
 * with SHIELD_ERR_UNSUPPORTED on shapes their kernel does not take; the
 * raw/unpacked choice is process-wide. For cross-checking the kernels against
 * each other. */
shield_status shield_set_gemm_path(shield_ctx *ctx, int32_t path);

/* Tile width of the tensor-core GEMM: 0 = automatic (64 output features per
 * tile when 128-wide tiles would leave more than half of the GPU's SMs idle,
 * i.e. few tokens; else 128), 64 or 128 = that width only. Process-wide; the
 * outputs are identical at either width. For cross-checking. */
shield_status shield_set_gemm_tile_width(shield_ctx *ctx, int32_t width);

/* Query rows per CTA of the attention kernel: 0 = automatic (128, or 64
 * when 128-row CTAs would be fewer than two per SM or less than half filled:
 * few tokens, or one token per request), 64 or 128 = that size only (a
 * multiple of the query heads per KV head, else later forwards fail with
 * SHIELD_ERR_UNSUPPORTED). Per context; outputs are identical at either
 * size. For cross-checking. */
shield_status shield_set_attention_rows(shield_ctx *ctx, int32_t rows);

/* Intermediate tensors of one layer, named as MinistralModel's
 * IActivationSink names them (MinistralModel.cs:212-237). */
enum {
    SHIELD_ACT_OUTPUT = 0,        /* blk.N.output         n x hidden */
    SHIELD_ACT_Q_ROPE = 1,        /* blk.N.q_rope         n x n_heads*head_dim */
    SHIELD_ACT_K_ROPE = 2,        /* blk.N.k_rope         n x n_kv_heads*head_dim */
    SHIELD_ACT_V = 3,             /* blk.N.v              n x n_kv_heads*head_dim */
    SHIELD_ACT_ATTN_WEIGHTED = 4, /* blk.N.attn_weighted  n x n_heads*head_dim */
    SHIELD_ACT_POST_ATTN = 5,     /* blk.N.post_attn      n x hidden */
    SHIELD_ACT_ATTN_NORM = 6      /* blk.N.attn_norm      n x hidden */
};

/* One request through the model on one GPU with tensor `what` of layer
 * `layer` copied out to `out`, for layer-by-layer parity checks. */
shield_status shield_debug_activation(shield_ctx *ctx, int32_t device, const int32_t *ids, int32_t n,
                                      int32_t layer, int32_t what, float *out);

/* Device-side accounting of the context's work, for benchmarks. */
typedef struct shield_timing {
    double forward_ms;      /* device time of forward passes, from the first kernel of a
                               micro-batch (its ids already on the GPU) to its verdict logits */
    double gemm_ms;         /* device time inside quantized-GEMM launches (level 2 only) */
    double gemm_ops;        /* their algorithmic ops, 2*M*N*K */
    double gemm_bytes;      /* their algorithmic bytes: packed weights + int8 activations and
                               scales + f32 outputs */
    int64_t gemm_launches;  /* quantized-GEMM launches */
    int64_t kernel_launches;/* every kernel the library launched */
    int64_t tokens;         /* tokens forwarded */
    int64_t requests;       /* requests scored */
    int64_t h2d_bytes;      /* host->device bytes of scoring calls */
    int64_t d2h_bytes;      /* device->host bytes of scoring calls */
    double attn_ms;         /* device time of the attention kernels (level 2 only) */
    double attn_flops;      /* their algorithmic flops: 4 * heads * head_dim per (query, key) pair */
} shield_timing;

/* level 0: off; 1: forward intervals and counters; 2: also every GEMM launch. */
shield_status shield_set_timing(shield_ctx *ctx, int32_t level);
/* Reads (after synchronizing) and optionally resets the accounting of one GPU. */
shield_status shield_read_timing(shield_ctx *ctx, int32_t device, shield_timing *out, int32_t reset);

/* The CUDA stream (cudaStream_t) the context enqueues work for `device` on. */
shield_status shield_device_stream(shield_ctx *ctx, int32_t device, void **stream);

/* Message of the calling thread's most recent failure ("" if none). */
const char *shield_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
