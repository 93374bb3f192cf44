// Host runtime of the Shieldstral scoring prefill and its C ABI
// (include/shield_b200.h): per-GPU weight store, micro-batched forward over a
// ragged batch of requests, request sharding across GPUs.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "ops.h"
#include "shield_b200.h"

namespace shield {

struct Error : std::runtime_error {
    shield_status code;
    Error(shield_status c, const std::string &m) : std::runtime_error(m), code(c) {}
};

static thread_local std::string g_last_error;

#define SHIELD_CUDA(x)                                                                                 \
    do {                                                                                               \
        cudaError_t e_ = (x);                                                                          \
        if (e_ != cudaSuccess)                                                                         \
            throw Error(e_ == cudaErrorMemoryAllocation ? SHIELD_ERR_NOMEM : SHIELD_ERR_CUDA,          \
                        std::string(#x) + " failed: " + cudaGetErrorString(e_));                     \
    } while (0)

static int64_t row_bytes_of(int type, int64_t cols) {
    switch (type) {
    case T_F32: return cols * 4;
    case T_F16: return cols * 2;
    default: {
        int bb = block_bytes_host(type);
        return bb && cols % 32 == 0 ? cols / 32 * bb : -1;
    }
    }
}

// ------------------------------------------------------------------ config

struct Config {
    int n_layers = 0, hidden = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, ffn = 0, vocab = 0;
    float eps = 1e-5f;
    int rope_half = 0;
    std::vector<float> freqs;
    float mscale = 1.0f;
    float temp_beta = 0.0f;
    int orig_ctx = 0;
    int max_positions = 8192;
    int max_batch_tokens = 16384;
    int qdim() const { return n_heads * head_dim; }
    int kvdim() const { return n_kv_heads * head_dim; }
    int max_k() const { return std::max(std::max(hidden, qdim()), ffn); }
};

static float mscale_term(float scale, float m) { return scale <= 1.0f ? 1.0f : 0.1f * m * logf(scale) + 1.0f; }

// The Rope constructor (Rope.cs:33-106), in float32 as the reference computes it.
static void rope_freqs(const shield_config &c, std::vector<float> &freqs, float &mscale) {
    int dim = c.rope_dim, half = dim / 2;
    freqs.assign(half, 0.0f);
    float freq_scale = 1.0f / c.rope_scale_factor;
    if (!c.rope_yarn) {
        for (int i = 0; i < half; i++) freqs[i] = freq_scale / powf(c.rope_freq_base, 2.0f * (float)i / (float)dim);
        mscale = c.rope_attn_factor;
        return;
    }
    float low, high;
    if (c.yarn_beta_fast == 0.0f && c.yarn_beta_slow == 0.0f) {
        low = 3.4028235e38f;
        high = (float)dim / 2.0f - 1.0f;
    } else {
        const float PI = 3.14159265358979323846f;
        float cf = (float)dim * logf((float)c.rope_orig_ctx / (c.yarn_beta_fast * 2.0f * PI)) /
                   (2.0f * logf(c.rope_freq_base));
        float cs = (float)dim * logf((float)c.rope_orig_ctx / (c.yarn_beta_slow * 2.0f * PI)) /
                   (2.0f * logf(c.rope_freq_base));
        low = fmaxf(0.0f, floorf(cf));
        high = fminf((float)dim / 2.0f - 1.0f, ceilf(cs));
    }
    for (int i = 0; i < half; i++) {
        float extrapolated = 1.0f / powf(c.rope_freq_base, 2.0f * (float)i / (float)dim);
        float interpolated = freq_scale * extrapolated;
        float y = ((float)i - low) / fmaxf(0.001f, high - low);
        float cl = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
        float mix = (1.0f - cl) * c.yarn_ext_factor;
        float a = interpolated * (1.0f - mix);
        float b = extrapolated * mix;
        freqs[i] = a + b;
    }
    float factor = c.rope_scale_factor;
    float m = c.yarn_mscale != 0.0f ? c.yarn_mscale : 1.0f;
    float ratio = c.yarn_mscale_all_dim != 0.0f ? mscale_term(factor, m) / mscale_term(factor, c.yarn_mscale_all_dim)
                                                : mscale_term(factor, 1.0f);
    mscale = ratio * c.rope_attn_factor;
}

// ------------------------------------------------------------------ device

struct Tensor {
    DevWeight w;             // matrices (raw bytes + derived planes)
    float *vec = nullptr;    // 1-D parameters widened to f32 (VectorParameter)
    void *raw = nullptr;
};

template <class T>
static void dev_alloc(T *&p, size_t count) {
    void *v = nullptr;
    SHIELD_CUDA(cudaMalloc(&v, std::max<size_t>(count, 1) * sizeof(T)));
    p = static_cast<T *>(v);
}
template <class T>
static void dev_free(T *&p) {
    if (p) cudaFree((void *)p);
    p = nullptr;
}

// int32 words of attention metadata per token of capacity (plus ATT_INTS_EXTRA):
// per work item (at most one per token and one per request) its request and
// first query (2) and scratch offset (2); per request start, len, pre (3),
// cache keys, values and stride (6) and the append flag (1)
constexpr int64_t ATT_INTS_PER_TOKEN = 16, ATT_INTS_EXTRA = 64;

struct Buffers {
    int64_t cap = 0;  // tokens
    float *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ctx = nullptr, *g = nullptr, *u = nullptr;
    float *kc = nullptr;       // keys after RoPE, chain-major per head (attention's layout)
    int8_t *a8 = nullptr;
    __half *a16 = nullptr;
    float *da = nullptr, *ds = nullptr;
    int32_t *sums = nullptr;
    int32_t *meta = nullptr;   // ids | pos | tok_start | last  (4 * cap)
    float *scores = nullptr;   // attention scores of a request group
    int64_t scores_cap = 0;    // floats
    int32_t *att = nullptr;    // attention work list | start | len | pre | base | caches (ATT_INTS_PER_TOKEN * cap)
    int32_t *h_att = nullptr;  // pinned
    float *logits = nullptr;
    int32_t *verdict = nullptr;
    int32_t *err = nullptr;
    int32_t *h_meta = nullptr;  // pinned
    float *h_logits = nullptr;  // pinned
    void free_all() {
        dev_free(h); dev_free(q); dev_free(k); dev_free(kc); dev_free(v); dev_free(ctx); dev_free(g); dev_free(u);
        dev_free(a8); dev_free(a16); dev_free(da); dev_free(ds); dev_free(sums); dev_free(meta);
        dev_free(logits); dev_free(verdict); dev_free(err); dev_free(scores); dev_free(att);
        if (h_att) cudaFreeHost(h_att);
        h_att = nullptr;
        scores_cap = 0;
        if (h_meta) cudaFreeHost(h_meta);
        if (h_logits) cudaFreeHost(h_logits);
        h_meta = nullptr;
        h_logits = nullptr;
        cap = 0;
    }
};

struct Scratch {  // grow-on-demand buffers of the single-GEMM entry points
    void *p = nullptr;
    size_t bytes = 0;
    void *get(size_t n) {
        if (n > bytes) {
            if (p) cudaFree(p);
            p = nullptr;
            bytes = 0;
            SHIELD_CUDA(cudaMalloc(&p, n));
            bytes = n;
        }
        return p;
    }
    ~Scratch() {
        if (p) cudaFree(p);
    }
};

// Device-side accounting (shield_set_timing / shield_read_timing).
struct Timing {
    int level = 0;
    std::vector<cudaEvent_t> pool;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> fwd, gemm, attn;
    double gemm_ops = 0, gemm_bytes = 0, attn_flops = 0;
    int64_t gemm_launches = 0, launches = 0, tokens = 0, requests = 0, h2d = 0, d2h = 0;
    cudaEvent_t event() {
        if (pool.empty()) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            return e;
        }
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    void recycle() {
        for (auto &p : fwd) { pool.push_back(p.first); pool.push_back(p.second); }
        for (auto &p : gemm) { pool.push_back(p.first); pool.push_back(p.second); }
        for (auto &p : attn) { pool.push_back(p.first); pool.push_back(p.second); }
        fwd.clear();
        gemm.clear();
        attn.clear();
    }
    void reset() {
        recycle();
        gemm_ops = gemm_bytes = attn_flops = 0;
        gemm_launches = launches = tokens = requests = h2d = d2h = 0;
    }
    ~Timing() {
        recycle();
        for (auto e : pool) cudaEventDestroy(e);
    }
};

struct Device {
    int ordinal = 0;
    int sms = 148;  // streaming multiprocessors
    cudaStream_t stream = nullptr;
    Timing timing;
    std::unordered_map<std::string, Tensor> tensors;
    float *cos_t = nullptr, *sin_t = nullptr, *temp = nullptr;
    Buffers buf;
    Scratch sx, sy, sa, sd;
    Scratch sl;  // full-vocabulary logits of a chunk of last positions
    // Upload staging: two pinned halves, so the host copy of one chunk
    // overlaps the DMA of the other (GgufFile mmap -> pinned -> HBM).
    static constexpr size_t STAGE_BYTES = (size_t)32 << 20;
    uint8_t *stage = nullptr;
    cudaEvent_t stage_free[2] = {nullptr, nullptr};
    // System-prompt prefix cache (SystemPromptCache.cs:51-75, KvCache.Snapshot):
    // the prefix's keys after RoPE (chain-major) and values, [layer][pos][kv-dim].
    float *pre_k = nullptr, *pre_v = nullptr;
    // Sequences for incremental forwards (MinistralModel.KvCache): each keeps
    // its keys (after RoPE, chain-major) and values, [layer][position][kv-dim].
    struct Sequence {
        float *k = nullptr, *v = nullptr;
        int32_t cap = 0, len = 0;
    };
    std::unordered_map<int64_t, Sequence> seqs;
    // Captured decode steps, by batch shape (see forward_batch).
    struct GraphEntry {
        cudaGraphExec_t exec = nullptr;
        float *d_logits = nullptr, *h_logits = nullptr;
    };
    std::unordered_map<std::string, GraphEntry> graphs;
    bool no_graphs = false;  // a capture failed on this device: plain launches only
    void clear_graphs() {
        for (auto &kv : graphs) {
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
            if (kv.second.d_logits) cudaFree(kv.second.d_logits);
            if (kv.second.h_logits) cudaFreeHost(kv.second.h_logits);
        }
        graphs.clear();
    }
    ~Device() {
        cudaSetDevice(ordinal);
        for (auto &kv : tensors) {
            if (kv.second.raw) cudaFree(kv.second.raw);
            if (kv.second.vec) cudaFree(kv.second.vec);
            if (kv.second.w.scale_plane) cudaFree(kv.second.w.scale_plane);
            if (kv.second.w.offset_plane) cudaFree(kv.second.w.offset_plane);
            if (kv.second.w.w16) cudaFree(kv.second.w.w16);
        }
        dev_free(cos_t);
        dev_free(sin_t);
        dev_free(temp);
        dev_free(pre_k);
        dev_free(pre_v);
        for (auto &kv : seqs) {
            dev_free(kv.second.k);
            dev_free(kv.second.v);
        }
        clear_graphs();
        if (stage) cudaFreeHost(stage);
        for (auto &e : stage_free)
            if (e) cudaEventDestroy(e);
        buf.free_all();
        if (stream) cudaStreamDestroy(stream);
    }
    const Tensor &get(const std::string &name) const {
        auto it = tensors.find(name);
        if (it == tensors.end()) throw Error(SHIELD_ERR_STATE, "tensor '" + name + "' has not been uploaded");
        return it->second;
    }
};

struct Ctx {
    std::vector<std::unique_ptr<Device>> devs;
    Config cfg;
    bool configured = false;
    int gemm_path = 0;
    int att_rows = 0;             // query rows per attention CTA: 0 = by the grid size
    std::vector<int32_t> prefix;  // token ids whose KV every device holds (empty: none)
    int64_t next_seq = 1;         // sequence ids: (device << 48) | serial
};

static void clear_prefix(Ctx &C) {
    C.prefix.clear();
    for (auto &d : C.devs) {
        cudaSetDevice(d->ordinal);
        dev_free(d->pre_k);
        dev_free(d->pre_v);
    }
}

// Cached keys and values are stale once the weights or the shapes change:
// sequences are emptied (new weights) or freed (new configuration).
static void drop_sequences(Ctx &C, bool free_them) {
    for (auto &d : C.devs) {
        cudaSetDevice(d->ordinal);
        d->clear_graphs();  // they hold the buffers' and the weights' addresses
        for (auto &kv : d->seqs) {
            kv.second.len = 0;
            if (free_them) {
                dev_free(kv.second.k);
                dev_free(kv.second.v);
            }
        }
        if (free_them) d->seqs.clear();
    }
}

// -------------------------------------------------------------- operations

static void check_launch(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Error(SHIELD_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Counts one launch (and, at timing level 2, brackets GEMM launches with events).
static void count_launch(Device &d) { d.timing.launches++; }

static void gemm(Ctx &C, Device &d, const Tensor &W, const QAct &q, float *y, int64_t ldy, int epi) {
    Timing &T = d.timing;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (T.level >= 2) {
        e0 = T.event();
        e1 = T.event();
        if (e0) cudaEventRecord(e0, d.stream);
    }
    bool done = false;
    // 1..16 tokens: the few-token kernels (decode steps, the last rows)
    if ((C.gemm_path == 0 || C.gemm_path == 4) && gemv_small_supports(W.w, q.M)) {
        cudaError_t e = launch_gemv_small(W.w, q, y, ldy, epi, d.stream);
        if (e == cudaSuccess)
            done = true;
        else if (e != cudaErrorNotSupported)
            check_launch(e, "few-token GEMM");
    }
    if (C.gemm_path == 4 && !done) throw Error(SHIELD_ERR_UNSUPPORTED, "the few-token GEMM does not take this shape");
    if (!done && C.gemm_path != 1 && C.gemm_path != 4 && gemm_tc_supports(W.w, q.M)) {
        cudaError_t e = launch_gemm_tc(W.w, q, y, ldy, epi, d.buf.err ? d.buf.err : nullptr, d.stream);
        if (e == cudaSuccess)
            done = true;
        else if (e != cudaErrorNotSupported)
            check_launch(e, "tensor-core GEMM");
    }
    if (!done) {
        if (C.gemm_path >= 2) throw Error(SHIELD_ERR_UNSUPPORTED, "the tensor-core GEMM does not take this shape");
        check_launch(launch_gemm_simt(W.w, nullptr, W.w.rows, q, y, ldy, epi, d.stream), "CUDA-core GEMM");
    }
    count_launch(d);
    if (T.level >= 1) {
        T.gemm_launches++;
        T.gemm_ops += 2.0 * (double)q.M * (double)W.w.rows * (double)W.w.cols;
        T.gemm_bytes += (double)W.w.rows * (double)W.w.row_bytes + (double)q.M * (double)W.w.cols * 1.125 +
                        (double)q.M * (double)W.w.rows * (epi == EPI_ADD ? 8.0 : 4.0);
    }
    if (e1 && e0) {
        cudaEventRecord(e1, d.stream);
        T.gemm.emplace_back(e0, e1);
    }
}

// Projections that share their activations (Q/K/V; gate/up): one
// tensor-core launch covering all of them when the kernel takes them (the
// tiles of every weight run side by side, which matters when few tokens make
// few tiles), else one gemm() each. The outputs are identical either way.
// Rows row_ids[0..n) of a weight for every token (the verdict head, row
// subsets): the few-token kernels up to 16 tokens (every block's dot in
// parallel, then each output's chain in block order), else the CUDA-core
// tiled kernel; the same arithmetic either way. Path 1 keeps the tiled kernel.
static cudaError_t launch_gemm_rows(const Ctx &C, const DevWeight &w, const int32_t *row_ids, int64_t n,
                                    const QAct &q, float *y, int64_t ldy, cudaStream_t s) {
    if (C.gemm_path != 1 && gemv_small_supports(w, q.M)) {
        const cudaError_t e = launch_gemv_rows(w, row_ids, n, q, y, ldy, EPI_STORE, s);
        if (e != cudaErrorNotSupported) return e;
    }
    return launch_gemm_simt(w, row_ids, n, q, y, ldy, EPI_STORE, s);
}

static void gemm_shared_input(Ctx &C, Device &d, int count, const Tensor *const *W, const QAct &q, float *const *ys,
                              const int64_t *lds) {
    const DevWeight *ws[3];
    for (int g = 0; g < count; g++) ws[g] = &W[g]->w;
    const bool tc_path = C.gemm_path == 0 || C.gemm_path == 2 || C.gemm_path == 3;
    bool grouped = count <= 3 && tc_path && !(C.gemm_path == 0 && gemv_small_supports(*ws[0], q.M));
    for (int g = 0; g < count && grouped; g++) grouped = gemm_tc_supports(*ws[g], q.M);
    if (grouped) {
        Timing &T = d.timing;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        if (T.level >= 2) {
            e0 = T.event();
            e1 = T.event();
            if (e0) cudaEventRecord(e0, d.stream);
        }
        const cudaError_t e = launch_gemm_tc_group(ws, ys, lds, count, q, EPI_STORE, d.buf.err, d.stream);
        if (e == cudaSuccess) {
            count_launch(d);
            if (T.level >= 1) {
                T.gemm_launches++;
                for (int g = 0; g < count; g++) {
                    T.gemm_ops += 2.0 * (double)q.M * (double)ws[g]->rows * (double)ws[g]->cols;
                    T.gemm_bytes += (double)ws[g]->rows * (double)ws[g]->row_bytes + (double)q.M * (double)ws[g]->rows * 4.0;
                }
                T.gemm_bytes += (double)q.M * (double)ws[0]->cols * 1.125;  // the shared activations, read once
            }
            if (e1 && e0) {
                cudaEventRecord(e1, d.stream);
                T.gemm.emplace_back(e0, e1);
            }
            return;
        }
        if (e != cudaErrorNotSupported) check_launch(e, "grouped tensor-core GEMM");
        if (e0) T.pool.push_back(e0);
        if (e1) T.pool.push_back(e1);
    }
    for (int g = 0; g < count; g++) gemm(C, d, *W[g], q, ys[g], lds[g], EPI_STORE);
}

static QAct qact(Buffers &b, int64_t M, int64_t K) {
    QAct q;
    q.a8 = b.a8;
    q.a16 = b.a16;
    q.da = b.da;
    q.ds = b.ds;
    q.sums = b.sums;
    q.M = M;
    q.K = K;
    return q;
}

static void ensure_buffers(Ctx &C, Device &d) {
    const Config &c = C.cfg;
    int64_t T = c.max_batch_tokens;
    if (d.buf.cap >= T) return;
    d.buf.free_all();
    int64_t K = c.max_k();
    dev_alloc(d.buf.h, (size_t)(T * c.hidden));
    dev_alloc(d.buf.q, (size_t)(T * c.qdim()));
    dev_alloc(d.buf.k, (size_t)(T * c.kvdim()));
    dev_alloc(d.buf.kc, (size_t)(T * c.kvdim()));
    dev_alloc(d.buf.v, (size_t)(T * c.kvdim()));
    dev_alloc(d.buf.ctx, (size_t)(T * c.qdim()));
    dev_alloc(d.buf.g, (size_t)(T * c.ffn));
    dev_alloc(d.buf.u, (size_t)(T * c.ffn));
    dev_alloc(d.buf.a8, (size_t)(T * K));
    dev_alloc(d.buf.a16, (size_t)(T * K));
    dev_alloc(d.buf.da, (size_t)(T * K / 32));
    dev_alloc(d.buf.ds, (size_t)(T * K / 32));
    dev_alloc(d.buf.sums, (size_t)(T * K / 32));
    dev_alloc(d.buf.meta, (size_t)(4 * T));
    dev_alloc(d.buf.logits, (size_t)(T * 64));
    dev_alloc(d.buf.verdict, 1024);
    dev_alloc(d.buf.err, 1);
    SHIELD_CUDA(cudaMemsetAsync(d.buf.err, 0, 4, d.stream));
    SHIELD_CUDA(cudaMallocHost((void **)&d.buf.h_meta, (size_t)(4 * T) * 4));
    SHIELD_CUDA(cudaMallocHost((void **)&d.buf.h_logits, (size_t)(T * 64) * 4));
    // attention scratch: at least one work item of the longest request, at
    // most 4 GiB (a micro-batch needing more is attended in several launches)
    int64_t one = attention_scratch_floats(c.max_positions, c.n_kv_heads, attention_rows_per_cta());
    int64_t all = std::min<int64_t>((int64_t)1 << 30, (int64_t)c.n_heads * T * c.max_positions);
    d.buf.scores_cap = std::max(one, all);
    dev_alloc(d.buf.scores, (size_t)d.buf.scores_cap);
    dev_alloc(d.buf.att, (size_t)(ATT_INTS_PER_TOKEN * T + ATT_INTS_EXTRA));
    SHIELD_CUDA(cudaMallocHost((void **)&d.buf.h_att, (size_t)(ATT_INTS_PER_TOKEN * T + ATT_INTS_EXTRA) * 4));
    d.buf.cap = T;
}

static void check_device_error(Device &d) {
    int32_t e = 0;
    SHIELD_CUDA(cudaMemcpyAsync(&e, d.buf.err, 4, cudaMemcpyDeviceToHost, d.stream));
    SHIELD_CUDA(cudaStreamSynchronize(d.stream));
    if (e) {
        SHIELD_CUDA(cudaMemsetAsync(d.buf.err, 0, 4, d.stream));
        if (e == 2) throw Error(SHIELD_ERR_RANGE, "a token id is outside the embedding table");
        throw Error(SHIELD_ERR_TIMEOUT, "a device-side wait gave up (error word " + std::to_string(e) + ")");
    }
}

struct Batch {  // one micro-batch of whole requests on one device
    std::vector<int32_t> req;     // indices into the caller's request list
    std::vector<int64_t> start;   // batch-local first token of each request
    std::vector<int32_t> len;     // tokens forwarded (after any cached positions)
    std::vector<int32_t> pre;     // cached positions in front of them
    // where those cached positions live when not the system-prompt prefix: a
    // sequence's cache (keys, values, floats per layer), and whether the
    // forwarded tokens are appended to it (empty vectors: the prefix)
    std::vector<const float *> ck, cv;
    std::vector<int64_t> cstride;
    std::vector<uint8_t> append;
    int64_t tokens = 0;
};

// MinistralModel.ForwardAsync (MinistralModel.cs:183-271) over a packed
// micro-batch. A request with pre > 0 continues from the cached system-prompt
// prefix (its tokens sit at positions pre, pre+1, ..); otherwise it starts at
// position 0 with an empty cache. Leaves verdict logits (R x nv) in
// d.buf.h_logits after a stream sync. full_logits (host, R x vocab): the whole
// tied head at every last position instead. store_prefix: the batch is the
// prefix alone; its per-layer keys and values are kept in d.pre_k / d.pre_v.
static void forward_batch(Ctx &C, Device &d, const int32_t *ids_host, const Batch &B, int nv,
                          const volatile int32_t *cancel, int capture_layer, int capture_what, float *capture,
                          float *full_logits = nullptr, bool store_prefix = false, bool graph = false) {
    const Config &c = C.cfg;
    const int64_t M = B.tokens;
    const int R = (int)B.req.size();
    cudaStream_t s = d.stream;
    Buffers &b = d.buf;
    int32_t *hm = b.h_meta;
    int32_t *h_ids = hm, *h_pos = hm + M, *h_start = hm + 2 * M, *h_last = hm + 3 * M;
    auto pre_of = [&](int r) { return B.pre.empty() ? 0 : B.pre[r]; };
    bool any_pre = false;
    for (int r = 0; r < R; r++) {
        int64_t st = B.start[r];
        const int32_t pre = pre_of(r);
        any_pre |= pre > 0;
        for (int32_t p = 0; p < B.len[r]; p++) {
            h_ids[st + p] = ids_host[st + p];
            h_pos[st + p] = pre + p;
            h_start[st + p] = (int32_t)st;
        }
        h_last[r] = (int32_t)(st + B.len[r] - 1);
    }
    const int64_t P = (int64_t)C.prefix.size();
    // each request's cache: its sequence's, else the system-prompt prefix
    std::vector<const float *> ck(R, nullptr), cv(R, nullptr);
    std::vector<int64_t> cstride(R, 0);
    std::vector<uint8_t> append(R, 0);
    bool any_append = false;
    for (int r = 0; r < R; r++) {
        if (!B.ck.empty() && B.ck[r]) {
            ck[r] = B.ck[r];
            cv[r] = B.cv[r];
            cstride[r] = B.cstride[r];
            append[r] = B.append[r];
            any_append |= append[r] != 0;
        } else if (pre_of(r) > 0) {
            if (!d.pre_k || !d.pre_v) throw Error(SHIELD_ERR_STATE, "no prefix cached on this device");
            ck[r] = d.pre_k;
            cv[r] = d.pre_v;
            cstride[r] = P * c.kvdim();
        }
    }
    const int32_t *d_ids = b.meta, *d_pos = b.meta + M, *d_last = b.meta + 3 * M;

    // attention: one work item per (request, rows/G query tokens), longest
    // first (the CTAs of long rows start early instead of forming a tail), in
    // groups whose scratch fits the buffer. 128 query rows per CTA, or 64
    // when 128-row items would give fewer than two CTAs per SM (a single
    // short request) or be less than half filled (decode steps: one token per
    // request). 32- and 16-row CTAs were slower in both cases (fewer threads
    // to load each key tile; config 1 +2% / +7%, one-sequence decode +21%).
    const int G = c.n_heads / c.n_kv_heads;
    int att_rows = C.att_rows ? C.att_rows : attention_rows_per_cta();
    if (!C.att_rows && (att_rows / 2) % G == 0) {
        int64_t items = 0, rows_used = 0;
        for (int r = 0; r < R; r++) {
            items += (B.len[r] + att_rows / G - 1) / (att_rows / G);
            rows_used += (int64_t)B.len[r] * G;
        }
        if (items * c.n_kv_heads < 2 * (int64_t)d.sms || 2 * rows_used < items * att_rows) att_rows /= 2;
    }
    if (att_rows % G) throw Error(SHIELD_ERR_UNSUPPORTED, "attention rows per CTA must be a multiple of heads per KV head");
    const int QT = att_rows / G;
    struct AttGroup { int w0, nw; };
    struct AttItem { int64_t kend; int32_t r, q0; };
    std::vector<AttItem> items;
    for (int r = 0; r < R; r++)
        for (int q0 = 0; q0 < B.len[r]; q0 += QT)
            items.push_back({(int64_t)pre_of(r) + std::min(q0 + QT, B.len[r]), r, q0});
    std::stable_sort(items.begin(), items.end(), [](const AttItem &a, const AttItem &b) { return a.kend > b.kend; });
    std::vector<AttGroup> groups;
    std::vector<int32_t> work;
    std::vector<int64_t> wbase;
    {
        int64_t used = 0;
        AttGroup cur{0, 0};
        for (const AttItem &it : items) {
            const int64_t need = attention_scratch_floats(it.kend, c.n_kv_heads, att_rows);
            if (used + need > b.scores_cap && cur.nw > 0) {
                groups.push_back(cur);
                cur = AttGroup{(int)wbase.size(), 0};
                used = 0;
            }
            wbase.push_back(used);
            used += need;
            work.push_back(it.r);
            work.push_back(it.q0);
            cur.nw++;
        }
        if (cur.nw > 0) groups.push_back(cur);
    }
    const int n_work = (int)(work.size() / 2);
    // algorithmic attention flops of one layer: q.k and p.v, 2 flops per
    // multiply-add, over every (query, key) pair a causal row attends to
    double attn_flops_layer = 0;
    for (int r = 0; r < R; r++) {
        const double len = B.len[r], pre = pre_of(r);
        attn_flops_layer += 4.0 * c.n_heads * c.head_dim * (len * pre + len * (len + 1) / 2);
    }
    if (4 * n_work + 12 * R + 8 > ATT_INTS_PER_TOKEN * b.cap + ATT_INTS_EXTRA)
        throw Error(SHIELD_ERR_RANGE, "attention work list exceeds its buffer");
    int32_t *ha = b.h_att;
    memcpy(ha, work.data(), work.size() * 4);
    int32_t *ha_start = ha + 2 * n_work, *ha_len = ha_start + R, *ha_pre = ha_len + R;
    for (int r = 0; r < R; r++) {
        ha_start[r] = (int32_t)B.start[r];
        ha_len[r] = B.len[r];
        ha_pre[r] = pre_of(r);
    }
    int64_t base_off = (2 * n_work + 3 * R + 1) / 2 * 2;  // int64 arrays on an 8-byte boundary
    memcpy(ha + base_off, wbase.data(), (size_t)n_work * 8);
    const int64_t ck_off = base_off + 2 * n_work, cv_off = ck_off + 2 * R, cs_off = cv_off + 2 * R,
                  ap_off = cs_off + 2 * R;
    memcpy(ha + ck_off, ck.data(), (size_t)R * 8);
    memcpy(ha + cv_off, cv.data(), (size_t)R * 8);
    memcpy(ha + cs_off, cstride.data(), (size_t)R * 8);
    memcpy(ha + ap_off, append.data(), (size_t)R);
    size_t att_bytes = (size_t)(ap_off * 4 + R);
    const int2 *d_work = reinterpret_cast<const int2 *>(b.att);
    const int32_t *d_rstart = b.att + 2 * n_work, *d_rlen = d_rstart + R, *d_rpre = d_rlen + R;
    const int64_t *d_wbase = reinterpret_cast<const int64_t *>(b.att + base_off);
    const float *const *d_ck = reinterpret_cast<const float *const *>(b.att + ck_off);
    const float *const *d_cv = reinterpret_cast<const float *const *>(b.att + cv_off);
    const int64_t *d_cs = reinterpret_cast<const int64_t *>(b.att + cs_off);
    const uint8_t *d_app = reinterpret_cast<const uint8_t *>(b.att + ap_off);

    // Everything from here on is stream work. A decode-shaped batch (graph)
    // replays a CUDA graph captured the first time its shape was seen: the
    // host arrays above are re-read from pinned memory by its copy nodes.
    Timing &T = d.timing;
    Device::GraphEntry *ge = nullptr;
    bool capturing = false;
    std::string graph_key;
    const int saved_level = T.level;
    if (graph) {
        std::string key = std::to_string(M) + "/" + std::to_string(R) + "/" + std::to_string(nv) + "/" +
                          std::to_string(att_rows) + "/" +
                          (full_logits ? "f" : "-") + (any_append ? "a" : "-");
        for (const AttGroup &ag : groups) key += "/" + std::to_string(ag.w0) + ":" + std::to_string(ag.nw);
        auto it = d.graphs.find(key);
        if (it != d.graphs.end()) {
            ge = &it->second;
            SHIELD_CUDA(cudaGraphLaunch(ge->exec, s));
            SHIELD_CUDA(cudaStreamSynchronize(s));
            check_device_error(d);
            if (full_logits) memcpy(full_logits, ge->h_logits, (size_t)R * c.vocab * 4);
            else if (nv > 0) memcpy(b.h_logits, ge->h_logits, (size_t)R * nv * 4);
            return;
        }
        Device::GraphEntry e;
        const size_t out_floats = (size_t)R * (full_logits ? c.vocab : nv);
        dev_alloc(e.d_logits, std::max<size_t>(out_floats, 1));
        SHIELD_CUDA(cudaMallocHost(reinterpret_cast<void **>(&e.h_logits), std::max<size_t>(out_floats, 1) * 4));
        ge = &d.graphs.emplace(key, e).first->second;
        graph_key = key;
        T.level = 0;
        SHIELD_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        capturing = true;
    }
    // a failure while capturing ends the capture and drops the half-made entry
    struct CaptureGuard {
        Device &d;
        Timing &T;
        bool &active;
        const std::string &key;
        int level;
        ~CaptureGuard() {
            if (!active) return;
            cudaGraph_t g = nullptr;
            cudaStreamEndCapture(d.stream, &g);
            if (g) cudaGraphDestroy(g);
            T.level = level;
            auto it = d.graphs.find(key);
            if (it != d.graphs.end()) {
                if (it->second.d_logits) cudaFree(it->second.d_logits);
                if (it->second.h_logits) cudaFreeHost(it->second.h_logits);
                d.graphs.erase(it);
            }
        }
    } guard{d, T, capturing, graph_key, saved_level};
    SHIELD_CUDA(cudaMemcpyAsync(b.meta, hm, (size_t)(3 * M + R) * 4, cudaMemcpyHostToDevice, s));
    SHIELD_CUDA(cudaMemcpyAsync(b.att, ha, att_bytes, cudaMemcpyHostToDevice, s));
    cudaEvent_t f0 = nullptr, f1 = nullptr;
    if (T.level >= 1) {
        T.h2d += (3 * M + R) * 4;
        T.tokens += M;
        T.requests += R;
        f0 = T.event();
        f1 = T.event();
        if (f0) cudaEventRecord(f0, s);
    }

    const Tensor &emb = d.get("token_embd.weight");
    count_launch(d), check_launch(launch_embed(emb.w, d_ids, M, b.h, b.err, s), "embedding gather");
    const float scale = 1.0f / sqrtf((float)c.head_dim);
    auto cap = [&](int l, int what, const float *src, int64_t width) {
        if (l == capture_layer && capture && capture_what == what)
            SHIELD_CUDA(cudaMemcpyAsync(capture, src, (size_t)(M * width) * 4, cudaMemcpyDeviceToHost, s));
    };
    for (int l = 0; l < c.n_layers; l++) {
        if (cancel && *cancel && !capturing) {
            cudaStreamSynchronize(s);
            throw Error(SHIELD_ERR_CANCELLED, "cancelled");
        }
        std::string p = "blk." + std::to_string(l) + ".";
        const Tensor &an = d.get(p + "attn_norm.weight"), &fn = d.get(p + "ffn_norm.weight");
        const Tensor &wq = d.get(p + "attn_q.weight"), &wk = d.get(p + "attn_k.weight");
        const Tensor &wv = d.get(p + "attn_v.weight"), &wo = d.get(p + "attn_output.weight");
        const Tensor &wg = d.get(p + "ffn_gate.weight"), &wu = d.get(p + "ffn_up.weight");
        const Tensor &wd = d.get(p + "ffn_down.weight");

        QAct qa = qact(b, M, c.hidden);
        bool want_norm = l == capture_layer && capture_what == SHIELD_ACT_ATTN_NORM;
        count_launch(d), check_launch(launch_rmsnorm_quant(b.h, nullptr, M, c.hidden, an.vec, c.eps, want_norm ? b.ctx : nullptr, qa, s),
                     "attn norm");
        cap(l, SHIELD_ACT_ATTN_NORM, b.ctx, c.hidden);
        {
            const Tensor *W[3] = {&wq, &wk, &wv};
            float *ys[3] = {b.q, b.k, b.v};
            const int64_t lds[3] = {c.qdim(), c.kvdim(), c.kvdim()};
            gemm_shared_input(C, d, 3, W, qa, ys, lds);
        }
        count_launch(d), check_launch(launch_rope_qk(b.q, c.n_heads, b.k, c.n_kv_heads, M, c.head_dim, d_pos, d.cos_t,
                                                    d.sin_t, c.rope_half, d.temp, b.ctx, b.kc,
                                                    l == capture_layer && capture_what == SHIELD_ACT_Q_ROPE,
                                                    l == capture_layer && capture_what == SHIELD_ACT_K_ROPE, s),
                                     "rope");
        cap(l, SHIELD_ACT_Q_ROPE, b.q, c.qdim());
        cap(l, SHIELD_ACT_K_ROPE, b.k, c.kvdim());
        cap(l, SHIELD_ACT_V, b.v, c.kvdim());
        const int64_t layer_kv = (int64_t)l * P * c.kvdim();
        if (store_prefix) {
            SHIELD_CUDA(cudaMemcpyAsync(d.pre_k + layer_kv, b.kc, (size_t)(M * c.kvdim()) * 4, cudaMemcpyDeviceToDevice, s));
            SHIELD_CUDA(cudaMemcpyAsync(d.pre_v + layer_kv, b.v, (size_t)(M * c.kvdim()) * 4, cudaMemcpyDeviceToDevice, s));
        }
        AttArgs A;
        // the chain-major queries live in ctx: a group's PV writes only its
        // own requests' rows, which no later group's scores read
        A.qc = b.ctx;
        A.kc = b.kc;
        A.v = b.v;
        A.ctx = b.ctx;
        A.scores = b.scores;
        A.req_start = d_rstart;
        A.req_len = d_rlen;
        A.req_pre = d_rpre;
        A.cache_k = d_ck;
        A.cache_v = d_cv;
        A.cache_stride = d_cs;
        A.layer = l;
        A.n_heads = c.n_heads;
        A.n_kv_heads = c.n_kv_heads;
        A.scale = scale;
        if (any_append)
            count_launch(d), check_launch(launch_append_kv(A, d_app, R, M, (int)c.kvdim(), s), "append to KV caches");
        cudaEvent_t a0 = nullptr, a1 = nullptr;
        if (T.level >= 2) {
            a0 = T.event();
            a1 = T.event();
            if (a0) cudaEventRecord(a0, s);
        }
        for (const AttGroup &ag : groups) {
            d.timing.launches += 1;
            A.work = d_work + ag.w0;
            A.work_base = d_wbase + ag.w0;
            check_launch(launch_attention(A, ag.nw, c.head_dim, att_rows, s), "attention");
        }
        if (a0 && a1) {
            cudaEventRecord(a1, s);
            T.attn.emplace_back(a0, a1);
            T.attn_flops += attn_flops_layer;
        }
        cap(l, SHIELD_ACT_ATTN_WEIGHTED, b.ctx, c.qdim());
        QAct qc = qact(b, M, c.qdim());
        count_launch(d), check_launch(launch_quantize(b.ctx, M, c.qdim(), c.qdim(), qc, s), "quantize context");
        gemm(C, d, wo, qc, b.h, c.hidden, EPI_ADD);
        cap(l, SHIELD_ACT_POST_ATTN, b.h, c.hidden);

        count_launch(d), check_launch(launch_rmsnorm_quant(b.h, nullptr, M, c.hidden, fn.vec, c.eps, nullptr, qa, s), "ffn norm");
        {
            const Tensor *W[2] = {&wg, &wu};
            float *ys[2] = {b.g, b.u};
            const int64_t lds[2] = {c.ffn, c.ffn};
            gemm_shared_input(C, d, 2, W, qa, ys, lds);
        }
        QAct qf = qact(b, M, c.ffn);
        count_launch(d), check_launch(launch_swiglu_quantize(b.g, b.u, M, c.ffn, qf, s), "swiglu + quantize");
        gemm(C, d, wd, qf, b.h, c.hidden, EPI_ADD);
        cap(l, SHIELD_ACT_OUTPUT, b.h, c.hidden);
    }
    if (full_logits) {
        // last position of every request -> final norm -> the whole tied head
        // (VerdictLogitsAsync, ShieldstralModerator.cs:269-277), in row chunks
        const Tensor &on = d.get("output_norm.weight");
        QAct qh = qact(b, R, c.hidden);
        count_launch(d), check_launch(launch_rmsnorm_quant(b.h, d_last, R, c.hidden, on.vec, c.eps, nullptr, qh, s), "final norm");
        const int64_t V = c.vocab, nb = c.hidden / 32;
        const int64_t chunk = ge ? R : std::max<int64_t>(1, std::min<int64_t>(R, ((int64_t)256 << 20) / (V * 4)));
        float *dl = ge ? ge->d_logits : static_cast<float *>(d.sl.get((size_t)(chunk * V) * 4));
        float *out = ge ? ge->h_logits : full_logits;
        for (int64_t r0 = 0; r0 < R; r0 += chunk) {
            QAct qc = qh;
            qc.M = std::min<int64_t>(chunk, R - r0);
            qc.a8 = qh.a8 + r0 * c.hidden;
            qc.a16 = qh.a16 + r0 * c.hidden;
            qc.da = qh.da + r0 * nb;
            qc.ds = qh.ds + r0 * nb;
            qc.sums = qh.sums + r0 * nb;
            gemm(C, d, emb, qc, dl, V, EPI_STORE);
            SHIELD_CUDA(cudaMemcpyAsync(out + r0 * V, dl, (size_t)(qc.M * V) * 4, cudaMemcpyDeviceToHost, s));
            if (T.level >= 1) T.d2h += qc.M * V * 4;
        }
        if (!ge) SHIELD_CUDA(cudaStreamSynchronize(s));
    } else if (nv > 0) {
        // last position of every request -> final norm -> verdict rows of the tied head
        const Tensor &on = d.get("output_norm.weight");
        QAct qh = qact(b, R, c.hidden);
        count_launch(d), check_launch(launch_rmsnorm_quant(b.h, d_last, R, c.hidden, on.vec, c.eps, nullptr, qh, s), "final norm");
        count_launch(d), check_launch(launch_gemm_rows(C, emb.w, b.verdict, nv, qh, b.logits, nv, s), "verdict head");
        if (f1 && f0) {
            cudaEventRecord(f1, s);
            T.fwd.emplace_back(f0, f1);
            f0 = f1 = nullptr;
        }
        SHIELD_CUDA(cudaMemcpyAsync(ge ? ge->h_logits : b.h_logits, b.logits, (size_t)R * nv * 4,
                                    cudaMemcpyDeviceToHost, s));
        if (T.level >= 1) T.d2h += (int64_t)R * nv * 4;
    }
    if (f1 && f0) {
        cudaEventRecord(f1, s);
        T.fwd.emplace_back(f0, f1);
    }
    if (capturing) {
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamEndCapture(s, &g);
        capturing = false;  // the guard has nothing left to undo
        T.level = saved_level;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&ge->exec, g, 0);
        if (g) cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            d.clear_graphs();
            throw Error(SHIELD_ERR_CUDA, std::string("decode graph: ") + cudaGetErrorString(e));
        }
        SHIELD_CUDA(cudaGraphLaunch(ge->exec, s));
        SHIELD_CUDA(cudaStreamSynchronize(s));
        check_device_error(d);
        if (full_logits) memcpy(full_logits, ge->h_logits, (size_t)R * c.vocab * 4);
        else if (nv > 0) memcpy(b.h_logits, ge->h_logits, (size_t)R * nv * 4);
        return;
    }
    check_device_error(d);
}

// ShieldstralModerator.Score (ShieldstralModerator.cs:348-364).
static void score_one(const float *v, int n_yes, int n_no, float &score, float &yes, float &no) {
    float y = -INFINITY, n = -INFINITY;
    for (int i = 0; i < n_yes; i++)
        if (v[i] > y) y = v[i];
    for (int i = 0; i < n_no; i++)
        if (v[n_yes + i] > n) n = v[n_yes + i];
    float m = fmaxf(y, n);
    float ey = expf(y - m), en = expf(n - m);
    score = ey / (ey + en);
    yes = y;
    no = n;
}

static void upload_rope_tables(Ctx &C, Device &d) {
    const Config &c = C.cfg;
    int P = c.max_positions, half = c.rope_half;
    std::vector<float> cs((size_t)P * half), sn((size_t)P * half), tp(P, 1.0f);
    bool any_temp = false;
    for (int p = 0; p < P; p++) {
        for (int i = 0; i < half; i++) {
            float theta = (float)p * c.freqs[i];
            cs[(size_t)p * half + i] = cosf(theta) * c.mscale;
            sn[(size_t)p * half + i] = sinf(theta) * c.mscale;
        }
        if (c.orig_ctx > 0 && c.temp_beta != 0.0f) {
            float interval = floorf((float)p / (float)c.orig_ctx);
            if (interval != 0.0f) {
                float lg = logf(1.0f + interval);
                float f = c.temp_beta * lg;
                tp[p] = 1.0f + f;
                any_temp = true;
            }
        }
    }
    SHIELD_CUDA(cudaSetDevice(d.ordinal));
    dev_free(d.cos_t);
    dev_free(d.sin_t);
    dev_free(d.temp);
    dev_alloc(d.cos_t, cs.size());
    dev_alloc(d.sin_t, sn.size());
    SHIELD_CUDA(cudaMemcpy(d.cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    SHIELD_CUDA(cudaMemcpy(d.sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    if (any_temp) {
        dev_alloc(d.temp, tp.size());
        SHIELD_CUDA(cudaMemcpy(d.temp, tp.data(), tp.size() * 4, cudaMemcpyHostToDevice));
    }
}

static void set_config(Ctx &C, const shield_config *in) {
    if (!in) throw Error(SHIELD_ERR_ARG, "config is null");
    const shield_config &c = *in;
    if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
        c.vocab <= 0)
        throw Error(SHIELD_ERR_ARG, "every model dimension must be positive");
    if (c.n_heads % c.n_kv_heads)
        throw Error(SHIELD_ERR_SHAPE, std::to_string(c.n_heads) + " attention heads do not divide into " +
                                          std::to_string(c.n_kv_heads) + " KV heads");
    if (c.hidden % 32 || c.ffn % 32 || (c.n_heads * c.head_dim) % 32)
        throw Error(SHIELD_ERR_UNSUPPORTED, "hidden, ffn and q dimensions must be multiples of 32");
    if (c.head_dim != 128 || 128 % (c.n_heads / c.n_kv_heads))
        throw Error(SHIELD_ERR_UNSUPPORTED, "the attention kernels take head_dim 128 and a power-of-two GQA group");
    Config cfg;
    cfg.n_layers = c.n_layers;
    cfg.hidden = c.hidden;
    cfg.n_heads = c.n_heads;
    cfg.n_kv_heads = c.n_kv_heads;
    cfg.head_dim = c.head_dim;
    cfg.ffn = c.ffn;
    cfg.vocab = c.vocab;
    cfg.eps = c.rms_eps;
    if (c.n_rope_freqs > 0) {
        if (!c.rope_freqs || c.n_rope_freqs * 2 > c.head_dim) throw Error(SHIELD_ERR_ARG, "bad rope frequency table");
        cfg.freqs.assign(c.rope_freqs, c.rope_freqs + c.n_rope_freqs);
        cfg.mscale = c.rope_mscale;
    } else {
        if (c.rope_dim <= 0 || c.rope_dim > c.head_dim || c.rope_dim % 2)
            throw Error(SHIELD_ERR_ARG, "rope_dim must be even and at most head_dim");
        rope_freqs(c, cfg.freqs, cfg.mscale);
    }
    cfg.rope_half = (int)cfg.freqs.size();
    cfg.temp_beta = c.attn_temperature_beta;
    cfg.orig_ctx = c.rope_orig_ctx;
    cfg.max_positions = c.max_positions > 0 ? c.max_positions : 8192;
    cfg.max_batch_tokens = c.max_batch_tokens > 0 ? c.max_batch_tokens : 16384;
    if (cfg.max_batch_tokens < cfg.max_positions) cfg.max_batch_tokens = cfg.max_positions;
    clear_prefix(C);
    drop_sequences(C, true);
    C.cfg = cfg;
    C.configured = true;
    for (auto &d : C.devs) {
        upload_rope_tables(C, *d);
        d->buf.free_all();
    }
}

// Host bytes (pageable, e.g. the GGUF mmap) to device memory in 32 MB chunks
// through the device's two pinned staging halves: the memcpy into one half
// runs while the DMA out of the other is in flight.
static void stage_to_device(Device &d, void *dst, const void *src, size_t nbytes) {
    if (!d.stage) {
        SHIELD_CUDA(cudaHostAlloc(reinterpret_cast<void **>(&d.stage), 2 * Device::STAGE_BYTES, cudaHostAllocDefault));
        for (auto &e : d.stage_free) SHIELD_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    const uint8_t *in = static_cast<const uint8_t *>(src);
    uint8_t *out = static_cast<uint8_t *>(dst);
    for (size_t off = 0, k = 0; off < nbytes; off += Device::STAGE_BYTES, k ^= 1) {
        const size_t n = std::min(Device::STAGE_BYTES, nbytes - off);
        uint8_t *half = d.stage + k * Device::STAGE_BYTES;
        SHIELD_CUDA(cudaEventSynchronize(d.stage_free[k]));  // its previous DMA has finished
        memcpy(half, in + off, n);
        SHIELD_CUDA(cudaMemcpyAsync(out + off, half, n, cudaMemcpyHostToDevice, d.stream));
        SHIELD_CUDA(cudaEventRecord(d.stage_free[k], d.stream));
    }
}

// Runs fn(device) for every GPU of the context, in parallel host threads when
// there are several; the first failure is rethrown.
template <class Fn>
static void for_each_device(Ctx &C, Fn fn) {
    const int D = (int)C.devs.size();
    if (D == 1) {
        fn(*C.devs[0]);
        return;
    }
    std::vector<std::string> errors(D);
    std::vector<shield_status> codes(D, SHIELD_OK);
    std::vector<std::thread> th;
    for (int di = 0; di < D; di++)
        th.emplace_back([&, di] {
            try {
                fn(*C.devs[di]);
            } catch (const Error &e) {
                codes[di] = e.code;
                errors[di] = e.what();
            } catch (const std::exception &e) {
                codes[di] = SHIELD_ERR_CUDA;
                errors[di] = e.what();
            }
        });
    for (auto &t : th) t.join();
    for (int di = 0; di < D; di++)
        if (codes[di] != SHIELD_OK) throw Error(codes[di], errors[di]);
}

static void upload(Ctx &C, const char *name, uint32_t type, int64_t rows, int64_t cols, const void *bytes,
                   size_t nbytes) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "shield_set_config must come before uploads");
    if (!name || !bytes) throw Error(SHIELD_ERR_ARG, "name and bytes must be non-null");
    if (rows <= 0 || cols <= 0) throw Error(SHIELD_ERR_ARG, "rows and cols must be positive");
    clear_prefix(C);  // cached keys and values were computed with the old weights
    drop_sequences(C, false);
    int64_t rb = row_bytes_of((int)type, cols);
    if (rb < 0) throw Error(SHIELD_ERR_UNSUPPORTED, std::string(name) + ": type " + std::to_string(type) +
                                                         " has no kernel, or cols is not a multiple of 32");
    if ((size_t)(rb * rows) != nbytes)
        throw Error(SHIELD_ERR_ARG, std::string(name) + ": expected " + std::to_string(rb * rows) + " bytes, got " +
                                        std::to_string(nbytes));
    std::string n(name);
    bool is_vector = n.size() > 11 && n.compare(n.size() - 11, 11, "norm.weight") == 0;
    const Config &c = C.cfg;
    if (n == "token_embd.weight" && (cols != c.hidden || rows != c.vocab))
        throw Error(SHIELD_ERR_SHAPE, "token_embd is " + std::to_string(rows) + "x" + std::to_string(cols) +
                                          " but the model is vocab " + std::to_string(c.vocab) + " x hidden " +
                                          std::to_string(c.hidden));
    if (is_vector && rows * cols != c.hidden) throw Error(SHIELD_ERR_SHAPE, n + " must have hidden elements");
    if (!is_vector && (type == T_F32 || type == T_F16))
        throw Error(SHIELD_ERR_UNSUPPORTED, n + ": float matrices are outside the integer path");
    // every GPU in its own host thread; bytes go through that GPU's pinned
    // staging, and the planes and the f16 copy are built on its stream
    auto one = [&](Device &d) {
        SHIELD_CUDA(cudaSetDevice(d.ordinal));
        SHIELD_CUDA(cudaStreamSynchronize(d.stream));
        auto old = d.tensors.find(n);
        if (old != d.tensors.end()) {
            if (old->second.raw) cudaFree(old->second.raw);
            if (old->second.vec) cudaFree(old->second.vec);
            if (old->second.w.scale_plane) cudaFree(old->second.w.scale_plane);
            if (old->second.w.offset_plane) cudaFree(old->second.w.offset_plane);
            if (old->second.w.w16) cudaFree(old->second.w.w16);
            d.tensors.erase(old);
        }
        Tensor t;
        if (is_vector) {
            std::vector<float> f((size_t)(rows * cols));
            if (type == T_F32) {
                memcpy(f.data(), bytes, f.size() * 4);
            } else {
                const uint16_t *hsrc = static_cast<const uint16_t *>(bytes);
                for (size_t i = 0; i < f.size(); i++) {
                    __half_raw r;
                    r.x = hsrc[i];
                    f[i] = __half2float(__half(r));
                }
            }
            dev_alloc(t.vec, f.size());
            SHIELD_CUDA(cudaMemcpy(t.vec, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
        } else {
            SHIELD_CUDA(cudaMalloc(&t.raw, nbytes + 64));
            stage_to_device(d, t.raw, bytes, nbytes);
            t.w.type = (int)type;
            t.w.rows = rows;
            t.w.cols = cols;
            t.w.row_bytes = rb;
            t.w.data = static_cast<const uint8_t *>(t.raw);
            dev_alloc(t.w.scale_plane, (size_t)(rows * (cols / 32)));
            if (type == T_Q4_1 || type == T_Q5_1) dev_alloc(t.w.offset_plane, (size_t)(rows * (cols / 32)));
            check_launch(launch_build_planes(t.w, d.stream), "scale planes");
            // layer matrices also get an f16 copy for long token batches (the tied
            // embedding/head is only ever read a few rows at a time)
            if (n.compare(0, 4, "blk.") == 0 && cols % 256 == 0 && rows % 16 == 0) {
                dev_alloc(t.w.w16, (size_t)(rows * cols));
                check_launch(launch_unpack_f16(t.w, d.stream), "f16 weight copy");
            }
            SHIELD_CUDA(cudaStreamSynchronize(d.stream));
        }
        d.tensors.emplace(n, t);
    };
    for_each_device(C, one);
}

static void validate_ids(const Ctx &C, const int32_t *ids, int64_t n) {
    for (int64_t i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= C.cfg.vocab)
            throw Error(SHIELD_ERR_RANGE, "token id " + std::to_string(ids[i]) + " is outside the " +
                                              std::to_string(C.cfg.vocab) + "-entry embedding table");
}

// Packs a device's requests (in the given order) into micro-batches.
static std::vector<Batch> make_batches(const Ctx &C, const std::vector<int32_t> &reqs, const int64_t *offsets,
                                       const std::vector<int32_t> &pre) {
    std::vector<Batch> out;
    Batch cur;
    for (int32_t r : reqs) {
        int32_t len = (int32_t)(offsets[r + 1] - offsets[r]) - pre[r];
        if (cur.tokens + len > C.cfg.max_batch_tokens && !cur.req.empty()) {
            out.push_back(cur);
            cur = Batch();
        }
        cur.req.push_back(r);
        cur.start.push_back(cur.tokens);
        cur.len.push_back(len);
        cur.pre.push_back(pre[r]);
        cur.tokens += len;
    }
    if (!cur.req.empty()) out.push_back(cur);
    return out;
}

// Requests sharded over the context's GPUs (longest-processing-time first),
// micro-batched per GPU and forwarded; on_batch(device, batch) consumes each
// micro-batch's results. A request whose ids start with the cached prefix and
// go beyond it forwards only the rest (SystemPromptCache.cs:51-75); the
// results are bit-identical either way.
template <class OnBatch>
static void forward_requests(Ctx &C, const int32_t *ids, const int64_t *offsets, int32_t n_req, int nv,
                             const volatile int32_t *cancel, OnBatch on_batch, bool full_head) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (n_req < 0 || (n_req > 0 && (!ids || !offsets))) throw Error(SHIELD_ERR_ARG, "null buffer");
    if (n_req == 0) return;
    if (offsets[0] != 0) throw Error(SHIELD_ERR_ARG, "offsets[0] must be 0");
    const int32_t P = (int32_t)C.prefix.size();
    std::vector<std::pair<double, int32_t>> cost(n_req);
    std::vector<int32_t> pre(n_req, 0);
    for (int32_t r = 0; r < n_req; r++) {
        int64_t len = offsets[r + 1] - offsets[r];
        if (len <= 0) throw Error(SHIELD_ERR_ARG, "request " + std::to_string(r) + " has no tokens");
        if (len > C.cfg.max_positions)
            throw Error(SHIELD_ERR_RANGE, "request " + std::to_string(r) + " has " + std::to_string(len) +
                                              " tokens, more than max_positions " +
                                              std::to_string(C.cfg.max_positions));
        if (P > 0 && len > P && std::equal(C.prefix.begin(), C.prefix.end(), ids + offsets[r])) pre[r] = P;
        const double own = (double)(len - pre[r]);
        cost[r] = {own * (1.0 + (double)len / 8192.0), r};
    }
    validate_ids(C, ids, offsets[n_req]);
    // longest-processing-time-first assignment of requests to GPUs
    int D = (int)C.devs.size();
    std::vector<std::vector<int32_t>> assign(D);
    if (D == 1) {
        assign[0].resize(n_req);
        std::iota(assign[0].begin(), assign[0].end(), 0);
    } else {
        std::vector<std::pair<double, int32_t>> sorted = cost;
        std::sort(sorted.begin(), sorted.end(), [](auto &a, auto &b) { return a.first > b.first; });
        std::vector<double> load(D, 0.0);
        for (auto &cr : sorted) {
            int best = (int)(std::min_element(load.begin(), load.end()) - load.begin());
            load[best] += cr.first;
            assign[best].push_back(cr.second);
        }
        for (auto &a : assign) std::sort(a.begin(), a.end());
    }
    std::vector<std::string> errors(D);
    std::vector<shield_status> codes(D, SHIELD_OK);
    auto run = [&](int di) {
        try {
            Device &d = *C.devs[di];
            SHIELD_CUDA(cudaSetDevice(d.ordinal));
            ensure_buffers(C, d);
            std::vector<int32_t> packed;
            std::vector<float> full;
            for (const Batch &B : make_batches(C, assign[di], offsets, pre)) {
                packed.resize(B.tokens);
                for (size_t i = 0; i < B.req.size(); i++)
                    memcpy(packed.data() + B.start[i], ids + offsets[B.req[i]] + B.pre[i], (size_t)B.len[i] * 4);
                if (full_head) full.resize(B.req.size() * (size_t)C.cfg.vocab);
                forward_batch(C, d, packed.data(), B, nv, cancel, -1, 0, nullptr, full_head ? full.data() : nullptr);
                on_batch(d, B, full_head ? full.data() : d.buf.h_logits);
            }
        } catch (const Error &e) {
            codes[di] = e.code;
            errors[di] = e.what();
        } catch (const std::exception &e) {
            codes[di] = SHIELD_ERR_CUDA;
            errors[di] = e.what();
        }
    };
    if (D == 1) {
        run(0);
    } else {
        std::vector<std::thread> th;
        for (int di = 0; di < D; di++) th.emplace_back(run, di);
        for (auto &t : th) t.join();
    }
    for (int di = 0; di < D; di++)
        if (codes[di] != SHIELD_OK) throw Error(codes[di], errors[di]);
}

static void score_batch(Ctx &C, const int32_t *ids, const int64_t *offsets, int32_t n_req, const int32_t *verdict,
                        int32_t n_yes, int32_t n_no, float *yes, float *no, float *score, float *logits,
                        const volatile int32_t *cancel) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (n_req < 0 || (n_req > 0 && (!ids || !offsets || !yes || !no || !score)))
        throw Error(SHIELD_ERR_ARG, "null buffer");
    if (n_yes <= 0 || n_no <= 0 || !verdict) throw Error(SHIELD_ERR_ARG, "need at least one yes and one no id");
    int nv = n_yes + n_no;
    if (nv > 64) throw Error(SHIELD_ERR_ARG, "at most 64 verdict ids");
    for (int i = 0; i < nv; i++)
        if (verdict[i] < 0 || verdict[i] >= C.cfg.vocab)
            throw Error(SHIELD_ERR_RANGE, "verdict id " + std::to_string(verdict[i]) + " is outside the vocabulary");
    if (n_req == 0) return;
    for (auto &d : C.devs) {
        SHIELD_CUDA(cudaSetDevice(d->ordinal));
        ensure_buffers(C, *d);
        SHIELD_CUDA(cudaMemcpyAsync(d->buf.verdict, verdict, (size_t)nv * 4, cudaMemcpyHostToDevice, d->stream));
    }
    forward_requests(
        C, ids, offsets, n_req, nv, cancel,
        [&](Device &, const Batch &B, const float *h_logits) {
            for (size_t i = 0; i < B.req.size(); i++) {
                int32_t r = B.req[i];
                const float *v = h_logits + i * nv;
                score_one(v, n_yes, n_no, score[r], yes[r], no[r]);
                if (logits) memcpy(logits + (int64_t)r * nv, v, (size_t)nv * 4);
            }
        },
        false);
}

// The whole tied head at every request's last position (VerdictLogitsAsync /
// TopVerdictTokenAsync, ShieldstralModerator.cs:269-277,370-378).
static void last_logits(Ctx &C, const int32_t *ids, const int64_t *offsets, int32_t n_req, float *logits,
                        const volatile int32_t *cancel) {
    if (n_req > 0 && !logits) throw Error(SHIELD_ERR_ARG, "null buffer");
    const int64_t V = C.cfg.vocab;
    forward_requests(
        C, ids, offsets, n_req, 0, cancel,
        [&](Device &, const Batch &B, const float *full) {
            for (size_t i = 0; i < B.req.size(); i++)
                memcpy(logits + (int64_t)B.req[i] * V, full + i * V, (size_t)V * 4);
        },
        true);
}

// SystemPromptCache.CaptureAsync (SystemPromptCache.cs:51-75): forwards the
// prefix once per GPU and keeps every layer's keys and values; n = 0 drops it.
static void set_prefix(Ctx &C, const int32_t *ids, int32_t n) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (n < 0 || (n > 0 && !ids)) throw Error(SHIELD_ERR_ARG, "bad prefix");
    if (n >= C.cfg.max_positions)
        throw Error(SHIELD_ERR_RANGE, "a prefix of " + std::to_string(n) + " tokens leaves no position below max_positions");
    validate_ids(C, ids, n);  // a rejected prefix leaves the cached one in place
    clear_prefix(C);
    if (n == 0) return;
    const Config &c = C.cfg;
    for (auto &dp : C.devs) {
        Device &d = *dp;
        SHIELD_CUDA(cudaSetDevice(d.ordinal));
        ensure_buffers(C, d);
        const size_t floats = (size_t)c.n_layers * n * c.kvdim();
        dev_alloc(d.pre_k, floats);
        dev_alloc(d.pre_v, floats);
        Batch B;
        B.req = {0};
        B.start = {0};
        B.len = {n};
        B.pre = {0};
        B.tokens = n;
        C.prefix.assign(ids, ids + n);  // forward_batch sizes the store from it
        try {
            forward_batch(C, d, ids, B, 0, nullptr, -1, 0, nullptr, nullptr, true);
            SHIELD_CUDA(cudaStreamSynchronize(d.stream));
        } catch (...) {
            clear_prefix(C);
            throw;
        }
    }
}

// Floats in a snapshot of n cached positions: KvCache.Snapshot's keys for
// every layer and kv head, then the values (KvCache.cs:102-118).
static int64_t prefix_state_floats(const Config &c, int64_t n) { return 2 * (int64_t)c.n_layers * c.kvdim() * n; }

// SystemPromptCache.RestoreInto / KvCache.Restore (SystemPromptCache.cs:66-74,
// KvCache.cs:121-136) onto every GPU. One layer's keys (and its values) are a
// contiguous range of the snapshot; each goes through the pinned staging
// buffers into a device scratch that a kernel reorders into the layout the
// attention reads. The scratch is reused layer after layer in stream order.
static void set_prefix_state(Ctx &C, const int32_t *ids, int32_t n, const float *state, int64_t n_floats) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (n < 0 || (n > 0 && (!ids || !state))) throw Error(SHIELD_ERR_ARG, "bad prefix");
    if (n >= C.cfg.max_positions)
        throw Error(SHIELD_ERR_RANGE, "a prefix of " + std::to_string(n) + " tokens leaves no position below max_positions");
    const Config &c = C.cfg;
    const int64_t want = prefix_state_floats(c, n);
    if (n_floats != want)
        throw Error(SHIELD_ERR_ARG, "Snapshot holds " + std::to_string(n_floats) + " floats; " + std::to_string(n) +
                                        " positions need " + std::to_string(want) + ".");
    validate_ids(C, ids, n);
    clear_prefix(C);
    if (n == 0) return;
    const int64_t layer = (int64_t)n * c.kvdim();  // floats of one layer's keys
    try {
        for_each_device(C, [&](Device &d) {
            SHIELD_CUDA(cudaSetDevice(d.ordinal));
            dev_alloc(d.pre_k, (size_t)(c.n_layers * layer));
            dev_alloc(d.pre_v, (size_t)(c.n_layers * layer));
            float *tmp = nullptr;
            dev_alloc(tmp, (size_t)(2 * layer));
            try {
                for (int l = 0; l < c.n_layers; l++) {
                    stage_to_device(d, tmp, state + l * layer, (size_t)layer * 4);
                    stage_to_device(d, tmp + layer, state + want / 2 + l * layer, (size_t)layer * 4);
                    check_launch(launch_prefix_state(d.pre_k + l * layer, d.pre_v + l * layer, tmp, tmp + layer, n,
                                                     c.n_kv_heads, c.head_dim, true, d.stream),
                                 "restore prefix state");
                }
                SHIELD_CUDA(cudaStreamSynchronize(d.stream));
            } catch (...) {
                dev_free(tmp);
                throw;
            }
            dev_free(tmp);
        });
    } catch (...) {
        clear_prefix(C);
        throw;
    }
    C.prefix.assign(ids, ids + n);
}

// KvCache.Snapshot of the cached prefix (KvCache.cs:102-118), as
// SystemPromptCache.CaptureAsync takes it (SystemPromptCache.cs:51-60), read
// from the first GPU layer by layer.
static void get_prefix_state(Ctx &C, float *state, int64_t n_floats) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (C.prefix.empty()) throw Error(SHIELD_ERR_STATE, "no prefix is cached");
    const Config &c = C.cfg;
    const int64_t n = (int64_t)C.prefix.size();
    const int64_t want = prefix_state_floats(c, n);
    if (!state || n_floats != want)
        throw Error(SHIELD_ERR_ARG, "the snapshot of " + std::to_string(n) + " positions holds " +
                                        std::to_string(want) + " floats; the buffer has " + std::to_string(n_floats) + ".");
    Device &d = *C.devs[0];
    SHIELD_CUDA(cudaSetDevice(d.ordinal));
    const int64_t layer = n * c.kvdim();
    float *tmp = nullptr;
    dev_alloc(tmp, (size_t)(2 * layer));
    try {
        for (int l = 0; l < c.n_layers; l++) {
            check_launch(launch_prefix_state(d.pre_k + l * layer, d.pre_v + l * layer, tmp, tmp + layer, n,
                                             c.n_kv_heads, c.head_dim, false, d.stream),
                         "read prefix state");
            SHIELD_CUDA(cudaMemcpyAsync(state + l * layer, tmp, (size_t)layer * 4, cudaMemcpyDeviceToHost, d.stream));
            SHIELD_CUDA(cudaMemcpyAsync(state + want / 2 + l * layer, tmp + layer, (size_t)layer * 4,
                                        cudaMemcpyDeviceToHost, d.stream));
        }
        SHIELD_CUDA(cudaStreamSynchronize(d.stream));
    } catch (...) {
        dev_free(tmp);
        throw;
    }
    dev_free(tmp);
}

// ---------------------------------------------------------- sequences

static Device &device_of(Ctx &C, int32_t device);

static Device::Sequence &sequence_of(Ctx &C, int64_t id, Device **dev) {
    const int64_t di = id >> 48;
    if (id <= 0 || di >= (int64_t)C.devs.size()) throw Error(SHIELD_ERR_ARG, "unknown sequence " + std::to_string(id));
    Device &d = *C.devs[di];
    auto it = d.seqs.find(id);
    if (it == d.seqs.end()) throw Error(SHIELD_ERR_ARG, "unknown sequence " + std::to_string(id));
    if (dev) *dev = &d;
    return it->second;
}

// A new, empty KV cache for up to capacity positions on one GPU of the context.
static int64_t seq_create(Ctx &C, int32_t device, int32_t capacity) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (capacity <= 0 || capacity > C.cfg.max_positions)
        throw Error(SHIELD_ERR_RANGE, "sequence capacity must be in 1.." + std::to_string(C.cfg.max_positions));
    Device &d = device_of(C, device);
    Device::Sequence sq;
    sq.cap = capacity;
    const size_t floats = (size_t)C.cfg.n_layers * capacity * C.cfg.kvdim();
    dev_alloc(sq.k, floats);
    dev_alloc(sq.v, floats);
    const int64_t id = ((int64_t)device << 48) | C.next_seq++;
    d.seqs.emplace(id, sq);
    return id;
}

// MinistralModel.ForwardAsync (MinistralModel.cs:179-271) on n sequences at
// once: sequence i appends ids[offsets[i] .. offsets[i+1]) to its cache, every
// new token attending to the cached positions and to the new ones before it;
// logits (optional) gets each sequence's whole tied head at its new last
// position. The results are bit-identical to forwarding each sequence's full
// history in one piece.
static void seq_forward(Ctx &C, const int64_t *seq, const int32_t *ids, const int64_t *offsets, int32_t n,
                        float *logits, const volatile int32_t *cancel) {
    if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
    if (n < 0 || (n > 0 && (!seq || !ids || !offsets))) throw Error(SHIELD_ERR_ARG, "null buffer");
    if (n == 0) return;
    if (offsets[0] != 0) throw Error(SHIELD_ERR_ARG, "offsets[0] must be 0");
    const int D = (int)C.devs.size();
    std::vector<std::vector<int32_t>> per_dev(D);
    std::unordered_map<int64_t, int32_t> seen;
    for (int32_t i = 0; i < n; i++) {
        Device *dp = nullptr;
        Device::Sequence &sq = sequence_of(C, seq[i], &dp);
        if (!seen.emplace(seq[i], i).second)
            throw Error(SHIELD_ERR_ARG, "sequence " + std::to_string(seq[i]) + " appears twice in one call");
        const int64_t len = offsets[i + 1] - offsets[i];
        if (len <= 0) throw Error(SHIELD_ERR_ARG, "sequence entry " + std::to_string(i) + " has no tokens");
        if (sq.len + len > sq.cap)
            throw Error(SHIELD_ERR_RANGE, "sequence " + std::to_string(seq[i]) + " would hold " +
                                              std::to_string(sq.len + len) + " positions, more than its capacity " +
                                              std::to_string(sq.cap));
        per_dev[seq[i] >> 48].push_back(i);
    }
    validate_ids(C, ids, offsets[n]);
    const int64_t V = C.cfg.vocab, stride_per_pos = C.cfg.kvdim();
    std::vector<std::string> errors(D);
    std::vector<shield_status> codes(D, SHIELD_OK);
    auto run = [&](int di) {
        try {
            Device &d = *C.devs[di];
            SHIELD_CUDA(cudaSetDevice(d.ordinal));
            ensure_buffers(C, d);
            const std::vector<int32_t> &mine = per_dev[di];
            size_t k = 0;
            std::vector<int32_t> packed;
            std::vector<float> full;
            while (k < mine.size()) {
                Batch B;
                while (k < mine.size()) {
                    const int32_t i = mine[k];
                    const int32_t len = (int32_t)(offsets[i + 1] - offsets[i]);
                    if (B.tokens + len > C.cfg.max_batch_tokens && !B.req.empty()) break;
                    Device::Sequence &sq = d.seqs.at(seq[i]);
                    B.req.push_back(i);
                    B.start.push_back(B.tokens);
                    B.len.push_back(len);
                    B.pre.push_back(sq.len);
                    B.ck.push_back(sq.k);
                    B.cv.push_back(sq.v);
                    B.cstride.push_back((int64_t)sq.cap * stride_per_pos);
                    B.append.push_back(1);
                    B.tokens += len;
                    k++;
                }
                packed.resize(B.tokens);
                for (size_t j = 0; j < B.req.size(); j++)
                    memcpy(packed.data() + B.start[j], ids + offsets[B.req[j]], (size_t)B.len[j] * 4);
                full.resize(B.req.size() * (size_t)V);
                const bool decode_step =
                    std::all_of(B.len.begin(), B.len.end(), [](int32_t l) { return l == 1; });
                try {
                    forward_batch(C, d, packed.data(), B, 0, cancel, -1, 0, nullptr, full.data(), false,
                                  decode_step && !d.no_graphs);
                } catch (const Error &e) {
                    // a step that could not be captured runs as plain launches (no
                    // GPU work ran yet; a replayed step only rewrites the same rows)
                    if (!decode_step || d.no_graphs || e.code == SHIELD_ERR_CANCELLED) throw;
                    d.no_graphs = true;
                    forward_batch(C, d, packed.data(), B, 0, cancel, -1, 0, nullptr, full.data());
                }
                for (size_t j = 0; j < B.req.size(); j++) {
                    d.seqs.at(seq[B.req[j]]).len += B.len[j];
                    if (logits) memcpy(logits + (int64_t)B.req[j] * V, full.data() + j * V, (size_t)V * 4);
                }
            }
        } catch (const Error &e) {
            codes[di] = e.code;
            errors[di] = e.what();
        } catch (const std::exception &e) {
            codes[di] = SHIELD_ERR_CUDA;
            errors[di] = e.what();
        }
    };
    if (D == 1) {
        run(0);
    } else {
        std::vector<std::thread> th;
        for (int di = 0; di < D; di++)
            if (!per_dev[di].empty()) th.emplace_back(run, di);
        for (auto &t : th) t.join();
    }
    for (int di = 0; di < D; di++)
        if (codes[di] != SHIELD_OK) throw Error(codes[di], errors[di]);
}

static void seq_reset(Ctx &C, int64_t id) { sequence_of(C, id, nullptr).len = 0; }

static void seq_release(Ctx &C, int64_t id) {
    Device *d = nullptr;
    Device::Sequence &sq = sequence_of(C, id, &d);
    SHIELD_CUDA(cudaSetDevice(d->ordinal));
    SHIELD_CUDA(cudaStreamSynchronize(d->stream));
    dev_free(sq.k);
    dev_free(sq.v);
    d->seqs.erase(id);
}

static int32_t seq_length(Ctx &C, int64_t id) { return sequence_of(C, id, nullptr).len; }

static Device &device_of(Ctx &C, int32_t device) {
    if (device < 0 || device >= (int32_t)C.devs.size())
        throw Error(SHIELD_ERR_RANGE, "device index " + std::to_string(device) + " is outside the context");
    Device &d = *C.devs[device];
    SHIELD_CUDA(cudaSetDevice(d.ordinal));
    return d;
}

static QAct scratch_qact(Device &d, int64_t M, int64_t K) {
    size_t n = (size_t)(M * K);
    size_t nb = (size_t)(M * K / 32);
    char *base = static_cast<char *>(d.sa.get(n * 3 + nb * 12 + 1024));
    QAct q;
    q.a8 = reinterpret_cast<int8_t *>(base);
    q.a16 = reinterpret_cast<__half *>(base + ((n + 255) & ~size_t(255)));
    char *sp = base + ((n + 255) & ~size_t(255)) + ((2 * n + 255) & ~size_t(255));
    q.da = reinterpret_cast<float *>(sp);
    q.ds = q.da + nb;
    q.sums = reinterpret_cast<int32_t *>(q.ds + nb);
    q.M = M;
    q.K = K;
    return q;
}

static void qmatmul_dev(Ctx &C, Device &d, const Tensor &W, const float *d_x, int64_t M, float *d_y,
                        const int32_t *d_rows, int32_t n_rows) {
    QAct q = scratch_qact(d, M, W.w.cols);
    check_launch(launch_quantize(d_x, M, W.w.cols, W.w.cols, q, d.stream), "quantize");
    if (d_rows) {
        check_launch(launch_gemm_rows(C, W.w, d_rows, n_rows, q, d_y, n_rows, d.stream), "row-subset GEMM");
    } else {
        if (!d.buf.err) {
            dev_alloc(d.buf.err, 1);
            SHIELD_CUDA(cudaMemsetAsync(d.buf.err, 0, 4, d.stream));
        }
        gemm(C, d, W, q, d_y, W.w.rows, EPI_STORE);
    }
}

static const Tensor &matrix(Device &d, const char *weight) {
    if (!weight) throw Error(SHIELD_ERR_ARG, "weight name is null");
    const Tensor &W = d.get(weight);
    if (!W.raw) throw Error(SHIELD_ERR_ARG, std::string(weight) + " is a vector, not a matrix");
    return W;
}

}  // namespace shield

using namespace shield;

struct shield_ctx {
    Ctx c;
};

template <class F>
static shield_status guarded(F &&f) {
    try {
        f();
        g_last_error.clear();
        return SHIELD_OK;
    } catch (const Error &e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc &) {
        g_last_error = "host memory exhausted";
        return SHIELD_ERR_NOMEM;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return SHIELD_ERR_CUDA;
    }
}

extern "C" {

shield_status shield_open(int32_t device_mask, shield_ctx **out) {
    return guarded([&] {
        if (!out) throw Error(SHIELD_ERR_ARG, "out is null");
        *out = nullptr;
        int n = 0;
        SHIELD_CUDA(cudaGetDeviceCount(&n));
        if (device_mask == 0) device_mask = 1;
        auto ctx = std::make_unique<shield_ctx>();
        for (int i = 0; i < 31; i++) {
            if (!(device_mask & (1 << i))) continue;
            if (i >= n) throw Error(SHIELD_ERR_RANGE, "device " + std::to_string(i) + " does not exist");
            auto d = std::make_unique<Device>();
            d->ordinal = i;
            SHIELD_CUDA(cudaSetDevice(i));
            SHIELD_CUDA(cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, i));
            SHIELD_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
            ctx->c.devs.push_back(std::move(d));
        }
        *out = ctx.release();
    });
}

void shield_close(shield_ctx *ctx) {
    if (!ctx) return;
    for (auto &d : ctx->c.devs) {
        cudaSetDevice(d->ordinal);
        cudaStreamSynchronize(d->stream);
    }
    delete ctx;
}

int32_t shield_device_count(const shield_ctx *ctx) { return ctx ? (int32_t)ctx->c.devs.size() : 0; }

shield_status shield_set_config(shield_ctx *ctx, const shield_config *cfg) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        set_config(ctx->c, cfg);
    });
}

shield_status shield_upload_tensor(shield_ctx *ctx, const char *name, uint32_t ggml_type, int64_t rows, int64_t cols,
                                   const void *bytes, size_t nbytes) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        upload(ctx->c, name, ggml_type, rows, cols, bytes, nbytes);
    });
}

shield_status shield_score_batch(shield_ctx *ctx, const int32_t *ids, const int64_t *offsets, int32_t n_req,
                                 const int32_t *verdict_ids, int32_t n_yes, int32_t n_no, float *yes, float *no,
                                 float *score, float *logits, const volatile int32_t *cancel) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        score_batch(ctx->c, ids, offsets, n_req, verdict_ids, n_yes, n_no, yes, no, score, logits, cancel);
    });
}

shield_status shield_last_logits(shield_ctx *ctx, const int32_t *ids, const int64_t *offsets, int32_t n_req,
                                 float *logits, const volatile int32_t *cancel) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        last_logits(ctx->c, ids, offsets, n_req, logits, cancel);
    });
}

shield_status shield_seq_create(shield_ctx *ctx, int32_t device, int32_t capacity, int64_t *seq) {
    return guarded([&] {
        if (!ctx || !seq) throw Error(SHIELD_ERR_ARG, "null argument");
        *seq = seq_create(ctx->c, device, capacity);
    });
}

shield_status shield_seq_forward(shield_ctx *ctx, const int64_t *seqs, const int32_t *ids, const int64_t *offsets,
                                 int32_t n, float *logits, const volatile int32_t *cancel) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        seq_forward(ctx->c, seqs, ids, offsets, n, logits, cancel);
    });
}

shield_status shield_seq_length(shield_ctx *ctx, int64_t seq, int32_t *length) {
    return guarded([&] {
        if (!ctx || !length) throw Error(SHIELD_ERR_ARG, "null argument");
        *length = seq_length(ctx->c, seq);
    });
}

shield_status shield_seq_reset(shield_ctx *ctx, int64_t seq) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        seq_reset(ctx->c, seq);
    });
}

shield_status shield_seq_release(shield_ctx *ctx, int64_t seq) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        seq_release(ctx->c, seq);
    });
}

shield_status shield_set_prefix(shield_ctx *ctx, const int32_t *ids, int32_t n) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        set_prefix(ctx->c, ids, n);
    });
}

shield_status shield_get_prefix_state(shield_ctx *ctx, float *state, int64_t n_floats) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        get_prefix_state(ctx->c, state, n_floats);
    });
}

shield_status shield_prefix_length(shield_ctx *ctx, int32_t *n) {
    return guarded([&] {
        if (!ctx || !n) throw Error(SHIELD_ERR_ARG, "ctx or n is null");
        *n = (int32_t)ctx->c.prefix.size();
    });
}

shield_status shield_set_prefix_state(shield_ctx *ctx, const int32_t *ids, int32_t n, const float *state,
                                      int64_t n_floats) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        set_prefix_state(ctx->c, ids, n, state, n_floats);
    });
}

shield_status shield_qmatmul(shield_ctx *ctx, int32_t device, const char *weight, const float *x, int64_t M,
                             float *y, const int32_t *row_ids, int32_t n_rows) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        Ctx &C = ctx->c;
        Device &d = device_of(C, device);
        const Tensor &W = matrix(d, weight);
        int64_t n_out = row_ids ? n_rows : W.w.rows;
        if (M < 0 || (row_ids && n_rows < 0)) throw Error(SHIELD_ERR_ARG, "negative size");
        if (row_ids)
            for (int32_t i = 0; i < n_rows; i++)
                if (row_ids[i] < 0 || row_ids[i] >= W.w.rows)
                    throw Error(SHIELD_ERR_RANGE, "Row " + std::to_string(row_ids[i]) + " is outside the matrix's " +
                                                      std::to_string(W.w.rows) + " rows.");
        if (M == 0 || n_out == 0) return;
        if (!x || !y) throw Error(SHIELD_ERR_ARG, "x and y must be non-null");
        float *dx = static_cast<float *>(d.sx.get((size_t)(M * W.w.cols) * 4));
        float *dy = static_cast<float *>(d.sy.get((size_t)(M * n_out) * 4));
        int32_t *drows = nullptr;
        if (row_ids) {
            drows = static_cast<int32_t *>(d.sd.get((size_t)n_rows * 4));
            SHIELD_CUDA(cudaMemcpyAsync(drows, row_ids, (size_t)n_rows * 4, cudaMemcpyHostToDevice, d.stream));
        }
        SHIELD_CUDA(cudaMemcpyAsync(dx, x, (size_t)(M * W.w.cols) * 4, cudaMemcpyHostToDevice, d.stream));
        qmatmul_dev(C, d, W, dx, M, dy, drows, n_rows);
        SHIELD_CUDA(cudaMemcpyAsync(y, dy, (size_t)(M * n_out) * 4, cudaMemcpyDeviceToHost, d.stream));
        check_device_error(d);
    });
}

shield_status shield_qmatmul_device(shield_ctx *ctx, int32_t device, const char *weight, const float *d_x, int64_t M,
                                    float *d_y) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        Ctx &C = ctx->c;
        Device &d = device_of(C, device);
        const Tensor &W = matrix(d, weight);
        if (M < 0) throw Error(SHIELD_ERR_ARG, "negative size");
        if (M == 0) return;
        if (!d_x || !d_y) throw Error(SHIELD_ERR_ARG, "x and y must be non-null");
        qmatmul_dev(C, d, W, d_x, M, d_y, nullptr, 0);
    });
}

shield_status shield_qmatmul_noalloc(shield_ctx *ctx, int32_t device, const char *weight, const float *d_x,
                                     int64_t M, float *d_y) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        Ctx &C = ctx->c;
        Device &d = device_of(C, device);
        const Tensor &W = matrix(d, weight);
        if (M < 0) throw Error(SHIELD_ERR_ARG, "negative size");
        if (M == 0) return;
        if (!d_x || !d_y) throw Error(SHIELD_ERR_ARG, "x and y must be non-null");
        if (M * W.w.cols > noalloc_max_elements())
            throw Error(SHIELD_ERR_ARG, "M * cols = " + std::to_string(M * W.w.cols) +
                                            " exceeds the no-allocation scratch limit of " +
                                            std::to_string(noalloc_max_elements()) + " activation elements");
        int32_t err = 0;
        cudaError_t e = launch_qmatmul_noalloc(W.w, d_x, M, d_y, C.gemm_path, &err, d.stream);
        if (e == cudaErrorNotSupported)
            throw Error(SHIELD_ERR_UNSUPPORTED, "the GEMM kernel selected by shield_set_gemm_path does not take this shape");
        check_launch(e, "no-allocation GEMM");
        if (err) throw Error(SHIELD_ERR_TIMEOUT, "a device-side wait gave up (error word " + std::to_string(err) + ")");
    });
}

shield_status shield_debug_block_dots(shield_ctx *ctx, int32_t device, const char *weight, const float *x, int64_t M,
                                      int32_t *dots, int32_t path) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        Ctx &C = ctx->c;
        Device &d = device_of(C, device);
        const Tensor &W = matrix(d, weight);
        if (M <= 0 || !x || !dots) throw Error(SHIELD_ERR_ARG, "bad arguments");
        int64_t nb = W.w.cols / 32;
        float *dx = static_cast<float *>(d.sx.get((size_t)(M * W.w.cols) * 4));
        int32_t *dd = static_cast<int32_t *>(d.sy.get((size_t)(M * W.w.rows * nb) * 4));
        SHIELD_CUDA(cudaMemcpyAsync(dx, x, (size_t)(M * W.w.cols) * 4, cudaMemcpyHostToDevice, d.stream));
        QAct q = scratch_qact(d, M, W.w.cols);
        check_launch(launch_quantize(dx, M, W.w.cols, W.w.cols, q, d.stream), "quantize");
        if (!d.buf.err) {
            dev_alloc(d.buf.err, 1);
            SHIELD_CUDA(cudaMemsetAsync(d.buf.err, 0, 4, d.stream));
        }
        bool tc = path == 2 || (path == 0 && C.gemm_path != 1 && gemm_tc_supports(W.w, M));
        if (tc) {
            cudaError_t e = launch_block_dots_tc(W.w, q, dd, d.buf.err, d.stream);
            if (e == cudaErrorNotSupported) throw Error(SHIELD_ERR_UNSUPPORTED, "tensor-core path does not take this shape");
            check_launch(e, "tensor-core block dots");
        } else {
            check_launch(launch_block_dots(W.w, q, dd, d.stream), "block dots");
        }
        SHIELD_CUDA(cudaMemcpyAsync(dots, dd, (size_t)(M * W.w.rows * nb) * 4, cudaMemcpyDeviceToHost, d.stream));
        check_device_error(d);
    });
}

shield_status shield_set_gemm_path(shield_ctx *ctx, int32_t path) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        if (path < 0 || path > 4) throw Error(SHIELD_ERR_ARG, "path must be 0, 1, 2, 3 or 4");
        ctx->c.gemm_path = path;
        gemm_tc_set_pre_min_tokens(path == 2 ? INT64_MAX : path == 3 ? 1 : -1);
    });
}

shield_status shield_set_gemm_tile_width(shield_ctx *ctx, int32_t width) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        if (width != 0 && width != 64 && width != 128) throw Error(SHIELD_ERR_ARG, "width must be 0, 64 or 128");
        gemm_tc_set_tile_width(width);
    });
}

shield_status shield_set_attention_rows(shield_ctx *ctx, int32_t rows) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        if (rows != 0 && rows != 64 && rows != 128) throw Error(SHIELD_ERR_ARG, "rows must be 0, 64 or 128");
        ctx->c.att_rows = rows;
    });
}

shield_status shield_debug_activation(shield_ctx *ctx, int32_t device, const int32_t *ids, int32_t n, int32_t layer,
                                      int32_t what, float *out) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        Ctx &C = ctx->c;
        if (!C.configured) throw Error(SHIELD_ERR_STATE, "no model configured");
        Device &d = device_of(C, device);
        if (n <= 0 || !ids || !out) throw Error(SHIELD_ERR_ARG, "bad arguments");
        if (n > C.cfg.max_positions) throw Error(SHIELD_ERR_RANGE, "request longer than max_positions");
        if (layer < 0 || layer >= C.cfg.n_layers) throw Error(SHIELD_ERR_RANGE, "layer out of range");
        if (what < SHIELD_ACT_OUTPUT || what > SHIELD_ACT_ATTN_NORM) throw Error(SHIELD_ERR_ARG, "unknown activation");
        validate_ids(C, ids, n);
        ensure_buffers(C, d);
        Batch B;
        B.req = {0};
        B.start = {0};
        B.len = {n};
        B.pre = {0};
        B.tokens = n;
        forward_batch(C, d, ids, B, 0, nullptr, layer, what, out);
    });
}

shield_status shield_set_timing(shield_ctx *ctx, int32_t level) {
    return guarded([&] {
        if (!ctx) throw Error(SHIELD_ERR_ARG, "ctx is null");
        if (level < 0 || level > 2) throw Error(SHIELD_ERR_ARG, "level must be 0, 1 or 2");
        for (auto &d : ctx->c.devs) d->timing.level = level;
    });
}

shield_status shield_read_timing(shield_ctx *ctx, int32_t device, shield_timing *out, int32_t reset) {
    return guarded([&] {
        if (!ctx || !out) throw Error(SHIELD_ERR_ARG, "null argument");
        Device &d = device_of(ctx->c, device);
        SHIELD_CUDA(cudaStreamSynchronize(d.stream));
        Timing &T = d.timing;
        shield_timing t{};
        for (auto &p : T.fwd) {
            float ms = 0;
            SHIELD_CUDA(cudaEventElapsedTime(&ms, p.first, p.second));
            t.forward_ms += ms;
        }
        for (auto &p : T.gemm) {
            float ms = 0;
            SHIELD_CUDA(cudaEventElapsedTime(&ms, p.first, p.second));
            t.gemm_ms += ms;
        }
        for (auto &p : T.attn) {
            float ms = 0;
            SHIELD_CUDA(cudaEventElapsedTime(&ms, p.first, p.second));
            t.attn_ms += ms;
        }
        t.attn_flops = T.attn_flops;
        t.gemm_ops = T.gemm_ops;
        t.gemm_bytes = T.gemm_bytes;
        t.gemm_launches = T.gemm_launches;
        t.kernel_launches = T.launches;
        t.tokens = T.tokens;
        t.requests = T.requests;
        t.h2d_bytes = T.h2d;
        t.d2h_bytes = T.d2h;
        *out = t;
        if (reset) T.reset();
    });
}

shield_status shield_device_stream(shield_ctx *ctx, int32_t device, void **stream) {
    return guarded([&] {
        if (!ctx || !stream) throw Error(SHIELD_ERR_ARG, "null argument");
        *stream = (void *)device_of(ctx->c, device).stream;
    });
}

const char *shield_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
