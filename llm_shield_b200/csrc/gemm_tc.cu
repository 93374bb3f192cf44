// tcgen05 tensor-core GEMM for GGUF legacy-quantized weights (sm_100a).
//
// y[t, n] = Σ_b fma-chain( float(i_b[t, n]) · (d_w[n, b] · d_a[t, b]) )     (+ Q4_1/Q5_1 offsets)
// with i_b the exact int32 dot of block b (IntegerGemm.cs:371-457): the same
// per-output operation sequence as the reference and the oracle, so outputs
// are bit-identical to theirs.
//
// Tile: 128 tokens (TMEM lanes / UMMA M) x 128 output features (UMMA N), or
// x 64 when 128-wide tiles would leave most SMs idle (few tokens). One launch
// can cover up to three weights that share the activations (Q/K/V, gate/up).
// Per 32-element quant block the tile needs its own int32 result, because the
// f32 chain scales every block separately; one block is one UMMA K-step.
//
//   warp 0      TMA producer: activation tiles (f16 holding the int8 values,
//               128B-swizzled K-major) and either the weights' once-unpacked
//               f16 copy (same layout; every layer matrix has one) or raw GGUF
//               weight chunks (8 blocks per row, bytes unchanged)
//   warp 1      TMEM owner + MMA issuer: two tcgen05.mma.kind::f16 (K=16) per
//               block into one of four 128-column TMEM slots, one commit per
//               block pair
//   warps 2-3   raw-chunk path: unpack raw blocks in registers (nibbles,
//               5th bits, Q8 bytes) to f16 integers in the canonical SW128
//               K-major layout; widen the f16 block scales (and offsets) to
//               f32. Copy path: warp 2 loads the scale tiles by TMA, so the
//               operand producer never waits on the epilogue
//   warps 4-19  epilogue, 32 (or 16) output features each: tcgen05.ld the slot, apply
//               the block's f32 scaling chain per output (packed f32x2
//               operations), write or add to y
//
// The activation scales reach shared memory by TMA beside the weight scales.
// The grid is persistent (one CTA per SM walking tiles), so a tile's pipeline
// fill and its final stores hide under its neighbours' work.
//
// kind::f16 rather than kind::i8: products of 8-bit integers summed over one
// block stay below 2^20, so the f32 accumulator holds the exact int32 sum and
// the epilogue needs no integer->float conversion (the epilogue's f32 pipe,
// not the tensor pipe, bounds this kernel).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "ops.h"

namespace shield {
namespace tc {

constexpr int BM = 128;          // tokens per tile (TMEM lanes)
constexpr int BN = 128;          // output features per tile (TMEM columns per slot); 64 for small grids
// Operand stages (2 blocks each: activations and f16 weights). An operand
// load takes about 2,700 SM cycles from issue to arrival (clock stamps inside
// the kernel), twice what a block pair takes, so the producer runs several
// pairs ahead. The copy path spends the shared memory the raw chunks would
// hold on it: 6 stages for 128-wide tiles, 8 for 64-wide ones; the raw-chunk
// path keeps 3.
constexpr int BASE_STAGES = 3;
constexpr int RAW_CHUNK_STAGES = 2;  // raw weight chunks in flight
template <int TN, bool PRE> constexpr int operand_stages() { return PRE ? (TN == 64 ? 8 : 6) : BASE_STAGES; }
constexpr int SC_STAGES = 2;     // f32 scale chunks in flight
constexpr int NSLOT = 4;         // TMEM accumulator slots (4 x 128 = 512 columns, or 4 x 64)
constexpr int CHUNK = 8;         // blocks per raw chunk (TMA inner box = 8 blocks)
constexpr int EPI_WARPS = 16;              // warp e owns lane quarter e%4 and columns EPI_COLS*(e/4)..
template <int TN> constexpr int epi_cols() { return TN / (EPI_WARPS / 4); }  // 32 or 16
constexpr int THREADS = 128 + 32 * EPI_WARPS;
constexpr int UNPACK_THREADS = 64;

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

template <int TYPE, int TN, bool PRE>
struct Smem {
    static constexpr int STAGES = operand_stages<TN, PRE>();
    static constexpr int RAW_STAGES = PRE ? 1 : RAW_CHUNK_STAGES;  // the copy path reserves no chunk memory
    static constexpr int BB = block_bytes(TYPE);
    static constexpr int RAW_ROW = CHUNK * BB;   // bytes of one row's chunk
    static constexpr int RAW_BYTES = TN * RAW_ROW;
    static constexpr int A_BYTES = BM * 128;     // 64 f16 per row
    static constexpr int B_BYTES = TN * 128;
    // one scale stage: weight scales [CHUNK][BN] (+ offsets), then the
    // activation scales [BM][CHUNK] (+ their offset terms)
    static constexpr int SC_DA = CHUNK * TN * (has_offset(TYPE) ? 2 : 1);
    static constexpr int DA_BYTES = CHUNK * BM * 4 * (has_offset(TYPE) ? 2 : 1);
    static constexpr int SC_FLOATS = SC_DA + DA_BYTES / 4;
    static_assert((SC_DA * 4) % 256 == 0 && (SC_FLOATS * 4) % 256 == 0, "swizzled TMA tiles need 256-byte alignment");
    static_assert(TN == 128 || TN == 64, "tiles are 128 or 64 features wide");
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
    static constexpr int OFF_RAW = OFF_B + STAGES * B_BYTES;
    static constexpr int OFF_SC = OFF_RAW + (PRE ? 0 : RAW_STAGES * align_up(RAW_BYTES, 1024));
    static constexpr int OFF_BAR = OFF_SC + SC_STAGES * SC_FLOATS * 4;
    // barriers: a_full, b_full, done (STAGES each), raw_full, raw_empty,
    // sc_full, sc_empty, t_empty (one per TMEM slot)
    static constexpr int NBAR = 3 * STAGES + 2 * RAW_STAGES + 2 * SC_STAGES + NSLOT;
    static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
    static_assert(BYTES <= 227 * 1024, "shared memory per CTA");
};

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after ~2 s of SM clock, raising the CTA's abort flag
// and the kernel's error word, so a lost arrival can never hang the GPU.
// Non-blocking test of a phase (the first look of a bounded wait, which on
// the hot path usually finds the phase complete).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, int32_t *err) {
    if (mbar_test(bar, parity)) return true;
    long long t0 = clock64();
    for (uint32_t i = 0;; i++) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 255) == 255) {
            if (*abort_flag) return false;
            if (clock64() - t0 > 4000000000LL) {
                *abort_flag = 1;
                if (err) atomicExch(err, 3);
                return false;
            }
        }
    }
}

// The same kind of bounded wait for a whole warp: every lane polls and a
// vote makes the outcome warp-uniform, so a loop around it needs no
// reconvergence point. It gives up after 2^26 polls (a quarter of a second
// or more; a preempted CTA does not poll, so time it is not running does not
// count), raising the abort flag and the error word.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort_flag, int32_t *err) {
    for (uint32_t i = 0;; i++) {
        if (__all_sync(0xffffffffu, mbar_try(bar, parity))) return true;
        if ((i & 255) == 255) {
            int stop = *abort_flag ? 1 : (i >= (1u << 26) ? 2 : 0);
            stop = __shfl_sync(0xffffffffu, stop, 0);
            if (stop) {
                if (stop == 2 && (threadIdx.x & 31) == 0) {
                    *abort_flag = 1;
                    if (err) atomicExch(err, 3);
                }
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128B-swizzled operand: 8-row groups 1024 B apart (SBO), LBO unused (1),
// descriptor version 1 (sm_100), layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, M=128, N=TN.
template <int TN>
constexpr uint32_t idesc() { return (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24); }

template <int TN>
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "n"(idesc<TN>()), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// tcgen05.ld 16x256b.x2: the same for 16 columns (registers 0-7).
__device__ __forceinline__ void tmem_ld16x256(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
}

// tcgen05.ld 16x256b.x4: 16 TMEM lanes x 32 columns. Register 4i + e holds
// column 8i + 2(lane%4) + (e&1) of lane lane/4 + 8(e>>1), relative to taddr.
// Load and wait are one asm statement, so the registers are defined after it.
__device__ __forceinline__ void tmem_ld16x256(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory loads at 32-bit shared addresses (kept in order with the
// barrier waits that publish the data).
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint64_t lds_b64(uint32_t a) {
    uint64_t v;
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
    return v;
}

// ------------------------------------------------------------ unpacking

// Four payload bytes (one per lane of a 32-bit word, each < 256) -> two f16x2
// words holding (byte - z) exactly: 0x6400|b is the f16 1024+b, minus 1024+z.
__device__ __forceinline__ void bytes_to_f16(uint32_t w, __half2 bias, uint32_t &lo, uint32_t &hi) {
    uint32_t a = __byte_perm(w, 0x64646464u, 0x4140);
    uint32_t b = __byte_perm(w, 0x64646464u, 0x4342);
    __half2 ha = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}

// bit i of the 4-bit x -> bit 4 of byte i (the Q5 fifth bits as 0x10 per byte)
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return ((x * 0x00204081u) & 0x01010101u) << 4; }

__device__ __forceinline__ uint32_t ld_smem_u32_2aligned(const uint8_t *p) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}

// One raw block -> 32 f16 integers (w = u - z) as 16 words, in weight order.
template <int TYPE>
__device__ __forceinline__ void unpack_block(const uint8_t *blk, uint32_t (&o)[16]) {
    constexpr int Z = zero_point(TYPE);
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)(0x6400 + Z)));
    if (TYPE == T_Q8_0) {
#pragma unroll
        for (int w = 0; w < 8; w++) {
            uint32_t v = ld_smem_u32_2aligned(blk + 2 + 4 * w) ^ 0x80808080u;  // u = q + 128
            bytes_to_f16(v, bias, o[2 * w], o[2 * w + 1]);
        }
    } else {
        const uint8_t *qs = blk + qs_offset(TYPE);
        uint32_t qh = 0;
        if (TYPE == T_Q5_0 || TYPE == T_Q5_1) qh = ld_smem_u32_2aligned(blk + qh_offset(TYPE));
#pragma unroll
        for (int w = 0; w < 4; w++) {
            uint32_t q = ld_smem_u32_2aligned(qs + 4 * w);
            uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;
            if (TYPE == T_Q5_0 || TYPE == T_Q5_1) {
                lo |= spread4((qh >> (4 * w)) & 0xFu);
                hi |= spread4((qh >> (16 + 4 * w)) & 0xFu);
            }
            // elements 4w..4w+3 (low nibbles) and 16+4w..16+4w+3 (high nibbles)
            bytes_to_f16(lo, bias, o[2 * w], o[2 * w + 1]);
            bytes_to_f16(hi, bias, o[8 + 2 * w], o[8 + 2 * w + 1]);
        }
    }
}

// ------------------------------------------------------------------ kernel

// One launch covers up to GMAX weights that share the activations, the
// weight type and K (the Q/K/V projections): tiles [tile0[g], tile0[g + 1])
// belong to weight g, whose outputs go to y[g] (row stride ldy[g]).
constexpr int GMAX = 3;
struct TcParams {
    CUtensorMap a, da, ds;  // activations (f16 integers) and their scales
    CUtensorMap w[GMAX], b[GMAX], sc[GMAX], off[GMAX];  // raw blocks, f16 copy, scale / offset planes
    float *y[GMAX];
    int64_t ldy[GMAX];
    int64_t tile0[GMAX + 1];
    int n[GMAX], ntn[GMAX];
    int count;
};

// The weight of tile t and the tile's first token and output feature.
template <int TN>
__device__ __forceinline__ int tile_weight(const TcParams &P, int64_t t, int &m0, int &n0) {
    int g = 0;
    while (g + 1 < P.count && t >= P.tile0[g + 1]) g++;
    const int64_t lt = t - P.tile0[g];
    n0 = (int)(lt % P.ntn[g]) * TN;
    m0 = (int)(lt / P.ntn[g]) * BM;
    return g;
}

// PRE: the weights come pre-unpacked (f16 copy) and their scales from the f32
// planes, both by TMA; the unpacker warps then idle.
//
// Persistent: CTA b takes tiles b, b + gridDim.x, ... (token tiles outer,
// feature tiles inner) and every ring (operand stages, scale stages, TMEM
// slots) runs on across tiles, so the next tile's loads and MMAs overlap the
// current tile's epilogue and final stores.
template <int TYPE, int EPI, bool DOTS, bool PRE, int TN>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc(const __grid_constant__ TcParams P, int M, int nb, int32_t *__restrict__ err, int32_t *__restrict__ dots) {
    using L = Smem<TYPE, TN, PRE>;
    constexpr int STAGES = L::STAGES, RAW_STAGES = L::RAW_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ntiles = P.tile0[P.count];

    uint32_t bar = sbase + L::OFF_BAR;
    // done(s): one tcgen05.commit per block pair, after its four MMAs. Its
    // completion frees operand stage s (producer, unpackers) and publishes the
    // pair's two TMEM slots (epilogue). Every waiter trails the commit by less
    // than STAGES pairs, so no phase can complete twice under a waiter.
    auto a_full = [&](int s) { return bar + 8 * s; };
    auto b_full = [&](int s) { return bar + 8 * (STAGES + s); };
    auto done = [&](int s) { return bar + 8 * (2 * STAGES + s); };
    auto raw_full = [&](int s) { return bar + 8 * (3 * STAGES + s); };
    auto raw_empty = [&](int s) { return bar + 8 * (3 * STAGES + RAW_STAGES + s); };
    auto sc_full = [&](int s) { return bar + 8 * (3 * STAGES + 2 * RAW_STAGES + s); };
    auto sc_empty = [&](int s) { return bar + 8 * (3 * STAGES + 2 * RAW_STAGES + SC_STAGES + s); };
    auto t_empty = [&](int s) { return bar + 8 * (3 * STAGES + 2 * RAW_STAGES + 2 * SC_STAGES + s); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::OFF_MISC + 4);
    float *sc_base = reinterpret_cast<float *>(smem + L::OFF_SC);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(a_full(s), 1);
            mbar_init(b_full(s), UNPACK_THREADS);
            mbar_init(done(s), 1);
        }
        for (int s = 0; s < RAW_STAGES; s++) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), UNPACK_THREADS);
        }
        for (int s = 0; s < SC_STAGES; s++) {
            // filled by TMA (PRE), or by the unpackers plus the producer's
            // TMA of the activation scales
            mbar_init(sc_full(s), PRE ? 1 : UNPACK_THREADS + (DOTS ? 0 : 1));
            mbar_init(sc_empty(s), EPI_WARPS * 32);
        }
        for (int s = 0; s < NSLOT; s++) mbar_init(t_empty(s), EPI_WARPS * 32);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(NSLOT * TN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int npairs = nb / 2, nchunks = nb / CHUNK;

    // One chunk's scales into scale stage cc % SC_STAGES: on the copy path the
    // weight-scale (and offset) plane tiles, and unless DOTS the token scales.
    // (On the raw path the unpackers write the weight scales.)
    auto load_scales = [&](uint32_t cc, int c, int gw, int m0, int n0) -> bool {
        const int ss = cc % SC_STAGES;
        if (!mbar_wait(sc_empty(ss), ((cc / SC_STAGES) & 1) ^ 1, abort_flag, err)) return false;
        const uint32_t dst = sbase + L::OFF_SC + ss * L::SC_FLOATS * 4;
        mbar_expect_tx(sc_full(ss), (PRE ? L::SC_DA * 4 : 0) + (DOTS ? 0 : L::DA_BYTES));
        if (PRE) {
            tma_load_2d(dst, &P.sc[gw], n0, c * CHUNK, sc_full(ss));
            if (has_offset(TYPE)) tma_load_2d(dst + CHUNK * TN * 4, &P.off[gw], n0, c * CHUNK, sc_full(ss));
        }
        if (!DOTS) {
            tma_load_2d(dst + L::SC_DA * 4, &P.da, c * CHUNK, m0, sc_full(ss));
            if (has_offset(TYPE)) tma_load_2d(dst + L::SC_DA * 4 + CHUNK * BM * 4, &P.ds, c * CHUNK, m0, sc_full(ss));
        }
        return true;
    };

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        // operand tiles (and on the raw path the raw chunks and token scales);
        // on the copy path warp 2 loads the scales, so this thread waits only
        // for operand stages to come free and runs up to STAGES pairs ahead
        if (lane == 0) {
            uint32_t pc = 0, cc = 0;  // pairs and chunks issued, over all tiles
            bool ok = true;
            for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                int m0, n0;
                const int gw = tile_weight<TN>(P, tile, m0, n0);
                for (int p = 0; p < npairs; p++, pc++) {
                    if ((2 * p) % CHUNK == 0) {
                        const int c = (2 * p) / CHUNK;
                        if (!PRE) {
                            const int rs = cc % RAW_STAGES;
                            if (!mbar_wait(raw_empty(rs), ((cc / RAW_STAGES) & 1) ^ 1, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            mbar_expect_tx(raw_full(rs), L::RAW_BYTES);
                            tma_load_2d(sbase + L::OFF_RAW + rs * align_up(L::RAW_BYTES, 1024), &P.w[gw],
                                        c * (L::RAW_ROW / 2), n0, raw_full(rs));
                        }
                        if (!PRE && !DOTS && !load_scales(cc, c, gw, m0, n0)) {
                            ok = false;
                            break;
                        }
                        cc++;
                    }
                    const int s = pc % STAGES;
                    if (!mbar_wait(done(s), ((pc / STAGES) & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(a_full(s), L::A_BYTES + (PRE ? L::B_BYTES : 0));
                    tma_load_2d(sbase + L::OFF_A + s * L::A_BYTES, &P.a, 2 * p * 32, m0, a_full(s));
                    if (PRE) tma_load_2d(sbase + L::OFF_B + s * L::B_BYTES, &P.b[gw], 2 * p * 32, n0, a_full(s));
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t pc = 0;  // block pairs consumed, over all tiles
            const uint64_t adesc0 = umma_desc_sw128(sbase + L::OFF_A), bdesc0 = umma_desc_sw128(sbase + L::OFF_B);
            bool ok = true;
            for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                for (int p = 0; p < npairs; p++, pc++) {
                    const int s = pc % STAGES, ps = pc % (NSLOT / 2);
                    const uint32_t ph = (pc / STAGES) & 1;
                    if (!mbar_wait(a_full(s), ph, abort_flag, err) ||
                        (!PRE && !mbar_wait(b_full(s), ph, abort_flag, err))) {
                        ok = false;
                        break;
                    }
                    // One wait for the pair's two slots, on the second: every
                    // epilogue thread releases the first before it, so its
                    // phase completing implies the first's (the slots come
                    // free ~1,200 cycles before they are needed). Descriptors
                    // advance in 16-byte units: +jb*64 bytes per block, +32
                    // bytes per K=16 step.
                    if (!mbar_wait(t_empty(2 * ps + 1), ((pc / (NSLOT / 2)) & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int jb = 0; jb < 2; jb++) {
#pragma unroll
                        for (int k = 0; k < 2; k++) {
                            const uint32_t off = (uint32_t)(jb * 64 + 32 * k) >> 4;
                            umma_f16<TN>(tmem_base + (2 * ps + jb) * TN, adesc0 + (uint32_t)(s * L::A_BYTES >> 4) + off,
                                     bdesc0 + (uint32_t)(s * L::B_BYTES >> 4) + off, k);
                        }
                    }
                    if (!ok) break;
                    umma_commit(done(s));
                }
            }
        }
    } else if (warp < 4) {
        // ------------------------------------------------------ unpackers
        if (PRE) {
            // copy path: warp 2 loads the scales, one chunk per scale stage
            if (warp == 2 && lane == 0) {
                uint32_t cc = 0;
                bool ok = true;
                for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                    int m0, n0;
                    const int gw = tile_weight<TN>(P, tile, m0, n0);
                    for (int c = 0; c < nchunks; c++, cc++)
                        if (!load_scales(cc, c, gw, m0, n0)) {
                            ok = false;
                            break;
                        }
                }
            }
            goto done;
        }
        const int ut = threadIdx.x - 64;
        uint32_t pc = 0, cc = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            for (int c = 0; c < nchunks; c++, cc++) {
                const int rs = cc % RAW_STAGES, ss = cc % SC_STAGES;
                if (!mbar_wait(raw_full(rs), (cc / RAW_STAGES) & 1, abort_flag, err) ||
                    !mbar_wait(sc_empty(ss), ((cc / SC_STAGES) & 1) ^ 1, abort_flag, err)) {
                    ok = false;
                    break;
                }
                const uint8_t *raw = smem + L::OFF_RAW + rs * align_up(L::RAW_BYTES, 1024);
                float *sc = sc_base + ss * L::SC_FLOATS;
                for (int pp = 0; pp < CHUNK / 2; pp++, pc++) {
                    const int s = pc % STAGES;
                    if (!mbar_wait(done(s), ((pc / STAGES) & 1) ^ 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *bst = smem + L::OFF_B + s * L::B_BYTES;
#pragma unroll
                    for (int rr = 0; rr < TN / 64; rr++) {
                        const int r = ut + rr * 64;
#pragma unroll
                        for (int jb = 0; jb < 2; jb++) {
                            const int j = 2 * pp + jb;
                            const uint8_t *blk = raw + r * L::RAW_ROW + j * L::BB;
                            uint32_t o[16];
                            unpack_block<TYPE>(blk, o);
#pragma unroll
                            for (int cq = 0; cq < 4; cq++) {
                                const int chunk16 = jb * 4 + cq;
                                const uint4 v = make_uint4(o[4 * cq], o[4 * cq + 1], o[4 * cq + 2], o[4 * cq + 3]);
                                *reinterpret_cast<uint4 *>(bst + r * 128 + ((chunk16 ^ (r & 7)) << 4)) = v;
                            }
                            sc[j * TN + r] = h2f(*reinterpret_cast<const uint16_t *>(blk));
                            if (has_offset(TYPE))
                                sc[CHUNK * TN + j * TN + r] = h2f(*reinterpret_cast<const uint16_t *>(blk + 2));
                        }
                    }
                    fence_proxy_async();
                    mbar_arrive(b_full(s));
                }
                if (!ok) break;
                mbar_arrive(raw_empty(rs));
                mbar_arrive(sc_full(ss));
            }
        }
    } else {
        // ------------------------------------------------------ epilogue
        // Warp (q, g) covers TMEM lane quarter q = warp % 4 (tokens 32q ..
        // 32q+31) and columns 32g .. 32g+31. A tcgen05.ld of shape 16x256b gives
        // each thread, per 8 columns, 2 adjacent columns (2(lane%4) + {0,1}) of
        // 2 tokens (lane/4 and lane/4 + 8 of a 16-lane half); two loads cover
        // the quarter. A thread so owns 4 tokens x 8 columns and reads each
        // weight scale once for 4 tokens and each token scale once for 8 columns.
        // (with 64-wide tiles, 16 columns: 2 tokens x 2 columns per load and the
        // thread's 4 tokens x 4 columns)
        constexpr int ECOLS = epi_cols<TN>(), NI = ECOLS / 8;
        const int q = warp & 3;
        const int g = (warp - 4) >> 2;
        const int tr = lane >> 2, tcol = g * ECOLS + (lane & 3) * 2;
        // byte offsets inside a scale stage: this thread's weight-scale pairs,
        // and its first token's scale row for blocks 0-3 / 4-7 (the 32-byte
        // swizzle moves the row's halves by +-16 bytes when bit 2 of tr is set)
        const uint32_t w_off = (uint32_t)tcol * 4;
        const uint32_t s16 = ((tr >> 2) & 1) << 4;
        const uint32_t d_off = L::SC_DA * 4 + (uint32_t)(q * 32 + tr) * (CHUNK * 4);
        const uint32_t d_lo = d_off + s16, d_hi = d_off - s16;
        const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16) + g * ECOLS;
        uint32_t cc = 0;               // chunks consumed, over all tiles
        uint32_t dstage = 0, dphase = 0;  // next block pair's commit barrier and parity
        bool ok = true;
        constexpr bool PAIRS = has_offset(TYPE);
        for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            int m0, n0;
            const int gw = tile_weight<TN>(P, tile, m0, n0);
            const int N = P.n[gw];
            const bool warp_live = m0 + q * 32 < M;
            // the accumulators of columns tcol + 8i and tcol + 8i + 1 of token k:
            // f[8k + 2i + e] as scalars, or (offset types, whose two chain steps
            // per block pair up better) f2[4k + i] as one f32 pair, each lane of
            // a packed fma being the scalar fma of its output
            float f[PAIRS ? 1 : 8 * NI];
            uint64_t f2[PAIRS ? 4 * NI : 1];
#pragma unroll
            for (int i = 0; i < (PAIRS ? 1 : 8 * NI); i++) f[i] = 0.0f;
#pragma unroll
            for (int i = 0; i < (PAIRS ? 4 * NI : 1); i++) f2[i] = 0;
            // One chunk of CHUNK blocks. LIVE: the warp's tokens exist (a warp
            // past the last token only keeps the barriers in step). The block
            // loop has no divergent branch: its waits are warp-uniform votes
            // and every lane arrives on the release barriers.
            auto chunk = [&](auto live, int c) -> bool {
                constexpr bool LIVE = decltype(live)::value;
                const int ss = cc % SC_STAGES;
                if (!mbar_wait_warp(sc_full(ss), (cc / SC_STAGES) & 1, abort_flag, err)) return false;
                const uint32_t sc_s = sbase + L::OFF_SC + ss * L::SC_FLOATS * 4;
                const uint32_t w_s = sc_s + w_off, dlo_s = sc_s + d_lo, dhi_s = sc_s + d_hi;
#pragma unroll
                for (int j = 0; j < CHUNK; j++) {
                    const int kb = c * CHUNK + j, slot = j % NSLOT;  // chunks start on slot 0
                    if (j % 2 == 0) {
                        const bool got = mbar_wait_warp(done(dstage), dphase, abort_flag, err);
                        if (++dstage == STAGES) dstage = 0, dphase ^= 1;
                        if (!got) return false;
                        tc_fence_after();
                    }
                    if (LIVE) {
                        uint64_t w2[NI], o2[NI];
                        float dav[4], dsv[4];
                        if (!DOTS) {
#pragma unroll
                            for (int i = 0; i < NI; i++) {
                                w2[i] = lds_b64(w_s + j * TN * 4 + 32 * i);
                                if (PAIRS) o2[i] = lds_b64(w_s + (CHUNK + j) * TN * 4 + 32 * i);
                            }
                            const uint32_t d_s = (j < 4 ? dlo_s : dhi_s) + 4 * j;
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                dav[k] = lds_f32(d_s + k * 8 * CHUNK * 4);
                                if (PAIRS) dsv[k] = lds_f32(d_s + CHUNK * BM * 4 + k * 8 * CHUNK * 4);
                            }
                        }
#pragma unroll
                        for (int hh = 0; hh < 2; hh++) {
                            uint32_t r[4 * NI];
                            tmem_ld16x256(t_lane + ((uint32_t)(16 * hh) << 16) + slot * TN, r);
                            if (DOTS) {
#pragma unroll
                                for (int kk = 0; kk < 2; kk++) {
                                    const int m = m0 + q * 32 + tr + 8 * (2 * hh + kk);
                                    if (m >= M) continue;
#pragma unroll
                                    for (int i = 0; i < NI; i++)
#pragma unroll
                                        for (int e = 0; e < 2; e++) {
                                            const int n = n0 + tcol + 8 * i + e;
                                            if (n < N)
                                                dots[((int64_t)m * N + n) * nb + kb] =
                                                    (int32_t)__uint_as_float(r[4 * i + 2 * kk + e]);
                                        }
                                }
                            } else {
#pragma unroll
                                for (int kk = 0; kk < 2; kk++) {
                                    const int k = 2 * hh + kk;
                                    const uint64_t da2 = pack2u(__float_as_uint(dav[k]), __float_as_uint(dav[k]));
#pragma unroll
                                    for (int i = 0; i < NI; i++) {
                                        // the two scale products as one f32x2 multiply
                                        const uint64_t p2 = mul2(w2[i], da2);
                                        if (PAIRS) {
                                            f2[NI * k + i] = fma2(pack2u(r[4 * i + 2 * kk], r[4 * i + 2 * kk + 1]),
                                                                 p2, f2[NI * k + i]);
                                        } else {
                                            float *fk = f + 2 * NI * k + 2 * i;
                                            fk[0] = __fmaf_rn(__uint_as_float(r[4 * i + 2 * kk]), lo_f(p2), fk[0]);
                                            fk[1] = __fmaf_rn(__uint_as_float(r[4 * i + 2 * kk + 1]), hi_f(p2),
                                                              fk[1]);
                                        }
                                    }
                                    if (PAIRS) {
                                        const uint64_t ds2 = pack2u(__float_as_uint(dsv[k]), __float_as_uint(dsv[k]));
#pragma unroll
                                        for (int i = 0; i < NI; i++) f2[NI * k + i] = fma2(o2[i], ds2, f2[NI * k + i]);
                                    }
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(t_empty(slot));
                }
                mbar_arrive(sc_empty(ss));
                return true;
            };
            for (int c = 0; c < nchunks; c++, cc++) {
                const bool good = warp_live ? chunk(std::true_type{}, c) : chunk(std::false_type{}, c);
                if (!good) {
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            if (!DOTS && !*abort_flag) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int m = m0 + q * 32 + tr + 8 * k;
                    if (m >= M) continue;
                    float *dst = P.y[gw] + (int64_t)m * P.ldy[gw] + n0 + tcol;
#pragma unroll
                    for (int i = 0; i < NI; i++) {
                        if (n0 + tcol + 8 * i >= N) break;
                        float2 v = PAIRS ? make_float2(lo_f(f2[NI * k + i]), hi_f(f2[NI * k + i]))
                                         : make_float2(f[2 * NI * k + 2 * i], f[2 * NI * k + 2 * i + 1]);
                        if (EPI == EPI_ADD) {
                            const float2 o = *reinterpret_cast<const float2 *>(dst + 8 * i);
                            v.x = __fadd_rn(o.x, v.x);
                            v.y = __fadd_rn(o.y, v.y);
                        }
                        *reinterpret_cast<float2 *>(dst + 8 * i) = v;
                    }
                }
            }
        }
    }
done:
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(NSLOT * TN));
    }
}

// ------------------------------------------------------------------ host

static int64_t g_pre_min = -1;
static int g_tile_width = 0;  // 0: by the grid size; 64 or 128: forced
static int64_t pre_min_tokens();

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Activations: f16 [M][K], box 64 x 128 rows, 128B swizzle.
static bool map_activations(CUtensorMap *m, const __half *a, int64_t M, int64_t K, int box_rows = BM) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)a, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw weights: rows of 16-bit units, box = one 8-block chunk x 128 rows.
static bool map_weights(CUtensorMap *m, const DevWeight &w, int raw_row, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)(w.row_bytes / 2), (cuuint64_t)w.rows};
    cuuint64_t strides[1] = {(cuuint64_t)w.row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(raw_row / 2), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)w.data, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// f32 scale (or offset) plane [K/32][rows], box = 128 features x 8 blocks.
static bool map_plane(CUtensorMap *m, const float *plane, int64_t rows, int64_t nb, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)rows, (cuuint64_t)nb};
    cuuint64_t strides[1] = {(cuuint64_t)(rows * 4)};
    cuuint32_t box[2] = {(cuuint32_t)box_rows, CHUNK};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)plane, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-token activation scales, [M][nb] f32 -> box of CHUNK blocks x BM tokens,
// 32-byte swizzled in shared memory: token T's scale for block j is word
// T * CHUNK + (j ^ 4 * bit 2 of T) (the 16-byte halves of a 32-byte row swap
// when bit 2 of the row is set), which spreads 8 consecutive tokens over all
// banks; the epilogue's d_lo / d_hi offsets encode it.
static bool map_token_scales(CUtensorMap *m, const float *d, int64_t M, int64_t nb) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)nb, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(nb * 4)};
    cuuint32_t box[2] = {CHUNK, BM};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)d, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

// SMs of the current device (persistent grid sizes, wave counts), cached per
// device.
int sm_count_of_device() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

namespace tc {
static int sm_count() { return sm_count_of_device(); }

// One weight of a launch: its matrix, where its outputs go and their row stride.
struct GemmOut {
    const DevWeight *w;
    float *y;
    int64_t ldy;
};

template <int TYPE, int EPI, bool DOTS, bool PRE, int TN>
static cudaError_t launch_t(const GemmOut *outs, int count, const QAct &q, int32_t *err, int32_t *dots,
                            cudaStream_t s) {
    using L = Smem<TYPE, TN, PRE>;
    if (count < 1 || count > GMAX) return cudaErrorInvalidValue;
    const int64_t K = outs[0].w->cols;
    TcParams P;
    memset(&P, 0, sizeof(P));
    if (!map_activations(&P.a, q.a16, q.M, K)) return cudaErrorInvalidValue;
    P.da = P.ds = P.a;  // placeholders for the maps a variant never reads
    if (!DOTS) {
        if (!map_token_scales(&P.da, q.da, q.M, K / 32)) return cudaErrorInvalidValue;
        if (has_offset(TYPE) && !map_token_scales(&P.ds, q.ds, q.M, K / 32)) return cudaErrorInvalidValue;
    }
    const int64_t ntm = (q.M + BM - 1) / BM;
    P.count = count;
    P.tile0[0] = 0;
    for (int g = 0; g < count; g++) {
        const DevWeight &w = *outs[g].w;
        if (w.type != TYPE || w.cols != K) return cudaErrorInvalidValue;
        if (!map_weights(&P.w[g], w, L::RAW_ROW, TN)) return cudaErrorInvalidValue;
        P.b[g] = P.sc[g] = P.off[g] = P.w[g];
        if (PRE) {
            if (!map_activations(&P.b[g], w.w16, w.rows, w.cols, TN) ||
                !map_plane(&P.sc[g], w.scale_plane, w.rows, w.cols / 32, TN))
                return cudaErrorInvalidValue;
            if (has_offset(TYPE) && !map_plane(&P.off[g], w.offset_plane, w.rows, w.cols / 32, TN))
                return cudaErrorInvalidValue;
        }
        P.y[g] = outs[g].y;
        P.ldy[g] = outs[g].ldy;
        P.n[g] = (int)w.rows;
        P.ntn[g] = (int)((w.rows + TN - 1) / TN);
        P.tile0[g + 1] = P.tile0[g] + (int64_t)P.ntn[g] * ntm;
    }
    auto kern = k_gemm_tc<TYPE, EPI, DOTS, PRE, TN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)std::min<int64_t>(P.tile0[count], sm_count());
    kern<<<grid, THREADS, L::BYTES, s>>>(P, (int)q.M, (int)(K / 32), err, dots);
    return cudaGetLastError();
}

template <int EPI, bool DOTS, bool PRE, int TN>
static cudaError_t dispatch_t(const GemmOut *outs, int count, const QAct &q, int32_t *err, int32_t *dots,
                              cudaStream_t s) {
    switch (outs[0].w->type) {
    case T_Q4_0: return launch_t<T_Q4_0, EPI, DOTS, PRE, TN>(outs, count, q, err, dots, s);
    case T_Q4_1: return launch_t<T_Q4_1, EPI, DOTS, PRE, TN>(outs, count, q, err, dots, s);
    case T_Q5_0: return launch_t<T_Q5_0, EPI, DOTS, PRE, TN>(outs, count, q, err, dots, s);
    case T_Q5_1: return launch_t<T_Q5_1, EPI, DOTS, PRE, TN>(outs, count, q, err, dots, s);
    case T_Q8_0: return launch_t<T_Q8_0, EPI, DOTS, PRE, TN>(outs, count, q, err, dots, s);
    default: return cudaErrorNotSupported;
    }
}

// Every token batch reads the pre-unpacked copy when the weight has one: on
// the raw blocks each 128-token tile unpacks the whole weight again, and two
// unpacker warps cannot keep up even at 17-255 tokens (the copy is 1.1-2.4x
// faster there). The raw-block kernel serves weights without a copy.
constexpr int64_t PRE_MIN_TOKENS = 1;
static int64_t pre_min_tokens() { return g_pre_min >= 0 ? g_pre_min : PRE_MIN_TOKENS; }

static bool has_copy(const DevWeight &w) {
    return w.w16 && w.scale_plane && (!has_offset(w.type) || w.offset_plane);
}

// 64-wide tiles when 128-wide ones would leave more than half of the SMs
// idle (few tokens): twice the tiles, half the epilogue work per block.
static bool narrow_tiles(const GemmOut *outs, int count, const QAct &q) {
    int64_t tiles = 0;
    for (int g = 0; g < count; g++) tiles += (outs[g].w->rows + BN - 1) / BN;
    tiles *= (q.M + BM - 1) / BM;
    return g_tile_width != 128 && (g_tile_width == 64 || 2 * tiles <= sm_count());
}

template <int EPI, bool DOTS>
static cudaError_t dispatch(const GemmOut *outs, int count, const QAct &q, int32_t *err, int32_t *dots,
                            cudaStream_t s) {
    bool pre = q.M >= pre_min_tokens();
    for (int g = 0; g < count; g++) pre = pre && has_copy(*outs[g].w);
    if (!DOTS && narrow_tiles(outs, count, q))
        return pre ? dispatch_t<EPI, DOTS, true, 64>(outs, count, q, err, dots, s)
                   : dispatch_t<EPI, DOTS, false, 64>(outs, count, q, err, dots, s);
    return pre ? dispatch_t<EPI, DOTS, true, 128>(outs, count, q, err, dots, s)
               : dispatch_t<EPI, DOTS, false, 128>(outs, count, q, err, dots, s);
}

}  // namespace tc

// Token count from which the tensor-core GEMM reads the pre-unpacked weights
// (negative: the built-in default). Used by tests to cover both paths.
void gemm_tc_set_pre_min_tokens(int64_t m) { tc::g_pre_min = m; }

// Tile width of the tensor-core GEMM: 0 chooses by the grid size, 64 or 128
// forces it (tests cover both).
void gemm_tc_set_tile_width(int w) { tc::g_tile_width = w; }

bool gemm_tc_supports(const DevWeight &w, int64_t M) {
    if (!block_bytes(w.type) || w.cols % 256 || w.rows % 16 || M < 1 || M > (1LL << 31) - 1) return false;
    if (w.row_bytes % 16 || reinterpret_cast<uintptr_t>(w.data) % 16) return false;
    if (w.rows / tc::BN > 65535 || (M + tc::BM - 1) / tc::BM > 65535) return false;
    return tc::encode_fn() != nullptr;
}

static bool tc_output_ok(const float *y, int64_t ldy) {
    return ldy % 4 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
}

static bool tc_activations_ok(const DevWeight &w, const QAct &q) {
    return q.a16 && reinterpret_cast<uintptr_t>(q.a16) % 16 == 0 && reinterpret_cast<uintptr_t>(q.da) % 16 == 0 &&
           (!has_offset(w.type) || reinterpret_cast<uintptr_t>(q.ds) % 16 == 0);
}

cudaError_t launch_gemm_tc(const DevWeight &w, const QAct &q, float *y, int64_t ldy, int epi, int32_t *err,
                           cudaStream_t s) {
    if (!gemm_tc_supports(w, q.M) || !tc_activations_ok(w, q) || !tc_output_ok(y, ldy)) return cudaErrorNotSupported;
    if (q.M == 0) return cudaSuccess;
    const tc::GemmOut out{&w, y, ldy};
    return epi == EPI_ADD ? tc::dispatch<EPI_ADD, false>(&out, 1, q, err, nullptr, s)
                          : tc::dispatch<EPI_STORE, false>(&out, 1, q, err, nullptr, s);
}

cudaError_t launch_gemm_tc_group(const DevWeight *const *ws, float *const *ys, const int64_t *ldys, int count,
                                 const QAct &q, int epi, int32_t *err, cudaStream_t s) {
    if (count < 1 || count > tc::GMAX) return cudaErrorNotSupported;
    tc::GemmOut outs[tc::GMAX];
    for (int g = 0; g < count; g++) {
        if (!gemm_tc_supports(*ws[g], q.M) || !tc_activations_ok(*ws[g], q) || !tc_output_ok(ys[g], ldys[g]) ||
            ws[g]->type != ws[0]->type || ws[g]->cols != ws[0]->cols)
            return cudaErrorNotSupported;
        outs[g] = tc::GemmOut{ws[g], ys[g], ldys[g]};
    }
    if (q.M == 0) return cudaSuccess;
    return epi == EPI_ADD ? tc::dispatch<EPI_ADD, false>(outs, count, q, err, nullptr, s)
                          : tc::dispatch<EPI_STORE, false>(outs, count, q, err, nullptr, s);
}

cudaError_t launch_block_dots_tc(const DevWeight &w, const QAct &q, int32_t *dots, int32_t *err, cudaStream_t s) {
    if (!gemm_tc_supports(w, q.M) || !q.a16) return cudaErrorNotSupported;
    const tc::GemmOut out{&w, nullptr, 0};
    return tc::dispatch<EPI_STORE, true>(&out, 1, q, err, dots, s);
}

}  // namespace shield
