// decode_kernel.cu -- the opt-125m decode step as ONE persistent kernel for sm_100a.
//
// Replaces the reference's per-token decode: rust/npu-whisper/src/bin/opt125m_decode.rs
// Opt::step (252-293) / Opt::generate (296-315) on the host, and the fused NPU decode ELF
// route_b_kernels/decode_fused/gen_decode.py (runlist 391-425).
//
// A batch-1 decode token is latency-bound (about 128 MB of weights, but dozens of dependent
// steps), so the design minimises the dependent global exchanges per layer -- two -- and
// keeps every step between them short:
//  * one CTA per SM, clusters of 2, each CTA = 8 consumer warps + 1 producer warp.  The roles
//    (head pair / FC / spare) and the exact-integer accumulator words are described in
//    decode.h.
//  * every weight byte a CTA needs for a token is pre-packed on the host into ONE contiguous
//    stream in consumption order and in mma.sync fragment order; the producer warp streams it
//    with 1-D bulk async copies (cp.async.bulk + mbarrier complete_tx, no multicast) through
//    an 8 x 16 KB ring.  Weights do not depend on activations, so HBM streaming runs ahead of
//    the layer chain and only stalls when the ring is full.
//  * GEMV = int8 tensor-core MMA (m16n8k32, weights = A, 16 output rows per MMA): the bf16
//    activation vector becomes a 29-bit fixed-point integer X split into four int8 limbs,
//    which are the four live columns of B.  Limb sums are combined exactly in int64 and
//    rounded once to f32: every dot product is exact, so the result does not depend on how K
//    is split and the CPU oracle reproduces it bit for bit.
//  * layer chain: [all CTAs: residual += fc2 of the previous layer (accumulator words)] ->
//    head pairs: LayerNorm (each warp redundantly, no block barrier), q|k|v of their 32 dims,
//    partial scores swapped with the other CTA of the pair by st.async into its shared memory,
//    softmax, P.V of their dims, K-split out projection added into the accumulator words ->
//    [all CTAs: residual += out projection] -> FC CTAs: LayerNorm, fc1 rows, ReLU, K-split fc2
//    added into the accumulator words.
//  * every wait is bounded (globaltimer deadline); a timeout records an error code in
//    RunState, the CTA's threads agree on leaving through a barrier reduction, the producer
//    drains its in-flight copies, and both CTAs of a cluster meet at a final cluster barrier
//    (so neither exits while the other may still write into its shared memory).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cmath>
#include <algorithm>

#include "decode.h"
#include "ptx.cuh"

namespace xdna {

// ------------------------------------------------------------------------------ smem map
struct SmemMap {
    static constexpr int ring = 0;
    static constexpr int kvst = ring + kSlots * kSlotBytes;              // staged K | V (32 KB)
    static constexpr int kvst_bytes = 2 * kStageKeys * kHalfDim * 2;
    static constexpr int ps = kvst + kvst_bytes;                         // [2][kMaxCtx] f32
    static constexpr int lnp = ps + 2 * kMaxCtx * 4;                     // [2][g|b][kDmax] f32
    static constexpr int part = lnp + 4 * kDmax * 4;                     // [8][96][4] int32
    static constexpr int part_rows = 96;
    static constexpr int xs = part + kConsumerWarps * part_rows * 4 * 4; // [kDmax] f32 residual
    static constexpr int limbs = xs + kDmax * 4;                         // [4][kLimbStride] int8
    static constexpr int own = limbs + kLimbs * kLimbStride;            // [kMaxCtx] f32
    static constexpr int misc = own + kMaxCtx * 4;
    static constexpr int misc_bytes = 2048;
    static constexpr int bars = misc + misc_bytes;
    static constexpr int total = bars + (2 * kSlots + 2) * 8;
};
static_assert(SmemMap::total <= 227 * 1024, "shared memory budget");
static_assert(kChunkKeys * kHalfDim * 2 <= SmemMap::kvst_bytes, "key chunk fits the staging area");
static_assert(kSliceTilesPerChunk * kFragBytes <= kSlotBytes, "slice chunk fits a slot");
static_assert(kTile * kDmax + kTile * 8 <= kSlotBytes, "row chunk fits a slot");
static_assert(kDmax / kTile * kFragBytes <= SmemMap::kvst_bytes, "slice epilogue scratch fits the staging area");

// limb column of the K-split GEMV inputs (attention context dims / fc1 rows)
constexpr int kSlimbOff = 1024;

extern __shared__ __align__(1024) uint8_t dsmem[];

struct Cta {
    uint8_t *ring;
    uint16_t *kst, *vst;        // staged K rows (64 B, 16-byte chunks swizzled by row & 3), V rows
    float *ps;                  // [2][kMaxCtx]: the pair's partial scores, then probabilities
    float *own;                 // [kMaxCtx]: this CTA's partial scores, then the full scores
    float *lnp;                 // [2 buffers][gamma | beta][kDmax]
    int *part;                  // [warp][row][limb] partial limb sums
    float *x;                   // residual stream
    int8_t *limbs;              // [limb][kLimbStride]
    float *qf;                  // [32] q of the own dims (bf16 values)
    uint16_t *kcur, *vcur;      // [32] k, v of the current position (kcur swizzled like kst)
    float *red;                 // [64] reductions
    float *accg;                // [8][32] P.V group partials
    unsigned long long *keys;   // [8] argmax keys
    int *pt;                    // [kMaxPages] page table
    int *flag;                  // [0] abort, [1] next token id
    uint64_t *full, *empty, *xchg;
    int tid, warp, lane;
};

__device__ __forceinline__ Cta make_cta() {
    uint8_t *s = dsmem;
    Cta S;
    S.ring = s + SmemMap::ring;
    S.kst = reinterpret_cast<uint16_t *>(s + SmemMap::kvst);
    S.vst = S.kst + kStageKeys * kHalfDim;
    S.ps = reinterpret_cast<float *>(s + SmemMap::ps);
    S.lnp = reinterpret_cast<float *>(s + SmemMap::lnp);
    S.part = reinterpret_cast<int *>(s + SmemMap::part);
    S.x = reinterpret_cast<float *>(s + SmemMap::xs);
    S.limbs = reinterpret_cast<int8_t *>(s + SmemMap::limbs);
    S.own = reinterpret_cast<float *>(s + SmemMap::own);
    uint8_t *m = s + SmemMap::misc;
    S.qf = reinterpret_cast<float *>(m);                          // 128 B
    S.kcur = reinterpret_cast<uint16_t *>(m + 128);               // 64 B
    S.vcur = reinterpret_cast<uint16_t *>(m + 192);               // 64 B
    S.red = reinterpret_cast<float *>(m + 256);                   // 256 B
    S.accg = reinterpret_cast<float *>(m + 512);                  // 1024 B
    S.keys = reinterpret_cast<unsigned long long *>(m + 1536);    // 64 B
    S.pt = reinterpret_cast<int *>(m + 1600);                     // 128 B
    S.flag = reinterpret_cast<int *>(m + 1728);                   // 32 B
    S.full = reinterpret_cast<uint64_t *>(s + SmemMap::bars);
    S.empty = S.full + kSlots;
    S.xchg = S.empty + kSlots;
    S.tid = threadIdx.x;
    S.warp = threadIdx.x >> 5;
    S.lane = threadIdx.x & 31;
    return S;
}

// ------------------------------------------------------------------ small PTX helpers
__device__ __forceinline__ void cbar() { named_bar(1, kConsumerThreads); }
// consumer barrier that also ORs a predicate over the 256 consumer threads (uniform result)
__device__ __forceinline__ bool cbar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ uint32_t mapa_peer(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_async_b32(uint32_t raddr, uint32_t v, uint32_t rbar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
                 "r"(v), "r"(rbar)
                 : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, uint32_t cnt) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(cnt) : "memory");
}
__device__ __forceinline__ void red_add_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------------- error handling
__device__ __forceinline__ uint32_t read_error(const RunState *st) {
    return *reinterpret_cast<const volatile uint32_t *>(&st->error);
}
__device__ __noinline__ void set_error_st(RunState *st, uint32_t code, uint32_t where) {
    if (atomicCAS(&st->error, 0u, code) == 0u) {
        st->error_cta = blockIdx.x;
        st->error_where = where;
    }
}
// Slow path of every bounded wait, called every few dozen polls: true when the waiter must
// give up -- the CTA's abort flag is up, another CTA already failed, or the deadline (counted
// from the first call, *t0) passed, in which case this CTA records the timeout.
__device__ __noinline__ bool wait_expired(RunState *st, uint64_t timeout_ns, int *sflag, uint64_t *t0,
                                          uint32_t code, uint32_t where) {
    if (*(volatile int *)sflag != 0 || read_error(st) != 0) { *(volatile int *)sflag = 1; return true; }
    const uint64_t now = globaltimer_ns();
    if (*t0 == 0) { *t0 = now; return false; }
    if (now - *t0 > timeout_ns) {
        set_error_st(st, code, where);
        *(volatile int *)sflag = 1;
        return true;
    }
    return false;
}

// Wait for the chunks with stream indices ctr .. ctr+n-1 (n <= kSlots) to be in their ring
// slots; false on timeout / abort.  Warp-collective: lane i watches chunk ctr + i itself (so
// every lane that reads a chunk has the completed phase ordered before its reads through the
// warp-wide vote), and all lanes get the same answer.
__device__ __forceinline__ bool wait_chunks(const DecodeParams &p, const Cta &S, uint32_t ctr, int n, uint32_t where) {
    const uint32_t q = ctr + (uint32_t)S.lane;
    bool mine = S.lane >= n || mbar_try_wait(&S.full[q % kSlots], (q / kSlots) & 1u);
    if (__all_sync(0xffffffffu, mine)) return true;
    uint64_t t0 = 0;
    uint32_t it = 0;
    while (true) {
        if (!mine) mine = mbar_try_wait(&S.full[q % kSlots], (q / kSlots) & 1u);
        if (__all_sync(0xffffffffu, mine)) return true;
        if ((++it & 15) == 0) {
            const bool gone = S.lane == 0 && wait_expired(p.state, p.timeout_ns, S.flag, &t0, ERR_TIMEOUT_FULL, where);
            if (__shfl_sync(0xffffffffu, gone, 0)) return false;
        }
    }
}
__device__ __forceinline__ bool wait_full(const DecodeParams &p, const Cta &S, uint32_t ctr, uint32_t where) {
    return wait_chunks(p, S, ctr, 1, where);
}
__device__ __forceinline__ const uint8_t *slot_ptr(const Cta &S, uint32_t ctr) {
    return S.ring + (ctr % kSlots) * kSlotBytes;
}
// the consumer warps release a slot: one arrival per warp
__device__ __forceinline__ void release_slot(const Cta &S, uint32_t ctr) {
    __syncwarp();
    if (S.lane == 0) mbar_arrive(&S.empty[ctr % kSlots]);
}

// optional phase timestamps (first two steps of a launch)
__device__ __forceinline__ void stamp(const DecodeParams &p, const Cta &S, int t, int slot) {
    if (p.timing == nullptr || t >= 2 || S.tid != 0) return;
    p.timing[((size_t)t * p.grid + blockIdx.x) * 128 + slot] = globaltimer_ns();
}
// SM cycle counter into slot 64 + k (same record)
__device__ __forceinline__ void stamp_clk(const DecodeParams &p, const Cta &S, int t, int k) {
    if (p.timing == nullptr || t >= 2 || S.tid != 0) return;
    p.timing[((size_t)t * p.grid + blockIdx.x) * 128 + 64 + k] = clock64();
}

// e^x for x <= 0 with the reference's own 2^floor x degree-5 polynomial
// (rust/npu-asr-host/src/lib.rs:38-58, the exp of its host softmax), every operation
// rounded separately so the CPU oracle reproduces it bit for bit.
__device__ __forceinline__ float fast_exp_nonpos(float x) {
    if (x < -87.0f) x = -87.0f;
    const float y = __fmul_rn(x, 1.442695040888963f);
    const float yf = floorf(y);
    const float f = __fsub_rn(y, yf);
    float p = __fadd_rn(0.009618129107628477f, __fmul_rn(f, 0.0013333558146428443f));
    p = __fadd_rn(0.05550410866482158f, __fmul_rn(f, p));
    p = __fadd_rn(0.2402265069591007f, __fmul_rn(f, p));
    p = __fadd_rn(0.6931471805599453f, __fmul_rn(f, p));
    p = __fadd_rn(1.0f, __fmul_rn(f, p));
    return __fmul_rn(p, __int_as_float((__float2int_rz(yf) + 127) << 23));
}

// ---------------------------------------------------------------------------- reductions
// xor butterfly: every lane ends with the same value; float addition is commutative, so the
// result is one well-defined sum (the CPU oracle replays it).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}
// max of non-negative floats: their bit patterns order like unsigned integers
__device__ __forceinline__ float warp_max_nonneg(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// ---------------------------------------------------------------- fixed point and limbs
// X = rint(x * 2^s) clamped to +-(2^30 - 64), split into four int8 limbs at column k
__device__ __forceinline__ void put_limbs4(int8_t *L, int k, float x, float sc) {
    float v = __fmul_rn(x, sc);
    v = fminf(fmaxf(v, -1073741760.0f), 1073741760.0f);
    const int X = __float2int_rn(v);
    const int d = ((X + 128) & 255) - 128;
    const int X1 = (X - d) >> 8;
    const int c = ((X1 + 128) & 255) - 128;
    const int X2 = (X1 - c) >> 8;
    const int b = ((X2 + 128) & 255) - 128;
    const int a = (X2 - b) >> 8;
    L[0 * kLimbStride + k] = (int8_t)a;
    L[1 * kLimbStride + k] = (int8_t)b;
    L[2 * kLimbStride + k] = (int8_t)c;
    L[3 * kLimbStride + k] = (int8_t)d;
}
// B fragment (32 k x 8 columns; columns 0..3 = limbs) of k-block kb at limb column base
__device__ __forceinline__ void load_bfrag(const int8_t *L, int base, int kb, int lane, uint32_t &b0, uint32_t &b1) {
    const int g = lane >> 2, tig = lane & 3;
    if (g < kLimbs) {
        const int8_t *r = L + g * kLimbStride + base + kb * 32 + tig * 4;
        b0 = *reinterpret_cast<const uint32_t *>(r);
        b1 = *reinterpret_cast<const uint32_t *>(r + 16);
    } else {
        b0 = b1 = 0u;
    }
}
// exact dot of the four limb columns: ((a * 256 + b) * 256 + c) * 256 + d, as two wide
// multiply-adds.  Every dot here has K <= 768 (the host limits an FC CTA's fc2 slice to 24
// k-blocks), so |a| <= 64 * 127 * 768 < 2^23 and |b| < 2^24: a * 256 + b fits in 32 bits.
__device__ __forceinline__ long long limb_dot(int a, int b, int c, int d) {
    const int hi = a * 256 + b;
    const long long lo = (long long)c * 256 + d;
    return (long long)hi * 65536 + lo;
}

// LayerNorm of the D-vector x by the 8 consumer warps together: warp w owns the 32-wide
// blocks [w*D/256, (w+1)*D/256) (the K range of its GEMV share); one pass gives the sum and
// the sum of squares (lane l adds its elements 32*kb + l in kb order, the warp adds its lanes
// with the xor butterfly, the 8 warp totals are added in warp order); mean = S1 / D,
// var = max(S2 / D - mean^2, 0) (population variance, the engine's single-pass form of
// rust/npu-asr-host/src/lib.rs:79-110), y = bf16((x - mean) * (1 / sqrt(var + eps)) * g + b).
// The GEMV input is y in fixed point 2^fix, an exponent derived from the LayerNorm
// parameters (|y_k| <= sqrt(D) |g_k| + |b_k|), so no max reduction is needed.  Each warp
// writes the limbs of its own blocks and, if `out` is given, those outputs.  One consumer
// barrier; every consumer thread calls it.
template <int D>
__device__ __forceinline__ void ln_limbs(const float *g, const float *b, float eps, int fix, float *out) {
    constexpr int KBW = D / 32 / kConsumerWarps;
    const Cta S = make_cta();
    const int lane = S.lane, kb0 = S.warp * KBW;
    float *red = S.red + 32;                      // [2][8]
    float v[KBW];
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int kk = 0; kk < KBW; kk++) {
        v[kk] = S.x[32 * (kb0 + kk) + lane];
        s1 = __fadd_rn(s1, v[kk]);
        s2 = __fadd_rn(s2, __fmul_rn(v[kk], v[kk]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, o));
        s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o));
    }
    if (lane == 0) { red[S.warp] = s1; red[8 + S.warp] = s2; }
    cbar();
    s1 = 0.0f;
    s2 = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) {
        s1 = __fadd_rn(s1, red[w]);
        s2 = __fadd_rn(s2, red[8 + w]);
    }
    const float mean = __fdiv_rn(s1, (float)D);
    const float var = fmaxf(__fsub_rn(__fdiv_rn(s2, (float)D), __fmul_rn(mean, mean)), 0.0f);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    const float sc = exp2i(fix);
#pragma unroll
    for (int kk = 0; kk < KBW; kk++) {
        const int i = 32 * (kb0 + kk) + lane;
        const float t = __fmul_rn(__fsub_rn(v[kk], mean), inv);
        const float y = bf16r(__fadd_rn(__fmul_rn(t, g[i]), b[i]));
        put_limbs4(S.limbs, i, y, sc);
        if (out) out[i] = y;
    }
    __syncwarp();
}

// ------------------------------------------------------------------------------ GEMVs
// Exact dot of one 16-row tile (chunk `ch`, K = 32 * NKB, fragment order) with the limbs at
// column 0, by one warp over the whole K (two accumulation chains).  Lanes with tig == 0 get
// the exact sums of rows g and g + 8 in P0, P1.
template <int NKB>
__device__ __forceinline__ void tile_dot(const Cta &S, const uint8_t *ch, long long &P0, long long &P1) {
    int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
#pragma unroll 4
    for (int kb = 0; kb < NKB; kb += 2) {
        uint32_t b0, b1, b2, b3;
        load_bfrag(S.limbs, 0, kb, S.lane, b0, b1);
        load_bfrag(S.limbs, 0, kb + 1, S.lane, b2, b3);
        const uint4 x0 = *reinterpret_cast<const uint4 *>(ch + kb * kFragBytes + S.lane * 16);
        const uint4 x1 = *reinterpret_cast<const uint4 *>(ch + (kb + 1) * kFragBytes + S.lane * 16);
        mma_s8_16832(a0, x0.x, x0.y, x0.z, x0.w, b0, b1);
        mma_s8_16832(a1, x1.x, x1.y, x1.z, x1.w, b2, b3);
    }
    int v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = a0[k] + a1[k];
    const int x0 = __shfl_down_sync(0xffffffffu, v[0], 1);
    const int x1 = __shfl_down_sync(0xffffffffu, v[1], 1);
    const int x2 = __shfl_down_sync(0xffffffffu, v[2], 1);
    const int x3 = __shfl_down_sync(0xffffffffu, v[3], 1);
    P0 = limb_dot(v[0], v[1], x0, x1);
    P1 = limb_dot(v[2], v[3], x2, x3);
}

// Row-tile GEMV with one warp per tile: warp w < nt takes chunk ctr + w (16 output rows, K =
// 32 * NKB) against the limbs at column 0 (all of them: the caller puts a consumer barrier
// after the LayerNorm).  Lanes with tig == 0 of warp w get y0 / y1 for rows 16w + g and
// 16w + g + 8: float(exact dot) * 2^-s * scale + bias.  No cross-warp partial sums.  The
// slots stay owned until release_tiles.
template <int NKB>
__device__ __forceinline__ bool rowtile_warp(const DecodeParams &p, uint32_t ctr, int nt, int s, uint32_t where,
                                          float *y) {
    const Cta S = make_cta();
    if (S.warp >= nt) return true;
    if (!wait_chunks(p, S, ctr + S.warp, 1, where)) return false;
    const uint8_t *ch = slot_ptr(S, ctr + S.warp);
    long long P0, P1;
    tile_dot<NKB>(S, ch, P0, P1);
    const int g = S.lane >> 2;
    const float *meta = reinterpret_cast<const float *>(ch + kTile * NKB * 32);
    const float2 m0 = *reinterpret_cast<const float2 *>(meta + 2 * g);
    const float2 m1 = *reinterpret_cast<const float2 *>(meta + 2 * (g + 8));
    const float inv = exp2i(-s);
    y[0] = __fadd_rn(__fmul_rn(__fmul_rn(__ll2float_rn(P0), inv), m0.x), m0.y);
    y[1] = __fadd_rn(__fmul_rn(__fmul_rn(__ll2float_rn(P1), inv), m1.x), m1.y);
    return true;
}

// release the nt row-tile slots from ctr: one arrival per warp on each
__device__ __forceinline__ void release_tiles(const Cta &S, uint32_t ctr, int nt) {
    __syncwarp();
    if (S.lane == 0)
        for (int t = 0; t < nt; t++) mbar_arrive(&S.empty[(ctr + t) % kSlots]);
}

// K-split slice GEMV with integer accumulation across CTAs: for each of nkb k-blocks (limb
// columns kSlimbOff + 32 kb), the slice chunks of D outputs; warp w owns the m-tiles w, w+8, ...
// Each output's exact partial is added as (partial + 2^bshift + 2^56) into words[n].
template <int D>
__device__ __forceinline__ bool slice_mma_red(const DecodeParams &p, uint32_t ctr, int nkb,
                                           unsigned long long *words, int bshift, uint32_t where,
                                           unsigned long long *clk = nullptr) {
    const Cta S = make_cta();
    constexpr int NT = D / kTile / kConsumerWarps;       // m-tiles per warp
    const int nch = slice_chunks(D);
    int acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;
    for (int kb = 0; kb < nkb; kb++) {
        uint32_t b0, b1;
        load_bfrag(S.limbs, kSlimbOff, kb, S.lane, b0, b1);
        if (!wait_chunks(p, S, ctr, nch, where)) return false;
        if (clk && S.tid == 0 && kb == 0) clk[0] = clock64();
        for (int c = 0; c < nch; c++) {
            const uint8_t *ch = slot_ptr(S, ctr);
#pragma unroll
            for (int i = 0; i < NT; i++) {
                const int tile = S.warp + kConsumerWarps * i;
                if (tile / kSliceTilesPerChunk == c) {
                    const uint4 a = *reinterpret_cast<const uint4 *>(
                        ch + (tile % kSliceTilesPerChunk) * kFragBytes + S.lane * 16);
                    mma_s8_16832(acc[i], a.x, a.y, a.z, a.w, b0, b1);
                }
            }
            release_slot(S, ctr);
            ctr++;
        }
    }
    if (clk && S.tid == 0) clk[1] = clock64();
    // Each lane parks its fragments (rows g / g + 8, limb pairs by tig) in the warp's scratch
    // with full-width stores; then lane L of round q owns output row L % 16 of tile 2q + L / 16
    // and gathers its four limb sums, so every red below is a full, coalesced warp operation.
    int4 *scr = reinterpret_cast<int4 *>(S.kst) + S.warp * NT * 32;
#pragma unroll
    for (int i = 0; i < NT; i++) scr[i * 32 + S.lane] = make_int4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    __syncwarp();
    const unsigned long long add = (1ull << bshift) + (1ull << kCountShift);
    const int r = S.lane & 15, gg = r & 7, hi = r >> 3;
#pragma unroll
    for (int q = 0; q < NT / 2; q++) {
        const int i = 2 * q + (S.lane >> 4);
        const int2 lo2 = reinterpret_cast<const int2 *>(scr + i * 32 + 4 * gg)[hi];       // limbs 0, 1
        const int2 hi2 = reinterpret_cast<const int2 *>(scr + i * 32 + 4 * gg + 1)[hi];   // limbs 2, 3
        const int n = (S.warp + kConsumerWarps * i) * kTile + r;
        red_add_u64(words + n, (unsigned long long)limb_dot(lo2.x, lo2.y, hi2.x, hi2.y) + add);
    }
    __syncwarp();
    return true;
}

// Read the D accumulator words of one exchange (complete when their count is `cnt`) and add
// the decoded values into the residual: x[n] += float(Y) * 2^-fix * scale[n] + bias[n].
// Thread t owns n = t + 256 i.  Returns false on timeout / abort.  The caller follows with a
// barrier.
template <int D>
__device__ __forceinline__ bool gather_acc(const DecodeParams &p, const unsigned long long *words, int cnt, int subs,
                                           int bshift, int fix, const float *sb, uint32_t where) {
    const Cta S = make_cta();
    constexpr int PER = D / kConsumerThreads;
    float sc[PER], bi[PER];
    unsigned long long v[PER][kMaxSubs];
    unsigned want[kMaxSubs];
#pragma unroll
    for (int k = 0; k < kMaxSubs; k++) want[k] = k < subs ? (unsigned)((cnt + subs - 1 - k) / subs) : 0u;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int n = S.tid + kConsumerThreads * i;
        sc[i] = sb[n];
        bi[i] = sb[D + n];
#pragma unroll
        for (int k = 0; k < kMaxSubs; k++) v[i][k] = k < subs ? ld_relaxed_u64(words + (size_t)k * D + n) : 0ull;
    }
    uint64_t t0 = 0;
    uint32_t it = 0;
    bool ok = true;
    while (true) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < PER; i++)
#pragma unroll
            for (int k = 0; k < kMaxSubs; k++) all &= (unsigned)(v[i][k] >> kCountShift) == want[k];
        if (all) break;
        __nanosleep(p.poll_ns);
#pragma unroll
        for (int i = 0; i < PER; i++)
#pragma unroll
            for (int k = 0; k < kMaxSubs; k++)
                if ((unsigned)(v[i][k] >> kCountShift) != want[k])
                    v[i][k] = ld_relaxed_u64(words + (size_t)k * D + S.tid + kConsumerThreads * i);
        if ((++it & 31) == 0 && wait_expired(p.state, p.timeout_ns, S.flag, &t0, ERR_TIMEOUT_FLAG, where)) {
            ok = false;
            break;
        }
    }
    const float inv = exp2i(-fix);
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int n = S.tid + kConsumerThreads * i;
        long long Y = 0;
#pragma unroll
        for (int k = 0; k < kMaxSubs; k++)
            Y += (long long)(v[i][k] & ((1ull << kCountShift) - 1)) - ((long long)want[k] << bshift);
        const float val = __fadd_rn(__fmul_rn(__fmul_rn(__ll2float_rn(Y), inv), sc[i]), bi[i]);
        S.x[n] = __fadd_rn(S.x[n], val);
    }
    return ok;
}

// ------------------------------------------------------------------------------ attention
__device__ __forceinline__ size_t kv_index(const DecodeParams &p, int layer, int phys, int head, int half,
                                           int kv, int row) {
    return (((((size_t)layer * p.n_phys_pages + phys) * p.n_heads + head) * 2 + half) * 2 + kv) *
               (size_t)(kPageTokens * kHalfDim) +
           (size_t)row * kHalfDim;
}
// cp.async rows [j0, j1) of this CTA's K (kv = 0) or V (kv = 1) dims to dst (row j at
// j - j0; K rows keep 16-byte chunk c at c ^ (j & 3) so the one-key-per-thread score loop is
// bank-conflict free); no commit
__device__ __forceinline__ void kv_stage(const DecodeParams &p, const Cta &S, int layer, int head, int half, int kv,
                                         int j0, int j1, uint16_t *dst) {
    for (int c = S.tid; c < (j1 - j0) * 4; c += kConsumerThreads) {
        const int j = j0 + (c >> 2), part = c & 3;
        const uint16_t *src =
            p.kv + kv_index(p, layer, S.pt[j / kPageTokens], head, half, kv, j % kPageTokens) + part * 8;
        const int pc = kv ? part : part ^ (j & 3);
        cp_async16(dst + (size_t)(j - j0) * kHalfDim + pc * 8, src);
    }
}
// partial score of key j over the own 32 dims: 4 chains of 8 dims (fma, d ascending),
// combined as (c0 + c1) + (c2 + c3); krow = the key's 64-byte row (chunks swizzled by j & 3)
__device__ __forceinline__ float part_score(const float *qf, const uint16_t *krow, int j) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(krow);
    const float4 *q4 = reinterpret_cast<const float4 *>(qf);
    float c[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 w = kr[i ^ (j & 3)];
        const float4 qa = q4[2 * i], qb = q4[2 * i + 1];
        float a = 0.0f;
        a = fmaf(qa.x, bf16lo(w.x), a);
        a = fmaf(qa.y, bf16hi(w.x), a);
        a = fmaf(qa.z, bf16lo(w.y), a);
        a = fmaf(qa.w, bf16hi(w.y), a);
        a = fmaf(qb.x, bf16lo(w.z), a);
        a = fmaf(qb.y, bf16hi(w.z), a);
        a = fmaf(qb.z, bf16lo(w.w), a);
        a = fmaf(qb.w, bf16hi(w.w), a);
        c[i] = a;
    }
    return __fadd_rn(__fadd_rn(c[0], c[1]), __fadd_rn(c[2], c[3]));
}

// One head pair's single-query attention over keys [0, pos] (mha_tile, mha_decode.cc:90-168,
// with one softmax over the whole context): this CTA's partial scores go to the other CTA by
// st.async; s_j = part_rank0 + part_rank1; M = max s; p_j = fast_exp(s_j - M); l = sum p
// (thread t sums keys j = t mod 256 in order, then the butterfly, then the warps in order);
// ctx_d = (sum over 8 key groups j = g mod 8, in group order, of fma chains) / l, bf16.  The
// ctx limbs (fixed point 2^fix) land at limb column kSlimbOff + d.  `xu` counts the pair
// exchanges of this launch (mbarrier buffer and parity).  Returns false on timeout / abort;
// the caller follows with a barrier.
__device__ __forceinline__ bool attention(const DecodeParams &p, int layer, int head, int half, int pos, bool staged,
                                       uint32_t xu, int fix, int t) {
    const Cta S = make_cta();
    const int tk = pos + 1;
    const int buf = xu & 1;
    const uint32_t par = (xu >> 1) & 1u;
    float *pbuf = S.ps + buf * kMaxCtx;
    const uint32_t peer = (uint32_t)half ^ 1u;
    const uint32_t rbuf = mapa_peer(pbuf, peer);
    const uint32_t rbar = mapa_peer(&S.xchg[buf], peer);
    float *own = S.own;
    // ---- partial scores of the own dims, sent to the peer as they are made
    if (staged) {
#pragma unroll 1
        for (int j = S.tid; j < tk; j += kConsumerThreads) {
            const float v = part_score(S.qf, j < pos ? S.kst + j * kHalfDim : S.kcur, j);
            own[j] = v;
            st_async_b32(rbuf + 4u * j, __float_as_uint(v), rbar);
        }
    } else {
        uint16_t *kchunk = S.kst;                         // the whole staging area holds K rows
#pragma unroll 1
        for (int j0 = 0; j0 < pos; j0 += kChunkKeys) {
            const int j1 = min(pos, j0 + kChunkKeys);
            cbar();                                       // previous chunk fully read
            kv_stage(p, S, layer, head, half, 0, j0, j1, kchunk);
            cp_async_commit();
            cp_async_wait_all();
            cbar();
#pragma unroll 1
            for (int j = j0 + S.tid; j < j1; j += kConsumerThreads)
                own[j] = part_score(S.qf, kchunk + (j - j0) * kHalfDim, j);
        }
        if (S.tid == pos % kConsumerThreads) own[pos] = part_score(S.qf, S.kcur, pos);
#pragma unroll 1
        for (int j = S.tid; j < tk; j += kConsumerThreads) st_async_b32(rbuf + 4u * j, __float_as_uint(own[j]), rbar);
    }
    if (layer == 1) stamp(p, S, t, 53);
    // ---- the peer's partials
    bool ok = true;
    if (!mbar_try_wait_cluster(&S.xchg[buf], par)) {
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (!mbar_try_wait_cluster(&S.xchg[buf], par))
            if ((++it & 15) == 0 &&
                wait_expired(p.state, p.timeout_ns, S.flag, &t0, ERR_TIMEOUT_PEER, 0x500u + layer)) {
                ok = false;
                break;
            }
    }
    if (layer == 1) stamp(p, S, t, 54);
    // every thread touches only its own keys j = tid mod 256 in own[] and pbuf[] until the
    // barrier before P.V
    float m = -INFINITY;
#pragma unroll 1
    for (int j = S.tid; j < tk; j += kConsumerThreads) {
        const float pr = pbuf[j];
        const float sj = half == 0 ? __fadd_rn(own[j], pr) : __fadd_rn(pr, own[j]);
        own[j] = sj;
        m = fmaxf(m, sj);
    }
    m = warp_max(m);
    if (S.lane == 0) S.red[S.warp] = m;
    if (cbar_or(!ok)) return false;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) m = fmaxf(m, S.red[w]);
    float l = 0.0f;
#pragma unroll 1
    for (int j = S.tid; j < tk; j += kConsumerThreads) {
        const float pj = fast_exp_nonpos(__fsub_rn(own[j], m));
        pbuf[j] = pj;
        l = __fadd_rn(l, pj);
    }
    l = warp_sum(l);
    if (S.lane == 0) S.red[8 + S.warp] = l;
    cbar();
    l = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) l = __fadd_rn(l, S.red[8 + w]);
    if (layer == 1) stamp(p, S, t, 55);
    // ---- P.V over the own dims: thread (d, g) chains keys j = g mod 8
    const int d = S.tid & 31, g = S.tid >> 5;
    float a = 0.0f;
    if (staged) {
#pragma unroll 4
        for (int j = g; j < tk; j += 8) {
            const uint16_t vv = j < pos ? S.vst[j * kHalfDim + d] : S.vcur[d];
            a = fmaf(pbuf[j], __uint_as_float((uint32_t)vv << 16), a);
        }
    } else {
        uint16_t *vchunk = S.kst;
        for (int j0 = 0; j0 < pos; j0 += kChunkKeys) {
            const int j1 = min(pos, j0 + kChunkKeys);
            cbar();
            kv_stage(p, S, layer, head, half, 1, j0, j1, vchunk);
            cp_async_commit();
            cp_async_wait_all();
            cbar();
            for (int j = j0 + ((g - j0 % 8) + 8) % 8; j < j1; j += 8)
                a = fmaf(pbuf[j], __uint_as_float((uint32_t)vchunk[(j - j0) * kHalfDim + d] << 16), a);
        }
        if (pos % 8 == g) a = fmaf(pbuf[pos], __uint_as_float((uint32_t)S.vcur[d] << 16), a);
    }
    S.accg[g * 32 + d] = a;
    cbar();
    if (S.tid < kHalfDim) {
        float tot = 0.0f;
#pragma unroll
        for (int gg = 0; gg < 8; gg++) tot = __fadd_rn(tot, S.accg[gg * 32 + S.tid]);
        put_limbs4(S.limbs, kSlimbOff + S.tid, bf16r(__fdiv_rn(tot, l)), exp2i(fix));
    }
    if (layer == 1) stamp(p, S, t, 56);
    return true;
}

// optional debugging record of the residual stream (CTA 0 only); after a consumer barrier
__device__ __forceinline__ void trace_x(const DecodeParams &p, const Cta &S, int t, int slot, const float *v) {
    if (p.trace == nullptr || blockIdx.x != 0) return;
    float *dst = p.trace + ((size_t)t * (2 * p.n_layers + 1) + slot) * p.d_model;
    for (int i = S.tid; i < p.d_model; i += kConsumerThreads) dst[i] = v[i];
}
// prefetch a LayerNorm's gamma and beta into S.lnp[buf] (cp.async, one commit group)
__device__ __forceinline__ void ln_prefetch(const Cta &S, int buf, const float *g, const float *b, int D) {
    float *dst = S.lnp + buf * 2 * kDmax;
    for (int c = S.tid; c < D / 2; c += kConsumerThreads) {   // D/4 16-byte pieces per vector
        const int v = c / (D / 4), q = c % (D / 4);
        cp_async16(dst + v * kDmax + 4 * q, (v ? b : g) + 4 * q);
    }
    cp_async_commit();
}

// LM head (the tied embedding as int8 rows) + greedy argmax for one token: warp w takes this
// CTA's row tiles w, w+8, ... (chunks ctr + i), all 24 k-blocks each; per CTA the best key
// (value order, then the larger index) is published as two flag-tagged words; then every CTA
// reads all CTAs' keys and leaves the winning id in S.flag[1] (CTA 0 also stores it in the
// token array).  Returns false on timeout / abort (uniform over the CTA).
template <int D>
__device__ __forceinline__ bool lm_head(const DecodeParams &p, uint32_t ctr, int t, int pos, uint32_t tau, int lm_t0,
                                     int lm_nt, int s) {
    const Cta S = make_cta();
    constexpr int NKB_D = D / 32;
    const int c = blockIdx.x, G = p.grid, V = p.vocab;
    const int lm_step = pos - max(p.start_pos, p.n_prompt - 1);
    float *lrow = p.logits ? p.logits + (size_t)lm_step * V : nullptr;
    unsigned long long best = 0ull;
    bool ok = true;
    const float inv = exp2i(-s);
    const int g = S.lane >> 2, tig = S.lane & 3;
    for (int i = S.warp; i < lm_nt; i += kConsumerWarps) {
        if (!wait_full(p, S, ctr + i, 0x100u)) { ok = false; break; }
        const uint8_t *ch = slot_ptr(S, ctr + i);
        int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
#pragma unroll 4
        for (int kb = 0; kb < NKB_D; kb += 2) {
            uint32_t b0, b1, b2, b3;
            load_bfrag(S.limbs, 0, kb, S.lane, b0, b1);
            load_bfrag(S.limbs, 0, kb + 1, S.lane, b2, b3);
            const uint4 x0 = *reinterpret_cast<const uint4 *>(ch + kb * kFragBytes + S.lane * 16);
            const uint4 x1 = *reinterpret_cast<const uint4 *>(ch + (kb + 1) * kFragBytes + S.lane * 16);
            mma_s8_16832(a0, x0.x, x0.y, x0.z, x0.w, b0, b1);
            mma_s8_16832(a1, x1.x, x1.y, x1.z, x1.w, b2, b3);
        }
        const float *meta = reinterpret_cast<const float *>(ch + kTile * D);
        const float2 m0 = *reinterpret_cast<const float2 *>(meta + 2 * g);
        const float2 m1 = *reinterpret_cast<const float2 *>(meta + 2 * (g + 8));
        __syncwarp();
        if (S.lane == 0) mbar_arrive_cnt(&S.empty[(ctr + i) % kSlots], kConsumerWarps);
        int v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = a0[k] + a1[k];
        const int x0 = __shfl_down_sync(0xffffffffu, v[0], 1);
        const int x1 = __shfl_down_sync(0xffffffffu, v[1], 1);
        const int x2 = __shfl_down_sync(0xffffffffu, v[2], 1);
        const int x3 = __shfl_down_sync(0xffffffffu, v[3], 1);
        if (tig == 0) {
            const int r0 = (lm_t0 + i) * kTile + g, r1 = r0 + 8;
            const float y0 = __fadd_rn(
                __fmul_rn(__fmul_rn(__ll2float_rn(limb_dot(v[0], v[1], x0, x1)), inv), m0.x), m0.y);
            const float y1 = __fadd_rn(
                __fmul_rn(__fmul_rn(__ll2float_rn(limb_dot(v[2], v[3], x2, x3)), inv), m1.x), m1.y);
            // key: value order (sign-flipped bits), then the larger index (ties -> last
            // max, Iterator::max_by in opt125m_decode.rs:303)
            if (r0 < V) {
                if (lrow) lrow[r0] = y0;
                const uint32_t u = __float_as_uint(y0);
                const unsigned long long k =
                    ((unsigned long long)(u & 0x80000000u ? ~u : u | 0x80000000u) << 32) | (uint32_t)r0;
                best = k > best ? k : best;
            }
            if (r1 < V) {
                if (lrow) lrow[r1] = y1;
                const uint32_t u = __float_as_uint(y1);
                const unsigned long long k =
                    ((unsigned long long)(u & 0x80000000u ? ~u : u | 0x80000000u) << 32) | (uint32_t)r1;
                best = k > best ? k : best;
            }
        }
    }
    best = warp_max_u64(best);
    if (S.lane == 0) S.keys[S.warp] = best;
    if (cbar_or(!ok)) return false;
    // global argmax: every CTA folds its best key into the token's max word, then counts
    // itself in with release order; one thread per CTA waits for the count to reach G
    unsigned long long *lmw = p.lm_words + 2 * (tau % kAccSlots);
    if (S.tid == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kConsumerWarps; w++) b = S.keys[w] > b ? S.keys[w] : b;
        atomicMax(lmw, b);
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(lmw + 1) : "memory");
    }
    stamp(p, S, t, 50);
    if (S.tid == 0) {
        uint64_t t0 = 0;
        uint32_t it = 0;
        unsigned long long n;
        while (true) {
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(n) : "l"(lmw + 1) : "memory");
            if (n >= (unsigned long long)G) break;
            __nanosleep(32);
            if ((++it & 31) == 0 && wait_expired(p.state, p.timeout_ns, S.flag, &t0, ERR_TIMEOUT_FLAG, 0x90u)) {
                ok = false;
                break;
            }
        }
        const unsigned long long b = ld_relaxed_u64(lmw);
        const int bi = (int)(uint32_t)b;
        S.flag[1] = bi;
        if (ok && c == 0) p.tokens[pos + 1] = bi;
    }
    if (cbar_or(!ok)) return false;
    return true;
}

// ------------------------------------------------------------------------------ producer
__device__ __forceinline__ void producer(const DecodeParams &p, Cta &S) {
    const int c = blockIdx.x;
    const ChunkRef *tab = p.chunks + (size_t)c * p.chunk_stride;
    const int nl = p.n_layer_chunks[c], nlm = p.n_lm_chunks[c];
    uint32_t ctr = 0;
    bool failed = false;
    for (int t = 0; t < p.n_steps && !failed; t++) {
        const int pos = p.start_pos + t;
        const int n = nl + (pos >= p.n_prompt - 1 ? nlm : 0);
        for (int i = 0; i < n; i++) {
            const int slot = ctr % kSlots;
            const uint32_t k = ctr / kSlots;
            if (k > 0 && !mbar_try_wait(&S.empty[slot], (k - 1) & 1u)) {
                uint64_t t0 = 0;
                uint32_t it = 0;
                // the producer runs a layer or more ahead of its consumers, so it can back off
                // between polls and leave the issue slots to them
                while (!mbar_try_wait(&S.empty[slot], (k - 1) & 1u)) {
                    __nanosleep(200);
                    if ((++it & 15) == 0 &&
                        wait_expired(p.state, p.timeout_ns, S.flag, &t0, ERR_TIMEOUT_EMPTY, 0x400u)) {
                        failed = true;
                        break;
                    }
                }
                if (failed) break;
            }
            const ChunkRef ch = tab[i];
            mbar_arrive_expect_tx(&S.full[slot], ch.bytes);
            bulk_g2s(S.ring + slot * kSlotBytes, p.stream + ch.off, ch.bytes, &S.full[slot]);
            ctr++;
        }
    }
    // drain: every issued copy must land before the CTA's shared memory is released
    const uint32_t first = ctr > (uint32_t)kSlots ? ctr - kSlots : 0u;
    for (uint32_t q = first; q < ctr; q++) {
        const uint64_t start = globaltimer_ns();
        while (!mbar_try_wait(&S.full[q % kSlots], (q / kSlots) & 1u))
            if (globaltimer_ns() - start > p.timeout_ns) break;
    }
}

// ------------------------------------------------------------------------------ consumer
template <int D, int F>
__device__ __forceinline__ void consumer(const DecodeParams &p, Cta &S) {
    const int c = blockIdx.x, G = p.grid;
    const int L = p.n_layers, V = p.vocab, H = p.n_heads;
    const bool is_head = c < 2 * H;
    const int head = c >> 1, half = c & 1;
    const int fci = c - 2 * H;
    const bool is_fc = !is_head && fci < p.n_fc;
    const int fc_kb_begin = is_fc ? fc_kb0(fci, F / 32, p.n_fc) : 0;
    const int fc_nkb = is_fc ? fc_kb0(fci + 1, F / 32, p.n_fc) - fc_kb_begin : 0;
    const uint32_t tok0 = p.state->tok_base;
    const int lm_t0 = lm_tile0(c, p.vocab_tiles, G);
    const int lm_nt = lm_tile0(c + 1, p.vocab_tiles, G) - lm_t0;
    uint32_t ctr = 0, xu = 0;
    int64_t next_id = 0;
    for (int i = S.tid; i < kMaxPages; i += kConsumerThreads) S.pt[i] = i < p.n_phys_pages ? p.page_table[i] : 0;
    if (S.tid == 0) { S.flag[0] = 0; S.flag[1] = 0; }
    cbar();

    for (int t = 0; t < p.n_steps; t++) {
        const int pos = p.start_pos + t;
        const uint32_t tau = tok0 + (uint32_t)t;
        const size_t XW = (size_t)D * kMaxSubs;            // words of one exchange
        unsigned long long *acc_tok = p.acc + (size_t)(tau % kAccSlots) * L * 2 * XW;
        const int64_t id = (t == 0 || pos < p.n_prompt) ? p.tokens[pos] : next_id;
        bool bad = false;
        if (id < 0 || id >= V || pos + 2 > p.max_pos + 1 || pos >= kMaxCtx) {
            bad = true;
            if (S.tid == 0) set_error_st(p.state, id < 0 || id >= V ? ERR_BAD_TOKEN : ERR_BAD_POS, pos);
        }
        cp_async_wait_all();                 // no stale prefetch may land after the next
        if (cbar_or(bad || *(volatile int *)S.flag != 0)) return;
        const bool lm_token = pos >= p.n_prompt - 1;
        if (!is_head && !is_fc && !lm_token) {
            // A spare CTA has no work in a token without an LM head, but it still waits for
            // the token's last fc2 words: that keeps it from running ahead into the slot of a
            // later token while the words there still hold an older token's complete sums.
            const bool ok = gather_acc<D>(p, acc_tok + (size_t)((L - 1) * 2 + 1) * XW, p.n_fc, p.f2_subs, p.f2_bias_shift,
                                          p.fix_h[L - 1], p.f2sb + (size_t)(L - 1) * 2 * D, 0x88u);
            if (cbar_or(!ok)) return;
            next_id = p.tokens[pos + 1];
            continue;
        }
        stamp(p, S, t, 0);
        stamp_clk(p, S, t, 0);
        for (int i = S.tid; i < D; i += kConsumerThreads)
            S.x[i] = __fadd_rn(p.emb_tok[(size_t)id * D + i], p.emb_pos[(size_t)(pos + 2) * D + i]);
        // the accumulator words of token tau + 2 (last used by token tau - 2, which every CTA
        // has finished: an FC CTA starts token tau only after all fc2 contributions of token
        // tau - 1, which needed every head pair's and FC CTA's work of that token) are cleared
        // by the FC CTAs and made visible before anything this CTA publishes later
        if (is_fc) {
            const int nz = p.n_fc, zi = fci;
            const size_t W = (size_t)L * 2 * XW;
            unsigned long long *z = p.acc + (size_t)((tau + 2) % kAccSlots) * W;
            const size_t z0 = W * zi / nz, z1 = W * (zi + 1) / nz;
            for (size_t i = z0 + S.tid; i < z1; i += kConsumerThreads) z[i] = 0ull;
            if (zi == 0 && S.tid < 2) p.lm_words[2 * ((tau + 2) % kAccSlots) + S.tid] = 0ull;
            __threadfence();
        }
        const float *ln_first = is_head ? p.ln : p.ln + 2 * D;
        ln_prefetch(S, 0, ln_first, ln_first + D, D);
        const bool staged = pos <= kStageKeys;

        for (int l = 0; l < L; l++) {
            unsigned long long *acc_o = acc_tok + (size_t)(l * 2 + 0) * XW;
            unsigned long long *acc_f = acc_tok + (size_t)(l * 2 + 1) * XW;
            // LayerNorm parameters of the next layer (or the final LN) into the other buffer
            {
                const float *nx = l + 1 < L ? p.ln + (size_t)(l + 1) * 4 * D + (is_head ? 0 : 2 * D) : p.lnf;
                ln_prefetch(S, (l + 1) & 1, nx, nx + D, D);
            }
            if (is_head) {
                // ---------------- head pair: x += fc2(l-1); LN1; q|k|v of the own dims
                if (staged) {
                    kv_stage(p, S, l, head, half, 0, 0, pos, S.kst);
                    kv_stage(p, S, l, head, half, 1, 0, pos, S.vst);
                }
                cp_async_commit();
                bool ok = true;
                if (l > 0)
                    ok = gather_acc<D>(p, acc_tok + (size_t)((l - 1) * 2 + 1) * XW, p.n_fc, p.f2_subs, p.f2_bias_shift,
                                       p.fix_h[l - 1], p.f2sb + (size_t)(l - 1) * 2 * D, 0x10u + l);
                cp_async_wait_group<2>();          // this layer's LN parameters
                if (cbar_or(!ok)) return;
                if (l > 0) trace_x(p, S, t, 2 * (l - 1) + 1, S.x);
                stamp(p, S, t, 1 + 4 * l);
                const float *lg = S.lnp + (l & 1) * 2 * kDmax;
                if (l == 1) stamp_clk(p, S, t, 1);
                const int s = p.fix_ln1[l];
                ln_limbs<D>(lg, lg + kDmax, p.eps, s, nullptr);
                cbar();                            // every warp's GEMV reads all limbs
                if (l == 1) stamp_clk(p, S, t, 2);
                if (l == 1) stamp(p, S, t, 57);
                float y[2];
                ok = rowtile_warp<D / 32>(p, ctr, 6, s, 0x20u + l, y);
                if (l == 1) stamp_clk(p, S, t, 3);
                if (l == 1) stamp(p, S, t, 58);
                // rows 16w + g and 16w + g + 8 of q | k | v (32 own dims each)
                if (ok && S.warp < 6 && (S.lane & 3) == 0) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        const int r = S.warp * kTile + (S.lane >> 2) + 8 * h2, part = r >> 5, i = r & 31;
                        if (part == 0) {
                            S.qf[i] = bf16r(__fmul_rn(y[h2], 0.125f));
                        } else {
                            const uint16_t bits = (uint16_t)bf16bits(y[h2]);
                            p.kv[kv_index(p, l, S.pt[pos / kPageTokens], head, half, part - 1, pos % kPageTokens) + i] = bits;
                            if (part == 1) S.kcur[(((i >> 3) ^ (pos & 3)) << 3) + (i & 7)] = bits;
                            else S.vcur[i] = bits;
                        }
                    }
                }
                if (cbar_or(!ok)) return;
                if (l == 1) stamp(p, S, t, 59);
                if (S.tid == 0) mbar_arrive_expect_tx(&S.xchg[xu & 1], 4u * (pos + 1));
                cp_async_wait_all();               // staged K / V rows
                cbar();
                release_tiles(S, ctr, 6);
                ctr += 6;
                stamp(p, S, t, 2 + 4 * l);
                // ---------------- attention over the own dims, then the K-split out projection
                ok = attention(p, l, head, half, pos, staged, xu, p.fix_ctx[l], t);
                xu++;
                if (cbar_or(!ok)) return;
                if (l == 1) stamp(p, S, t, 60);
                if (l == 1) stamp_clk(p, S, t, 10);
                ok = slice_mma_red<D>(p, ctr, 1, acc_o + (size_t)(c % p.o_subs) * D, p.o_bias_shift, 0x30u + l,
                                      (p.timing && l == 1 && t < 2) ? p.timing + ((size_t)t * p.grid + blockIdx.x) * 128 + 75 : nullptr);
                if (l == 1) stamp_clk(p, S, t, 13);
                ctr += slice_chunks(D);
                stamp(p, S, t, 3 + 4 * l);
                // ---------------- x += out projection
                ok = ok && gather_acc<D>(p, acc_o, 2 * H, p.o_subs, p.o_bias_shift, p.fix_ctx[l],
                                         p.osb + (size_t)l * 2 * D, 0x40u + l);
                if (cbar_or(!ok)) return;
                trace_x(p, S, t, 2 * l, S.x);
                stamp(p, S, t, 4 + 4 * l);
            } else {
                // ---------------- x += out projection; LN2; fc1 rows; ReLU; K-split fc2
                cp_async_commit();                 // (keeps the group count of the head path)
                bool ok = gather_acc<D>(p, acc_o, 2 * H, p.o_subs, p.o_bias_shift, p.fix_ctx[l],
                                        p.osb + (size_t)l * 2 * D, 0x40u + l);
                cp_async_wait_group<2>();
                if (cbar_or(!ok)) return;
                trace_x(p, S, t, 2 * l, S.x);
                stamp(p, S, t, 1 + 4 * l);
                if (is_fc) {
                    const float *lg = S.lnp + (l & 1) * 2 * kDmax;
                    const int s = p.fix_ln2[l];
                    ln_limbs<D>(lg, lg + kDmax, p.eps, s, nullptr);
                    cbar();                        // every warp's GEMV reads all limbs
                    if (l == 1) stamp(p, S, t, 57);
                    const float hsc = exp2i(p.fix_h[l]);
                    const int ntile = 2 * fc_nkb;
                    for (int t0 = 0; t0 < ntile; t0 += kConsumerWarps) {
                        const int nt = min(kConsumerWarps, ntile - t0);
                        float y[2];
                        ok = rowtile_warp<D / 32>(p, ctr, nt, s, 0x50u + l, y);
                        if (ok && S.warp < nt && (S.lane & 3) == 0) {
                            const int r = (t0 + S.warp) * kTile + (S.lane >> 2);
                            put_limbs4(S.limbs, kSlimbOff + r, bf16r(fmaxf(y[0], 0.0f)), hsc);
                            put_limbs4(S.limbs, kSlimbOff + r + 8, bf16r(fmaxf(y[1], 0.0f)), hsc);
                        }
                        if (l == 1) stamp(p, S, t, 58);
                        if (cbar_or(!ok)) return;
                        if (l == 1) stamp(p, S, t, 59);
                        release_tiles(S, ctr, nt);
                        ctr += nt;
                    }
                    stamp(p, S, t, 2 + 4 * l);
                    if (l == 1) stamp(p, S, t, 60);
                    ok = slice_mma_red<D>(p, ctr, fc_nkb, acc_f + (size_t)(fci % p.f2_subs) * D, p.f2_bias_shift, 0x60u + l);
                    ctr += fc_nkb * slice_chunks(D);
                    stamp(p, S, t, 3 + 4 * l);
                }
                // ---------------- x += fc2
                ok = ok && gather_acc<D>(p, acc_f, p.n_fc, p.f2_subs, p.f2_bias_shift, p.fix_h[l],
                                         p.f2sb + (size_t)l * 2 * D, 0x70u + l);
                if (cbar_or(!ok)) return;
                trace_x(p, S, t, 2 * l + 1, S.x);
                stamp(p, S, t, 4 + 4 * l);
            }
            // the LM-head rows of this CTA go to L2 a few layers before they are needed
            if (l == p.lm_prefetch_layer && lm_token && S.tid < lm_nt) {
                const ChunkRef ch = p.chunks[(size_t)c * p.chunk_stride + p.n_layer_chunks[c] + S.tid];
                prefetch_l2(p.stream + ch.off, ch.bytes);
            }
        }
        if (is_head) {
            const bool ok = gather_acc<D>(p, acc_tok + (size_t)((L - 1) * 2 + 1) * XW, p.n_fc, p.f2_subs, p.f2_bias_shift,
                                          p.fix_h[L - 1], p.f2sb + (size_t)(L - 1) * 2 * D, 0x80u);
            if (cbar_or(!ok)) return;
            trace_x(p, S, t, 2 * L - 1, S.x);
            stamp(p, S, t, 49);
        }
        // ---------------- final LN, LM head + greedy argmax
        if (lm_token) {
            cp_async_wait_all();
            cbar();
            const float *lg = S.lnp + (L & 1) * 2 * kDmax;
            float *tr = (p.trace && c == 0) ? p.trace + ((size_t)t * (2 * L + 1) + 2 * L) * D : nullptr;
            const int s = p.fix_lnf;
            ln_limbs<D>(lg, lg + kDmax, p.eps, s, tr);
            cbar();
            if (!lm_head<D>(p, ctr, t, pos, tau, lm_t0, lm_nt, s)) return;
            ctr += lm_nt;
            cbar();
            next_id = S.flag[1];
            stamp(p, S, t, 51);
            stamp_clk(p, S, t, 4);
        } else {
            next_id = p.tokens[pos + 1];
        }
    }
    if (c == 0 && S.tid == 0) p.state->tok_base = tok0 + (uint32_t)p.n_steps;
}

template <int D, int F>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) opt_decode_kernel(const __grid_constant__ DecodeParams p) {
    Cta S = make_cta();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; i++) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], kConsumerWarps);
        }
        mbar_init(&S.xchg[0], 1);
        mbar_init(&S.xchg[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    cluster_sync_all();                      // the pair's mbarriers exist before any st.async
    if (S.warp == kConsumerWarps) {
        if (S.lane == 0) producer(p, S);
        __syncwarp();
    } else {
        consumer<D, F>(p, S);
        // after the last token, or after an agreed early exit: a producer still waiting for a
        // free slot sees the flag at its next poll and stops
        if (S.tid == 0) *(volatile int *)S.flag = 1;
    }
    cluster_sync_all();                      // neither CTA leaves while its pair may write into it
}


// ------------------------------------------------------------------------------ prefill
// The prompt's positions before the last one need no LM head, only their K / V rows, and their
// layers do not depend on one another within a layer's linear maps: so they run as a batch of
// up to kPrefillTokens positions per launch sequence instead of one decode step each
// (rust/npu-whisper/src/bin/opt125m_decode.rs:296-315 steps the prompt one token at a time).
// Every number is the decode kernel's: the same LayerNorm reduction order, the same fixed-point
// inputs and exact integer dots (the int8 MMA over the four limbs, combined in 64 bits), the same
// epilogue roundings, the same partial-score chains, softmax sums and P.V chains; so the K / V
// rows written here, and every later token, are bit-identical to a run that steps the prompt.
__global__ void prefill_embed_kernel(const int64_t *tokens, int pos0, int D, int V, const float *emb_tok,
                                     const float *emb_pos, float *x, RunState *state) {
    const int t = blockIdx.x, pos = pos0 + t;
    int64_t id = tokens[pos];
    if (id < 0 || id >= V) {                       // reported like the decode kernel; row 0 stands in
        if (threadIdx.x == 0) set_error_st(state, ERR_BAD_TOKEN, pos);
        id = 0;
    }
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        x[(size_t)t * D + i] = __fadd_rn(emb_tok[(size_t)id * D + i], emb_pos[(size_t)(pos + 2) * D + i]);
}

// limbs of rint(x * sc) (put_limbs4's rule) into [4][K] rows at column k
__device__ __forceinline__ void put_limbs_rows(int8_t *L, int K, int k, float x, float sc) {
    float v = __fmul_rn(x, sc);
    v = fminf(fmaxf(v, -1073741760.0f), 1073741760.0f);
    const int X = __float2int_rn(v);
    const int d = ((X + 128) & 255) - 128;
    const int X1 = (X - d) >> 8;
    const int c = ((X1 + 128) & 255) - 128;
    const int X2 = (X1 - c) >> 8;
    const int b = ((X2 + 128) & 255) - 128;
    const int a = (X2 - b) >> 8;
    L[k] = (int8_t)a;
    L[K + k] = (int8_t)b;
    L[2 * K + k] = (int8_t)c;
    L[3 * K + k] = (int8_t)d;
}

// ln_limbs for one position per CTA (256 threads): same per-lane sums, butterfly, warp order
template <int D>
__global__ void __launch_bounds__(256) prefill_ln_kernel(const float *x, const float *g, const float *b, float eps,
                                                         int fix, int8_t *limbs) {
    constexpr int KBW = D / 32 / kConsumerWarps;
    __shared__ float red[16];
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, kb0 = warp * KBW;
    const float *xr = x + (size_t)t * D;
    float v[KBW];
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int kk = 0; kk < KBW; kk++) {
        v[kk] = xr[32 * (kb0 + kk) + lane];
        s1 = __fadd_rn(s1, v[kk]);
        s2 = __fadd_rn(s2, __fmul_rn(v[kk], v[kk]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, o));
        s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o));
    }
    if (lane == 0) { red[warp] = s1; red[8 + warp] = s2; }
    __syncthreads();
    s1 = 0.0f;
    s2 = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) {
        s1 = __fadd_rn(s1, red[w]);
        s2 = __fadd_rn(s2, red[8 + w]);
    }
    const float mean = __fdiv_rn(s1, (float)D);
    const float var = fmaxf(__fsub_rn(__fdiv_rn(s2, (float)D), __fmul_rn(mean, mean)), 0.0f);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    const float sc = exp2i(fix);
    int8_t *L = limbs + (size_t)t * 4 * D;
#pragma unroll
    for (int kk = 0; kk < KBW; kk++) {
        const int i = 32 * (kb0 + kk) + lane;
        const float tt = __fmul_rn(__fsub_rn(v[kk], mean), inv);
        put_limbs_rows(L, D, i, bf16r(__fadd_rn(__fmul_rn(tt, g[i]), b[i])), sc);
    }
}

// One CTA per (16-row tile, K slice), its 8 warps splitting the slice again, all positions at
// once.  The slice's input limbs of every position are staged in shared memory first (rows padded
// by 16 bytes, so a fragment load hits 32 distinct banks) and each warp holds its weight
// fragments in registers before the MMAs, so no load waits inside the MMA chain.  B columns =
// (position pair, limb): one m16n8k32 covers two positions' four limbs; limb sums are exact in
// 32 bits (|sum| <= K * 128 * 127 < 2^31 for K <= 3072) and combine exactly in 64 bits.  The
// warps' partials are added in shared memory, the slices' in 64-bit integer atomics (any order
// gives the same sum); the tile's last slice applies the epilogue.
constexpr int kPfWarps = 8;
constexpr int kPfMaxKbWarp = 4;                   // k-blocks per warp at most

__global__ void __launch_bounds__(kPfWarps * 32) prefill_gemv_kernel(const PrefillGemv a) {
    constexpr int NCG = kPrefillTokens / 2;
    extern __shared__ __align__(16) uint8_t pf_smem[];
    __shared__ unsigned last_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x, n0 = tile * kTile;
    const int nkb = a.K / 32;
    const int kbA = blockIdx.y * nkb / a.nsplit, kbB = (blockIdx.y + 1) * nkb / a.nsplit;
    const int ks = (kbB - kbA) * 32, stride = ks + 16;
    // this warp's k-blocks and their weight fragments (requested before the staging wait)
    const int w0k = kbA + warp * (kbB - kbA) / kPfWarps, w1k = kbA + (warp + 1) * (kbB - kbA) / kPfWarps;
    const int nk = w1k - w0k;
    uint32_t af[kPfMaxKbWarp][4];
    {
        const int8_t *r0 = a.w + (size_t)(n0 + g) * a.K + tig * 4, *r1 = r0 + (size_t)8 * a.K;
#pragma unroll
        for (int i = 0; i < kPfMaxKbWarp; i++)
            if (i < nk) {
                const int kb = w0k + i;
                af[i][0] = __ldg(reinterpret_cast<const unsigned int *>(r0 + kb * 32));
                af[i][1] = __ldg(reinterpret_cast<const unsigned int *>(r1 + kb * 32));
                af[i][2] = __ldg(reinterpret_cast<const unsigned int *>(r0 + kb * 32 + 16));
                af[i][3] = __ldg(reinterpret_cast<const unsigned int *>(r1 + kb * 32 + 16));
            }
    }
    // stage limbs [position][limb][slice] (positions >= T as zeros)
    {
        const int vec = ks / 16, rows = kPrefillTokens * 4;
        for (int i = threadIdx.x; i < rows * vec; i += kPfWarps * 32) {
            const int row = i / vec, c = i - row * vec, t = row >> 2;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (t < a.T)
                v = __ldg(reinterpret_cast<const uint4 *>(a.limbs + (size_t)row * a.K + (size_t)kbA * 32) + c);
            *reinterpret_cast<uint4 *>(pf_smem + (size_t)row * stride + c * 16) = v;
        }
    }
    __syncthreads();
    int acc[NCG][4];
#pragma unroll
    for (int i = 0; i < NCG; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0;
    // column g of a pair tile: position 2 cg + (g >> 2), limb g & 3 -> staged row 8 cg + g
#pragma unroll
    for (int i = 0; i < kPfMaxKbWarp; i++) {
        if (i >= nk) break;
        const uint8_t *bb = pf_smem + (size_t)g * stride + (w0k + i - kbA) * 32 + tig * 4;
#pragma unroll
        for (int cg = 0; cg < NCG; cg++) {
            const uint8_t *r = bb + (size_t)(8 * cg) * stride;
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(r);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(r + 16);
            mma_s8_16832(acc[cg], af[i][0], af[i][1], af[i][2], af[i][3], b0, b1);
        }
    }
    __syncthreads();                        // the staged limbs are dead: their space holds partials
    long long(*part)[kPrefillTokens][kTile] = reinterpret_cast<long long(*)[kPrefillTokens][kTile]>(pf_smem);
    // lanes with even tig hold rows g, g + 8 of position 2 cg + tig / 2
    const bool owner = (tig & 1) == 0;
#pragma unroll
    for (int cg = 0; cg < NCG; cg++) {
        const int x0 = __shfl_down_sync(0xffffffffu, acc[cg][0], 1);
        const int x1 = __shfl_down_sync(0xffffffffu, acc[cg][1], 1);
        const int x2 = __shfl_down_sync(0xffffffffu, acc[cg][2], 1);
        const int x3 = __shfl_down_sync(0xffffffffu, acc[cg][3], 1);
        const int t = 2 * cg + (tig >> 1);
        if (owner) {
            part[warp][t][g] = ((long long)acc[cg][0] << 24) + ((long long)acc[cg][1] << 16) + ((long long)x0 << 8) + x1;
            part[warp][t][g + 8] =
                ((long long)acc[cg][2] << 24) + ((long long)acc[cg][3] << 16) + ((long long)x2 << 8) + x3;
        }
    }
    __syncthreads();
    // thread i of the CTA: items (position, row) i, i + 256, ...
    const int items = a.T * kTile;
    auto warp_total = [&](int t, int r) {
        long long y = 0;
#pragma unroll
        for (int w = 0; w < kPfWarps; w++) y += part[w][t][r];
        return y;
    };
    if (a.nsplit > 1) {
        for (int i = threadIdx.x; i < items; i += kPfWarps * 32) {
            const int t = i / kTile, r = i % kTile;
            atomicAdd(a.acc + (size_t)t * a.N + n0 + r, (unsigned long long)warp_total(t, r));
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last_s = atomicAdd(a.cnt + tile, 1u) == (unsigned)(a.nsplit - 1);
        __syncthreads();
        if (!last_s) return;
        __threadfence();
    }
    const float inv = exp2i(-a.fix);
    for (int i = threadIdx.x; i < items; i += kPfWarps * 32) {
        const int t = i / kTile, r = i % kTile, n = n0 + r;
        const long long Y = a.nsplit > 1 ? (long long)atomicExch(a.acc + (size_t)t * a.N + n, 0ull) : warp_total(t, r);
        const float y = __fadd_rn(__fmul_rn(__fmul_rn(__ll2float_rn(Y), inv), a.sc[n]), a.bi[n]);
        if (a.mode == PF_QKV) {
            const int part_i = n / a.D, rr = n - part_i * a.D;
            const int pos = a.pos0 + t;
            if (part_i == 0) {
                a.q[(size_t)t * a.D + rr] = bf16r(__fmul_rn(y, 0.125f));
            } else {
                const int head = rr / kHeadDim, half = (rr % kHeadDim) / kHalfDim, k = rr % kHalfDim;
                const size_t idx =
                    (((((size_t)a.layer * a.n_phys + a.pt[pos / kPageTokens]) * a.n_heads + head) * 2 + half) * 2 +
                     (part_i - 1)) * (size_t)(kPageTokens * kHalfDim) + (size_t)(pos % kPageTokens) * kHalfDim + k;
                a.kv[idx] = (uint16_t)bf16bits(y);
            }
        } else if (a.mode == PF_FC1) {
            put_limbs_rows(a.limbs_out + (size_t)t * 4 * a.N, a.N, n, bf16r(fmaxf(y, 0.0f)), exp2i(a.fix_out));
        } else {
            float *xr = a.x + (size_t)t * a.N + n;
            *xr = __fadd_rn(*xr, y);
        }
    }
    if (a.nsplit > 1 && threadIdx.x == 0) a.cnt[tile] = 0u;
}

// partial score over 32 dims of an unswizzled cache row: part_score's four fma chains
__device__ __forceinline__ float part_score_row(const float *qf, const uint16_t *krow) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(krow);
    float c[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 w = kr[i];
        const float *qq = qf + 8 * i;
        float a = 0.0f;
        a = fmaf(qq[0], bf16lo(w.x), a);
        a = fmaf(qq[1], bf16hi(w.x), a);
        a = fmaf(qq[2], bf16lo(w.y), a);
        a = fmaf(qq[3], bf16hi(w.y), a);
        a = fmaf(qq[4], bf16lo(w.z), a);
        a = fmaf(qq[5], bf16hi(w.z), a);
        a = fmaf(qq[6], bf16lo(w.w), a);
        a = fmaf(qq[7], bf16hi(w.w), a);
        c[i] = a;
    }
    return __fadd_rn(__fadd_rn(c[0], c[1]), __fadd_rn(c[2], c[3]));
}

// attention() for one (position, head) per CTA of 256 threads, both halves of the head:
// s_j = part_0 + part_1, the max, fast_exp, the per-thread / butterfly / warp-order sum,
// P.V chains over keys j = g mod 8 per half, ctx limbs at 2^fix
__global__ void __launch_bounds__(256) prefill_attn_kernel(const float *q, const uint16_t *kv, const int *pt,
                                                           int layer, int n_phys, int n_heads, int pos0, int D,
                                                           int fix, int8_t *limbs) {
    __shared__ float sp[kMaxCtx];
    __shared__ __align__(16) float qf[kHeadDim];
    __shared__ float red[16], accg[8 * kHalfDim];
    const int t = blockIdx.x, head = blockIdx.y, pos = pos0 + t, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    if (tid < kHeadDim) qf[tid] = q[(size_t)t * D + head * kHeadDim + tid];
    __syncthreads();
    auto row = [&](int j, int half, int kvsel) {
        return kv + (((((size_t)layer * n_phys + pt[j / kPageTokens]) * n_heads + head) * 2 + half) * 2 + kvsel) *
                        (size_t)(kPageTokens * kHalfDim) +
               (size_t)(j % kPageTokens) * kHalfDim;
    };
    float m = -INFINITY;
    for (int j = tid; j <= pos; j += 256) {
        const float s = __fadd_rn(part_score_row(qf, row(j, 0, 0)), part_score_row(qf + kHalfDim, row(j, 1, 0)));
        sp[j] = s;
        m = fmaxf(m, s);
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) m = fmaxf(m, red[w]);
    float l = 0.0f;
    for (int j = tid; j <= pos; j += 256) {
        const float pj = fast_exp_nonpos(__fsub_rn(sp[j], m));
        sp[j] = pj;
        l = __fadd_rn(l, pj);
    }
    l = warp_sum(l);
    __syncthreads();                       // every red[] max read before the sums overwrite
    if (lane == 0) red[8 + warp] = l;
    __syncthreads();
    l = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) l = __fadd_rn(l, red[8 + w]);
    const int d = tid & 31, g = tid >> 5;
    int8_t *L = limbs + (size_t)t * 4 * D;
    for (int half = 0; half < 2; half++) {
        float a = 0.0f;
        for (int j = g; j <= pos; j += 8) {
            const uint16_t vv = row(j, half, 1)[d];
            a = fmaf(sp[j], __uint_as_float((uint32_t)vv << 16), a);
        }
        accg[g * 32 + d] = a;
        __syncthreads();
        if (tid < kHalfDim) {
            float tot = 0.0f;
#pragma unroll
            for (int gg = 0; gg < 8; gg++) tot = __fadd_rn(tot, accg[gg * 32 + tid]);
            put_limbs_rows(L, D, head * kHeadDim + half * kHalfDim + tid, bf16r(__fdiv_rn(tot, l)), exp2i(fix));
        }
        __syncthreads();
    }
}

cudaError_t launch_prefill_embed(const int64_t *tokens, int pos0, int T, int D, int V, const float *emb_tok,
                                 const float *emb_pos, float *x, RunState *state, cudaStream_t st) {
    prefill_embed_kernel<<<T, 256, 0, st>>>(tokens, pos0, D, V, emb_tok, emb_pos, x, state);
    return cudaGetLastError();
}
cudaError_t launch_prefill_ln(const float *x, int T, int D, const float *g, const float *b, float eps, int fix,
                              int8_t *limbs, cudaStream_t st) {
    if (D == 768) prefill_ln_kernel<768><<<T, 256, 0, st>>>(x, g, b, eps, fix, limbs);
    else if (D == 256) prefill_ln_kernel<256><<<T, 256, 0, st>>>(x, g, b, eps, fix, limbs);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}
cudaError_t launch_prefill_gemv(const PrefillGemv &a, cudaStream_t st) {
    const int nkb = a.K / 32;
    if (a.T < 1 || a.T > kPrefillTokens || a.K % 32 || a.N % kTile || a.nsplit < 1 || a.nsplit > nkb ||
        (nkb + a.nsplit - 1) / a.nsplit > kPfWarps * kPfMaxKbWarp)
        return cudaErrorInvalidValue;
    // the largest slice's staged limbs, or the warps' partials, whichever is larger
    const int ks = (nkb + a.nsplit - 1) / a.nsplit * 32;
    const size_t smem = std::max((size_t)kPrefillTokens * 4 * (ks + 16),
                                 (size_t)kPfWarps * kPrefillTokens * kTile * sizeof(long long));
    cudaError_t e = cudaFuncSetAttribute(prefill_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    prefill_gemv_kernel<<<dim3(a.N / kTile, a.nsplit), kPfWarps * 32, smem, st>>>(a);
    return cudaGetLastError();
}
cudaError_t launch_prefill_attn(const float *q, const uint16_t *kv, const int *pt, int layer, int n_phys, int n_heads,
                                int pos0, int T, int D, int fix, int8_t *limbs, cudaStream_t st) {
    prefill_attn_kernel<<<dim3(T, n_heads), 256, 0, st>>>(q, kv, pt, layer, n_phys, n_heads, pos0, D, fix, limbs);
    return cudaGetLastError();
}

// model widths the decode kernel is compiled for (d_model, ffn)
#define XDNA_DECODE_SHAPES(X) X(768, 3072) X(256, 512)

int decode_smem_bytes() { return SmemMap::total; }

static const void *decode_kernel_for(int d, int f) {
#define XDNA_PICK(DD, FF) if (d == DD && f == FF) return (const void *)opt_decode_kernel<DD, FF>;
    XDNA_DECODE_SHAPES(XDNA_PICK)
#undef XDNA_PICK
    return nullptr;
}

bool decode_shape_supported(int d, int f) { return decode_kernel_for(d, f) != nullptr; }

cudaError_t launch_opt_decode(const DecodeParams &p, cudaStream_t st) {
    const void *fn = decode_kernel_for(p.d_model, p.ffn);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemMap::total);
    if (e != cudaSuccess) return e;
    DecodeParams pp = p;
    void *args[] = {&pp};
    return cudaLaunchKernel(fn, dim3(p.grid), dim3(kThreads), args, SmemMap::total, st);
}

// largest even grid whose clusters of 2 are all co-resident (one CTA per SM)
cudaError_t max_coresident_ctas(int d, int f, int *out) {
    const void *fn = decode_kernel_for(d, f);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemMap::total);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms & ~1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = SmemMap::total;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg);
    if (e != cudaSuccess) return e;
    *out = 2 * clusters;
    return cudaSuccess;
}

}  // namespace xdna
