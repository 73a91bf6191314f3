// decode_kernel.cu -- the opt-125m decode step as ONE persistent kernel for sm_100a.
//
// Replaces the reference's per-token decode: rust/npu-whisper/src/bin/opt125m_decode.rs
// Opt::step (252-293) / Opt::generate (296-315) on the host, and the fused NPU decode ELF
// route_b_kernels/decode_fused/gen_decode.py (runlist 391-425).
//
// Design (B200-first):
//  * one CTA per SM, all co-resident (cooperative launch); each CTA = 8 consumer warps + 1
//    producer warp.
//  * every weight byte of a token is pre-packed on the host into ONE contiguous stream per
//    CTA, in the order the CTA consumes it (QKV, O, FC1, FC2 rows of each layer, then its
//    slice of the LM head).  The producer warp streams it with 1-D bulk async copies
//    (cp.async.bulk + mbarrier complete_tx) through a 5 x 32 KB shared-memory ring.  Weights
//    do not depend on activations, so HBM streaming never waits for the layer chain: it only
//    stalls when the ring is full.
//  * GEMV = int8 tensor-core MMA (m16n8k32): the bf16 activation vector is turned into a
//    22-bit fixed-point integer (per-vector power-of-two scale) split into three int8 limbs,
//    the limbs are the A operand rows, the int8 weight rows straight from the ring are the B
//    operand.  The int32 limb sums are combined exactly (int64) and rounded once to f32:
//    the dot product is exact, so the kernel reproduces the CPU oracle bit for bit.
//  * consecutive phases exchange their small output vectors through flag-tagged 64-bit
//    words (data | epoch) in global memory: a consumer polls the words it needs until their
//    epoch matches; no grid barrier, no fence on the critical path.
//  * attention: item (page p, head h) -> CTA (p*H + h) mod grid, statically, so the CTA
//    that appends a position's K/V to a page is the one that later reads that page: the KV
//    cache never crosses CTAs within a launch.  The page's cached rows are prefetched with
//    cp.async at the start of the layer.  Partial (max, sum, acc) per page are combined
//    flash-decode style by the O-projection CTAs.
//  * every wait is bounded (globaltimer deadline); a timeout records an error code in
//    RunState, makes all CTAs leave at their next phase boundary, and the producer drains
//    its in-flight copies before exiting.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cmath>

#include "decode.h"
#include "ptx.cuh"

namespace xdna {

// ------------------------------------------------------------------------------ smem map
struct SmemMap {
    static constexpr int ring = 0;
    static constexpr int limbs = ring + kStages * kStageBytes;           // 3 x kKmax int8
    static constexpr int act = limbs + 3 * kKmax;                        // kKmax bf16 / words
    static constexpr int xs = act + kKmax * 2;                           // 2 x kDmax f32
    static constexpr int lnp = xs + 2 * kDmax * 4;                       // [2][g|b][kDmax] f32
    static constexpr int kvbuf = lnp + 4 * kDmax * 4;                    // [page][K|V][64][64] bf16
    static constexpr int kvbuf_bytes = kGroupPages * 2 * kPageTokens * kHeadDim * 2;
    static constexpr int part = kvbuf + kvbuf_bytes;                     // 2 x partial MMA sums
    static constexpr int part_ints = kConsumerWarps * kMaxTilesPerChunk * 3 * 8;
    static constexpr int misc = part + 2 * part_ints * 4;
    static constexpr int misc_floats = 64 + 64 + 64 * kGroupPages + 4 * 64 * kGroupPages + 96 + 32 + kMaxPages + 8;
    static constexpr int bars = (misc + misc_floats * 4 + 15) & ~15;
    static constexpr int total = bars + 2 * kStages * 8 + 16;
};
static_assert(SmemMap::total <= 227 * 1024, "shared memory budget");

struct Cta {
    uint8_t *ring;
    int8_t *limbs;
    uint16_t *act;              // GEMV input vector (bf16) / gather buffer (32-bit words)
    float *xs;                  // residual stream, double buffered: xs[0..kDmax), xs[kDmax..)
    float *lnp;                 // LayerNorm parameters: [buf][0 = gamma, 1 = beta][kDmax]
    uint16_t *kvbuf;            // [kGroupPages][2][64][64] bf16: K rows then V rows per page (also a gather buffer)
    int *part;                  // [2][warps][tiles][3][8] partial limb sums
    float *red, *qf, *sc, *accp, *pst;   // pst: per-page (m, l)
    uint32_t *qkvw;             // 96 words: q, k, v of one head
    int *flag;                  // [0] abort flag, [1] greedy id
    int *pt;                    // page table copy
    uint64_t *full, *empty;
    int tid, warp, lane;
};

// the kernels' dynamic shared memory; out-of-line helpers rebuild their Cta view from it
extern __shared__ __align__(1024) uint8_t dsmem[];

__device__ __forceinline__ Cta make_cta(uint8_t *smem = dsmem) {
    Cta S;
    S.ring = smem + SmemMap::ring;
    S.limbs = reinterpret_cast<int8_t *>(smem + SmemMap::limbs);
    S.act = reinterpret_cast<uint16_t *>(smem + SmemMap::act);
    S.xs = reinterpret_cast<float *>(smem + SmemMap::xs);
    S.lnp = reinterpret_cast<float *>(smem + SmemMap::lnp);
    S.kvbuf = reinterpret_cast<uint16_t *>(smem + SmemMap::kvbuf);
    S.part = reinterpret_cast<int *>(smem + SmemMap::part);
    float *m = reinterpret_cast<float *>(smem + SmemMap::misc);
    S.red = m;
    S.qf = m + 64;
    S.sc = m + 128;                                   // [kGroupPages][64]
    S.accp = S.sc + 64 * kGroupPages;                 // [kGroupPages][4][64]
    S.qkvw = reinterpret_cast<uint32_t *>(S.accp + 256 * kGroupPages);
    S.flag = reinterpret_cast<int *>(S.qkvw + 96);
    S.pt = S.flag + 32;
    S.pst = reinterpret_cast<float *>(S.pt + kMaxPages);
    S.full = reinterpret_cast<uint64_t *>(smem + SmemMap::bars);
    S.empty = S.full + kStages;
    S.tid = threadIdx.x;
    S.warp = threadIdx.x >> 5;
    S.lane = threadIdx.x & 31;
    return S;
}

__device__ __forceinline__ void cbar() { named_bar(1, kConsumerThreads); }

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
#define set_error(p, code, where) set_error_st((p).state, (code), (where))
// Slow path of every bounded wait, called every few dozen polls: returns true when the
// waiter must give up -- another CTA already failed, or the deadline (counted from the
// first call, *t0) passed, in which case this CTA records the timeout.  Either way the
// CTA's shared abort flag is raised, so every consumer thread leaves at the next phase
// boundary without another global read.
__device__ __noinline__ bool wait_expired_st(RunState *st, uint64_t timeout_ns, int *sflag,
                                             uint64_t *t0, uint32_t code, uint32_t where) {
    if (read_error(st) != 0) { *(volatile int *)sflag = 1; return true; }
    const uint64_t now = globaltimer_ns();
    if (*t0 == 0) { *t0 = now; return false; }
    if (now - *t0 > timeout_ns) {
        set_error_st(st, code, where);
        *(volatile int *)sflag = 1;
        return true;
    }
    return false;
}
#define wait_expired(p, sflag, t0, code, where) \
    wait_expired_st((p).state, (p).timeout_ns, (sflag), &(t0), (code), (where))

__device__ __forceinline__ void wait_full(const DecodeParams &p, Cta &S, int slot, uint32_t parity,
                                          uint32_t where) {
    if (mbar_try_wait(&S.full[slot], parity)) return;
    uint64_t t0 = 0;
    while (!mbar_try_wait(&S.full[slot], parity))
        if (wait_expired(p, S.flag, t0, ERR_TIMEOUT_FULL, where)) return;
}

// Poll n flag-tagged words [src, src+n) until they all carry `epoch`; store their data to
// dst.  The words are spread over the warps in units of 4 per lane (at most 8 in flight
// per lane), and a lane re-polls only its words still missing, with a short sleep between
// rounds: 148 CTAs spinning on the same few L2 lines would otherwise saturate the L2 slices
// that hold them.  The caller follows with a consumer barrier.
// (out of line: one copy of the code, called by every phase, stays in the instruction cache)
__device__ __forceinline__ void ll_gather_impl(RunState *state, uint64_t timeout_ns, const uint64_t *src,
                                            uint32_t *dst, int n, uint32_t epoch, uint32_t where) {
    Cta S = make_cta();
    constexpr int B = 8;
    const int nw = min(kConsumerWarps, (n + 32 * 4 - 1) / (32 * 4));
    if (S.warp >= nw) return;
    const int stride = nw * 32;
    for (int base = 0; base < n; base += B * stride) {
        uint64_t v[B];
#pragma unroll
        for (int j = 0; j < B; j++) {
            const int i = base + S.tid + j * stride;
            v[j] = i < n ? ll_load(src + i) : (static_cast<uint64_t>(epoch) << 32);
        }
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (true) {
            bool all = true;
#pragma unroll
            for (int j = 0; j < B; j++) all &= static_cast<uint32_t>(v[j] >> 32) == epoch;
            if (all) break;
            __nanosleep(32);
#pragma unroll
            for (int j = 0; j < B; j++) {
                const int i = base + S.tid + j * stride;
                if (i < n && static_cast<uint32_t>(v[j] >> 32) != epoch) v[j] = ll_load(src + i);
            }
            if ((++it & 63) == 0 && wait_expired_st(state, timeout_ns, S.flag, &t0, ERR_TIMEOUT_FLAG, where)) break;
        }
#pragma unroll
        for (int j = 0; j < B; j++) {
            const int i = base + S.tid + j * stride;
            if (i < n) dst[i] = static_cast<uint32_t>(v[j]);
        }
    }
}
#define ll_gather(p, S, src, dst, n, epoch, where) \
    ll_gather_impl((p).state, (p).timeout_ns, (src), (dst), (n), (epoch), (where))

// uniform "should this CTA stop" decision among the consumer threads (shared flag only)
__device__ __forceinline__ bool abort_check(Cta &S) {
    cbar();
    const bool stop = *(volatile int *)S.flag != 0;
    cbar();
    return stop;
}

// optional phase timestamps: slot 0 token start, 1 + 5l + phase after each phase's publish,
// 5L + 1 after the LM head, 5L + 2 after the greedy id is known
__device__ __forceinline__ void stamp(const DecodeParams &p, const Cta &S, int t, int slot) {
    if (p.timing == nullptr || t >= 2 || S.tid != 0) return;
    p.timing[((size_t)t * p.grid + blockIdx.x) * 128 + slot] = globaltimer_ns();
    if (slot == 0 || slot == 5 * p.n_layers + 2)
        p.timing[((size_t)t * p.grid + blockIdx.x) * 128 + 120 + (slot != 0)] = clock64();
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
// max is order-free, so the single-instruction warp reductions give the butterfly's value
__device__ __forceinline__ float warp_max(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}
// max of non-negative floats: their bit patterns order like unsigned integers
__device__ __forceinline__ float warp_max_nonneg(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}

// 22-bit fixed-point exponent for a vector whose max |x| is m: X = rint(x * 2^s), |X| < 2^22
__device__ __forceinline__ int limb_exponent(float m) {
    const int E = m >= 0x1p-100f ? (int)((__float_as_uint(m) >> 23) & 0xff) - 126 : 0;   // m < 2^E
    return 22 - E;
}
// write the three int8 limbs of element i = lane + 32*kb: logical byte i of each limb row,
// 32-byte block kb of row j stored at block kb ^ j (bank-conflict-free MMA fragment loads)
__device__ __forceinline__ void put_limbs(int8_t *limbs, int kb, int lane, float x, float sc) {
    const int X = __float2int_rn(x * sc);
    const int c = ((X + 128) & 255) - 128;
    const int X1 = (X - c) >> 8;
    const int b = ((X1 + 128) & 255) - 128;
    const int a = (X1 - b) >> 8;
    limbs[0 * kKmax + ((kb ^ 0) << 5) + lane] = (int8_t)a;
    limbs[1 * kKmax + ((kb ^ 1) << 5) + lane] = (int8_t)b;
    limbs[2 * kKmax + ((kb ^ 2) << 5) + lane] = (int8_t)c;
}

// Residual add + LayerNorm + limbs, fused: x_new = x_old (+ add), h = bf16(LN(x_new))
// (rust/npu-asr-host/src/lib.rs:79-110: population variance, (x - mean) * inv * g + b, each
// op rounded), then the limbs of h.  Thread (warp w, lane l) owns elements 32*(w + 8j) + l;
// sums run over the thread's elements in j order, then the warp's xor butterfly, then the 8
// warp totals in warp order (the CPU oracle replays exactly this tree).  Three consumer
// barriers; returns the fixed-point exponent s.  The caller ends with a consumer barrier.
template <int D>
__device__ __forceinline__ int resid_ln_limbs_impl(const float *xo, float *xn, const uint32_t *add,
                                               const float *g, const float *b, float eps) {
    Cta S = make_cta();
    constexpr int PER = D / kConsumerThreads;
    static_assert(D % kConsumerThreads == 0, "d_model must be a multiple of 256");
    float xv[PER];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = 32 * (S.warp + 8 * j) + S.lane;
        float x = xo[i];
        if (add) { x = __fadd_rn(x, __uint_as_float(add[i])); xn[i] = x; }
        xv[j] = x;
        sum = __fadd_rn(sum, x);
    }
    sum = warp_sum(sum);
    if (S.lane == 0) S.red[S.warp] = sum;
    cbar();
    sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) sum = __fadd_rn(sum, S.red[w]);
    const float mean = __fdiv_rn(sum, (float)D);
    float var = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const float c = __fsub_rn(xv[j], mean);
        var = __fadd_rn(var, __fmul_rn(c, c));
    }
    var = warp_sum(var);
    if (S.lane == 0) S.red[8 + S.warp] = var;
    cbar();
    var = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) var = __fadd_rn(var, S.red[8 + w]);
    var = __fdiv_rn(var, (float)D);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = 32 * (S.warp + 8 * j) + S.lane;
        const float t = __fmul_rn(__fsub_rn(xv[j], mean), inv);
        xv[j] = bf16r(__fadd_rn(__fmul_rn(t, g[i]), b[i]));
        m = fmaxf(m, fabsf(xv[j]));
    }
    m = warp_max_nonneg(m);
    if (S.lane == 0) S.red[16 + S.warp] = m;
    cbar();
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) m = fmaxf(m, S.red[16 + w]);
    const int s = limb_exponent(m);
    const float sc = exp2i(s);
#pragma unroll
    for (int j = 0; j < PER; j++) put_limbs(S.limbs, S.warp + 8 * j, S.lane, xv[j], sc);
    return s;
}

template <int D>
__device__ __forceinline__ int resid_ln_limbs(Cta &, const float *xo, float *xn, const uint32_t *add,
                                              const float *g, const float *b, float eps) {
    return resid_ln_limbs_impl<D>(xo, xn, add, g, b, eps);
}

// Limbs of a length-K vector already in shared memory (bf16 or f32), same ownership as
// resid_ln_limbs.  One consumer barrier; the caller ends with another.
template <int K, class Load>
__device__ __forceinline__ int limbs_of(Cta &S, Load ld) {
    constexpr int PER = K / kConsumerThreads;
    static_assert(K % kConsumerThreads == 0, "length must be a multiple of 256");
    float v[PER];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        v[j] = ld(32 * (S.warp + 8 * j) + S.lane);
        m = fmaxf(m, fabsf(v[j]));
    }
    m = warp_max_nonneg(m);
    if (S.lane == 0) S.red[24 + S.warp] = m;
    cbar();
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) m = fmaxf(m, S.red[24 + w]);
    const int s = limb_exponent(m);
    const float sc = exp2i(s);
#pragma unroll
    for (int j = 0; j < PER; j++) put_limbs(S.limbs, S.warp + 8 * j, S.lane, v[j], sc);
    return s;
}

// limbs of the bf16 vector in S.act[0..K) (out of line)
template <int K>
__device__ __forceinline__ int limbs_of_act() {
    Cta S = make_cta();
    return limbs_of<K>(S, [&](int i) { return __uint_as_float((uint32_t)S.act[i] << 16); });
}

__device__ __forceinline__ void gemv_partials(const uint8_t *stage, int rows, int K, int pb) {
    Cta S = make_cta();
    const int g = S.lane >> 2, tig = S.lane & 3;
    const int ntiles = rows >> 3;
    const int KS = K >> 5;
    const int kb0 = S.warp * KS / kConsumerWarps, kb1 = (S.warp + 1) * KS / kConsumerWarps;
    int acc[kMaxTilesPerChunk][4];
#pragma unroll
    for (int t = 0; t < kMaxTilesPerChunk; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const int8_t *arow = S.limbs + (g < 3 ? g : 0) * kKmax;
#pragma unroll 4
    for (int kb = kb0; kb < kb1; kb++) {
        uint2 av = make_uint2(0u, 0u);
        if (g < 3) av = *reinterpret_cast<const uint2 *>(arow + ((kb ^ g) << 5) + tig * 8);
#pragma unroll
        for (int t = 0; t < kMaxTilesPerChunk; t++) {
            if (t < ntiles) {
                const uint8_t *br = stage + (size_t)(t * 8 + g) * K;
                uint2 bv = *reinterpret_cast<const uint2 *>(br + ((kb ^ (g & 3)) << 5) + tig * 8);
                mma_s8_16832(acc[t], av.x, 0u, av.y, 0u, bv.x, bv.y);
            }
        }
    }
    int *part = S.part + pb * SmemMap::part_ints;
    if (g < 3) {
#pragma unroll
        for (int t = 0; t < kMaxTilesPerChunk; t++) {
            if (t < ntiles) {
                int *pp = part + ((S.warp * kMaxTilesPerChunk + t) * 3 + g) * 8 + 2 * tig;
                pp[0] = acc[t][0];
                pp[1] = acc[t][1];
            }
        }
    }
}

// output row r of a chunk: float(exact dot) * 2^-s * scale + bias
__device__ __forceinline__ float gemv_row(const uint8_t *stage, int rows, int K, int s, int pb, int r) {
    const int *part = reinterpret_cast<const int *>(dsmem + SmemMap::part) + pb * SmemMap::part_ints;
    const float *meta = reinterpret_cast<const float *>(stage + (size_t)rows * K);
    const int t = r >> 3, col = r & 7;
    long long A = 0, B = 0, C = 0;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) {
        const int *pp = part + ((w * kMaxTilesPerChunk + t) * 3) * 8 + col;
        A += pp[0];
        B += pp[8];
        C += pp[16];
    }
    const float y = __fmul_rn(__ll2float_rn(A * 65536 + B * 256 + C), exp2i(-s));
    return __fadd_rn(__fmul_rn(y, meta[2 * r]), meta[2 * r + 1]);
}

// One weight chunk: rows (multiple of 8) x K int8 (row r swizzled by r & 3) followed by
// rows x (f32 scale, f32 bias).  Warps split K; their int32 limb partials meet in S.part
// (double buffered by `pb`, so one barrier per chunk suffices); then each output
// y = float(exact dot) * 2^-s * scale + bias goes to epi(row, y) -- or, with PAIR, rows
// 2j and 2j+1 go together to epi(2j, y0, y1) from one thread.
template <bool PAIR, class Epi>
__device__ __forceinline__ void gemv_chunk(Cta &S, const uint8_t *stage, int rows, int K, int s, int pb,
                                           Epi epi) {
    gemv_partials(stage, rows, K, pb);
    cbar();
    if (PAIR) {
        if (S.tid < (rows >> 1))
            epi(2 * S.tid, gemv_row(stage, rows, K, s, pb, 2 * S.tid), gemv_row(stage, rows, K, s, pb, 2 * S.tid + 1));
    } else {
        if (S.tid < rows) epi(S.tid, gemv_row(stage, rows, K, s, pb, S.tid), 0.0f);
    }
}

// Consume one phase's chunks from the ring (rows of reduction length K).
template <bool PAIR, class Epi>
__device__ __forceinline__ void gemv_phase(const DecodeParams &p, Cta &S, uint32_t &ctr, int rows, int K, int s,
                           uint32_t where, Epi epi) {
    const int rpc = rows_per_chunk(K);
    for (int r0 = 0; r0 < rows; r0 += rpc) {
        const int rr = min(rpc, rows - r0);
        const int slot = ctr % kStages;
        const uint32_t parity = (ctr / kStages) & 1u;
        wait_full(p, S, slot, parity, where);
        gemv_chunk<PAIR>(S, S.ring + slot * kStageBytes, rr, K, s, (int)(ctr & 1u),
                         [&](int r, float y0, float y1) { epi(r0 + r, y0, y1); });
        __syncwarp();
        if (S.lane == 0) mbar_arrive(&S.empty[slot]);
        ctr++;
    }
}

// ------------------------------------------------------------------------------ attention
__device__ __forceinline__ size_t kv_index(const DecodeParams &p, int layer, int phys, int kv,
                                           int head, int row) {
    return ((((size_t)layer * p.n_phys_pages + phys) * 2 + kv) * p.n_heads + head) *
               (size_t)(kPageTokens * kHeadDim) +
           (size_t)row * kHeadDim;
}

// cp.async the cached rows [j0, min(pos, j0 + 64 * kGroupPages)) of (layer, head) into
// kvbuf, j0 = first position of the item's page group.
__device__ __forceinline__ void kv_prefetch(const DecodeParams &p, Cta &S, int layer, int item, int pos) {
    const int H = p.n_heads;
    const int grp = item / H, h = item % H;
    const int j0 = grp * kGroupPages * kPageTokens;
    const int nrows = min(pos, j0 + kGroupPages * kPageTokens) - j0;   // cached rows (current pos excluded)
    for (int c = S.tid; c < nrows * 16; c += kConsumerThreads) {
        const int row = c >> 4, kv = (c >> 3) & 1, part = c & 7;
        const int pl = row / kPageTokens, r = row % kPageTokens;
        const int phys = S.pt[grp * kGroupPages + pl];
        const uint16_t *src = p.kv + kv_index(p, layer, phys, kv, h, r) + part * 8;
        // K rows keep their 16-byte chunk c at c ^ (row & 7): the score loop reads one row per
        // lane, and the swizzle spreads a quarter-warp's reads over all banks
        const int pc = kv ? part : part ^ (r & 7);
        uint16_t *dst = S.kvbuf + ((pl * 2 + kv) * kPageTokens + r) * kHeadDim + pc * 8;
        cp_async16(dst, src);
    }
    cp_async_commit();
}

// One (page group, head) item of single-query attention (mha_tile, mha_decode.cc:90-168, in
// its split form).  Per page of the group: scores of the page's keys against q (already
// * 1/sqrt(64) and bf16), the page max m, l = sum exp(s - m), acc = sum exp(s - m) v; the
// page partials are then merged in page order (flash-decode merge).  With one group in the
// context (`single`) the item publishes ctx = bf16(acc / l) of its head as 32 words at
// ll_att[h*32..]; otherwise it publishes the group partial [m, l, acc[64]] at ll_att[item*66].
__device__ __forceinline__ void att_item(const DecodeParams &p, Cta &S, int layer, int item, int pos,
                         bool prefetched, bool single, uint32_t ep_qkv, uint32_t ep_att, int t) {
    const int H = p.n_heads, D = p.d_model;
    const int grp = item / H, h = item % H;
    const int j0 = grp * kGroupPages * kPageTokens;
    const int ntok = min(pos + 1, j0 + kGroupPages * kPageTokens) - j0;   // keys, current included
    const int np = (ntok + kPageTokens - 1) / kPageTokens;
    const bool has_cur = pos < j0 + kGroupPages * kPageTokens;
    if (!prefetched) kv_prefetch(p, S, layer, item, pos);
    // q, k, v of head h: words [part*D/2 + h*32, +32)
    if (S.tid < 96) {
        const int part = S.tid >> 5, wi = S.tid & 31;
        const uint64_t *src = p.ll_qkv + part * (D / 2) + h * 32 + wi;
        uint64_t v = ll_load(src);
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (static_cast<uint32_t>(v >> 32) != ep_qkv) {
            v = ll_load(src);
            if ((++it & 63) == 0 && wait_expired(p, S.flag, t0, ERR_TIMEOUT_FLAG, 0x200u + layer)) break;
            __nanosleep(32);
        }
        S.qkvw[S.tid] = static_cast<uint32_t>(v);
    }
    if (layer == 1) stamp(p, S, t, 86);
    cp_async_wait_all();
    cbar();
    if (layer == 1) stamp(p, S, t, 80);
    if (S.tid < 32) {
        uint32_t w = S.qkvw[S.tid];
        S.qf[2 * S.tid] = bf16lo(w);
        S.qf[2 * S.tid + 1] = bf16hi(w);
    }
    if (has_cur && S.tid >= 32 && S.tid < 96) {
        // append this position's K (tid 32..63) or V (tid 64..95) row: kvbuf and the cache
        const int kv = (S.tid - 32) >> 5, wi = S.tid & 31, row = pos - j0;
        const int pl = row / kPageTokens, r = row % kPageTokens;
        const uint32_t w = S.qkvw[S.tid];
        const int swi = kv ? wi : (wi ^ ((r & 7) << 2));    // K: chunk (wi / 4) ^ (row & 7)
        reinterpret_cast<uint32_t *>(S.kvbuf + ((pl * 2 + kv) * kPageTokens + r) * kHeadDim)[swi] = w;
        const int phys = S.pt[grp * kGroupPages + pl];
        reinterpret_cast<uint32_t *>(p.kv + kv_index(p, layer, phys, kv, h, r))[wi] = w;
    }
    cbar();
    // scores: one key per thread (thread k -> page k / 64, key k % 64), four chains of 16
    // dims (d ascending) combined as (s0 + s1) + (s2 + s3)
    if (S.tid < np * kPageTokens) {
        const int pl = S.tid / kPageTokens, key = S.tid % kPageTokens;
        const int nk = min(kPageTokens, ntok - pl * kPageTokens);
        float sd = -INFINITY;
        if (key < nk) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(S.kvbuf + ((pl * 2) * kPageTokens + key) * kHeadDim);
            const float4 *q4p = reinterpret_cast<const float4 *>(S.qf);
            float s4[4];
#pragma unroll
            for (int q4 = 0; q4 < 4; q4++) {
                float acc = 0.0f;
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    const int c = 2 * q4 + half;
                    const uint4 kv8 = kr[c ^ (key & 7)];
                    const float4 qa = q4p[2 * c], qb = q4p[2 * c + 1];
                    acc = fmaf(qa.x, bf16lo(kv8.x), acc);
                    acc = fmaf(qa.y, bf16hi(kv8.x), acc);
                    acc = fmaf(qa.z, bf16lo(kv8.y), acc);
                    acc = fmaf(qa.w, bf16hi(kv8.y), acc);
                    acc = fmaf(qb.x, bf16lo(kv8.z), acc);
                    acc = fmaf(qb.y, bf16hi(kv8.z), acc);
                    acc = fmaf(qb.z, bf16lo(kv8.w), acc);
                    acc = fmaf(qb.w, bf16hi(kv8.w), acc);
                }
                s4[q4] = acc;
            }
            sd = __fadd_rn(__fadd_rn(s4[0], s4[1]), __fadd_rn(s4[2], s4[3]));
        }
        S.sc[pl * 64 + key] = sd;
    }
    cbar();
    if (layer == 1) stamp(p, S, t, 84);
    // page statistics: warp pl owns page pl; probabilities replace the scores in place
    if (S.warp < np) {
        const int pl = S.warp;
        const int nk = min(kPageTokens, ntok - pl * kPageTokens);
        float *sc = S.sc + pl * 64;
        const float s0 = sc[S.lane], s1 = sc[S.lane + 32];
        const float m = warp_max(fmaxf(s0, s1));
        const float p0 = S.lane < nk ? fast_exp_nonpos(__fsub_rn(s0, m)) : 0.0f;
        const float p1 = S.lane + 32 < nk ? fast_exp_nonpos(__fsub_rn(s1, m)) : 0.0f;
        const float l = warp_sum(p0 + p1);
        __syncwarp();
        sc[S.lane] = p0;
        sc[S.lane + 32] = p1;
        if (S.lane == 0) { S.pst[2 * pl] = m; S.pst[2 * pl + 1] = l; }
    }
    cbar();
    if (layer == 1) stamp(p, S, t, 85);
    // P.V: thread (d, q4) runs the chains over keys q4*16 .. q4*16+15 of every page (j ascending)
    {
        const int d = S.tid & 63, q4 = S.tid >> 6;
        float a[kGroupPages];
        int nkp[kGroupPages];
#pragma unroll
        for (int pl = 0; pl < kGroupPages; pl++) {
            a[pl] = 0.0f;
            nkp[pl] = pl < np ? min(kPageTokens, ntok - pl * kPageTokens) : 0;
        }
#pragma unroll 4
        for (int jj = 0; jj < 16; jj++) {
            const int j = q4 * 16 + jj;
#pragma unroll
            for (int pl = 0; pl < kGroupPages; pl++) {
                if (j < nkp[pl]) {
                    const uint16_t v = S.kvbuf[((pl * 2 + 1) * kPageTokens + j) * kHeadDim + d];
                    a[pl] = fmaf(S.sc[pl * 64 + j], __uint_as_float((uint32_t)v << 16), a[pl]);
                }
            }
        }
#pragma unroll
        for (int pl = 0; pl < kGroupPages; pl++)
            if (pl < np) S.accp[(pl * 4 + q4) * 64 + d] = a[pl];
    }
    cbar();
    if (layer == 1) stamp(p, S, t, 81);
    if (S.tid < 64) {
        float M = -INFINITY, L = 0.0f, A = 0.0f;
        for (int pl = 0; pl < np; pl++) {
            const float *ap = S.accp + pl * 256 + S.tid;
            const float a = __fadd_rn(__fadd_rn(__fadd_rn(ap[0], ap[64]), ap[128]), ap[192]);
            const float mp = S.pst[2 * pl], lp = S.pst[2 * pl + 1];
            const float mn = fmaxf(M, mp);
            const float c0 = fast_exp_nonpos(__fsub_rn(M, mn));
            const float c1 = fast_exp_nonpos(__fsub_rn(mp, mn));
            L = __fadd_rn(__fmul_rn(L, c0), __fmul_rn(lp, c1));
            A = __fadd_rn(__fmul_rn(A, c0), __fmul_rn(a, c1));
            M = mn;
        }
        if (single) {
            const float ctx = __fdiv_rn(A, L);
            const uint32_t mine = bf16bits(ctx);
            const uint32_t hi = __shfl_down_sync(0xffffffffu, mine, 1);
            if ((S.tid & 1) == 0) ll_store(p.ll_att + h * 32 + (S.tid >> 1), mine | (hi << 16), ep_att);
        } else {
            uint64_t *dst = p.ll_att + (size_t)item * (2 + kHeadDim);
            ll_store(dst + 2 + S.tid, __float_as_uint(A), ep_att);
            if (S.tid == 0) ll_store(dst, __float_as_uint(M), ep_att);
            if (S.tid == 1) ll_store(dst + 1, __float_as_uint(L), ep_att);
        }
    }
    // no trailing barrier: what follows writes none of sc / accp / pst before its own barrier
}

// n_groups page groups cover positions [0, pos]
__device__ __forceinline__ int att_groups(int pos) { return pos / (kGroupPages * kPageTokens) + 1; }

// Combine the group partials of every head (flash-decode merge, in group order) into
// ctx = bf16(acc / l) in S.act[0..D).  Partials are staged through kvbuf in batches of whole
// items.  The caller ends with a consumer barrier.
__device__ __forceinline__ void att_combine(const DecodeParams &p, Cta &S, int pos, uint32_t ep_att, int layer) {
    const int H = p.n_heads, D = p.d_model;
    const int n_items = att_groups(pos) * H;
    constexpr int W = 2 + kHeadDim;
    const int per_batch = (SmemMap::kvbuf_bytes / 4) / W;   // items per kvbuf load
    float M[4], L[4], A[4];
#pragma unroll
    for (int k = 0; k < 4; k++) { M[k] = -INFINITY; L[k] = 0.0f; A[k] = 0.0f; }
    uint32_t *buf = reinterpret_cast<uint32_t *>(S.kvbuf);
    for (int b0 = 0; b0 < n_items; b0 += per_batch) {
        const int b1 = min(n_items, b0 + per_batch);
        if (b0 > 0) cbar();                       // previous batch fully read
        ll_gather(p, S, p.ll_att + (size_t)b0 * W, buf, (b1 - b0) * W, ep_att, 0x300u + layer);
        cbar();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int i = S.tid + k * kConsumerThreads;
            if (i < D) {
                const int h = i / kHeadDim, d = i % kHeadDim;
                int it = b0 + ((h - b0 % H) + H) % H;       // first item of head h in batch
                for (; it < b1; it += H) {
                    const uint32_t *w = buf + (size_t)(it - b0) * W;
                    const float mp = __uint_as_float(w[0]), lp = __uint_as_float(w[1]);
                    const float ap = __uint_as_float(w[2 + d]);
                    const float mn = fmaxf(M[k], mp);
                    const float c0 = fast_exp_nonpos(__fsub_rn(M[k], mn));
                    const float c1 = fast_exp_nonpos(__fsub_rn(mp, mn));
                    L[k] = __fadd_rn(__fmul_rn(L[k], c0), __fmul_rn(lp, c1));
                    A[k] = __fadd_rn(__fmul_rn(A[k], c0), __fmul_rn(ap, c1));
                    M[k] = mn;
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = S.tid + k * kConsumerThreads;
        if (i < D) S.act[i] = (uint16_t)bf16bits(__fdiv_rn(A[k], L[k]));
    }
}

// optional debugging record of the residual stream (CTA 0 only); after a consumer barrier
__device__ __forceinline__ void trace_x(const DecodeParams &p, Cta &S, int t, int slot, const float *v) {
    if (p.trace == nullptr || blockIdx.x != 0) return;
    float *dst = p.trace + ((size_t)t * (2 * p.n_layers + 1) + slot) * p.d_model;
    for (int i = S.tid; i < p.d_model; i += kConsumerThreads) dst[i] = v[i];
}
// prefetch a LayerNorm's gamma and beta into S.lnp[buf] (cp.async, generic proxy)
__device__ __forceinline__ void ln_prefetch(Cta &S, int buf, const float *g, const float *b, int D) {
    float *dst = S.lnp + buf * 2 * kDmax;
    for (int c = S.tid; c < D / 2; c += kConsumerThreads) {   // D/4 16-byte pieces per vector
        const int v = c / (D / 4), q = c % (D / 4);
        cp_async16(dst + v * kDmax + 4 * q, (v ? b : g) + 4 * q);
    }
    cp_async_commit();
}

__device__ __forceinline__ void producer(const DecodeParams &p, Cta &S) {
    if (S.lane != 0) return;
    const int c = blockIdx.x;
    const ChunkRef *tab = p.chunks + (size_t)c * p.chunk_stride;
    const int nl = p.n_layer_chunks[c], nlm = p.n_lm_chunks[c];
    uint32_t ctr = 0;
    bool failed = false;
    for (int t = 0; t < p.n_steps && !failed; t++) {
        const int pos = p.start_pos + t;
        const int n = nl + (pos >= p.n_prompt - 1 ? nlm : 0);
        for (int i = 0; i < n; i++) {
            const int slot = ctr % kStages;
            const uint32_t k = ctr / kStages;
            if (k > 0 && !mbar_try_wait(&S.empty[slot], (k - 1) & 1u)) {
                uint64_t t0 = 0;
                while (!mbar_try_wait(&S.empty[slot], (k - 1) & 1u))
                    if (wait_expired(p, S.flag, t0, ERR_TIMEOUT_EMPTY, 0x400u)) { failed = true; break; }
                if (failed) break;
            }
            const ChunkRef ch = tab[i];
            mbar_arrive_expect_tx(&S.full[slot], ch.bytes);
            bulk_g2s(S.ring + slot * kStageBytes, p.stream + ch.off, ch.bytes, &S.full[slot]);
            ctr++;
        }
    }
    // drain: every issued copy must land before the CTA's shared memory is released
    const uint32_t first = ctr > (uint32_t)kStages ? ctr - kStages : 0u;
    for (uint32_t q = first; q < ctr; q++) {
        const int slot = q % kStages;
        const uint32_t par = (q / kStages) & 1u;
        uint64_t t0 = 0;
        const uint64_t start = globaltimer_ns();
        while (!mbar_try_wait(&S.full[slot], par)) {
            (void)t0;
            if (globaltimer_ns() - start > p.timeout_ns) break;
        }
    }
}

template <int D, int F>
__device__ __forceinline__ void consumer(const DecodeParams &p, Cta &S) {
    const int c = blockIdx.x, G = p.grid;
    const int L = p.n_layers, V = p.vocab, H = p.n_heads;
    const uint32_t base = p.state->epoch_base;
    const int PHT = kPhasesPerLayer * L + 1;
    const int q_row0 = part_row0(c, 3 * D, G), q_rows = part_rows(c, 3 * D, G);
    const int o_row0 = part_row0(c, D, G), o_rows = part_rows(c, D, G);
    const int f1_row0 = part_row0(c, F, G), f1_rows = part_rows(c, F, G);
    const int f2_row0 = part_row0(c, D, G), f2_rows = part_rows(c, D, G);
    const int lm_row0 = part_row0(c, V, G), lm_rows = part_rows(c, V, G);
    uint32_t ctr = 0;
    int64_t next_id = 0;
    uint32_t *actw = reinterpret_cast<uint32_t *>(S.act);
    const float *lng = S.lnp, *lnb = S.lnp + kDmax;                     // buffer 0: LN1 / LNf
    const float *ln2g = S.lnp + 2 * kDmax, *ln2b = S.lnp + 3 * kDmax;  // buffer 1: LN2
    for (int i = S.tid; i < kMaxPages; i += kConsumerThreads)
        S.pt[i] = i < p.n_phys_pages ? p.page_table[i] : 0;
    if (S.tid == 0) { S.flag[0] = 0; S.flag[1] = 0; }
    cbar();

    for (int t = 0; t < p.n_steps; t++) {
        const int pos = p.start_pos + t;
        const uint32_t ep0 = base + (uint32_t)(t * PHT) + 1u;
        const int64_t id = (t == 0 || pos < p.n_prompt) ? p.tokens[pos] : next_id;
        if (id < 0 || id >= V || pos + 2 > p.max_pos + 1) {
            if (S.tid == 0) {
                set_error(p, id < 0 || id >= V ? ERR_BAD_TOKEN : ERR_BAD_POS, pos);
                S.flag[0] = 1;
            }
        }
        cp_async_wait_all();                 // no stale LN prefetch may land after the next
        if (abort_check(S)) return;
        stamp(p, S, t, 0);
        ln_prefetch(S, 0, p.ln, p.ln + D, D);
        float *xcur = S.xs;                  // x lives in xs[0..D) or xs[kDmax..kDmax+D)
        for (int i = S.tid; i < D; i += kConsumerThreads)
            xcur[i] = __fadd_rn(p.emb_tok[(size_t)id * D + i], p.emb_pos[(size_t)(pos + 2) * D + i]);
        const int n_items = att_groups(pos) * H;
        const bool single = n_items == H;

        for (int l = 0; l < L; l++) {
            const uint32_t ep = ep0 + (uint32_t)(l * kPhasesPerLayer);
            const float *ln = p.ln + (size_t)l * 4 * D;
            // cp.async groups, oldest first: LN1 params (issued one phase group earlier),
            // LN2 params, this CTA's KV pages (always committed, possibly empty)
            ln_prefetch(S, 1, ln + 2 * D, ln + 3 * D, D);
            if (c < n_items) kv_prefetch(p, S, l, c, pos);
            else cp_async_commit();
            // ---------------- QKV: x += fc2(prev layer); LN1; q, k, v rows
            if (l > 0) ll_gather(p, S, p.ll_f2, actw, D, ep - kPhasesPerLayer + PH_FC2, 0x10u + l);
            cp_async_wait_group<2>();          // LN1 params in; LN2 and KV may still be in flight
            cbar();
            if (l == 1) stamp(p, S, t, 70);
            if (*(volatile int *)S.flag) return;
            float *xnext = xcur == S.xs ? S.xs + kDmax : S.xs;
            int s = resid_ln_limbs<D>(S, xcur, xnext, l > 0 ? actw : nullptr, lng, lnb, p.eps);
            if (l > 0) xcur = xnext;
            cbar();
            if (l == 1) stamp(p, S, t, 71);
            if (l > 0) trace_x(p, S, t, 2 * (l - 1) + 1, xcur);
            gemv_phase<true>(p, S, ctr, q_rows, D, s, 0x20u + l, [&](int r, float y0, float y1) {
                const int n = q_row0 + r;
                if (n < D) { y0 = __fmul_rn(y0, 0.125f); y1 = __fmul_rn(y1, 0.125f); }
                ll_store(p.ll_qkv + n / 2, bf16bits(y0) | (bf16bits(y1) << 16), ep + PH_QKV);
            });
            stamp(p, S, t, 1 + 5 * l + PH_QKV);
            if (l == 1) stamp(p, S, t, 72);
            // ---------------- ATT: this CTA's (page, head) items
            for (int it = c, k = 0; it < n_items; it += G, k++)
                att_item(p, S, l, it, pos, k == 0, single, ep + PH_QKV, ep + PH_ATT, t);
            stamp(p, S, t, 1 + 5 * l + PH_ATT);
            // LN1 of the next layer (or the final LN) into buffer 0, read by nothing until then
            if (l + 1 < L) ln_prefetch(S, 0, ln + 4 * D, ln + 5 * D, D);
            else ln_prefetch(S, 0, p.lnf, p.lnf + D, D);
            // ---------------- O: merge partials -> ctx; O rows
            if (o_rows > 0) {
                if (single) ll_gather(p, S, p.ll_att, actw, D / 2, ep + PH_ATT, 0x300u + l);
                else att_combine(p, S, pos, ep + PH_ATT, l);
                cbar();
                if (l == 1) stamp(p, S, t, 82);
                s = limbs_of_act<D>();
                cbar();
                if (l == 1) stamp(p, S, t, 83);
                gemv_phase<false>(p, S, ctr, o_rows, D, s, 0x30u + l, [&](int r, float y, float) {
                    ll_store(p.ll_o + o_row0 + r, __float_as_uint(y), ep + PH_O);
                });
            }
            stamp(p, S, t, 1 + 5 * l + PH_O);
            // ---------------- FC1: x += o; LN2; relu(fc1) -> bf16
            if (l == 1) stamp(p, S, t, 63);
            ll_gather(p, S, p.ll_o, actw, D, ep + PH_O, 0x40u + l);
            cp_async_wait_group<1>();          // LN2 params in; the next LN1 may still be in flight
            cbar();
            if (l == 1) stamp(p, S, t, 64);
            if (*(volatile int *)S.flag) return;
            xnext = xcur == S.xs ? S.xs + kDmax : S.xs;
            s = resid_ln_limbs<D>(S, xcur, xnext, actw, ln2g, ln2b, p.eps);
            xcur = xnext;
            cbar();
            if (l == 1) stamp(p, S, t, 65);
            trace_x(p, S, t, 2 * l, xcur);
            gemv_phase<true>(p, S, ctr, f1_rows, D, s, 0x50u + l, [&](int r, float y0, float y1) {
                y0 = fmaxf(y0, 0.0f);
                y1 = fmaxf(y1, 0.0f);
                ll_store(p.ll_h + (f1_row0 + r) / 2, bf16bits(y0) | (bf16bits(y1) << 16), ep + PH_FC1);
            });
            stamp(p, S, t, 1 + 5 * l + PH_FC1);
            // ---------------- FC2
            if (f2_rows > 0) {
                if (l == 1) stamp(p, S, t, 66);
                ll_gather(p, S, p.ll_h, actw, F / 2, ep + PH_FC1, 0x60u + l);
                cbar();
                if (l == 1) stamp(p, S, t, 67);
                s = limbs_of_act<F>();
                cbar();
                if (l == 1) stamp(p, S, t, 68);
                gemv_phase<false>(p, S, ctr, f2_rows, F, s, 0x70u + l, [&](int r, float y, float) {
                    ll_store(p.ll_f2 + f2_row0 + r, __float_as_uint(y), ep + PH_FC2);
                });
            }
            stamp(p, S, t, 1 + 5 * l + PH_FC2);
        }
        // ---------------- final residual, LN, LM head + greedy argmax
        const uint32_t ep_last = ep0 + (uint32_t)((L - 1) * kPhasesPerLayer) + PH_FC2;
        if (pos >= p.n_prompt - 1) {
            const uint32_t ep_lm = ep0 + (uint32_t)(L * kPhasesPerLayer);
            ll_gather(p, S, p.ll_f2, actw, D, ep_last, 0x80u);
            cp_async_wait_all();
            cbar();
            if (*(volatile int *)S.flag) return;
            float *xnext = xcur == S.xs ? S.xs + kDmax : S.xs;
            const int s = resid_ln_limbs<D>(S, xcur, xnext, actw, lng, lnb, p.eps);
            cbar();
            trace_x(p, S, t, 2 * L - 1, xnext);
            float best = -INFINITY;
            int best_i = -1;
            const int lm_step = pos - max(p.start_pos, p.n_prompt - 1);
            float *lrow = p.logits ? p.logits + (size_t)lm_step * V : nullptr;
            gemv_phase<false>(p, S, ctr, lm_rows, D, s, 0x100u, [&](int r, float y, float) {
                const int idx = lm_row0 + r;
                if (lrow) lrow[idx] = y;
                if (y > best || (y == best && idx > best_i)) { best = y; best_i = idx; }
            });
            // CTA-level argmax (ties -> larger index: Iterator::max_by, opt125m_decode.rs:303)
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                if (ob > best || (ob == best && oi > best_i)) { best = ob; best_i = oi; }
            }
            if (S.lane == 0) { S.red[S.warp] = best; S.red[32 + S.warp] = __int_as_float(best_i); }
            cbar();
            if (S.tid == 0) {
                float b = S.red[0];
                int bi = __float_as_int(S.red[32]);
                for (int w = 1; w < kConsumerWarps; w++) {
                    const float ob = S.red[w];
                    const int oi = __float_as_int(S.red[32 + w]);
                    if (ob > b || (ob == b && oi > bi)) { b = ob; bi = oi; }
                }
                ll_store(p.ll_lm + 2 * c, __float_as_uint(b), ep_lm);
                ll_store(p.ll_lm + 2 * c + 1, (uint32_t)bi, ep_lm);
            }
            stamp(p, S, t, 5 * L + 1);
            // global argmax over all CTAs (every CTA computes it in the same order)
            ll_gather(p, S, p.ll_lm, actw, 2 * G, ep_lm, 0x90u);
            cbar();
            if (S.tid == 0) {
                float b = -INFINITY;
                int bi = -1;
                for (int q = 0; q < G; q++) {
                    const float ob = __uint_as_float(actw[2 * q]);
                    const int oi = (int)actw[2 * q + 1];
                    if (oi < 0) continue;
                    if (bi < 0 || ob > b || (ob == b && oi > bi)) { b = ob; bi = oi; }
                }
                S.flag[1] = bi;
                if (c == 0) p.tokens[pos + 1] = bi;
            }
            cbar();
            next_id = S.flag[1];
            stamp(p, S, t, 5 * L + 2);
        } else {
            next_id = p.tokens[pos + 1];
        }
    }
    if (c == 0 && S.tid == 0) p.state->epoch_base = base + (uint32_t)(p.n_steps * PHT);
}

template <int D, int F>
__global__ void __launch_bounds__(kThreads, 1) opt_decode_kernel(const DecodeParams p) {
    Cta S = make_cta();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    if (S.warp == kConsumerWarps) producer(p, S);
    else consumer<D, F>(p, S);
}

// model widths the decode kernel is compiled for (d_model, ffn)
#define XDNA_DECODE_SHAPES(X) X(768, 3072) X(256, 512)

// ------------------------------------------------------------------ standalone GEMV (op API)
// y[N] = exact-int8-GEMV(x[K]) * scale + bias over a packed chunk list: one CTA per chunk,
// the decode kernel's limb and MMA code (for parity tests and the op-level C ABI).
__global__ void __launch_bounds__(kThreads, 1)
gemv_i8_kernel(const float *x, int K, const uint8_t *packed, const ChunkRef *chunks, int N, float *y) {
    Cta S = make_cta();
    const int rpc = rows_per_chunk(K);
    const int row0 = blockIdx.x * rpc;
    const int rows = min(rpc, N - row0);
    if (threadIdx.x == 0) {
        mbar_init(&S.full[0], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == kConsumerThreads) {
        const ChunkRef ch = chunks[blockIdx.x];
        mbar_arrive_expect_tx(&S.full[0], ch.bytes);
        bulk_g2s(S.ring, packed + ch.off, ch.bytes, &S.full[0]);
    }
    if (S.warp == kConsumerWarps) return;
    float *xf = reinterpret_cast<float *>(S.kvbuf);
    for (int i = S.tid; i < K; i += kConsumerThreads) xf[i] = x[i];
    cbar();
    int s = 0;
    switch (K) {
#define XDNA_GEMV_K(KK) case KK: s = limbs_of<KK>(S, [&](int i) { return xf[i]; }); break;
        XDNA_GEMV_K(256) XDNA_GEMV_K(512) XDNA_GEMV_K(768) XDNA_GEMV_K(1024) XDNA_GEMV_K(1536)
        XDNA_GEMV_K(2048) XDNA_GEMV_K(2560) XDNA_GEMV_K(3072)
#undef XDNA_GEMV_K
        default: return;
    }
    cbar();
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(&S.full[0], 0u))
        if (globaltimer_ns() - start > 1000000000ull) return;   // bounded (1 s)
    gemv_chunk<false>(S, S.ring, rows, K, s, 0, [&](int r, float v, float) { y[row0 + r] = v; });
}

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
    return cudaLaunchCooperativeKernel(fn, dim3(p.grid), dim3(kThreads), args, SmemMap::total, st);
}

cudaError_t launch_gemv_i8(const float *x, int K, const uint8_t *packed, const ChunkRef *chunks,
                           int N, float *y, cudaStream_t st) {
    // per-device attribute: set on every launch (cheap), so a second device is covered too
    cudaError_t e = cudaFuncSetAttribute(gemv_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SmemMap::total);
    if (e != cudaSuccess) return e;
    const int nch = (N + rows_per_chunk(K) - 1) / rows_per_chunk(K);
    gemv_i8_kernel<<<nch, kThreads, SmemMap::total, st>>>(x, K, packed, chunks, N, y);
    return cudaGetLastError();
}

cudaError_t max_coresident_ctas(int *out) {
    const void *fn = decode_kernel_for(768, 3072);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemMap::total);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, kThreads, SmemMap::total);
    if (e != cudaSuccess) return e;
    *out = sms * per;
    return cudaSuccess;
}

}  // namespace xdna
