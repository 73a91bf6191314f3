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
    static constexpr int kvbuf = lnp + 4 * kDmax * 4;                    // 2 x 64 x 64 bf16
    static constexpr int part = kvbuf + 2 * kPageTokens * kHeadDim * 2;  // 2 x partial MMA sums
    static constexpr int part_ints = kConsumerWarps * kMaxTilesPerChunk * 3 * 8;
    static constexpr int misc = part + 2 * part_ints * 4;
    static constexpr int misc_floats = 64 + 64 + 64 + 4 * 64 + 96 + 32 + kMaxPages;
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
    uint16_t *kvbuf;            // [2][64][64] bf16: K rows then V rows (also a gather buffer)
    int *part;                  // [2][warps][tiles][3][8] partial limb sums
    float *red, *qf, *sc, *accp;
    uint32_t *qkvw;             // 96 words: q, k, v of one head
    int *flag;                  // [0] abort flag, [1] greedy id
    int *pt;                    // page table copy
    uint64_t *full, *empty;
    int tid, warp, lane;
};

__device__ __forceinline__ Cta make_cta(uint8_t *smem) {
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
    S.sc = m + 128;
    S.accp = m + 192;
    S.qkvw = reinterpret_cast<uint32_t *>(m + 448);
    S.flag = reinterpret_cast<int *>(m + 544);
    S.pt = reinterpret_cast<int *>(m + 576);
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
// dst.  Only as many warps as needed poll (16 words in flight per lane), with a short sleep
// between rounds: 148 CTAs spinning with every thread on the same few L2 lines saturate the
// L2 slices that hold them.  The caller follows with a consumer barrier.
__device__ __forceinline__ void ll_gather(const DecodeParams &p, Cta &S, const uint64_t *src, uint32_t *dst,
                          int n, uint32_t epoch, uint32_t where) {
    constexpr int B = 16;
    const int nw = min(kConsumerWarps, (n + 32 * B - 1) / (32 * B));
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
            if ((++it & 63) == 0 && wait_expired(p, S.flag, t0, ERR_TIMEOUT_FLAG, where)) break;
        }
#pragma unroll
        for (int j = 0; j < B; j++) {
            const int i = base + S.tid + j * stride;
            if (i < n) dst[i] = static_cast<uint32_t>(v[j]);
        }
    }
}

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
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
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
__device__ __forceinline__ int resid_ln_limbs(Cta &S, const float *xo, float *xn, const uint32_t *add,
                                              const float *g, const float *b, float eps) {
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
    m = warp_max(m);
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
    m = warp_max(m);
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

// One weight chunk: rows (multiple of 8) x K int8 (row r swizzled by r & 3) followed by
// rows x (f32 scale, f32 bias).  Warps split K; their int32 limb partials meet in S.part
// (double buffered by `pb`, so one barrier per chunk suffices); then each output
// y = float(exact dot) * 2^-s * scale + bias goes to epi(row, y) -- or, with PAIR, rows
// 2j and 2j+1 go together to epi(2j, y0, y1) from one thread.
template <bool PAIR, class Epi>
__device__ __forceinline__ void gemv_chunk(Cta &S, const uint8_t *stage, int rows, int K, int s, int pb,
                                           Epi epi) {
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
    cbar();
    const float *meta = reinterpret_cast<const float *>(stage + (size_t)rows * K);
    const float down = exp2i(-s);
    auto row = [&](int r) {
        const int t = r >> 3, col = r & 7;
        long long A = 0, B = 0, C = 0;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) {
            const int *pp = part + ((w * kMaxTilesPerChunk + t) * 3) * 8 + col;
            A += pp[0];
            B += pp[8];
            C += pp[16];
        }
        const float y = __fmul_rn(__ll2float_rn(A * 65536 + B * 256 + C), down);
        return __fadd_rn(__fmul_rn(y, meta[2 * r]), meta[2 * r + 1]);
    };
    if (PAIR) {
        if (S.tid < (rows >> 1)) epi(2 * S.tid, row(2 * S.tid), row(2 * S.tid + 1));
    } else {
        if (S.tid < rows) epi(S.tid, row(S.tid), 0.0f);
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

// cp.async the cached rows [page*64, min(pos, page*64+64)) of (layer, head) into kvbuf.
__device__ __forceinline__ void kv_prefetch(const DecodeParams &p, Cta &S, int layer, int item, int pos) {
    const int H = p.n_heads;
    const int pg = item / H, h = item % H;
    const int j0 = pg * kPageTokens;
    const int nrows = min(pos, j0 + kPageTokens) - j0;   // cached rows (current pos excluded)
    if (nrows <= 0) return;
    const int phys = S.pt[pg];
    const uint16_t *srcK = p.kv + kv_index(p, layer, phys, 0, h, 0);
    const uint16_t *srcV = p.kv + kv_index(p, layer, phys, 1, h, 0);
    for (int c = S.tid; c < nrows * 16; c += kConsumerThreads) {
        const int row = c >> 4, kv = (c >> 3) & 1, part = c & 7;
        const uint16_t *src = (kv ? srcV : srcK) + row * kHeadDim + part * 8;
        uint16_t *dst = S.kvbuf + kv * kPageTokens * kHeadDim + row * kHeadDim + part * 8;
        cp_async16(dst, src);
    }
    cp_async_commit();
}

// One (page, head) item of single-query attention (mha_tile, mha_decode.cc:90-168, in its
// split form): scores of the page's keys against q (already * 1/sqrt(64) and bf16), the page
// max m, l = sum exp(s - m), acc = sum exp(s - m) v.  Publishes [m, l, acc[64]].
__device__ __forceinline__ void att_item(const DecodeParams &p, Cta &S, int layer, int item, int pos,
                         bool prefetched, uint32_t ep_qkv, uint32_t ep_att) {
    const int H = p.n_heads, D = p.d_model;
    const int pg = item / H, h = item % H;
    const int j0 = pg * kPageTokens;
    const int nk = min(pos + 1, j0 + kPageTokens) - j0;
    const bool has_cur = pos < j0 + kPageTokens;
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
    cp_async_wait_all();
    cbar();
    if (layer == 1) stamp(p, S, 0, 80);
    if (S.tid < 32) {
        uint32_t w = S.qkvw[S.tid];
        S.qf[2 * S.tid] = bf16lo(w);
        S.qf[2 * S.tid + 1] = bf16hi(w);
    }
    if (has_cur && S.tid >= 32 && S.tid < 96) {
        // append this position's K (tid 32..63) or V (tid 64..95) row: kvbuf and the cache
        const int kv = (S.tid - 32) >> 5, wi = S.tid & 31, row = pos - j0;
        const uint32_t w = S.qkvw[S.tid];
        reinterpret_cast<uint32_t *>(S.kvbuf + kv * kPageTokens * kHeadDim + row * kHeadDim)[wi] = w;
        const int phys = S.pt[pg];
        reinterpret_cast<uint32_t *>(p.kv + kv_index(p, layer, phys, kv, h, row))[wi] = w;
    }
    cbar();
    // scores: warp w -> keys 8w..8w+7, 4 lanes per key, 16 dims per lane
    {
        const int key = S.warp * 8 + (S.lane >> 2), d0 = (S.lane & 3) * 16;
        float sd = 0.0f;
        if (key < nk) {
            const uint16_t *kr = S.kvbuf + key * kHeadDim + d0;
#pragma unroll
            for (int d = 0; d < 16; d++) sd = fmaf(S.qf[d0 + d], __uint_as_float((uint32_t)kr[d] << 16), sd);
        }
        sd += __shfl_xor_sync(0xffffffffu, sd, 1);
        sd += __shfl_xor_sync(0xffffffffu, sd, 2);
        if ((S.lane & 3) == 0) S.sc[key] = key < nk ? sd : -INFINITY;
    }
    cbar();
    float m = warp_max(fmaxf(S.sc[S.lane], S.sc[S.lane + 32]));
    float p0 = S.lane < nk ? fast_exp_nonpos(__fsub_rn(S.sc[S.lane], m)) : 0.0f;
    float p1 = S.lane + 32 < nk ? fast_exp_nonpos(__fsub_rn(S.sc[S.lane + 32], m)) : 0.0f;
    float l = warp_sum(p0 + p1);
    cbar();                      // everyone has read the scores
    if (S.warp == 0) { S.sc[S.lane] = p0; S.sc[S.lane + 32] = p1; }
    cbar();
    {
        const int d = S.tid & 63, q4 = S.tid >> 6;
        float a = 0.0f;
        const uint16_t *vb = S.kvbuf + kPageTokens * kHeadDim;
        for (int j = q4 * 16; j < q4 * 16 + 16 && j < nk; j++)
            a = fmaf(S.sc[j], __uint_as_float((uint32_t)vb[j * kHeadDim + d] << 16), a);
        S.accp[q4 * 64 + d] = a;
    }
    cbar();
    if (layer == 1) stamp(p, S, 0, 81);
    uint64_t *dst = p.ll_att + (size_t)item * (2 + kHeadDim);
    if (S.tid < 64) {
        float a = S.accp[S.tid] + S.accp[64 + S.tid] + S.accp[128 + S.tid] + S.accp[192 + S.tid];
        ll_store(dst + 2 + S.tid, __float_as_uint(a), ep_att);
    } else if (S.tid == 64) {
        ll_store(dst, __float_as_uint(m), ep_att);
    } else if (S.tid == 65) {
        ll_store(dst + 1, __float_as_uint(l), ep_att);
    }
    cbar();
}

// Combine the page partials of every head (flash-decode merge, in page order) into
// ctx = bf16(acc / l) in S.act[0..D).  Partials are staged through kvbuf in batches of whole
// items.  The caller ends with a consumer barrier.
__device__ __forceinline__ void att_combine(const DecodeParams &p, Cta &S, int pos, uint32_t ep_att, int layer) {
    const int H = p.n_heads, D = p.d_model;
    const int n_items = (pos / kPageTokens + 1) * H;
    constexpr int W = 2 + kHeadDim;
    const int per_batch = (2 * kPageTokens * kHeadDim * 2 / 4) / W;   // items per kvbuf load
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
        const int n_items = (pos / kPageTokens + 1) * H;

        for (int l = 0; l < L; l++) {
            const uint32_t ep = ep0 + (uint32_t)(l * kPhasesPerLayer);
            const float *ln = p.ln + (size_t)l * 4 * D;
            if (c < n_items) kv_prefetch(p, S, l, c, pos);
            // ---------------- QKV: x += fc2(prev layer); LN1; q, k, v rows
            if (l > 0) ll_gather(p, S, p.ll_f2, actw, D, ep - kPhasesPerLayer + PH_FC2, 0x10u + l);
            cp_async_wait_all();
            cbar();
            if (l == 1) stamp(p, S, t, 70);
            if (*(volatile int *)S.flag) return;
            float *xnext = xcur == S.xs ? S.xs + kDmax : S.xs;
            int s = resid_ln_limbs<D>(S, xcur, xnext, l > 0 ? actw : nullptr, lng, lnb, p.eps);
            if (l > 0) xcur = xnext;
            cbar();
            if (l == 1) stamp(p, S, t, 71);
            if (l > 0) trace_x(p, S, t, 2 * (l - 1) + 1, xcur);
            ln_prefetch(S, 1, ln + 2 * D, ln + 3 * D, D);
            gemv_phase<true>(p, S, ctr, q_rows, D, s, 0x20u + l, [&](int r, float y0, float y1) {
                const int n = q_row0 + r;
                if (n < D) { y0 = __fmul_rn(y0, 0.125f); y1 = __fmul_rn(y1, 0.125f); }
                ll_store(p.ll_qkv + n / 2, bf16bits(y0) | (bf16bits(y1) << 16), ep + PH_QKV);
            });
            stamp(p, S, t, 1 + 5 * l + PH_QKV);
            if (l == 1) stamp(p, S, t, 72);
            // ---------------- ATT: this CTA's (page, head) items
            for (int it = c, k = 0; it < n_items; it += G, k++)
                att_item(p, S, l, it, pos, k == 0, ep + PH_QKV, ep + PH_ATT);
            stamp(p, S, t, 1 + 5 * l + PH_ATT);
            // ---------------- O: merge partials -> ctx; O rows
            if (o_rows > 0) {
                att_combine(p, S, pos, ep + PH_ATT, l);
                cbar();
                if (l == 1) stamp(p, S, t, 82);
                s = limbs_of<D>(S, [&](int i) { return __uint_as_float((uint32_t)S.act[i] << 16); });
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
            cp_async_wait_all();
            cbar();
            if (l == 1) stamp(p, S, t, 64);
            if (*(volatile int *)S.flag) return;
            xnext = xcur == S.xs ? S.xs + kDmax : S.xs;
            s = resid_ln_limbs<D>(S, xcur, xnext, actw, ln2g, ln2b, p.eps);
            xcur = xnext;
            cbar();
            if (l == 1) stamp(p, S, t, 65);
            trace_x(p, S, t, 2 * l, xcur);
            if (l + 1 < L) ln_prefetch(S, 0, ln + 4 * D, ln + 5 * D, D);
            else ln_prefetch(S, 0, p.lnf, p.lnf + D, D);
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
                s = limbs_of<F>(S, [&](int i) { return __uint_as_float((uint32_t)S.act[i] << 16); });
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
    extern __shared__ __align__(1024) uint8_t smem[];
    Cta S = make_cta(smem);
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
    extern __shared__ __align__(1024) uint8_t smem[];
    Cta S = make_cta(smem);
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
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SmemMap::total);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
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
