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
    static constexpr int act = limbs + 3 * kKmax;                        // kKmax f32
    static constexpr int xs = act + kKmax * 4;                           // kDmax f32
    static constexpr int kvbuf = xs + kDmax * 4;                         // 2 x 64 x 64 bf16
    static constexpr int part = kvbuf + 2 * kPageTokens * kHeadDim * 2;  // partial MMA sums
    static constexpr int part_bytes = kConsumerWarps * kMaxTilesPerChunk * 3 * 8 * 4;
    static constexpr int outv = part + part_bytes;                       // 1024 f32
    static constexpr int misc = outv + 1024 * 4;                         // scratch floats
    static constexpr int misc_floats = 64 + 64 + 64 + 4 * 64 + 96 + 32;
    static constexpr int bars = (misc + misc_floats * 4 + 15) & ~15;
    static constexpr int total = bars + 2 * kStages * 8 + 16;
};
static_assert(SmemMap::total <= 227 * 1024, "shared memory budget");

struct Cta {
    uint8_t *ring;
    int8_t *limbs;
    float *act, *xs;
    uint16_t *kvbuf;            // [2][64][64] bf16: K rows then V rows
    int *part;
    float *outv;
    float *red;                 // 64 reduction slots
    float *qf;                  // 64 query floats
    float *sc;                  // 64 scores / probabilities
    float *accp;                // 4 x 64 partial contexts
    uint32_t *qkvw;             // 96 words: q, k, v of one head
    int *flag;                  // [0] abort flag
    uint64_t *full, *empty;
    int tid, warp, lane;
};

__device__ __forceinline__ Cta make_cta(uint8_t *smem) {
    Cta S;
    S.ring = smem + SmemMap::ring;
    S.limbs = reinterpret_cast<int8_t *>(smem + SmemMap::limbs);
    S.act = reinterpret_cast<float *>(smem + SmemMap::act);
    S.xs = reinterpret_cast<float *>(smem + SmemMap::xs);
    S.kvbuf = reinterpret_cast<uint16_t *>(smem + SmemMap::kvbuf);
    S.part = reinterpret_cast<int *>(smem + SmemMap::part);
    S.outv = reinterpret_cast<float *>(smem + SmemMap::outv);
    float *m = reinterpret_cast<float *>(smem + SmemMap::misc);
    S.red = m;
    S.qf = m + 64;
    S.sc = m + 128;
    S.accp = m + 192;
    S.qkvw = reinterpret_cast<uint32_t *>(m + 192 + 256);
    S.flag = reinterpret_cast<int *>(m + 192 + 256 + 96);
    S.full = reinterpret_cast<uint64_t *>(smem + SmemMap::bars);
    S.empty = S.full + kStages;
    S.tid = threadIdx.x;
    S.warp = threadIdx.x >> 5;
    S.lane = threadIdx.x & 31;
    return S;
}

__device__ __forceinline__ void cbar() { named_bar(1, kConsumerThreads); }

// ------------------------------------------------------------------------- error handling
__device__ __forceinline__ uint32_t read_error(const DecodeParams &p) {
    return *reinterpret_cast<volatile uint32_t *>(&p.state->error);
}
__device__ void set_error(const DecodeParams &p, uint32_t code, uint32_t where) {
    if (atomicCAS(&p.state->error, 0u, code) == 0u) {
        p.state->error_cta = blockIdx.x;
        p.state->error_where = where;
    }
}
// Returns true when a waiter must give up: another CTA already failed, or the deadline
// (started at the first call) passed -- then this CTA records the timeout.
__device__ __noinline__ bool wait_expired(const DecodeParams &p, uint64_t &t0, uint32_t code,
                                          uint32_t where) {
    if (read_error(p) != 0) return true;
    uint64_t now = globaltimer_ns();
    if (t0 == 0) { t0 = now; return false; }
    if (now - t0 > p.timeout_ns) { set_error(p, code, where); return true; }
    return false;
}

__device__ __forceinline__ void wait_full(const DecodeParams &p, Cta &S, int slot, uint32_t parity,
                                          uint32_t where) {
    if (mbar_try_wait(&S.full[slot], parity)) return;
    uint64_t t0 = 0;
    while (!mbar_try_wait(&S.full[slot], parity))
        if (wait_expired(p, t0, ERR_TIMEOUT_FULL, where)) return;
}

// Poll n flag-tagged words [src, src+n) until they all carry `epoch`; store their data to
// dst.  Each consumer thread keeps up to 8 words in flight at once.
__device__ void ll_gather(const DecodeParams &p, const Cta &S, const uint64_t *src,
                          uint32_t *dst, int n, uint32_t epoch, uint32_t where) {
    constexpr int B = 8;
    for (int base = 0; base < n; base += B * kConsumerThreads) {
        uint64_t v[B];
#pragma unroll
        for (int j = 0; j < B; j++) {
            int i = base + S.tid + j * kConsumerThreads;
            v[j] = i < n ? ll_load(src + i) : (static_cast<uint64_t>(epoch) << 32);
        }
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (true) {
            bool all = true;
#pragma unroll
            for (int j = 0; j < B; j++) all &= static_cast<uint32_t>(v[j] >> 32) == epoch;
            if (all) break;
#pragma unroll
            for (int j = 0; j < B; j++) {
                int i = base + S.tid + j * kConsumerThreads;
                if (i < n && static_cast<uint32_t>(v[j] >> 32) != epoch) v[j] = ll_load(src + i);
            }
            if ((++it & 31) == 0 && wait_expired(p, t0, ERR_TIMEOUT_FLAG, where)) break;
        }
#pragma unroll
        for (int j = 0; j < B; j++) {
            int i = base + S.tid + j * kConsumerThreads;
            if (i < n) dst[i] = static_cast<uint32_t>(v[j]);
        }
    }
}

// uniform "should this CTA stop" decision among the consumer threads
__device__ __forceinline__ bool abort_check(const DecodeParams &p, Cta &S) {
    if (S.tid == 0) S.flag[0] = read_error(p) != 0;
    cbar();
    bool stop = S.flag[0] != 0;
    cbar();
    return stop;
}

// ---------------------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// block-wide sum over the consumer threads; every thread gets the same value (fixed order)
__device__ float block_sum(Cta &S, float v) {
    v = warp_sum(v);
    if (S.lane == 0) S.red[S.warp] = v;
    cbar();
    float r = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) r += S.red[w];
    cbar();
    return r;
}
__device__ float block_max(Cta &S, float v) {
    v = warp_max(v);
    if (S.lane == 0) S.red[S.warp] = v;
    cbar();
    float r = S.red[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; w++) r = fmaxf(r, S.red[w]);
    cbar();
    return r;
}

// LayerNorm of S.xs[0..D) (rust/npu-asr-host/src/lib.rs:79-110: population variance,
// y = (x - mean) * inv * g + b, each op rounded) -> S.act, rounded to bf16.
__device__ void layer_norm_bf16(Cta &S, int D, const float *g, const float *b, float eps) {
    float s = 0.0f;
    for (int i = S.tid; i < D; i += kConsumerThreads) s += S.xs[i];
    float mean = __fdiv_rn(block_sum(S, s), (float)D);
    float v = 0.0f;
    for (int i = S.tid; i < D; i += kConsumerThreads) {
        float c = __fsub_rn(S.xs[i], mean);
        v = __fadd_rn(v, __fmul_rn(c, c));
    }
    float var = __fdiv_rn(block_sum(S, v), (float)D);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int i = S.tid; i < D; i += kConsumerThreads) {
        float t = __fmul_rn(__fsub_rn(S.xs[i], mean), inv);
        t = __fadd_rn(__fmul_rn(t, g[i]), b[i]);
        S.act[i] = bf16r(t);
    }
    cbar();
}

// S.act[0..K) -> three swizzled int8 limb rows of the 22-bit fixed-point vector.  Returns
// the power-of-two exponent s (X = rint(x * 2^s)).  Row j, 32-byte block kb is stored at
// block kb ^ j so that the MMA fragment loads are bank-conflict free.
__device__ int make_limbs(Cta &S, int K) {
    float m = 0.0f;
    for (int i = S.tid; i < K; i += kConsumerThreads) m = fmaxf(m, fabsf(S.act[i]));
    m = block_max(S, m);
    int E = 0;
    if (m >= 0x1p-100f) E = (int)((__float_as_uint(m) >> 23) & 0xff) - 126;   // m < 2^E
    int s = 22 - E;
    float sc = exp2i(s);
    for (int i4 = S.tid; i4 < K / 4; i4 += kConsumerThreads) {
        float4 v = reinterpret_cast<const float4 *>(S.act)[i4];
        float vv[4] = {v.x, v.y, v.z, v.w};
        uint32_t wa = 0, wb = 0, wc = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            int X = __float2int_rn(vv[e] * sc);
            int c = ((X + 128) & 255) - 128;
            int X1 = (X - c) >> 8;
            int b = ((X1 + 128) & 255) - 128;
            int a = (X1 - b) >> 8;
            wa |= (uint32_t)(a & 255) << (8 * e);
            wb |= (uint32_t)(b & 255) << (8 * e);
            wc |= (uint32_t)(c & 255) << (8 * e);
        }
        int o = i4 * 4, kb = o >> 5, w = o & 31;
        *reinterpret_cast<uint32_t *>(S.limbs + 0 * kKmax + ((kb ^ 0) << 5) + w) = wa;
        *reinterpret_cast<uint32_t *>(S.limbs + 1 * kKmax + ((kb ^ 1) << 5) + w) = wb;
        *reinterpret_cast<uint32_t *>(S.limbs + 2 * kKmax + ((kb ^ 2) << 5) + w) = wc;
    }
    cbar();
    return s;
}

// One weight chunk: rows (multiple of 8) x K int8 (row r swizzled by r & 3) followed by
// rows x (f32 scale, f32 bias).  Writes y[r] = float(exact dot) * 2^-s * scale + bias to
// out[r].  Ends with a consumer barrier.
__device__ void gemv_chunk(Cta &S, const uint8_t *stage, int rows, int K, int s, float *out) {
    const int g = S.lane >> 2, tig = S.lane & 3;
    const int ntiles = rows >> 3;
    const int KS = K >> 5;
    const int kb0 = S.warp * KS / kConsumerWarps, kb1 = (S.warp + 1) * KS / kConsumerWarps;
    int acc[kMaxTilesPerChunk][4];
#pragma unroll
    for (int t = 0; t < kMaxTilesPerChunk; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const int8_t *arow = S.limbs + (g < 3 ? g : 0) * kKmax;
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
    if (g < 3) {
#pragma unroll
        for (int t = 0; t < kMaxTilesPerChunk; t++) {
            if (t < ntiles) {
                int *pp = S.part + ((S.warp * kMaxTilesPerChunk + t) * 3 + g) * 8 + 2 * tig;
                pp[0] = acc[t][0];
                pp[1] = acc[t][1];
            }
        }
    }
    cbar();
    if (S.tid < rows) {
        const int r = S.tid, t = r >> 3, col = r & 7;
        long long A = 0, B = 0, C = 0;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) {
            const int *pp = S.part + ((w * kMaxTilesPerChunk + t) * 3) * 8 + col;
            A += pp[0];
            B += pp[8];
            C += pp[16];
        }
        long long X = A * 65536 + B * 256 + C;
        float y = __fmul_rn(__ll2float_rn(X), exp2i(-s));
        const float *meta = reinterpret_cast<const float *>(stage + (size_t)rows * K);
        y = __fadd_rn(__fmul_rn(y, meta[2 * r]), meta[2 * r + 1]);
        out[r] = y;
    }
}

// Consume one phase's chunks from the ring: rows of reduction length K, outputs to out[].
__device__ void gemv_phase(const DecodeParams &p, Cta &S, uint32_t &ctr, int rows, int K, int s,
                           float *out, uint32_t where) {
    const int rpc = rows_per_chunk(K);
    for (int r0 = 0; r0 < rows; r0 += rpc) {
        const int rr = min(rpc, rows - r0);
        const int slot = ctr % kStages;
        const uint32_t parity = (ctr / kStages) & 1u;
        wait_full(p, S, slot, parity, where);
        gemv_chunk(S, S.ring + slot * kStageBytes, rr, K, s, out + r0);
        __syncwarp();
        if (S.lane == 0) mbar_arrive(&S.empty[slot]);
        cbar();
        ctr++;
    }
}

// LM head phase: like gemv_phase, but each row's logit feeds a running argmax whose ties go
// to the LAST index (Iterator::max_by, opt125m_decode.rs:303).
__device__ void lm_phase(const DecodeParams &p, Cta &S, uint32_t &ctr, int row0, int rows, int K,
                         int s, float *logits_row, float &best, int &best_i) {
    const int rpc = rows_per_chunk(K);
    for (int r0 = 0; r0 < rows; r0 += rpc) {
        const int rr = min(rpc, rows - r0);
        const int slot = ctr % kStages;
        const uint32_t parity = (ctr / kStages) & 1u;
        wait_full(p, S, slot, parity, 0x100u);
        gemv_chunk(S, S.ring + slot * kStageBytes, rr, K, s, S.outv);
        __syncwarp();
        if (S.lane == 0) mbar_arrive(&S.empty[slot]);
        if (S.tid < rr) {
            float v = S.outv[S.tid];
            int idx = row0 + r0 + S.tid;
            if (logits_row) logits_row[idx] = v;
            if (v > best || (v == best && idx > best_i)) { best = v; best_i = idx; }
        }
        cbar();
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
__device__ void kv_prefetch(const DecodeParams &p, Cta &S, int layer, int item, int pos) {
    const int H = p.n_heads;
    const int pg = item / H, h = item % H;
    const int j0 = pg * kPageTokens;
    const int nrows = min(pos, j0 + kPageTokens) - j0;   // cached rows (current pos excluded)
    if (nrows <= 0) return;
    const int phys = p.page_table[pg];
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
__device__ void att_item(const DecodeParams &p, Cta &S, int layer, int item, int pos,
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
            if ((++it & 31) == 0 && wait_expired(p, t0, ERR_TIMEOUT_FLAG, 0x200u + layer)) break;
        }
        S.qkvw[S.tid] = static_cast<uint32_t>(v);
    }
    cp_async_wait_all();
    cbar();
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
        const int phys = p.page_table[pg];
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
    float p0 = S.lane < nk ? expf(S.sc[S.lane] - m) : 0.0f;
    float p1 = S.lane + 32 < nk ? expf(S.sc[S.lane + 32] - m) : 0.0f;
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

// Combine the page partials of every head (flash-decode merge) into ctx = bf16(acc / l) in
// S.act[0..D).  Partials are staged through kvbuf in batches of whole items.
__device__ void att_combine(const DecodeParams &p, Cta &S, int pos, uint32_t ep_att, int layer) {
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
                    const float c0 = expf(M[k] - mn), c1 = expf(mp - mn);
                    L[k] = L[k] * c0 + lp * c1;
                    A[k] = A[k] * c0 + ap * c1;
                    M[k] = mn;
                }
            }
        }
        cbar();
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = S.tid + k * kConsumerThreads;
        if (i < D) S.act[i] = bf16r(A[k] / L[k]);
    }
    cbar();
}

// optional debugging record of the residual stream (CTA 0 only)
__device__ __forceinline__ void trace_x(const DecodeParams &p, Cta &S, int t, int slot, const float *v) {
    if (p.trace == nullptr || blockIdx.x != 0) return;
    float *dst = p.trace + ((size_t)t * (2 * p.n_layers + 1) + slot) * p.d_model;
    for (int i = S.tid; i < p.d_model; i += kConsumerThreads) dst[i] = v[i];
}

// ---------------------------------------------------------------------------------- roles
__device__ void producer(const DecodeParams &p, Cta &S) {
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
                    if (wait_expired(p, t0, ERR_TIMEOUT_EMPTY, 0x400u)) { failed = true; break; }
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

__device__ void consumer(const DecodeParams &p, Cta &S) {
    const int c = blockIdx.x, G = p.grid;
    const int L = p.n_layers, D = p.d_model, F = p.ffn, V = p.vocab, H = p.n_heads;
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

    for (int t = 0; t < p.n_steps; t++) {
        const int pos = p.start_pos + t;
        const uint32_t ep0 = base + (uint32_t)(t * PHT) + 1u;
        const int64_t id = (t == 0 || pos < p.n_prompt) ? p.tokens[pos] : next_id;
        if (id < 0 || id >= V || pos + 2 > p.max_pos + 1) {
            if (S.tid == 0) set_error(p, id < 0 || id >= V ? ERR_BAD_TOKEN : ERR_BAD_POS, pos);
        }
        if (abort_check(p, S)) return;
        for (int i = S.tid; i < D; i += kConsumerThreads)
            S.xs[i] = __fadd_rn(p.emb_tok[(size_t)id * D + i], p.emb_pos[(size_t)(pos + 2) * D + i]);
        cbar();
        const int n_items = (pos / kPageTokens + 1) * H;

        for (int l = 0; l < L; l++) {
            const uint32_t ep = ep0 + (uint32_t)(l * kPhasesPerLayer);
            const float *ln = p.ln + (size_t)l * 4 * D;
            // attention page prefetch for this layer (first item of this CTA)
            if (c < n_items) kv_prefetch(p, S, l, c, pos);
            // ---------------- QKV: x += fc2(prev layer); LN1; q,k,v rows
            if (l > 0) {
                ll_gather(p, S, p.ll_f2, actw, D, ep - kPhasesPerLayer + PH_FC2, 0x10u + l);
                cbar();
                for (int i = S.tid; i < D; i += kConsumerThreads) S.xs[i] = __fadd_rn(S.xs[i], S.act[i]);
                cbar();
                trace_x(p, S, t, 2 * (l - 1) + 1, S.xs);
            }
            if (abort_check(p, S)) return;
            layer_norm_bf16(S, D, ln, ln + D, p.eps);
            int s = make_limbs(S, D);
            gemv_phase(p, S, ctr, q_rows, D, s, S.outv, 0x20u + l);
            for (int w = S.tid; w < q_rows / 2; w += kConsumerThreads) {
                const int n = q_row0 + 2 * w;
                float y0 = S.outv[2 * w], y1 = S.outv[2 * w + 1];
                if (n < D) { y0 = __fmul_rn(y0, 0.125f); y1 = __fmul_rn(y1, 0.125f); }
                ll_store(p.ll_qkv + n / 2, bf16bits(y0) | (bf16bits(y1) << 16), ep + PH_QKV);
            }
            // ---------------- ATT: this CTA's (page, head) items
            for (int it = c, k = 0; it < n_items; it += G, k++)
                att_item(p, S, l, it, pos, k == 0, ep + PH_QKV, ep + PH_ATT);
            // ---------------- O: merge partials -> ctx; O rows
            if (o_rows > 0) {
                att_combine(p, S, pos, ep + PH_ATT, l);
                s = make_limbs(S, D);
                gemv_phase(p, S, ctr, o_rows, D, s, S.outv, 0x30u + l);
                for (int r = S.tid; r < o_rows; r += kConsumerThreads)
                    ll_store(p.ll_o + o_row0 + r, __float_as_uint(S.outv[r]), ep + PH_O);
            }
            // ---------------- FC1: x += o; LN2; relu(fc1) -> bf16
            ll_gather(p, S, p.ll_o, actw, D, ep + PH_O, 0x40u + l);
            cbar();
            for (int i = S.tid; i < D; i += kConsumerThreads) S.xs[i] = __fadd_rn(S.xs[i], S.act[i]);
            cbar();
            trace_x(p, S, t, 2 * l, S.xs);
            if (abort_check(p, S)) return;
            layer_norm_bf16(S, D, ln + 2 * D, ln + 3 * D, p.eps);
            s = make_limbs(S, D);
            gemv_phase(p, S, ctr, f1_rows, D, s, S.outv, 0x50u + l);
            for (int w = S.tid; w < f1_rows / 2; w += kConsumerThreads) {
                const float y0 = fmaxf(S.outv[2 * w], 0.0f), y1 = fmaxf(S.outv[2 * w + 1], 0.0f);
                ll_store(p.ll_h + (f1_row0 / 2) + w, bf16bits(y0) | (bf16bits(y1) << 16), ep + PH_FC1);
            }
            // ---------------- FC2
            if (f2_rows > 0) {
                ll_gather(p, S, p.ll_h, actw + F / 2, F / 2, ep + PH_FC1, 0x60u + l);
                cbar();
                // (two-pass unpack: read all pairs first, then write, so in-place is safe)
                {
                    float tmp[12][2];
                    int cnt = 0;
                    for (int w = S.tid; w < F / 2 && cnt < 12; w += kConsumerThreads, cnt++) {
                        const uint32_t v = actw[F / 2 + w];
                        tmp[cnt][0] = bf16lo(v);
                        tmp[cnt][1] = bf16hi(v);
                    }
                    cbar();
                    cnt = 0;
                    for (int w = S.tid; w < F / 2 && cnt < 12; w += kConsumerThreads, cnt++) {
                        S.act[2 * w] = tmp[cnt][0];
                        S.act[2 * w + 1] = tmp[cnt][1];
                    }
                    cbar();
                }
                s = make_limbs(S, F);
                gemv_phase(p, S, ctr, f2_rows, F, s, S.outv, 0x70u + l);
                for (int r = S.tid; r < f2_rows; r += kConsumerThreads)
                    ll_store(p.ll_f2 + f2_row0 + r, __float_as_uint(S.outv[r]), ep + PH_FC2);
            }
        }
        // ---------------- final residual, LN, LM head + greedy argmax
        {
            const uint32_t ep_last = ep0 + (uint32_t)((L - 1) * kPhasesPerLayer) + PH_FC2;
            ll_gather(p, S, p.ll_f2, actw, D, ep_last, 0x80u);
            cbar();
            for (int i = S.tid; i < D; i += kConsumerThreads) S.xs[i] = __fadd_rn(S.xs[i], S.act[i]);
            cbar();
            trace_x(p, S, t, 2 * L - 1, S.xs);
        }
        if (pos >= p.n_prompt - 1) {
            const uint32_t ep_lm = ep0 + (uint32_t)(L * kPhasesPerLayer);
            if (abort_check(p, S)) return;
            layer_norm_bf16(S, D, p.lnf, p.lnf + D, p.eps);
            trace_x(p, S, t, 2 * L, S.act);
            const int s = make_limbs(S, D);
            float best = -INFINITY;
            int best_i = -1;
            const int lm_step = pos - max(p.start_pos, p.n_prompt - 1);
            float *lrow = p.logits ? p.logits + (size_t)lm_step * V : nullptr;
            lm_phase(p, S, ctr, lm_row0, lm_rows, D, s, lrow, best, best_i);
            // CTA-level argmax (ties -> larger index)
            {
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
                cbar();
            }
            // global argmax over all CTAs (every CTA computes it; same order -> same id)
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
        } else {
            next_id = p.tokens[pos + 1];
        }
    }
    if (c == 0 && S.tid == 0) p.state->epoch_base = base + (uint32_t)(p.n_steps * PHT);
}

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
    else consumer(p, S);
}

// ------------------------------------------------------------------ standalone GEMV (op API)
// y[N] = exact-int8-GEMV(x[K]) * scale + bias over a packed [N/rows_per_chunk] chunk list:
// one CTA per chunk, same device code as the decode kernel (for parity tests and the op-level
// C ABI).
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
    for (int i = S.tid; i < K; i += kConsumerThreads) S.act[i] = x[i];
    cbar();
    const int s = make_limbs(S, K);
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(&S.full[0], 0u))
        if (globaltimer_ns() - start > 1000000000ull) return;   // bounded (1 s)
    gemv_chunk(S, S.ring, rows, K, s, S.outv);
    cbar();
    for (int r = S.tid; r < rows; r += kConsumerThreads) y[row0 + r] = S.outv[r];
}

int decode_smem_bytes() { return SmemMap::total; }

cudaError_t launch_opt_decode(const DecodeParams &p, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(opt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SmemMap::total);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    DecodeParams pp = p;
    void *args[] = {&pp};
    return cudaLaunchCooperativeKernel((const void *)opt_decode_kernel, dim3(p.grid), dim3(kThreads),
                                       args, SmemMap::total, st);
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
    cudaError_t e = cudaFuncSetAttribute(opt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SmemMap::total);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, opt_decode_kernel, kThreads, SmemMap::total);
    if (e != cudaSuccess) return e;
    *out = sms * per;
    return cudaSuccess;
}

}  // namespace xdna
