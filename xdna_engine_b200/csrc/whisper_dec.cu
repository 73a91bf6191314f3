// whisper_dec.cu -- the Whisper-small greedy decoder on B200, B streams in lockstep.
//
// Replaces the reference's decoder (rust/npu-engine/src/asr/whisper_decoder.rs):
//   precompute_cross 388-399  -> one bf16 tcgen05 GEMM for all layers' cross K and V
//                                ([B*T_enc, 768] x [768, 12 * 2 * 768])
//   HostDecoder::step 401-560 / the fused per-token ELF (route_b_kernels/decode_fused/
//   gen_decode.py runlist 391-425) -> per token: embed, then per layer LN -> bfp16 GEMV (q|k|v)
//   -> self attention over the bf16 cache -> GEMV out (+x) -> LN -> GEMV cross q -> split cross
//   attention + ordered merge -> GEMV cross out (+x) -> LN -> GEMV fc1 (+GELU) -> GEMV fc2 (+x);
//   ln_post -> GEMV over the tied proj_out (the device lm-head of gen_projout.py) -> argmax
//   (whisper.rs:749-757: first maximum).  The ~150 launches of a token are one CUDA graph.
// Weights are the reference's bfp16 format (route_b_kernels/ffn_bfp16/golden_ffn_gemm.py:34-49:
// blocks of 8 along K, shared exponent e = floor(log2 max|x|), mantissa round-half-even of
// x / 2^(e-6)), stored as int8 mantissas + one byte per block (1.125 bytes per weight) in the
// order the tensor-core GEMV consumes them, and dequantised in registers (exactly: every bfp16
// value is a bf16 value).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"
#include "ptx.cuh"

namespace xdna {
void set_last_error_message(const std::string &m);
cudaError_t gemm_bf16(const uint16_t *A, int lda, const uint16_t *B, int ldb, int M, int N, int K,
                      const float *bias, const uint16_t *residual, int ldr, int act, uint16_t *C, int ldc,
                      cudaStream_t st, int res_mod = 0, float *C_f32 = nullptr);
unsigned gemm_error_and_clear();

namespace wdec {
namespace cg = cooperative_groups;

constexpr int D = 768, H = 12, HD = 64, F = 3072;
constexpr int MAXB = 32;              // streams per decoder
constexpr int GEMV_WARPS = 8;

enum { OUT_F32 = 0, OUT_RESID = 1, OUT_GELU_BF16 = 2 };

__device__ __forceinline__ float gelu_erf_as(float v) {   // npu-asr-host/src/lib.rs:464-495
    const float x = v * 0.70710678118654752440f;
    const float ax = fabsf(x);
    const float t = __frcp_rn(fmaf(0.3275911f, ax, 1.0f));
    float p = fmaf(1.061405429f, t, -1.453152027f);
    p = fmaf(p, t, 1.421413741f);
    p = fmaf(p, t, -0.284496736f);
    p = fmaf(p, t, 0.254829592f);
    const float y = fmaf(-p * t, expf(-ax * ax), 1.0f);
    return 0.5f * v * (1.0f + copysignf(y, x));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// two int8 mantissas of one block -> bf16x2 (exact): code byte e: bits 0-5 = exponent + 32,
// bit 7 = the block's mantissas are stored negated
__device__ __forceinline__ uint32_t deq2(uint32_t m2, uint32_t ecode) {
    const float sc = __int_as_float((int)(((ecode & 63u) - 32u + 127u - 6u) << 23)) * ((ecode & 128u) ? -1.0f : 1.0f);
    const float lo = (float)(int8_t)(m2 & 255u) * sc, hi = (float)(int8_t)(m2 >> 8) * sc;
    return bf16bits(lo) | (bf16bits(hi) << 16);
}

struct GemvArgs {
    const uint8_t *mant;        // [row groups][K/16 k-steps][32 lanes][8]
    const uint8_t *ecode;       // [row groups][K/16][8 quads][4]
    const float *bias;          // [N] or null
    const uint16_t *x;          // bf16 [B][K]
    int B, N, K;
    int R, Wk, nsplit;          // row groups per CTA, warps per row group (along K), K ranges = cluster size
    int red_off;                // float offset of the partial-sum area in shared memory (0: aliases X)
    int mode;
    float *out;                 // OUT_F32: [B][ldo]; OUT_RESID: x f32 [B][ldo] (+=)
    uint16_t *out_bf16;         // OUT_GELU_BF16: [B][ldo]
    int ldo;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// Y[b][n] = X[b] . W[n] + bias for b < B on the bf16 tensor cores (bfp16 values are exact in
// bf16).  Grid (row-group blocks, K ranges); the K ranges of one row-group block form a
// thread-block cluster.  CTA = GEMV_WARPS warps = R row groups x Wk warps along the CTA's K
// range; warp = 16 output rows whose weight fragments come straight from HBM in mma order
// (8 bytes of mantissas + a quad-shared 4-byte exponent word per lane and k-step), 8 k-steps at
// a time with the next 8 in flight.  The first 8 are requested before the wait for the previous
// grid (programmatic dependent launch); the X range is staged with cp.async in one round trip
// and read with ldmatrix.  Partial sums meet in shared memory, are added over the Wk warps and
// then over the cluster's CTAs through DSMEM in rank order (deterministic).
template <int NT>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) bfp_gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint16_t xs[];
    float *red = reinterpret_cast<float *>(xs) + a.red_off;
    const uint32_t xs_a = smem_u32(xs);
    griddep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int n_rg = (a.N + 15) / 16, nks = a.K / 16, split = blockIdx.y;
    const int ks0 = split * nks / a.nsplit, nkc = (split + 1) * nks / a.nsplit - ks0, xld = nkc * 16 + 8;
    const int r = warp / a.Wk, wk = warp % a.Wk;
    const int w0 = wk * nkc / a.Wk, nst = (wk + 1) * nkc / a.Wk - w0, ngrp = (nst + 7) / 8;
    const int rstride = gridDim.x * a.R;
    uint2 mv[8], mn[8];
    uint32_t ev[8], en[8];
    auto fetch = [&](uint2 (&dm)[8], uint32_t (&de)[8], int rg, int s0) {
        const bool live = rg < n_rg;
        const size_t base = (size_t)(live ? rg : 0) * nks + ks0 + w0 + s0;
        const uint2 *mp = reinterpret_cast<const uint2 *>(a.mant) + base * 32 + lane;
        const uint32_t *ep = reinterpret_cast<const uint32_t *>(a.ecode) + base * 8 + g;
#pragma unroll
        for (int s = 0; s < 8; s++) {
            const bool ok = live && s0 + s < nst;
            dm[s] = ok ? __ldcs(mp + s * 32) : make_uint2(0, 0);
            de[s] = ok ? __ldcs(ep + s * 8) : 0u;
        }
    };
    fetch(mv, ev, blockIdx.x * a.R + r, 0);
    griddep_wait();
    {
        const int cpr = nkc * 2;                        // 16-byte pieces per row
        for (int b = warp; b < NT * 8; b += GEMV_WARPS)
            for (int c = lane; c < cpr; c += 32) {
                uint16_t *d = &xs[b * xld + c * 8];
                if (b < a.B) cp_async16(d, a.x + (size_t)b * a.K + ks0 * 16 + c * 8);
                else *reinterpret_cast<uint4 *>(d) = make_uint4(0, 0, 0, 0);
            }
        cp_async_commit();
        cp_async_wait_all();
    }
    __syncthreads();
    cg::cluster_group cl = cg::this_cluster();
    for (int rg0 = blockIdx.x * a.R; rg0 < n_rg; rg0 += rstride) {
        const int rg = rg0 + r;
        if (rg0 != (int)blockIdx.x * a.R) fetch(mv, ev, rg, 0);
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (int gi = 0; gi < ngrp; gi++) {
            if (gi + 1 < ngrp) fetch(mn, en, rg, (gi + 1) * 8);
#pragma unroll
            for (int s = 0; s < 8; s++) {
                if (gi * 8 + s >= nst) break;
                // a0 (row g, k 2t..) a1 (row g+8, k 2t..) block 0; a2, a3 (k 2t+8..) block 1
                const uint32_t e = ev[s];
                const uint32_t a0 = deq2(mv[s].x & 0xffffu, e & 255u), a1 = deq2(mv[s].x >> 16, (e >> 8) & 255u);
                const uint32_t a2 = deq2(mv[s].y & 0xffffu, (e >> 16) & 255u), a3 = deq2(mv[s].y >> 16, e >> 24);
                const int kk = (w0 + gi * 8 + s) * 16;
                if constexpr (NT == 1) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(&xs[g * xld + kk + 2 * t]);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t *>(&xs[g * xld + kk + 8 + 2 * t]);
                    mma16816(acc[0], a0, a1, a2, a3, b0, b1);
                } else {
#pragma unroll
                    for (int n = 0; n < NT; n += 2) {
                        uint32_t r0, r1, r2, r3;
                        ldsm_x4(xs_a + 2u * ((n * 8 + ((lane >> 4) << 3) + (lane & 7)) * xld + kk + (((lane >> 3) & 1) << 3)),
                                r0, r1, r2, r3);
                        mma16816(acc[n], a0, a1, a2, a3, r0, r1);
                        mma16816(acc[n + 1], a0, a1, a2, a3, r2, r3);
                    }
                }
            }
#pragma unroll
            for (int s = 0; s < 8; s++) { mv[s] = mn[s]; ev[s] = en[s]; }
        }
        if (a.red_off == 0) __syncthreads();            // the partials overwrite the staged X
        float *rw = red + warp * NT * 128;
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) rw[(n * 4 + e) * 32 + lane] = acc[n][e];
        __syncthreads();
        if (a.Wk > 1)
            for (int i = threadIdx.x; i < a.R * NT * 128; i += blockDim.x) {
                const int rr = i / (NT * 128), e = i - rr * (NT * 128);
                float sum = red[rr * a.Wk * NT * 128 + e];
                for (int k = 1; k < a.Wk; k++) sum += red[(rr * a.Wk + k) * NT * 128 + e];
                red[rr * a.Wk * NT * 128 + e] = sum;
            }
        if (a.nsplit > 1) cl.sync(); else __syncthreads();
        // outputs: item = (row group, n tile, column c, lane) -> rows g and g + 8, stream n*8 + 2t + c;
        // this CTA takes its share of the items and adds the K ranges in rank order
        const int items = a.R * NT * 64, i0 = split * items / a.nsplit, i1 = (split + 1) * items / a.nsplit;
        for (int it = i0 + threadIdx.x; it < i1; it += blockDim.x) {
            const int rr = it / (NT * 64), rem = it - rr * (NT * 64), n = rem >> 6, c = (rem >> 5) & 1, ln = rem & 31;
            const int off = rr * a.Wk * NT * 128 + (n * 4 + c) * 32 + ln;
            float v0 = 0.0f, v1 = 0.0f;
            if (a.nsplit > 1) {
                float p0[8], p1[8];
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (q < a.nsplit) {
                        const float *rp = cl.map_shared_rank(red, q);
                        p0[q] = rp[off];
                        p1[q] = rp[off + 64];
                    }
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (q < a.nsplit) { v0 += p0[q]; v1 += p1[q]; }
            } else {
                v0 = red[off];
                v1 = red[off + 64];
            }
            const int orow = rg0 + rr, b = n * 8 + 2 * (ln & 3) + c, n0 = orow * 16 + (ln >> 2);
            if (orow >= n_rg || b >= a.B) continue;
            const float vv[2] = {v0, v1};
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int row = n0 + 8 * h;
                if (row >= a.N) continue;
                const float y = vv[h] + (a.bias ? a.bias[row] : 0.0f);
                if (a.mode == OUT_F32) a.out[(size_t)b * a.ldo + row] = y;
                else if (a.mode == OUT_RESID) a.out[(size_t)b * a.ldo + row] += y;
                else a.out_bf16[(size_t)b * a.ldo + row] = (uint16_t)bf16bits(gelu_erf_as(y));
            }
        }
        if (a.nsplit > 1) cl.sync(); else __syncthreads();   // partials stay until every CTA has read them
    }
}

// positions: pos[b * pos_stride] (stride 0: one shared position; 1: per stream); a negative
// position marks an empty slot, which gets a zero row
__global__ void embed_kernel(const int64_t *tok, const int *pos, int pos_stride, const float *et, const float *ep,
                             float *x) {
    const int b = blockIdx.x, p = pos[b * pos_stride];
    const int64_t id = tok[b];
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        x[(size_t)b * D + d] = p < 0 ? 0.0f : et[(size_t)id * D + d] + ep[(size_t)p * D + d];
}

// y = bf16(LN(x)) per stream row (ln_row: population variance, eps 1e-5); one warp per row
__global__ void ln_kernel(const float *__restrict__ x, int B, const float *__restrict__ gm,
                          const float *__restrict__ bt, uint16_t *__restrict__ y) {
    griddep_launch();                                 // the next GEMV may start its weight fetch
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    float v[24], gv[24], bv[24];
#pragma unroll
    for (int i = 0; i < 24; i++) {
        v[i] = x[(size_t)b * D + lane + 32 * i];
        gv[i] = gm[lane + 32 * i];
        bv[i] = bt[lane + 32 * i];
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; i++) s += v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mu = s / (float)D;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; i++) { const float c = v[i] - mu; q += c * c; }
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.0f / sqrtf(q / (float)D + 1e-5f);
#pragma unroll
    for (int i = 0; i < 24; i++) {
        y[(size_t)b * D + lane + 32 * i] = (uint16_t)bf16bits((v[i] - mu) * inv * gv[i] + bv[i]);
    }
}

// Self attention of (head h, stream b) over positions 0..pos (attend_one, whisper_decoder.rs:
// 242-278): appends this position's k, v (bf16) to the cache, stages the head's cached K and V
// in shared memory by bulk copies, then scores / softmax / P.V from there.  qkv f32
// [B][3D]; cache [B][H][max_tgt][64] (K) and the same for V; ctx bf16 [B][D].
// set by a kernel whose bounded wait expired; read and cleared by the synchronous entry points
__device__ unsigned int g_wdec_error;
// bounded wait on a bulk-copy mbarrier (1 s): false, with the error word set, when it expires
__device__ __forceinline__ bool wait_copy(uint64_t *bar) {
    if (mbar_try_wait(bar, 0)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, 0))
        if (globaltimer_ns() - t0 > 1000000000ull) {
            atomicCAS(&g_wdec_error, 0u, 1u);
            return false;
        }
    return true;
}
constexpr int SA_MAX = 448;
constexpr int SA_SMEM = 2 * SA_MAX * HD * 2;
__global__ void __launch_bounds__(128) self_attn_kernel(const float *qkv, const int *posp, int pos_stride, int max_tgt,
                                                        uint16_t *kc, uint16_t *vc, uint16_t *ctx) {
    griddep_launch();                                 // the next GEMV may start its weight fetch
    extern __shared__ __align__(16) uint16_t kvs[];        // K rows then V rows
    __shared__ float q[HD], sc[SA_MAX], red[8], part[2][HD];
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, pos = posp[b * pos_stride];
    if (pos < 0) {                                    // an empty slot: no cache row, zero context
        if (tid < HD) ctx[(size_t)b * D + h * HD + tid] = 0;
        return;
    }
    const float *r = qkv + (size_t)b * 3 * D + h * HD;
    const size_t cb = ((size_t)b * H + h) * max_tgt * HD;
    const int S = pos + 1;
    uint16_t *ks = kvs, *vs = kvs + SA_MAX * HD;
    __shared__ __align__(8) uint64_t bar;
    __shared__ int ok_s;
    // cached rows 0 .. pos-1 (contiguous: two bulk copies on one mbarrier), and this position's
    // row from the projection
    if (tid == 0) {
        ok_s = 1;
        if (pos > 0) {
            mbar_init(&bar, 1);
            mbar_fence_init();
            const uint32_t bytes = (uint32_t)pos * HD * 2;
            mbar_arrive_expect_tx(&bar, 2 * bytes);
            bulk_g2s(ks, kc + cb, bytes, &bar);
            bulk_g2s(vs, vc + cb, bytes, &bar);
        }
    }
    __syncthreads();
    if (tid < HD) {
        q[tid] = r[tid];
        const uint16_t kb = (uint16_t)bf16bits(r[D + tid]), vb = (uint16_t)bf16bits(r[2 * D + tid]);
        kc[cb + (size_t)pos * HD + tid] = kb;
        vc[cb + (size_t)pos * HD + tid] = vb;
        ks[pos * HD + tid] = kb;
        vs[pos * HD + tid] = vb;
    }
    if (pos > 0 && !wait_copy(&bar)) ok_s = 0;
    __syncthreads();
    if (!ok_s) return;
    float mx = -INFINITY;
    for (int j = tid; j < S; j += 128) {
        const uint4 *kr = reinterpret_cast<const uint4 *>(ks + j * HD);
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const uint4 w = kr[(c + j) & 7];               // rotate: lanes start on different banks
            const int d0 = 8 * ((c + j) & 7);
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; e++) dot += q[d0 + 2 * e] * bf16lo(u[e]) + q[d0 + 2 * e + 1] * bf16hi(u[e]);
        }
        sc[j] = dot * 0.125f;
        mx = fmaxf(mx, sc[j]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float sum = 0.0f;
    for (int j = tid; j < S; j += 128) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0) red[4 + (tid >> 5)] = sum;
    __syncthreads();
    const float inv = 1.0f / (red[4] + red[5] + red[6] + red[7]);
    const int d = tid & 63, half = tid >> 6;
    float acc = 0.0f;
    for (int j = half; j < S; j += 2) acc += sc[j] * inv * bf16lo(vs[j * HD + d]);
    part[half][d] = acc;
    __syncthreads();
    if (tid < HD) ctx[(size_t)b * D + h * HD + tid] = (uint16_t)bf16bits(part[0][tid] + part[1][tid]);
}

// Cross attention, split: block (h, b, s) takes encoder positions [128 s, 128 s + 128) and
// writes (max, sum, acc[64]); cross_merge folds the splits in order.  kv rows: [B][T_enc][ldkv]
// with this layer's K at column koff + h*64 and V at koff + D + h*64.  The chunk's K and V
// rows are staged in shared memory by bulk copies first.
constexpr int XCH = 128;
// The cross K/V of one layer, head-major: ckl[b][h][K | V][T][64] bf16 (cross_relayout_kernel), so
// a split's 128 keys are one contiguous 16 KB block of K and one of V.
__global__ void __launch_bounds__(128) cross_attn_kernel(const float *q, const uint16_t *ckl, int T, float *part,
                                                         int nsplit) {
    __shared__ __align__(128) uint16_t ks[XCH * HD], vs[XCH * HD];
    __shared__ float qs[HD], sc[XCH], red[4], pacc[2][HD];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int ok_s;
    const int h = blockIdx.x, b = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
    const int jn = min(XCH, T - s * XCH);
    const uint16_t *kb = ckl + (((size_t)b * H + h) * 2 * T + (size_t)s * XCH) * HD;
    const uint16_t *vb = kb + (size_t)T * HD;
    // the chunk's K and V rows are contiguous (head-major relayout): two bulk copies
    // (cp.async.bulk, no multicast) complete on one mbarrier while q is read
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        const uint32_t bytes = (uint32_t)jn * HD * 2;
        mbar_arrive_expect_tx(&bar, 2 * bytes);
        bulk_g2s(ks, kb, bytes, &bar);
        bulk_g2s(vs, vb, bytes, &bar);
        ok_s = 1;
    }
    if (tid < HD) qs[tid] = q[(size_t)b * D + h * HD + tid];
    __syncthreads();
    if (!wait_copy(&bar)) ok_s = 0;          // bounded: 1 s, then the launch is reported failed
    __syncthreads();
    if (!ok_s) return;
    float v = -INFINITY;
    if (tid < jn) {
        const uint4 *kr = reinterpret_cast<const uint4 *>(ks + tid * HD);
        float dot = 0.0f;
#pragma unroll
        for (int c0 = 0; c0 < 8; c0++) {
            const int c = (c0 + tid) & 7;                   // rotate: lanes start on different banks
            const uint4 w = kr[c];
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; e++) dot += qs[8 * c + 2 * e] * bf16lo(u[e]) + qs[8 * c + 2 * e + 1] * bf16hi(u[e]);
        }
        v = dot * 0.125f;
    }
    float mx = v;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float p = tid < jn ? expf(v - mx) : 0.0f;
    sc[tid] = p;
    float sum = p;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    const int d = tid & 63, half = tid >> 6;
    float acc = 0.0f;
    for (int jj = half; jj < jn; jj += 2) acc += sc[jj] * bf16lo(vs[jj * HD + d]);
    pacc[half][d] = acc;
    __syncthreads();
    float *pp = part + (((size_t)b * H + h) * nsplit + s) * (HD + 2);
    if (tid < HD) pp[2 + tid] = pacc[0][tid] + pacc[1][tid];
    if (tid == 0) { pp[0] = mx; pp[1] = red[0] + red[1] + red[2] + red[3]; }
}
// continuous batching: each slot's greedy next token (first maximum), -1 for an empty slot;
// the logits rows optionally copied to logits_out [B][V]
__global__ void __launch_bounds__(1024) slot_argmax_kernel(const float *logits, int V, int ldl, const int *pos,
                                                           int64_t *next, float *logits_out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float *lr = logits + (size_t)b * ldl;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
        const float v = lr[i];
        if (v > best) { best = v; idx = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if ((tid & 31) == 0) { bv[tid >> 5] = best; bi[tid >> 5] = idx; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        next[b] = pos[b] < 0 ? -1 : idx;
    }
    if (logits_out)
        for (int i = tid; i < V; i += blockDim.x) logits_out[(size_t)b * V + i] = lr[i];
}

// ckv [B * T][L][K | V][768] (the cross K/V GEMM's output) -> ckh [L][B][12 heads][K | V][T][64]:
// 16-byte chunks, reads coalesced along a row, writes in 128-byte head rows
// (streams b0 .. b0 + B - 1 of ckv's rows, into a layout of BL streams)
__global__ void cross_relayout_kernel(const uint16_t *__restrict__ ckv, int b0, int B, int BL, int T, int L,
                                      uint16_t *__restrict__ ckh) {
    const size_t row_chunks = (size_t)L * 2 * D / 8, n = (size_t)B * T * row_chunks;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t bt = i / row_chunks, r = i % row_chunks;
        const int b = b0 + (int)(bt / T), t = (int)(bt % T);
        const int l = (int)(r / (2 * D / 8)), kv = (int)((r / (D / 8)) & 1), h = (int)((r % (D / 8)) / 8), c = (int)(r % 8);
        const size_t dst = (((((size_t)l * BL + b) * H + h) * 2 + kv) * T + t) * HD + 8 * c;
        *reinterpret_cast<uint4 *>(ckh + dst) = *reinterpret_cast<const uint4 *>(ckv + ((size_t)b0 * T) * (row_chunks * 8) + i * 8);
    }
}

__global__ void cross_merge_kernel(const float *__restrict__ part, int nsplit, uint16_t *__restrict__ ctx) {
    griddep_launch();                                 // the next GEMV may start its weight fetch
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const float *pp = part + ((size_t)b * H + h) * nsplit * (HD + 2);
    constexpr int MAXS = 16;                           // encoder positions <= 16 x 128
    float m[MAXS], l[MAXS], a[MAXS];
#pragma unroll
    for (int s = 0; s < MAXS; s++)
        if (s < nsplit) { m[s] = pp[s * (HD + 2)]; l[s] = pp[s * (HD + 2) + 1]; a[s] = pp[s * (HD + 2) + 2 + d]; }
    float M = -INFINITY, L = 0.0f, A = 0.0f;
#pragma unroll
    for (int s = 0; s < MAXS; s++) {
        if (s >= nsplit) break;
        const float mn = fmaxf(M, m[s]);
        const float c0 = M == -INFINITY ? 0.0f : expf(M - mn), c1 = expf(m[s] - mn);
        L = L * c0 + l[s] * c1;
        A = A * c0 + a[s] * c1;
        M = mn;
    }
    ctx[(size_t)b * D + h * HD + d] = (uint16_t)bf16bits(A / L);
}

// next token per stream: prompt[pos + 1] while the prompt lasts, else the first maximum of the
// logits (whisper.rs argmax, strict >); records generated tokens; one block per stream.  The
// last block to finish advances *pos.
__global__ void __launch_bounds__(1024) argmax_kernel(const float *logits, int V, int ldl, int B, const int64_t *prompt,
                                                      int n_prompt, int *posp, int64_t *tok, int64_t *out, int n_new,
                                                      float *logits_rec, unsigned *done) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x, tid = threadIdx.x, pos = *posp;
    const float *lr = logits + (size_t)b * ldl;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
        const float v = lr[i];
        if (v > best) { best = v; idx = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if ((tid & 31) == 0) { bv[tid >> 5] = best; bi[tid >> 5] = idx; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        const int step = pos + 1 - n_prompt;
        int64_t next;
        if (pos + 1 < n_prompt) next = prompt[pos + 1];
        else {
            next = idx;
            if (step < n_new) out[(size_t)b * n_new + step] = idx;
        }
        tok[b] = next;
        __threadfence();
        if (atomicAdd(done, 1u) == (unsigned)B - 1) { *done = 0; *posp = pos + 1; }
    }
    if (logits_rec && pos + 1 >= n_prompt && pos + 1 - n_prompt < n_new)
        for (int i = tid; i < V; i += blockDim.x)
            logits_rec[((size_t)b * n_new + (pos + 1 - n_prompt)) * V + i] = lr[i];
}

// f32 -> bf16 copy
__global__ void to_bf16_kernel(const float *x, size_t n, uint16_t *y) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = (uint16_t)bf16bits(x[i]);
}

}  // namespace wdec

// ====================================================================================== host
namespace {
struct CudaFail : std::runtime_error {
    using std::runtime_error::runtime_error;
};
void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw CudaFail(std::string(what) + ": " + cudaGetErrorString(e));
}
template <class T>
T *dalloc(size_t n) {
    void *p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)), "cudaMalloc");
    return static_cast<T *>(p);
}
template <class T>
T *dupload(const std::vector<T> &v) {
    T *p = dalloc<T>(v.size());
    ck(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
    return p;
}
uint16_t bf16_host(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
// bfp16 of one block of 8 (golden_ffn_gemm.py:34-49): exponent e and mantissas (-128..128)
void bfp16_block(const float *x, int &e, int (&m)[8]) {
    float mx = 0.0f;
    for (int i = 0; i < 8; i++) mx = std::max(mx, std::fabs(x[i]));
    if (mx == 0.0f) mx = 1.0f;
    int ex;
    (void)std::frexp(mx, &ex);
    e = ex - 1;
    const float q = std::ldexp(1.0f, e - 6);
    for (int i = 0; i < 8; i++) m[i] = (int)std::nearbyint(x[i] / q);
}
}  // namespace
}  // namespace xdna

using namespace xdna;

// one bfp16 weight [N, K] (rows = outputs) in the GEMV's fragment order
struct BfpMat {
    uint8_t *mant = nullptr, *ecode = nullptr;
    float *bias = nullptr;
    int N = 0, K = 0;
};

struct XdnaWhisperDec {
    XdnaWhisperDecConfig cfg{};
    int max_batch = 0;
    size_t clamped = 0;                     // blocks that held both +128 and -128 (see pack)
    struct Layer {
        BfpMat qkv, out, cq, cout, fc1, fc2;
        float *ln;                          // [3][2][D]: self, cross, final
    };
    std::vector<Layer> layers;
    BfpMat lm;
    float *et = nullptr, *ep = nullptr, *lnpost = nullptr;
    uint16_t *ckv_w = nullptr;              // [L * 2 * D][D] bf16 cross k|v weights (rows = outputs)
    float *ckv_b = nullptr;                 // [L * 2 * D]
    // state
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *logits = nullptr, *xpart = nullptr;
    uint16_t *xn = nullptr, *ctx = nullptr, *h = nullptr, *kcache = nullptr, *vcache = nullptr, *ckv = nullptr,
             *ckh = nullptr,
             *enc_bf = nullptr;
    float *enc_f = nullptr;
    unsigned *done = nullptr;
    int *pos = nullptr;
    int64_t *tok = nullptr, *prompt = nullptr, *out_tok = nullptr, *tok_out = nullptr;
    // continuous batching: per-slot token, position and next token; logits rows [max_batch][V]
    int *spos = nullptr;
    int64_t *stok = nullptr, *snext = nullptr;
    float *slog = nullptr;
    std::vector<std::pair<int, cudaGraphExec_t>> slot_graphs[2];   // [with logits] (n_slots, graph)
    float *lrec = nullptr;                  // logits record of xdna_whisper_dec_generate
    size_t lrec_n = 0;
    int B_enc = 0;
    std::vector<void *> owned;
    struct Graph {
        int B, n_prompt, n_new;
        float *lrec;
        cudaGraphExec_t exec;
    };
    std::vector<Graph> graphs;
    cudaStream_t cap = nullptr;
    ~XdnaWhisperDec() {
        if (lrec) cudaFree(lrec);
        for (auto &v : slot_graphs)
            for (auto &g : v) cudaGraphExecDestroy(g.second);
        for (auto &g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        if (cap) cudaStreamDestroy(cap);
        for (void *p : owned) cudaFree(p);
    }
};

namespace {
// W given as [K, N] ([in, out]) with optional bias; or (rows_kn == false) as [N, K]
BfpMat pack_bfp(XdnaWhisperDec *m, const float *w, const float *bias, int K, int N, bool kn) {
    const int nrg = (N + 15) / 16, nks = K / 16;
    std::vector<uint8_t> mant((size_t)nrg * nks * 32 * 8), ecode((size_t)nrg * nks * 32);
    std::vector<int> qm((size_t)nrg * 16 * K);
    std::vector<int> qe((size_t)nrg * 16 * (K / 8));
    std::vector<float> row(K);
    for (int n = 0; n < nrg * 16; n++) {
        for (int k = 0; k < K; k++) row[k] = n < N ? (kn ? w[(size_t)k * N + n] : w[(size_t)n * K + k]) : 0.0f;
        for (int b0 = 0; b0 < K; b0 += 8) {
            int e, mm[8];
            bfp16_block(&row[b0], e, mm);
            bool pos128 = false, neg128 = false;
            for (int i = 0; i < 8; i++) { pos128 |= mm[i] == 128; neg128 |= mm[i] == -128; }
            int neg = 0;
            if (pos128) {
                neg = 1;                              // store the block negated: +128 -> -128
                if (neg128) m->clamped++;             // both extremes: -(-128) cannot be stored
            }
            for (int i = 0; i < 8; i++) {
                int v = neg ? -mm[i] : mm[i];
                v = std::min(127, std::max(-128, v));
                qm[(size_t)n * K + b0 + i] = v;
            }
            const int ec = std::min(31, std::max(-32, e)) + 32;
            qe[(size_t)n * (K / 8) + b0 / 8] = ec | (neg << 7);
        }
    }
    for (int rg = 0; rg < nrg; rg++)
        for (int ks = 0; ks < nks; ks++) {
            uint8_t *mp = &mant[(((size_t)rg * nks + ks) * 32) * 8];
            uint8_t *epp = &ecode[(((size_t)rg * nks + ks) * 32)];
            for (int lane = 0; lane < 32; lane++) {
                const int g = lane >> 2, t = lane & 3;
                const int r0 = rg * 16 + g, r1 = r0 + 8, k = ks * 16 + 2 * t;
                const int vals[8] = {qm[(size_t)r0 * K + k], qm[(size_t)r0 * K + k + 1], qm[(size_t)r1 * K + k],
                                     qm[(size_t)r1 * K + k + 1], qm[(size_t)r0 * K + k + 8], qm[(size_t)r0 * K + k + 9],
                                     qm[(size_t)r1 * K + k + 8], qm[(size_t)r1 * K + k + 9]};
                for (int i = 0; i < 8; i++) mp[lane * 8 + i] = (uint8_t)(int8_t)vals[i];
            }
            for (int g = 0; g < 8; g++) {
                const int r0 = rg * 16 + g, r1 = r0 + 8, blk = ks * 2;
                epp[g * 4 + 0] = (uint8_t)qe[(size_t)r0 * (K / 8) + blk];
                epp[g * 4 + 1] = (uint8_t)qe[(size_t)r1 * (K / 8) + blk];
                epp[g * 4 + 2] = (uint8_t)qe[(size_t)r0 * (K / 8) + blk + 1];
                epp[g * 4 + 3] = (uint8_t)qe[(size_t)r1 * (K / 8) + blk + 1];
            }
        }
    BfpMat o;
    o.N = N;
    o.K = K;
    o.mant = dupload(mant);
    o.ecode = dupload(ecode);
    m->owned.push_back(o.mant);
    m->owned.push_back(o.ecode);
    if (bias) {
        std::vector<float> bv(bias, bias + N);
        o.bias = dupload(bv);
        m->owned.push_back(o.bias);
    }
    return o;
}

// GEMV launch shape: the largest row-group block per CTA (more reuse of the staged X) and the
// fewest K ranges that still give about 1.3 CTAs per SM, within the shared memory that lets two
// CTAs share an SM.  One pass when the grid covers every row group, else CTAs loop over row-group
// blocks with the staged X kept (then the partial sums get their own area).
struct GemvPlan {
    int R, nsplit, gx, red_off;
    size_t smem;
};
constexpr size_t kGemvSmemCap = 113 * 1024;
GemvPlan plan_of(int N, int K, int nt) {
    const int nrg = (N + 15) / 16, ks = K / 16;
    GemvPlan best{1, 1, 1, 0, 0};
    long best_ctas = -1;
    for (int R : {8, 4, 2, 1})
        for (int ns : {1, 2, 4, 8}) {
            if (ns > ks) continue;
            const int kc = (ks + ns - 1) / ns * 16, blocks = (nrg + R - 1) / R;
            const size_t xsb = (size_t)nt * 8 * (kc + 8) * 2, redb = (size_t)wdec::GEMV_WARPS * nt * 128 * 4;
            const int gx = std::min(blocks, std::max(1, 296 / ns));
            const bool loop = gx < blocks;
            const size_t smem = loop ? xsb + redb : std::max(xsb, redb);
            if (smem > kGemvSmemCap) continue;
            const long ctas = (long)blocks * ns;
            const GemvPlan p{R, ns, gx, loop ? (int)(xsb / 4) : 0, smem};
            if (ctas >= 190) return p;
            if (ctas > best_ctas) { best = p; best_ctas = ctas; }
        }
    if (best_ctas < 0) throw std::runtime_error("GEMV shape does not fit shared memory");
    return best;
}

cudaError_t gemv(XdnaWhisperDec *m, const BfpMat &w, const uint16_t *x, int B, int mode, float *out, uint16_t *ob,
                 int ldo, cudaStream_t st) {
    (void)m;
    const int nt = B <= 8 ? 1 : (B <= 16 ? 2 : 4);
    GemvPlan p;
    try { p = plan_of(w.N, w.K, nt); } catch (...) { return cudaErrorInvalidValue; }
    wdec::GemvArgs a{w.mant, w.ecode, w.bias, x, B, w.N, w.K, p.R, wdec::GEMV_WARPS / p.R, p.nsplit, p.red_off,
                     mode, out, ob, ldo};
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(p.gx, p.nsplit);
    lc.blockDim = dim3(wdec::GEMV_WARPS * 32);
    lc.dynamicSmemBytes = p.smem;
    lc.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = p.nsplit;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 2;
    if (nt == 1) return cudaLaunchKernelEx(&lc, wdec::bfp_gemv_kernel<1>, a);
    if (nt == 2) return cudaLaunchKernelEx(&lc, wdec::bfp_gemv_kernel<2>, a);
    return cudaLaunchKernelEx(&lc, wdec::bfp_gemv_kernel<4>, a);
}

// one token for B streams.  Lockstep (slots == false): reads *pos and tok on the device and
// advances both.  Slots: stream b feeds stok[b] at its own position spos[b] (< 0: empty slot) and
// writes its greedy next token to snext[b] (logits rows to slog when not null).
cudaError_t step(XdnaWhisperDec *m, int B, int n_prompt, int n_new, float *lrec, cudaStream_t st, bool slots = false) {
    using namespace wdec;
    const auto &c = m->cfg;
    const int nsplit = (c.n_enc + XCH - 1) / XCH;
    const int *posp = slots ? m->spos : m->pos;
    const int pstride = slots ? 1 : 0;
    cudaError_t e = cudaSuccess;
    embed_kernel<<<B, 256, 0, st>>>(slots ? m->stok : m->tok, posp, pstride, m->et, m->ep, m->x);
    for (int l = 0; l < c.n_layers && !e; l++) {
        const auto &L = m->layers[l];
        ln_kernel<<<(B + 7) / 8, 256, 0, st>>>(m->x, B, L.ln, L.ln + D, m->xn);
        if ((e = gemv(m, L.qkv, m->xn, B, OUT_F32, m->qkv, nullptr, 3 * D, st))) break;
        self_attn_kernel<<<dim3(H, B), 128, SA_SMEM, st>>>(m->qkv, posp, pstride, c.max_tgt,
                                                     m->kcache + (size_t)l * m->max_batch * H * c.max_tgt * HD,
                                                     m->vcache + (size_t)l * m->max_batch * H * c.max_tgt * HD, m->ctx);
        if ((e = gemv(m, L.out, m->ctx, B, OUT_RESID, m->x, nullptr, D, st))) break;
        ln_kernel<<<(B + 7) / 8, 256, 0, st>>>(m->x, B, L.ln + 2 * D, L.ln + 3 * D, m->xn);
        if ((e = gemv(m, L.cq, m->xn, B, OUT_F32, m->q, nullptr, D, st))) break;
        cross_attn_kernel<<<dim3(H, B, nsplit), 128, 0, st>>>(m->q, m->ckh + (size_t)l * m->max_batch * H * 2 * c.n_enc * HD,
                                                               c.n_enc, m->xpart, nsplit);
        cross_merge_kernel<<<dim3(H, B), HD, 0, st>>>(m->xpart, nsplit, m->ctx);
        if ((e = gemv(m, L.cout, m->ctx, B, OUT_RESID, m->x, nullptr, D, st))) break;
        ln_kernel<<<(B + 7) / 8, 256, 0, st>>>(m->x, B, L.ln + 4 * D, L.ln + 5 * D, m->xn);
        if ((e = gemv(m, L.fc1, m->xn, B, OUT_GELU_BF16, nullptr, m->h, F, st))) break;
        if ((e = gemv(m, L.fc2, m->h, B, OUT_RESID, m->x, nullptr, D, st))) break;
    }
    if (e) return e;
    ln_kernel<<<(B + 7) / 8, 256, 0, st>>>(m->x, B, m->lnpost, m->lnpost + D, m->xn);
    const int ldl = (c.vocab + 15) / 16 * 16;
    if ((e = gemv(m, m->lm, m->xn, B, OUT_F32, m->logits, nullptr, ldl, st))) return e;
    if (slots)
        slot_argmax_kernel<<<B, 1024, 0, st>>>(m->logits, c.vocab, ldl, m->spos, m->snext, lrec);
    else
        argmax_kernel<<<B, 1024, 0, st>>>(m->logits, c.vocab, ldl, B, m->prompt, n_prompt, m->pos, m->tok, m->out_tok,
                                          n_new, lrec, m->done);
    return cudaGetLastError();
}
}  // namespace

// true (and cleared) if a decoder kernel's bounded wait expired since the last check
static bool wdec_error_and_clear() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, wdec::g_wdec_error, sizeof v) != cudaSuccess || !v) return false;
    const unsigned z = 0;
    cudaMemcpyToSymbol(wdec::g_wdec_error, &z, sizeof z);
    return true;
}

extern "C" {

XdnaWhisperDec *xdna_whisper_dec_create(XdnaDevice *dev_unused, const XdnaWhisperDecConfig *cfg,
                                        const XdnaWhisperDecWeights *w, int max_batch) {
    (void)dev_unused;
    using namespace wdec;
    if (!cfg || !w || !w->layers || !w->embed_tokens || !w->embed_positions || !w->proj_out || !w->ln_post_w ||
        !w->ln_post_b) {
        set_last_error_message("xdna_whisper_dec_create: null pointer");
        return nullptr;
    }
    const XdnaWhisperDecConfig c = *cfg;
    if (c.d_model != D || c.n_heads != H || c.ffn != F || c.n_layers < 1 || c.vocab < 2 || c.max_tgt < 2 ||
        c.max_tgt > 448 || c.n_enc < 1 || max_batch < 1 || max_batch > MAXB) {
        set_last_error_message("xdna_whisper_dec_create: supported shape is d_model 768, 12 heads, ffn 3072, "
                               "max_tgt <= 448, 1..32 streams");
        return nullptr;
    }
    auto *m = new XdnaWhisperDec();
    try {
        m->cfg = c;
        m->max_batch = max_batch;
        auto keep = [&](void *p) { m->owned.push_back(p); return p; };
        auto f32 = [&](std::initializer_list<std::pair<const float *, size_t>> parts) {
            std::vector<float> v;
            for (auto &pr : parts) v.insert(v.end(), pr.first, pr.first + pr.second);
            return static_cast<float *>(keep(dupload(v)));
        };
        std::vector<uint16_t> ckw;
        std::vector<float> ckb;
        for (int l = 0; l < c.n_layers; l++) {
            const XdnaWhisperDecLayer &L = w->layers[l];
            XdnaWhisperDec::Layer o{};
            {
                std::vector<float> cat((size_t)D * 3 * D), cb(3 * D);
                for (int k = 0; k < D; k++)
                    for (int n = 0; n < D; n++) {
                        cat[(size_t)k * 3 * D + n] = L.q_w[(size_t)k * D + n];
                        cat[(size_t)k * 3 * D + D + n] = L.k_w[(size_t)k * D + n];
                        cat[(size_t)k * 3 * D + 2 * D + n] = L.v_w[(size_t)k * D + n];
                    }
                for (int n = 0; n < D; n++) {
                    cb[n] = L.q_b[n];
                    cb[D + n] = L.k_b ? L.k_b[n] : 0.0f;
                    cb[2 * D + n] = L.v_b[n];
                }
                o.qkv = pack_bfp(m, cat.data(), cb.data(), D, 3 * D, true);
            }
            o.out = pack_bfp(m, L.out_w, L.out_b, D, D, true);
            o.cq = pack_bfp(m, L.cross_q_w, L.cross_q_b, D, D, true);
            o.cout = pack_bfp(m, L.cross_out_w, L.cross_out_b, D, D, true);
            o.fc1 = pack_bfp(m, L.fc1_w, L.fc1_b, D, F, true);
            o.fc2 = pack_bfp(m, L.fc2_w, L.fc2_b, F, D, true);
            o.ln = f32({{L.ln_self_w, (size_t)D}, {L.ln_self_b, (size_t)D}, {L.ln_cross_w, (size_t)D},
                        {L.ln_cross_b, (size_t)D}, {L.ln_final_w, (size_t)D}, {L.ln_final_b, (size_t)D}});
            // cross k | v: bfp16 values (exact in bf16), rows = outputs, for the tcgen05 GEMM
            for (int which = 0; which < 2; which++) {
                const float *wk = which ? L.cross_v_w : L.cross_k_w;
                const float *bk = which ? L.cross_v_b : L.cross_k_b;
                std::vector<float> col(D);
                for (int n = 0; n < D; n++) {
                    for (int k = 0; k < D; k++) col[k] = wk[(size_t)k * D + n];
                    for (int b0 = 0; b0 < D; b0 += 8) {
                        int e, mm[8];
                        bfp16_block(&col[b0], e, mm);
                        for (int i = 0; i < 8; i++) ckw.push_back(bf16_host(std::ldexp((float)mm[i], e - 6)));
                    }
                    ckb.push_back(bk ? bk[n] : 0.0f);
                }
            }
            m->layers.push_back(o);
        }
        m->ckv_w = static_cast<uint16_t *>(keep(dupload(ckw)));
        m->ckv_b = static_cast<float *>(keep(dupload(ckb)));
        m->lm = pack_bfp(m, w->proj_out, nullptr, D, c.vocab, true);
        m->et = f32({{w->embed_tokens, (size_t)c.vocab * D}});
        m->ep = f32({{w->embed_positions, (size_t)c.max_tgt * D}});
        m->lnpost = f32({{w->ln_post_w, (size_t)D}, {w->ln_post_b, (size_t)D}});
        const size_t B = (size_t)max_batch, L = c.n_layers;
        const size_t ldl = (size_t)(c.vocab + 15) / 16 * 16;
        m->x = static_cast<float *>(keep(dalloc<float>(B * D)));
        m->qkv = static_cast<float *>(keep(dalloc<float>(B * 3 * D)));
        m->q = static_cast<float *>(keep(dalloc<float>(B * D)));
        m->logits = static_cast<float *>(keep(dalloc<float>(B * ldl)));
        for (int nt : {1, 2, 4}) {                 // every GEMV shape has a launch plan
            plan_of(3 * D, D, nt); plan_of(D, D, nt); plan_of(F, D, nt); plan_of(D, F, nt);
            plan_of(c.vocab, D, nt);
        }
        const int nsplit = (c.n_enc + XCH - 1) / XCH;
        m->xpart = static_cast<float *>(keep(dalloc<float>(B * H * nsplit * (HD + 2))));
        m->xn = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * D)));
        m->ctx = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * D)));
        m->h = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * F)));
        m->kcache = static_cast<uint16_t *>(keep(dalloc<uint16_t>(L * B * H * c.max_tgt * HD)));
        m->vcache = static_cast<uint16_t *>(keep(dalloc<uint16_t>(L * B * H * c.max_tgt * HD)));
        m->ckv = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * c.n_enc * L * 2 * D)));
        m->ckh = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * c.n_enc * L * 2 * D)));
        m->enc_bf = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * c.n_enc * D)));
        m->enc_f = static_cast<float *>(keep(dalloc<float>(B * c.n_enc * D)));
        m->done = static_cast<unsigned *>(keep(dalloc<unsigned>(1)));
        m->pos = static_cast<int *>(keep(dalloc<int>(1)));
        m->tok = static_cast<int64_t *>(keep(dalloc<int64_t>(B)));
        m->prompt = static_cast<int64_t *>(keep(dalloc<int64_t>(c.max_tgt)));
        m->out_tok = static_cast<int64_t *>(keep(dalloc<int64_t>(B * c.max_tgt)));
        m->tok_out = static_cast<int64_t *>(keep(dalloc<int64_t>(B * c.max_tgt)));
        m->spos = static_cast<int *>(keep(dalloc<int>(B)));
        m->stok = static_cast<int64_t *>(keep(dalloc<int64_t>(B)));
        m->snext = static_cast<int64_t *>(keep(dalloc<int64_t>(B)));
        m->slog = static_cast<float *>(keep(dalloc<float>(B * (size_t)c.vocab)));
        ck(cudaMemset(m->done, 0, sizeof(unsigned)), "memset");
        ck(cudaFuncSetAttribute(self_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SA_SMEM), "smem");
        const int gsm = (int)kGemvSmemCap;
        ck(cudaFuncSetAttribute(bfp_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(bfp_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(bfp_gemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaDeviceSynchronize(), "create sync");
        return m;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_whisper_dec_create: ") + ex.what());
        delete m;
        return nullptr;
    }
}

void xdna_whisper_dec_free(XdnaWhisperDec *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    delete m;
}

long long xdna_whisper_dec_clamped_blocks(const XdnaWhisperDec *m) { return m ? (long long)m->clamped : -1; }

int xdna_whisper_dec_set_encoder(XdnaWhisperDec *m, const float *enc_dev, int B, void *stream) {
    if (!m || !enc_dev) { set_last_error_message("xdna_whisper_dec_set_encoder: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch) { set_last_error_message("xdna_whisper_dec_set_encoder: bad batch"); return -1; }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const auto &c = m->cfg;
    const size_t n = (size_t)B * c.n_enc * wdec::D;
    wdec::to_bf16_kernel<<<1184, 256, 0, st>>>(enc_dev, n, m->enc_bf);
    const int NKV = c.n_layers * 2 * wdec::D;
    cudaError_t e = cudaGetLastError();
    if (!e) e = gemm_bf16(m->enc_bf, wdec::D, m->ckv_w, wdec::D, B * c.n_enc, NKV, wdec::D, m->ckv_b, nullptr, 0, 0,
                          m->ckv, NKV, st);
    if (!e) {
        wdec::cross_relayout_kernel<<<148 * 8, 256, 0, st>>>(m->ckv, 0, B, m->max_batch, c.n_enc, c.n_layers, m->ckh);
        e = cudaGetLastError();
    }
    if (e) { set_last_error_message(std::string("xdna_whisper_dec_set_encoder: ") + cudaGetErrorString(e)); return -1; }
    m->B_enc = B;
    return 0;
}

// ---- continuous batching: streams join and leave slots; every slot runs at its own position
int xdna_whisper_dec_set_encoder_slot(XdnaWhisperDec *m, int slot, const float *enc_dev, void *stream) {
    if (!m || !enc_dev) { set_last_error_message("xdna_whisper_dec_set_encoder_slot: null pointer"); return -1; }
    if (slot < 0 || slot >= m->max_batch) {
        set_last_error_message("xdna_whisper_dec_set_encoder_slot: slot outside 0 .. max_batch - 1");
        return -1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const auto &c = m->cfg;
    const size_t n = (size_t)c.n_enc * wdec::D;
    const int NKV = c.n_layers * 2 * wdec::D;
    uint16_t *enc_bf = m->enc_bf + (size_t)slot * n, *ckv = m->ckv + (size_t)slot * c.n_enc * NKV;
    wdec::to_bf16_kernel<<<1184, 256, 0, st>>>(enc_dev, n, enc_bf);
    cudaError_t e = cudaGetLastError();
    if (!e) e = gemm_bf16(enc_bf, wdec::D, m->ckv_w, wdec::D, c.n_enc, NKV, wdec::D, m->ckv_b, nullptr, 0, 0, ckv, NKV, st);
    if (!e) {
        wdec::cross_relayout_kernel<<<148 * 8, 256, 0, st>>>(m->ckv, slot, 1, m->max_batch, c.n_enc, c.n_layers, m->ckh);
        e = cudaGetLastError();
    }
    if (e) { set_last_error_message(std::string("xdna_whisper_dec_set_encoder_slot: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

int xdna_whisper_dec_step_slots(XdnaWhisperDec *m, int n_slots, const int64_t *tokens, const int *positions,
                                int64_t *next, float *logits) {
    if (!m || !tokens || !positions || !next) { set_last_error_message("xdna_whisper_dec_step_slots: null pointer"); return -1; }
    const auto &c = m->cfg;
    if (n_slots < 1 || n_slots > m->max_batch) {
        set_last_error_message("xdna_whisper_dec_step_slots: n_slots outside 1 .. max_batch");
        return -1;
    }
    for (int b = 0; b < n_slots; b++)
        if (positions[b] >= 0 && (positions[b] >= c.max_tgt || tokens[b] < 0 || tokens[b] >= c.vocab)) {
            set_last_error_message("xdna_whisper_dec_step_slots: slot " + std::to_string(b) +
                                   ": position beyond max_tgt or token out of range");
            return -1;
        }
    cudaStream_t st = nullptr;
    cudaError_t e = cudaMemcpy(m->stok, tokens, sizeof(int64_t) * n_slots, cudaMemcpyHostToDevice);
    if (!e) e = cudaMemcpy(m->spos, positions, sizeof(int) * n_slots, cudaMemcpyHostToDevice);
    auto &graphs = m->slot_graphs[logits ? 1 : 0];
    cudaGraphExec_t exec = nullptr;
    for (auto &g : graphs)
        if (g.first == n_slots) exec = g.second;
    if (!e && exec) e = cudaGraphLaunch(exec, st);
    else if (!e) {
        // the first step of a width runs eagerly (kernel attributes set before any capture), then
        // the width is recorded as a graph for the following steps
        e = step(m, n_slots, 0, 0, logits ? m->slog : nullptr, st, true);
        if (!e && !m->cap) e = cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking);
        cudaGraph_t graph = nullptr;
        if (!e) e = cudaStreamSynchronize(st);
        if (!e) e = cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal);
        if (!e) {
            const cudaError_t e2 = step(m, n_slots, 0, 0, logits ? m->slog : nullptr, m->cap, true);
            e = cudaStreamEndCapture(m->cap, &graph);
            if (!e) e = e2;
        }
        cudaGraphExec_t g = nullptr;
        if (!e) e = cudaGraphInstantiate(&g, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (!e) graphs.push_back({n_slots, g});
    }
    if (!e) e = cudaMemcpy(next, m->snext, sizeof(int64_t) * n_slots, cudaMemcpyDeviceToHost);
    if (!e && wdec_error_and_clear()) {
        set_last_error_message("xdna_whisper_dec_step_slots: an attention copy wait expired");
        return -1;
    }
    if (!e && logits) e = cudaMemcpy(logits, m->slog, sizeof(float) * n_slots * (size_t)c.vocab, cudaMemcpyDeviceToHost);
    if (e) { set_last_error_message(std::string("xdna_whisper_dec_step_slots: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

// Decode n_new tokens for B streams after a shared prompt (positions 0 .. n_prompt + n_new - 2
// are run).  Tokens go to tokens_dev [B][n_new] (device), logits_dev [B][n_new][vocab] if not
// null.  The first run of a (B, n_prompt, n_new, logits_dev) runs its steps eagerly and
// records them as a graph; later runs replay the graph once per step.
int xdna_whisper_dec_run(XdnaWhisperDec *m, int B, const int64_t *prompt_host, int n_prompt, int n_new,
                         int64_t *tokens_dev, float *logits_dev, void *stream) {
    if (!m || !prompt_host || !tokens_dev) { set_last_error_message("xdna_whisper_dec_run: null pointer"); return -1; }
    if (B != m->B_enc) { set_last_error_message("xdna_whisper_dec_run: batch differs from set_encoder"); return -1; }
    if (n_prompt < 1 || n_new < 1 || n_prompt + n_new > m->cfg.max_tgt) {
        set_last_error_message("xdna_whisper_dec_run: prompt + new tokens beyond max_tgt");
        return -1;
    }
    for (int i = 0; i < n_prompt; i++)
        if (prompt_host[i] < 0 || prompt_host[i] >= m->cfg.vocab) {
            set_last_error_message("xdna_whisper_dec_run: prompt token out of range");
            return -1;
        }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::vector<int64_t> t0(B, prompt_host[0]);
    const int zero = 0;
    cudaError_t e = cudaMemcpyAsync(m->prompt, prompt_host, sizeof(int64_t) * n_prompt, cudaMemcpyHostToDevice, st);
    if (!e) e = cudaMemcpyAsync(m->tok, t0.data(), sizeof(int64_t) * B, cudaMemcpyHostToDevice, st);
    if (!e) e = cudaMemcpyAsync(m->pos, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    if (!e) e = cudaStreamSynchronize(st);   // the host staging above is pageable
    if (e) { set_last_error_message(std::string("xdna_whisper_dec_run: ") + cudaGetErrorString(e)); return -1; }
    XdnaWhisperDec::Graph *g = nullptr;
    for (auto &x : m->graphs)
        if (x.B == B && x.n_prompt == n_prompt && x.n_new == n_new && x.lrec == logits_dev) g = &x;
    const int steps = n_prompt + n_new - 1;
    if (!g) {
        for (int s = 0; s < steps && !e; s++) e = step(m, B, n_prompt, n_new, logits_dev, st);
        if (!e) {
            m->graphs.push_back({B, n_prompt, n_new, logits_dev, nullptr});
            g = &m->graphs.back();
            if (!m->cap) e = cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking);
            cudaGraph_t graph = nullptr;
            if (!e) e = cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal);
            if (!e) {
                const cudaError_t e2 = step(m, B, n_prompt, n_new, logits_dev, m->cap);
                e = cudaStreamEndCapture(m->cap, &graph);
                if (!e) e = e2;
            }
            if (!e) e = cudaGraphInstantiate(&g->exec, graph, 0);
            if (graph) cudaGraphDestroy(graph);
        }
    } else {
        for (int s = 0; s < steps && !e; s++) e = cudaGraphLaunch(g->exec, st);
    }
    if (!e) e = cudaMemcpyAsync(tokens_dev, m->out_tok, sizeof(int64_t) * B * n_new, cudaMemcpyDeviceToDevice, st);
    if (e) { set_last_error_message(std::string("xdna_whisper_dec_run: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

int xdna_whisper_dec_generate(XdnaWhisperDec *m, const float *enc_host, int B, const int64_t *prompt, int n_prompt,
                              int n_new, int64_t *tokens_host, float *logits_host) {
    if (!m || !enc_host || !prompt || !tokens_host) {
        set_last_error_message("xdna_whisper_dec_generate: null pointer");
        return -1;
    }
    if (B < 1 || B > m->max_batch) { set_last_error_message("xdna_whisper_dec_generate: bad batch"); return -1; }
    try {
        const size_t ne = (size_t)B * m->cfg.n_enc * wdec::D;
        ck(cudaMemcpy(m->enc_f, enc_host, sizeof(float) * ne, cudaMemcpyHostToDevice), "copy encoder states");
        if (xdna_whisper_dec_set_encoder(m, m->enc_f, B, nullptr) != 0) return -1;
        float *lg = nullptr;
        if (logits_host) {
            const size_t need = (size_t)B * n_new * m->cfg.vocab;
            if (need > m->lrec_n) {      // grown once, reused by later calls (and their graphs)
                if (m->lrec) {
                    ck(cudaDeviceSynchronize(), "sync");
                    for (auto &g : m->graphs)
                        if (g.lrec == m->lrec) g.lrec = nullptr, g.B = -1;
                    cudaFree(m->lrec);
                }
                m->lrec = dalloc<float>(need);
                m->lrec_n = need;
            }
            lg = m->lrec;
        }
        if (xdna_whisper_dec_run(m, B, prompt, n_prompt, n_new, m->tok_out, lg, nullptr) != 0) return -1;
        ck(cudaMemcpy(tokens_host, m->tok_out, sizeof(int64_t) * B * n_new, cudaMemcpyDeviceToHost), "copy tokens");
        if (lg) ck(cudaMemcpy(logits_host, lg, sizeof(float) * B * n_new * m->cfg.vocab, cudaMemcpyDeviceToHost), "copy logits");
        if (gemm_error_and_clear()) { set_last_error_message("xdna_whisper_dec_generate: a GEMM wait expired"); return -1; }
        if (wdec_error_and_clear()) {
            set_last_error_message("xdna_whisper_dec_generate: an attention copy wait expired");
            return -1;
        }
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_whisper_dec_generate: ") + ex.what());
        return -1;
    }
}

}  // extern "C"
