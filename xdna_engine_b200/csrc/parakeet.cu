// parakeet.cu -- the Parakeet FastConformer encoder (parakeet-tdt-0.6b-v3 shapes) on B200 for
// batches of clips.
//
// Replaces the reference's FastConformerEncoder (rust/npu-parakeet/src/encoder.rs):
//   subsample      encoder.rs:200-237, conv2d ops.rs:38-89:
//                    conv.0 (1 -> 256, k3 s2 p1) + ReLU and conv.2 (depthwise k3 s2 p1) fused
//                    -> sub_conv02_kernel (channels-last bf16)
//                    conv.3 / conv.6 (pointwise + ReLU) -> bf16 tcgen05 GEMM, ReLU epilogue
//                    conv.5 (depthwise k3 s2 p1)     -> dw_s2_kernel
//                    flatten [t, c*F + f] + out linear -> bf16 GEMM over the channels-last
//                    rows [t, f*256 + c] with the out weight's rows permuted to match
//   block          encoder.rs:572-654, every weight linear on the int8 GEMM engine
//                  (tcgen05 kind::i8, the reference's rust/npu-asr/src/ctx2.rs int8 rule):
//                    LayerNorm + per-clip dynamic quantisation -> ln_quant_kernel (a cluster
//                    of 8 CTAs per clip; the clip's max |y| is reduced over DSMEM)
//                    feed_forward 102-168 -> int8 GEMM (SiLU epilogue) -> quant_kernel ->
//                    int8 GEMM (x + 0.5 y epilogue)
//                    mhsa 238-253 + attention_core 285-414 -> int8 QKV GEMM -> relpos_attention
//                    (tensor-core rel-pos MHA, rel_shift by index) -> int8 out GEMM (x + y)
//                    conv_module 416-570 -> int8 pw1 GEMM with the GLU epilogue ->
//                    dwconv_silu_quant_kernel (k9 'same' + bias + SiLU + quantise, cluster per
//                    clip) -> int8 pw2 GEMM (x + y)
//                    norm_out -> ln_quant_kernel in its f32 mode
// Activations between kernels are f32 (the residual stream and every int8 GEMM input before
// quantisation), so each quantisation sees the values the reference's rule sees.
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

namespace cg = cooperative_groups;

namespace xdna {
void set_last_error_message(const std::string &m);
cudaError_t gemm_bf16(const uint16_t *A, int lda, const uint16_t *B, int ldb, int M, int N, int K,
                      const float *bias, const uint16_t *residual, int ldr, int act, uint16_t *C, int ldc,
                      cudaStream_t st, int res_mod = 0, float *C_f32 = nullptr);
cudaError_t gemm_i8(const int8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, const float *sa,
                    int rows_per_clip, const float *ws, const float *bias, int act, const float *residual, int ldr,
                    float alpha, float *C, int ldc, unsigned *amax, cudaStream_t st);
unsigned gemm_error_and_clear();

namespace parakeet {

constexpr int D = 1024, H = 8, DK = 128, F = 4096, C = 256, KC = 9;
constexpr int CLUSTER = 8, ROWS_PER_CTA = 16, MAX_T = CLUSTER * ROWS_PER_CTA;   // 128 frames per clip

__device__ __forceinline__ float quant_scale(float amax) { return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f; }
// quant_i8 (ctx2.rs:1352-1354): round half away from zero of x / s, clamped to +-127
__device__ __forceinline__ int quant_i8(float x, float s) {
    const float v = roundf(__fdiv_rn(x, s));
    return (int)fminf(fmaxf(v, -127.0f), 127.0f);
}
__device__ __forceinline__ float silu(float v) { return __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)))); }
__device__ __forceinline__ uint32_t pack_i8x4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) | ((uint32_t)(d & 255) << 24);
}

// ------------------------------------------------------------------------------ subsample
// out2[b][h2][w2][c] (bf16, channels last) = conv.2(relu(conv.0(mel^T)))[c][h2][w2].  One CTA
// per (b, 2 rows of h2, 8 columns of w2), one thread per channel: the thread first computes
// the 5 x 17 conv.0 outputs its 16 conv.2 outputs read (conv.0 has one input channel, so this
// is cheap), keeps them in registers, then applies conv.2.  The accumulations follow conv2d of
// ops.rs: bias first, then + w * x tap by tap in (i, j) order; conv.0's zero padding of the
// input is in the staged patch (adding w * 0 leaves a finite sum unchanged, the same as the
// reference's skipped taps), conv.2 skips conv.0 positions outside the image.
constexpr int SH = 2, SW = 8;                                  // conv.2 outputs per CTA
constexpr int PH = 4 * SH + 3, PW = 4 * SW + 3;                // mel patch (time x freq)
constexpr int C0H = 2 * SH + 1, C0W = 2 * SW + 1;              // conv.0 outputs per thread
__global__ void __launch_bounds__(C) sub_conv02_kernel(const float *mel, int NM, int T0, int H1, int W1, int H2,
                                                       int W2, const float *w0, const float *b0, const float *w2,
                                                       const float *b2, uint16_t *out) {
    __shared__ float patch[PH][PW];
    const int h2_0 = blockIdx.y * SH, w2_0 = blockIdx.x * SW, b = blockIdx.z, c = threadIdx.x;
    const int t_0 = 4 * h2_0 - 3, f_0 = 4 * w2_0 - 3;           // patch origin
    const float *m = mel + (size_t)b * NM * T0;
    for (int i = threadIdx.x; i < PH * PW; i += C) {
        const int t = t_0 + i / PW, f = f_0 + i % PW;
        patch[i / PW][i % PW] = (t >= 0 && t < T0 && f >= 0 && f < NM) ? m[(size_t)f * T0 + t] : 0.0f;
    }
    __syncthreads();
    float k0[9];
#pragma unroll
    for (int i = 0; i < 9; i++) k0[i] = w0[c * 9 + i];
    const float bias0 = b0[c];
    // conv.0 output (h1, w1) = (2 h2_0 - 1 + u, 2 w2_0 - 1 + v); its taps read patch rows 2u + i
    // and columns 2v + j
    float a0[C0H][C0W];
#pragma unroll
    for (int u = 0; u < C0H; u++)
#pragma unroll
        for (int v = 0; v < C0W; v++) {
            float acc = bias0;
#pragma unroll
            for (int i = 0; i < 3; i++)
#pragma unroll
                for (int j = 0; j < 3; j++) acc = __fadd_rn(acc, __fmul_rn(k0[3 * i + j], patch[2 * u + i][2 * v + j]));
            const int h1 = 2 * h2_0 - 1 + u, w1 = 2 * w2_0 - 1 + v;
            a0[u][v] = (h1 >= 0 && h1 < H1 && w1 >= 0 && w1 < W1) ? fmaxf(acc, 0.0f) : 0.0f;
        }
    float k2[9];
#pragma unroll
    for (int i = 0; i < 9; i++) k2[i] = w2[c * 9 + i];
    const float bias2 = b2[c];
#pragma unroll
    for (int oh = 0; oh < SH; oh++)
#pragma unroll
        for (int ow = 0; ow < SW; ow++) {
            const int h2 = h2_0 + oh, w2o = w2_0 + ow;
            float acc = bias2;
#pragma unroll
            for (int i = 0; i < 3; i++)
#pragma unroll
                for (int j = 0; j < 3; j++) {
                    const int h1 = 2 * h2 + i - 1, w1 = 2 * w2o + j - 1;
                    if (h1 < 0 || h1 >= H1 || w1 < 0 || w1 >= W1) continue;
                    acc = __fadd_rn(acc, __fmul_rn(k2[3 * i + j], a0[2 * oh + i][2 * ow + j]));
                }
            if (h2 < H2 && w2o < W2) out[(((size_t)b * H2 + h2) * W2 + w2o) * C + c] = (uint16_t)bf16bits(acc);
        }
}

// depthwise k3 s2 p1 over channels-last bf16 [b][hin][win][C] -> [b][hout][wout][C]
__global__ void __launch_bounds__(C) dw_s2_kernel(const uint16_t *in, int Hin, int Win, int Hout, int Wout,
                                                  const float *w, const float *bias, uint16_t *out) {
    const int ow = blockIdx.x, oh = blockIdx.y, b = blockIdx.z, c = threadIdx.x;
    float acc = bias[c];
#pragma unroll
    for (int i = 0; i < 3; i++)
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const int ih = 2 * oh + i - 1, iw = 2 * ow + j - 1;
            const float wv = w[c * 9 + 3 * i + j];
            if (ih < 0 || ih >= Hin || iw < 0 || iw >= Win || wv == 0.0f) continue;
            const float x = bf16lo(in[(((size_t)b * Hin + ih) * Win + iw) * C + c]);
            acc = __fadd_rn(acc, __fmul_rn(wv, x));
        }
    out[(((size_t)b * Hout + oh) * Wout + ow) * C + c] = (uint16_t)bf16bits(acc);
}

// ------------------------------------------------------------ per-clip rows, cluster of 8
// Row layout inside a warp: lane holds columns 128 j + 4 lane + e (j < 8, e < 4).
__device__ __forceinline__ float cluster_max(float m, float *slot, cg::cluster_group &cl) {
    // slot: 33 floats of shared memory (one per warp, [32] = this CTA's maximum)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    if (lane == 0) slot[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float cm = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) cm = fmaxf(cm, slot[w]);
        slot[32] = cm;
    }
    cl.sync();
    float tot = 0.0f;
    for (unsigned r = 0; r < cl.num_blocks(); r++) tot = fmaxf(tot, *cl.map_shared_rank(slot + 32, r));
    cl.sync();   // every CTA has read every other CTA's slot before any of them moves on
    return tot;
}

// y = LN(x) per row (ops.rs:17-35: mean, population variance, (x - mu) * inv * g + b, eps
// 1e-5); quantise: q int8 with the clip's dynamic scale (sa[clip]), or (q == null) y f32 to
// yf (may alias x).  Cluster of 8 CTAs per clip, each 16 rows (2 per warp).
__global__ void __cluster_dims__(CLUSTER, 1, 1) __launch_bounds__(256, 2)
    ln_quant_kernel(const float *x, int T, const float *g, const float *bt, int8_t *q, float *sa, float *yf) {
    __shared__ float slot[33];
    cg::cluster_group cl = cg::this_cluster();
    const int clip = blockIdx.x / CLUSTER, rank = blockIdx.x % CLUSTER;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float v[2][32];
    float m = 0.0f;
    // both rows are requested before any arithmetic (one round trip)
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        const int t = rank * ROWS_PER_CTA + warp * 2 + rr;
        const float *xr = x + ((size_t)clip * T + min(t, T - 1)) * D;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 a = *reinterpret_cast<const float4 *>(xr + 128 * j + 4 * lane);
            v[rr][4 * j] = a.x; v[rr][4 * j + 1] = a.y; v[rr][4 * j + 2] = a.z; v[rr][4 * j + 3] = a.w;
        }
    }
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        const int t = rank * ROWS_PER_CTA + warp * 2 + rr;
        if (t >= T) continue;
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++) s += v[rr][i];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mu = __fdiv_rn(s, (float)D);
        float var = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++) { const float c = v[rr][i] - mu; var += c * c; }
#pragma unroll
        for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, (float)D), 1e-5f)));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 g4 = *reinterpret_cast<const float4 *>(g + 128 * j + 4 * lane);
            const float4 b4 = *reinterpret_cast<const float4 *>(bt + 128 * j + 4 * lane);
            const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float y = (v[rr][4 * j + e] - mu) * inv * gv[e] + bv[e];
                v[rr][4 * j + e] = y;
                m = fmaxf(m, fabsf(y));
            }
        }
        if (!q) {
            float *yr = yf + ((size_t)clip * T + t) * D;
#pragma unroll
            for (int j = 0; j < 8; j++)
                *reinterpret_cast<float4 *>(yr + 128 * j + 4 * lane) =
                    make_float4(v[rr][4 * j], v[rr][4 * j + 1], v[rr][4 * j + 2], v[rr][4 * j + 3]);
        }
    }
    if (!q) return;
    const float s = quant_scale(cluster_max(m, slot, cl));
    if (rank == 0 && threadIdx.x == 0) sa[clip] = s;
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        const int t = rank * ROWS_PER_CTA + warp * 2 + rr;
        if (t >= T) continue;
        int8_t *qr = q + ((size_t)clip * T + t) * D;
#pragma unroll
        for (int j = 0; j < 8; j++)
            *reinterpret_cast<uint32_t *>(qr + 128 * j + 4 * lane) =
                pack_i8x4(quant_i8(v[rr][4 * j], s), quant_i8(v[rr][4 * j + 1], s), quant_i8(v[rr][4 * j + 2], s),
                          quant_i8(v[rr][4 * j + 3], s));
    }
}

// conv_module's depthwise conv (ops.rs:92-110: k 9 'same', acc = bias then + taps[j] * x
// for valid j in order) + SiLU, then quantised with the clip's dynamic scale.  x = GLU output
// f32 [clip*T + t][D]; thread owns channels 2 tid, 2 tid + 1 for the CTA's 16 rows.
__global__ void __cluster_dims__(CLUSTER, 1, 1) __launch_bounds__(512)
    dwconv_silu_quant_kernel(const float *x, int T, const float *taps, const float *bias, int8_t *q, float *sa) {
    __shared__ float slot[33];
    cg::cluster_group cl = cg::this_cluster();
    const int clip = blockIdx.x / CLUSTER, rank = blockIdx.x % CLUSTER;
    const int c0 = 2 * threadIdx.x;
    float tp[2][KC];
#pragma unroll
    for (int e = 0; e < 2; e++)
#pragma unroll
        for (int j = 0; j < KC; j++) tp[e][j] = taps[(c0 + e) * KC + j];
    const float2 bb = *reinterpret_cast<const float2 *>(bias + c0);
    float o[ROWS_PER_CTA][2];
    float m = 0.0f;
    const float *xc = x + (size_t)clip * T * D + c0;
    constexpr int HALO = (KC - 1) / 2, NIN = ROWS_PER_CTA + KC - 1;
    const int t0 = rank * ROWS_PER_CTA;
    float2 xin[NIN];      // input rows t0 - 4 .. t0 + 19, all requested up front
#pragma unroll
    for (int u = 0; u < NIN; u++) {
        const int s = t0 - HALO + u;
        xin[u] = (s >= 0 && s < T) ? *reinterpret_cast<const float2 *>(xc + (size_t)s * D) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < ROWS_PER_CTA; r++) {
        const int t = t0 + r;
        float a[2] = {bb.x, bb.y};
        if (t < T) {
#pragma unroll
            for (int j = 0; j < KC; j++) {
                const int s = t + j - HALO;
                if (s < 0 || s >= T) continue;
                a[0] = __fadd_rn(a[0], __fmul_rn(tp[0][j], xin[r + j].x));
                a[1] = __fadd_rn(a[1], __fmul_rn(tp[1][j], xin[r + j].y));
            }
            a[0] = silu(a[0]);
            a[1] = silu(a[1]);
            m = fmaxf(m, fmaxf(fabsf(a[0]), fabsf(a[1])));
        }
        o[r][0] = a[0];
        o[r][1] = a[1];
    }
    const float s = quant_scale(cluster_max(m, slot, cl));
    if (rank == 0 && threadIdx.x == 0) sa[clip] = s;
#pragma unroll
    for (int r = 0; r < ROWS_PER_CTA; r++) {
        const int t = rank * ROWS_PER_CTA + r;
        if (t >= T) continue;
        *reinterpret_cast<uint16_t *>(q + ((size_t)clip * T + t) * D + c0) =
            (uint16_t)((quant_i8(o[r][0], s) & 255) | ((quant_i8(o[r][1], s) & 255) << 8));
    }
}

// q = quant_i8(x, s[clip]) for a GEMM-produced f32 tensor whose per-clip max |x| is in amax;
// also records s[clip].  x [clips * T, K], K % 4 == 0.
__global__ void quant_kernel(const float *x, int T, int K, int clips, const unsigned *amax, int8_t *q, float *sa) {
    const int clip = blockIdx.y;
    const float s = quant_scale(__uint_as_float(amax[clip]));
    if (blockIdx.x == 0 && threadIdx.x == 0) sa[clip] = s;
    const int n4 = T * K / 4;
    const float4 *xs = reinterpret_cast<const float4 *>(x) + (size_t)clip * n4;
    uint32_t *qs = reinterpret_cast<uint32_t *>(q) + (size_t)clip * n4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const float4 v = xs[i];
        qs[i] = pack_i8x4(quant_i8(v.x, s), quant_i8(v.y, s), quant_i8(v.z, s), quant_i8(v.w, s));
    }
}

// -------------------------------------------------------------------- rel-pos attention
// attention_core (encoder.rs:285-414) for one (head, clip): qu = q + u[h], qv = q + v[h];
// scores[i][j] = (qu_i . k_j + qv_i . p_(T-1-i+j)) / sqrt(128) -- rel_shift (ops.rs:113-133)
// picks exactly BD[i][T-1-i+j] -- softmax over j < T, ctx = P V.  Tensor cores (mma.sync
// m16n8k16, bf16 operands, f32 accumulation); warp w owns query rows 16w .. 16w+15.  For its
// rows a warp computes BD over the 144 positions it can need, r0 = T-16-16w .. r0+143, parks
// them in its shared scratch, and reads BD[i][T-1-i+j] from there next to the AC fragment.
constexpr int ATT_THREADS = 256;
constexpr int P_OFF = 32;                       // sP row of position r is r + P_OFF
constexpr int P_ROWS = 2 * MAX_T + P_OFF + 16;  // 288
constexpr int BD_COLS = 144;
constexpr int ATT_SMEM = (2 * MAX_T + P_ROWS) * DK * 2 + 8 * 16 * BD_COLS * 4;

__device__ __forceinline__ uint32_t swz256(int row, int chunk) {
    return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pk(float lo, float hi) { return bf16bits(lo) | (bf16bits(hi) << 16); }

// rows [0, nrows) of a [*, ld] f32 matrix (columns col0 .. col0+127) -> bf16 swizzled tile rows
// dst_row0 + r; other rows of [dst_row0 + r_lo, dst_row0 + r_hi) zero
__device__ __forceinline__ void load_rows_bf16(uint8_t *tile, const float *src, int ld, int r_lo, int r_hi,
                                               int nrows, int dst_row0) {
    // 8 pieces (16 floats each) per thread in flight before any is converted
    const int n = (r_hi - r_lo) * 16;
    for (int c0 = threadIdx.x; c0 < n; c0 += 8 * ATT_THREADS) {
        float4 a[8], b[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int c = c0 + u * ATT_THREADS, r = r_lo + c / 16, ch = c % 16;
            a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c < n && r >= 0 && r < nrows) {
                a[u] = *reinterpret_cast<const float4 *>(src + (size_t)r * ld + ch * 8);
                b[u] = *reinterpret_cast<const float4 *>(src + (size_t)r * ld + ch * 8 + 4);
            }
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int c = c0 + u * ATT_THREADS, r = r_lo + c / 16, ch = c % 16;
            if (c < n)
                *reinterpret_cast<uint4 *>(tile + swz256(dst_row0 + r, ch)) =
                    make_uint4(pk(a[u].x, a[u].y), pk(a[u].z, a[u].w), pk(b[u].x, b[u].y), pk(b[u].z, b[u].w));
        }
    }
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    relpos_attention_kernel(const float *qkv, const float *pm, const float *pos_u, const float *pos_v, int T,
                            float *ctx, unsigned *amax) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t *sK = sm, *sV = sm + MAX_T * 256, *sP = sm + 2 * MAX_T * 256;
    float *scratch = reinterpret_cast<float *>(sm + (2 * MAX_T + P_ROWS) * 256);
    const int h = blockIdx.x, clip = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    constexpr int LD = 3 * D;
    const float *Q = qkv + (size_t)clip * T * LD + h * DK;
    load_rows_bf16(sK, Q + D, LD, 0, MAX_T, T, 0);
    load_rows_bf16(sV, Q + 2 * D, LD, 0, MAX_T, T, 0);
    load_rows_bf16(sP, pm + h * DK, D, -P_OFF, P_ROWS - P_OFF, 2 * T - 1, P_OFF);
    __syncthreads();
    const int i0 = warp * 16;
    if (i0 >= T) return;
    float *scr = scratch + warp * 16 * BD_COLS;

    // A fragments of q + bias for this warp's rows (rows >= T are zero)
    auto q_frags = [&](const float *bias, uint32_t (&a)[8][4]) {
#pragma unroll
        for (int kc = 0; kc < 8; kc++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {          // hh: column half (k 0-7 / 8-15)
                const int d = kc * 16 + hh * 8 + 2 * tq;
                const float b0 = bias[h * DK + d], b1 = bias[h * DK + d + 1];
#pragma unroll
                for (int rh = 0; rh < 2; rh++) {      // rh: row g / g + 8
                    const int i = i0 + g + 8 * rh;
                    float x0 = 0.0f, x1 = 0.0f;
                    if (i < T) {
                        const float2 qq = *reinterpret_cast<const float2 *>(Q + (size_t)i * LD + d);
                        x0 = qq.x + b0;
                        x1 = qq.y + b1;
                    }
                    a[kc][hh * 2 + rh] = pk(x0, x1);
                }
            }
    };
    uint32_t qa[8][4];
    // ---- BD over positions r0 .. r0 + 143 -> scratch[16][144]
    q_frags(pos_v, qa);
    const int r0 = T - 16 - i0;
    {
        float bd[18][4];
#pragma unroll
        for (int n = 0; n < 18; n++) bd[n][0] = bd[n][1] = bd[n][2] = bd[n][3] = 0.0f;
        const uint32_t p_base = smem_u32(sP);
#pragma unroll
        for (int kc = 0; kc < 8; kc++)
#pragma unroll
            for (int np = 0; np < 9; np++) {
                const int row = P_OFF + r0 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = kc * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(p_base + swz256(row, ch), b0, b1, b2, b3);
                mma16816(bd[2 * np], qa[kc], b0, b1);
                mma16816(bd[2 * np + 1], qa[kc], b2, b3);
            }
#pragma unroll
        for (int n = 0; n < 18; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) scr[(g + 8 * (e >> 1)) * BD_COLS + n * 8 + 2 * tq + (e & 1)] = bd[n][e];
    }
    // ---- AC over the 128 key slots
    q_frags(pos_u, qa);
    float sc[16][4];
#pragma unroll
    for (int n = 0; n < 16; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
    {
        const uint32_t k_base = smem_u32(sK);
#pragma unroll
        for (int kc = 0; kc < 8; kc++)
#pragma unroll
            for (int np = 0; np < 8; np++) {
                const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = kc * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(k_base + swz256(key, ch), b0, b1, b2, b3);
                mma16816(sc[2 * np], qa[kc], b0, b1);
                mma16816(sc[2 * np + 1], qa[kc], b2, b3);
            }
    }
    __syncwarp();
    // ---- scores, softmax (rows g and g + 8)
    const float scale = sqrtf((float)DK);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 16; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int il = g + 8 * (e >> 1), j = n * 8 + 2 * tq + (e & 1);
            float s = -INFINITY;
            if (j < T) s = __fdiv_rn(__fadd_rn(sc[n][e], scr[il * BD_COLS + j + 15 - il]), scale);
            sc[n][e] = s;
            mx[e >> 1] = fmaxf(mx[e >> 1], s);
        }
    float sum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 2; r++) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    uint32_t pa[8][4];
#pragma unroll
    for (int n = 0; n < 16; n++) {
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            p[e] = sc[n][e] == -INFINITY ? 0.0f : expf(sc[n][e] - mx[e >> 1]);
            sum[e >> 1] += p[e];
        }
        const int kc = n >> 1, hi = n & 1;
        pa[kc][hi * 2 + 0] = pk(p[0], p[1]);
        pa[kc][hi * 2 + 1] = pk(p[2], p[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 1);
        sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], 2);
    }
    // ---- ctx = P V
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    const uint32_t v_base = smem_u32(sV);
#pragma unroll
    for (int kc = 0; kc < 8; kc++)
#pragma unroll
        for (int np = 0; np < 8; np++) {
            const int key = kc * 16 + (lane & 15);
            const int ch = np * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(v_base + swz256(key, ch), b0, b1, b2, b3);
            mma16816(o[2 * np], pa[kc], b0, b1);
            mma16816(o[2 * np + 1], pa[kc], b2, b3);
        }
    float m = 0.0f;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = i0 + g + 8 * r;
        if (i >= T) continue;
        const float inv = __fdiv_rn(1.0f, sum[r]);
        float *dst = ctx + ((size_t)clip * T + i) * D + h * DK;
#pragma unroll
        for (int n = 0; n < 16; n++) {
            const float a = o[n][2 * r] * inv, b = o[n][2 * r + 1] * inv;
            *reinterpret_cast<float2 *>(dst + n * 8 + 2 * tq) = make_float2(a, b);
            m = fmaxf(m, fmaxf(fabsf(a), fabsf(b)));
        }
    }
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    if (lane == 0 && amax) atomicMax(amax + clip, __float_as_uint(m));
}

}  // namespace parakeet

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
uint16_t bf16_bits_host(float f) {   // round to nearest even
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
float q_round(float x, float s) {    // quant_i8 on the host: round half away, clamp +-127
    float v = std::round(x / s);
    return v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
}
// W [K, N] ([in, out]) -> per-output-channel int8 [N, K] and scales (ctx2.rs:549-584); column
// n of the result is column perm[n] of W
void quant_cols(const float *w, int K, int N, const std::vector<int> &perm, std::vector<int8_t> &q,
                std::vector<float> &s) {
    q.resize((size_t)N * K);
    s.resize(N);
    for (int n = 0; n < N; n++) {
        const int src = perm.empty() ? n : perm[n];
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = std::max(amax, std::fabs(w[(size_t)k * N + src]));
        s[n] = amax > 0.0f ? amax / 127.0f : 1.0f;
        for (int k = 0; k < K; k++) q[(size_t)n * K + k] = (int8_t)q_round(w[(size_t)k * N + src], s[n]);
    }
}

}  // namespace
}  // namespace xdna

using namespace xdna;

struct XdnaParakeet {
    XdnaParakeetConfig cfg{};
    int max_batch = 0, T = 0, H1 = 0, W1 = 0, H2 = 0, W2 = 0, W3 = 0;
    float *c0w = nullptr, *c0b = nullptr, *c2w = nullptr, *c2b = nullptr, *c5w = nullptr, *c5b = nullptr;
    uint16_t *c3w = nullptr, *c6w = nullptr, *outw = nullptr;
    float *c3b = nullptr, *c6b = nullptr, *outb = nullptr;
    struct Lin {
        int8_t *q;
        float *s;
    };
    struct Layer {
        Lin ff1a, ff1b, qkv, out, pw1, pw2, ff2a, ff2b;
        float *ln_ff1, *ln_att, *ln_conv, *ln_ff2, *ln_out;   // [2][D]
        float *pos_u, *pos_v, *dw_w, *dw_b, *pm;              // pm [2T-1][D]
    };
    std::vector<Layer> layers;
    // activations
    float *mel = nullptr, *x = nullptr, *h = nullptr, *qkvb = nullptr, *ctx = nullptr, *outf = nullptr;
    int8_t *q8 = nullptr;
    float *sa = nullptr;
    unsigned *amax = nullptr;
    uint16_t *a2 = nullptr, *a3 = nullptr, *a5 = nullptr, *a6 = nullptr;
    std::vector<void *> owned;
    // replay graphs of the whole forward, one per (batch, input, output) seen twice
    struct Graph {
        int B;
        const float *mel;
        float *out;
        int calls;
        cudaGraphExec_t exec;
    };
    std::vector<Graph> graphs;
    cudaStream_t cap = nullptr;
    ~XdnaParakeet() {
        for (auto &g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        if (cap) cudaStreamDestroy(cap);
        for (void *p : owned) cudaFree(p);
    }
};

namespace {
constexpr int kD = parakeet::D, kF = parakeet::F, kC = parakeet::C;

void run_ln(XdnaParakeet *m, const float *g, int B, bool quant, cudaStream_t st) {
    parakeet::ln_quant_kernel<<<B * parakeet::CLUSTER, 256, 0, st>>>(m->x, m->T, g, g + kD, quant ? m->q8 : nullptr,
                                                                     m->sa, m->x);
}
cudaError_t lin(XdnaParakeet *m, const XdnaParakeet::Lin &L, int M, int N, int K, int act, const float *res,
                float alpha, float *out, unsigned *amax, cudaStream_t st) {
    const int ldc = act == 3 ? N / 2 : N;
    return gemm_i8(m->q8, K, L.q, K, M, N, K, m->sa, m->T, L.s, nullptr, act, res, ldc, alpha, out, ldc, amax, st);
}
cudaError_t quant(XdnaParakeet *m, const float *src, int K, int B, cudaStream_t st) {
    parakeet::quant_kernel<<<dim3(std::max(1, 148 * 8 / B), B), 256, 0, st>>>(src, m->T, K, B, m->amax, m->q8, m->sa);
    return cudaGetLastError();
}
cudaError_t ffn(XdnaParakeet *m, const float *ln, const XdnaParakeet::Lin &a, const XdnaParakeet::Lin &b, int B,
                cudaStream_t st) {
    const int M = B * m->T;
    run_ln(m, ln, B, true, st);
    cudaError_t e = cudaMemsetAsync(m->amax, 0, sizeof(unsigned) * B, st);
    if (!e) e = lin(m, a, M, kF, kD, 1, nullptr, 1.0f, m->h, m->amax, st);
    if (!e) e = quant(m, m->h, kF, B, st);
    if (!e) e = lin(m, b, M, kD, kF, 0, m->x, 0.5f, m->x, nullptr, st);
    return e;
}
}  // namespace

extern "C" {

XdnaParakeet *xdna_parakeet_create(XdnaDevice *dev_unused, const XdnaParakeetConfig *cfg,
                                   const XdnaParakeetWeights *w, int max_batch) {
    (void)dev_unused;
    if (!cfg || !w || !w->layers) { set_last_error_message("xdna_parakeet_create: null pointer"); return nullptr; }
    const XdnaParakeetConfig c = *cfg;
    auto sub2 = [](int v) { return (v - 1) / 2 + 1; };
    const int H1 = sub2(c.n_frames), H2 = sub2(H1), T = sub2(H2);
    const int W1 = sub2(c.n_mels), W2 = sub2(W1), W3 = sub2(W2);
    if (c.d_model != kD || c.n_heads != parakeet::H || c.ffn != kF || c.sub_ch != kC || c.kconv != parakeet::KC ||
        c.n_layers < 1 || c.n_mels < 2 || c.n_frames < 2 || T > parakeet::MAX_T || max_batch < 1) {
        set_last_error_message("xdna_parakeet_create: supported shape is d_model 1024, 8 heads, ffn 4096, 256 "
                               "subsample channels, conv kernel 9, at most 128 frames after subsampling");
        return nullptr;
    }
    auto *m = new XdnaParakeet();
    try {
        m->cfg = c;
        m->max_batch = max_batch;
        m->T = T; m->H1 = H1; m->W1 = W1; m->H2 = H2; m->W2 = W2; m->W3 = W3;
        auto keep = [&](void *p) { m->owned.push_back(p); return p; };
        auto f32 = [&](std::initializer_list<std::pair<const float *, size_t>> parts) {
            std::vector<float> v;
            for (auto &pr : parts) v.insert(v.end(), pr.first, pr.first + pr.second);
            return static_cast<float *>(keep(dupload(v)));
        };
        auto bf_rows = [&](const float *src, size_t n) {   // plain copy to bf16
            std::vector<uint16_t> v(n);
            for (size_t i = 0; i < n; i++) v[i] = bf16_bits_host(src[i]);
            return static_cast<uint16_t *>(keep(dupload(v)));
        };
        m->c0w = f32({{w->c0_w, (size_t)kC * 9}}); m->c0b = f32({{w->c0_b, (size_t)kC}});
        m->c2w = f32({{w->c2_w, (size_t)kC * 9}}); m->c2b = f32({{w->c2_b, (size_t)kC}});
        m->c5w = f32({{w->c5_w, (size_t)kC * 9}}); m->c5b = f32({{w->c5_b, (size_t)kC}});
        m->c3w = bf_rows(w->c3_w, (size_t)kC * kC); m->c3b = f32({{w->c3_b, (size_t)kC}});   // [out][in]
        m->c6w = bf_rows(w->c6_w, (size_t)kC * kC); m->c6b = f32({{w->c6_b, (size_t)kC}});
        {   // out linear [C*W3, D] ([in, out], in = c*W3 + f) -> [D][W3*C] with in' = f*C + c
            const int Kin = kC * W3;
            std::vector<uint16_t> v((size_t)kD * Kin);
            for (int n = 0; n < kD; n++)
                for (int f = 0; f < W3; f++)
                    for (int ch = 0; ch < kC; ch++)
                        v[(size_t)n * Kin + f * kC + ch] = bf16_bits_host(w->out_w[(size_t)(ch * W3 + f) * kD + n]);
            m->outw = static_cast<uint16_t *>(keep(dupload(v)));
            m->outb = f32({{w->out_b, (size_t)kD}});
        }
        // rel-pos table (pos.rs:7-47) and its int8 quantisation (one tensor, one scale)
        const int P = 2 * T - 1;
        std::vector<float> pe((size_t)P * kD);
        for (int k = 0; k < P; k++) {
            const double pos = k < T ? (double)(T - 1 - k) : -(double)(k - T + 1);
            for (int i = 0; i < kD / 2; i++) {
                const double dv = std::exp(-std::log(10000.0) * (double)(2 * i) / (double)kD);
                pe[(size_t)k * kD + 2 * i] = (float)std::sin(pos * dv);
                pe[(size_t)k * kD + 2 * i + 1] = (float)std::cos(pos * dv);
            }
        }
        float pe_amax = 0.0f;
        for (float v : pe) pe_amax = std::max(pe_amax, std::fabs(v));
        const float pe_s = pe_amax > 0.0f ? pe_amax / 127.0f : 1.0f;
        std::vector<int8_t> peq(pe.size());
        for (size_t i = 0; i < pe.size(); i++) peq[i] = (int8_t)q_round(pe[i], pe_s);
        int8_t *d_peq = dalloc<int8_t>(((size_t)P + 127) / 128 * 128 * kD);
        keep(d_peq);
        ck(cudaMemcpy(d_peq, peq.data(), peq.size(), cudaMemcpyHostToDevice), "upload pe");
        float *d_pes = f32({{&pe_s, 1}});

        auto lin = [&](const float *wk, int K, int N, const std::vector<int> &perm) {
            std::vector<int8_t> q;
            std::vector<float> s;
            quant_cols(wk, K, N, perm, q, s);
            XdnaParakeet::Lin L;
            L.q = static_cast<int8_t *>(keep(dupload(q)));
            L.s = static_cast<float *>(keep(dupload(s)));
            return L;
        };
        std::vector<int> glu_perm(2 * kD);
        for (int ch = 0; ch < kD; ch++) { glu_perm[2 * ch] = ch; glu_perm[2 * ch + 1] = kD + ch; }
        for (int l = 0; l < c.n_layers; l++) {
            const XdnaParakeetLayer &L = w->layers[l];
            XdnaParakeet::Layer o{};
            o.ff1a = lin(L.ff1_w1, kD, kF, {}); o.ff1b = lin(L.ff1_w2, kF, kD, {});
            o.ff2a = lin(L.ff2_w1, kD, kF, {}); o.ff2b = lin(L.ff2_w2, kF, kD, {});
            {   // q, k, v share one GEMM: columns [q | k | v], each its own per-channel scale
                std::vector<float> cat((size_t)kD * 3 * kD);
                for (int k = 0; k < kD; k++)
                    for (int n = 0; n < kD; n++) {
                        cat[(size_t)k * 3 * kD + n] = L.wq[(size_t)k * kD + n];
                        cat[(size_t)k * 3 * kD + kD + n] = L.wk[(size_t)k * kD + n];
                        cat[(size_t)k * 3 * kD + 2 * kD + n] = L.wv[(size_t)k * kD + n];
                    }
                o.qkv = lin(cat.data(), kD, 3 * kD, {});
            }
            o.out = lin(L.wout, kD, kD, {});
            o.pw1 = lin(L.pw1, kD, 2 * kD, glu_perm);
            o.pw2 = lin(L.pw2, kD, kD, {});
            o.ln_ff1 = f32({{L.ff1_ln_w, (size_t)kD}, {L.ff1_ln_b, (size_t)kD}});
            o.ln_att = f32({{L.att_ln_w, (size_t)kD}, {L.att_ln_b, (size_t)kD}});
            o.ln_conv = f32({{L.conv_ln_w, (size_t)kD}, {L.conv_ln_b, (size_t)kD}});
            o.ln_ff2 = f32({{L.ff2_ln_w, (size_t)kD}, {L.ff2_ln_b, (size_t)kD}});
            o.ln_out = f32({{L.out_ln_w, (size_t)kD}, {L.out_ln_b, (size_t)kD}});
            o.pos_u = f32({{L.pos_u, (size_t)kD}});
            o.pos_v = f32({{L.pos_v, (size_t)kD}});
            o.dw_w = f32({{L.dw_w, (size_t)kD * parakeet::KC}});
            o.dw_b = f32({{L.dw_b, (size_t)kD}});
            // pm = pos_enc . W_pos on the int8 engine, once (it depends on weights and T only)
            XdnaParakeet::Lin lp = lin(L.wpos, kD, kD, {});
            o.pm = static_cast<float *>(keep(dalloc<float>((size_t)P * kD)));
            ck(gemm_i8(d_peq, kD, lp.q, kD, P, kD, kD, d_pes, P, lp.s, nullptr, 0, nullptr, kD, 1.0f, o.pm, kD,
                       nullptr, nullptr), "pos projection");
            m->layers.push_back(o);
        }
        const size_t B = (size_t)max_batch, M = B * T;
        m->mel = static_cast<float *>(keep(dalloc<float>(B * c.n_mels * c.n_frames)));
        m->x = static_cast<float *>(keep(dalloc<float>(M * kD)));
        m->h = static_cast<float *>(keep(dalloc<float>(M * kF)));
        m->qkvb = static_cast<float *>(keep(dalloc<float>(M * 3 * kD)));
        m->ctx = static_cast<float *>(keep(dalloc<float>(M * kD)));
        m->outf = static_cast<float *>(keep(dalloc<float>(M * kD)));
        m->q8 = static_cast<int8_t *>(keep(dalloc<int8_t>(M * kF)));
        m->sa = static_cast<float *>(keep(dalloc<float>(B)));
        m->amax = static_cast<unsigned *>(keep(dalloc<unsigned>(B)));
        m->a2 = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * H2 * W2 * kC)));
        m->a3 = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * H2 * W2 * kC)));
        m->a5 = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * T * W3 * kC)));
        m->a6 = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * T * W3 * kC)));
        ck(cudaFuncSetAttribute(parakeet::relpos_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                parakeet::ATT_SMEM), "attention smem");
        ck(cudaDeviceSynchronize(), "create sync");
        if (gemm_error_and_clear()) throw CudaFail("a GEMM wait expired");
        return m;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_parakeet_create: ") + ex.what());
        delete m;
        return nullptr;
    }
}

void xdna_parakeet_free(XdnaParakeet *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    delete m;
}

int xdna_parakeet_frames_out(const XdnaParakeet *m) { return m ? m->T : -1; }

}  // extern "C"

// the forward's ~500 launches, in stream order on st
static int parakeet_enqueue(XdnaParakeet *m, const float *mel_dev, int B, float *out_dev, cudaStream_t st) {
    const int T = m->T, M = B * T, NM = m->cfg.n_mels, T0 = m->cfg.n_frames;
    cudaError_t e = cudaSuccess;
    // ---- subsample
    parakeet::sub_conv02_kernel<<<dim3((m->W2 + parakeet::SW - 1) / parakeet::SW, (m->H2 + parakeet::SH - 1) / parakeet::SH, B), kC, 0, st>>>(
        mel_dev, NM, T0, m->H1, m->W1, m->H2, m->W2, m->c0w, m->c0b, m->c2w, m->c2b, m->a2);
    const int R2 = B * m->H2 * m->W2, R3 = B * T * m->W3;
    e = gemm_bf16(m->a2, kC, m->c3w, kC, R2, kC, kC, m->c3b, nullptr, 0, 2, m->a3, kC, st);
    if (!e) {
        parakeet::dw_s2_kernel<<<dim3(m->W3, T, B), kC, 0, st>>>(m->a3, m->H2, m->W2, T, m->W3, m->c5w, m->c5b, m->a5);
        e = gemm_bf16(m->a5, kC, m->c6w, kC, R3, kC, kC, m->c6b, nullptr, 0, 2, m->a6, kC, st);
    }
    if (!e) e = gemm_bf16(m->a6, kC * m->W3, m->outw, kC * m->W3, M, kD, kC * m->W3, m->outb, nullptr, 0, 0, nullptr,
                          kD, st, 0, m->x);
    // ---- blocks
    for (size_t li = 0; li < m->layers.size() && !e; li++) {
        const auto &L = m->layers[li];
        if ((e = ffn(m, L.ln_ff1, L.ff1a, L.ff1b, B, st))) break;
        // rel-pos MHSA
        run_ln(m, L.ln_att, B, true, st);
        if ((e = lin(m, L.qkv, M, 3 * kD, kD, 0, nullptr, 1.0f, m->qkvb, nullptr, st))) break;
        if ((e = cudaMemsetAsync(m->amax, 0, sizeof(unsigned) * B, st))) break;
        parakeet::relpos_attention_kernel<<<dim3(parakeet::H, B), parakeet::ATT_THREADS, parakeet::ATT_SMEM, st>>>(
            m->qkvb, L.pm, L.pos_u, L.pos_v, T, m->ctx, m->amax);
        if ((e = quant(m, m->ctx, kD, B, st))) break;
        if ((e = lin(m, L.out, M, kD, kD, 0, m->x, 1.0f, m->x, nullptr, st))) break;
        // conv module
        run_ln(m, L.ln_conv, B, true, st);
        if ((e = lin(m, L.pw1, M, 2 * kD, kD, 3, nullptr, 1.0f, m->ctx, nullptr, st))) break;
        parakeet::dwconv_silu_quant_kernel<<<B * parakeet::CLUSTER, 512, 0, st>>>(m->ctx, T, L.dw_w, L.dw_b, m->q8,
                                                                                 m->sa);
        if ((e = lin(m, L.pw2, M, kD, kD, 0, m->x, 1.0f, m->x, nullptr, st))) break;
        if ((e = ffn(m, L.ln_ff2, L.ff2a, L.ff2b, B, st))) break;
        run_ln(m, L.ln_out, B, false, st);
    }
    if (!e) e = cudaMemcpyAsync(out_dev, m->x, sizeof(float) * (size_t)M * kD, cudaMemcpyDeviceToDevice, st);
    if (!e) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_parakeet_encode_device: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" {

// The rel-pos attention brick alone (relpos_mha.cc's contract; attention_core, encoder.rs:285-414)
int xdna_relpos_mha(const float *qkv_dev, const float *pm_dev, const float *pos_u_dev, const float *pos_v_dev, int T,
                    int B, float *ctx_dev, void *stream) {
    if (!qkv_dev || !pm_dev || !pos_u_dev || !pos_v_dev || !ctx_dev || T < 1 || T > parakeet::MAX_T || B < 1 ||
        B > 65535) {
        set_last_error_message("xdna_relpos_mha: null pointer, or T outside 1..128, or B outside 1..65535");
        return -1;
    }
    cudaError_t e = cudaFuncSetAttribute(parakeet::relpos_attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, parakeet::ATT_SMEM);
    if (e == cudaSuccess) {
        parakeet::relpos_attention_kernel<<<dim3(parakeet::H, B), parakeet::ATT_THREADS, parakeet::ATT_SMEM,
                                            static_cast<cudaStream_t>(stream)>>>(qkv_dev, pm_dev, pos_u_dev,
                                                                                  pos_v_dev, T, ctx_dev, nullptr);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_relpos_mha: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// The second call with the same (batch, input, output) captures the forward into a CUDA graph
// on a private stream; that call and later ones replay it on `stream` (one launch instead of
// ~500).  The first call runs eagerly, so every kernel attribute is set before any capture.
int xdna_parakeet_encode_device(XdnaParakeet *m, const float *mel_dev, int B, float *out_dev, void *stream) {
    if (!m || !mel_dev || !out_dev) { set_last_error_message("xdna_parakeet_encode_device: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch) {
        set_last_error_message("xdna_parakeet_encode_device: batch beyond max_batch");
        return -1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    XdnaParakeet::Graph *g = nullptr;
    for (auto &x : m->graphs)
        if (x.B == B && x.mel == mel_dev && x.out == out_dev) g = &x;
    if (!g) {
        m->graphs.push_back({B, mel_dev, out_dev, 0, nullptr});
        g = &m->graphs.back();
    }
    if (g->calls++ == 0) return parakeet_enqueue(m, mel_dev, B, out_dev, st);
    if (!g->exec) {
        cudaError_t e = m->cap ? cudaSuccess : cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking);
        cudaGraph_t graph = nullptr;
        if (!e) e = cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal);
        if (e) {
            set_last_error_message(std::string("xdna_parakeet_encode_device: capture: ") + cudaGetErrorString(e));
            return -1;
        }
        const int rc = parakeet_enqueue(m, mel_dev, B, out_dev, m->cap);
        e = cudaStreamEndCapture(m->cap, &graph);
        if (rc != 0) { if (graph) cudaGraphDestroy(graph); return -1; }
        if (!e) e = cudaGraphInstantiate(&g->exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e) {
            g->exec = nullptr;
            set_last_error_message(std::string("xdna_parakeet_encode_device: graph: ") + cudaGetErrorString(e));
            return -1;
        }
    }
    const cudaError_t e = cudaGraphLaunch(g->exec, st);
    if (e) {
        set_last_error_message(std::string("xdna_parakeet_encode_device: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int xdna_parakeet_encode(XdnaParakeet *m, const float *mel, int B, float *out) {
    if (!m || !mel || !out) { set_last_error_message("xdna_parakeet_encode: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch) { set_last_error_message("xdna_parakeet_encode: batch beyond max_batch"); return -1; }
    try {
        const size_t nm = (size_t)B * m->cfg.n_mels * m->cfg.n_frames, no = (size_t)B * m->T * kD;
        ck(cudaMemcpy(m->mel, mel, sizeof(float) * nm, cudaMemcpyHostToDevice), "copy mel");
        if (xdna_parakeet_encode_device(m, m->mel, B, m->outf, nullptr) != 0) return -1;
        ck(cudaMemcpy(out, m->outf, sizeof(float) * no, cudaMemcpyDeviceToHost), "copy out");
        if (gemm_error_and_clear()) { set_last_error_message("xdna_parakeet_encode: a GEMM wait expired"); return -1; }
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_parakeet_encode: ") + ex.what());
        return -1;
    }
}

}  // extern "C"
