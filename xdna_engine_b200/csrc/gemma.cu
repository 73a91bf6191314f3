// gemma.cu -- Gemma-3 text decoder (GEMMA3_1B shapes) on B200: B streams in lockstep, int8
// per-channel weights, optional tensor parallelism across GPUs.
//
// The reference has no Gemma decode step (rust/npu-gemma/src/lib.rs:30-43 lists what to
// reuse); this is the HF Gemma-3 text model with npu-gemma's pieces (rmsnorm_ref lib.rs:55-64,
// geglu_ref 68-77, is_global_layer config.rs:131-133).  Per token and layer:
//   in-norm (bf16 out) -> int8 GEMV q | k | v (tensor cores, row scales in the epilogue)
//   -> q/k RMS norms + RoPE + cache append -> split GQA attention (the 4 q heads share the one
//   K/V head; local layers over the last 512 positions of a ring buffer, global layers over
//   all) + ordered merge -> GEMV o -> [all-reduce] -> post-attention norm + residual + pre-FFN
//   norm -> GEMV gate|up (rows interleaved in groups of 8, GeGLU in the epilogue)
//   -> GEMV down -> [all-reduce] -> post-FFN norm + residual + next in-norm;
//   final norm -> vocabulary-sharded int8 LM head -> per-rank argmax -> [gather] -> token.
// Tensor parallel (rank r of P): q heads, gate/up columns, the o / down input rows and the
// LM head's vocabulary rows are split; the single K/V head is replicated.  The all-reduce sums
// the P partial vectors in rank order from every peer's buffer (CUDA IPC peer pointers,
// flag-tagged words with bounded waits), so every rank gets the same bits.
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

namespace gm {

constexpr int HD = 256;              // head dim
constexpr int MAXB = 64;             // streams
constexpr int GW = 16;               // warps per GEMV CTA (one staged input range, 16 row groups)
constexpr int AK = 64;               // keys per attention split
constexpr int MAXTP = 8;

enum { OUT_F32 = 0, OUT_GEGLU_BF16 = 1 };

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// two int8 weights -> bf16x2 (exact: |q| <= 127)
__device__ __forceinline__ uint32_t i8x2_bf16(uint32_t m2) {
    return bf16bits((float)(int8_t)(m2 & 255u)) | (bf16bits((float)(int8_t)(m2 >> 8)) << 16);
}
__device__ __forceinline__ float gelu_tanh(float x) {   // npu-gemma lib.rs:74-77
    const float C = 0.79788456f;
    return 0.5f * x * (1.0f + tanhf(C * (x + 0.044715f * x * x * x)));
}

struct GemvArgs {
    const uint8_t *w;           // [row groups][K/16][32 lanes][8] int8 in mma fragment order
    const float *scale;         // [Np] per output row
    const uint16_t *x;          // bf16 [B][K]
    int B, N, K, nsplit, kchunk;
    float *part;                // [nsplit][Np][MAXB]
    unsigned *count;            // [row groups]
    int mode;
    float *out;                 // OUT_F32: [B][ldo]
    uint16_t *out_bf16;         // OUT_GEGLU_BF16: [B][ldo], column = row group * 8 + g
    int ldo;
};

// Y[b][n] = (X[b] . Wq[n]) * scale[n]: the bfp16 GEMV design of whisper_dec.cu with per-row
// int8 scales (warp = 16 rows x one K range, the next 8 k-steps in flight, deterministic
// split-K reduction by the last warp).  OUT_GEGLU_BF16: row group = 8 gate rows then the 8
// matching up rows; the epilogue writes gelu_tanh(gate) * up.
template <int NT>
__global__ void __launch_bounds__(GW * 32) i8_gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint16_t xs[];
    __shared__ int last_flag[GW];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int split = blockIdx.y, n_rg = (a.N + 15) / 16;
    const int k0 = split * a.kchunk, xld = a.kchunk + 8;
    for (int i = threadIdx.x; i < NT * 8 * (a.kchunk / 8); i += blockDim.x) {
        const int b = i / (a.kchunk / 8), c = i % (a.kchunk / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (b < a.B) v = *reinterpret_cast<const uint4 *>(a.x + (size_t)b * a.K + k0 + c * 8);
        *reinterpret_cast<uint4 *>(&xs[b * xld + c * 8]) = v;
    }
    __syncthreads();
    // the staged input range serves every row group this warp owns (grid-strided)
    for (int rg = blockIdx.x * GW + warp; rg < n_rg; rg += gridDim.x * GW) {
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    const int nks = a.K / 16, nst = a.kchunk / 16, ngrp = (nst + 7) / 8;
    const uint2 *mp = reinterpret_cast<const uint2 *>(a.w) + ((size_t)rg * nks + k0 / 16) * 32 + lane;
    uint2 mv[8], mn[8];
#pragma unroll
    for (int s = 0; s < 8; s++) mv[s] = s < nst ? __ldcs(mp + s * 32) : make_uint2(0, 0);
    for (int gi = 0; gi < ngrp; gi++) {
        if (gi + 1 < ngrp) {
#pragma unroll
            for (int s = 0; s < 8; s++)
                mn[s] = (gi + 1) * 8 + s < nst ? __ldcs(mp + ((gi + 1) * 8 + s) * 32) : make_uint2(0, 0);
        }
#pragma unroll
        for (int s = 0; s < 8; s++) {
            if (gi * 8 + s >= nst) break;
            const uint32_t a0 = i8x2_bf16(mv[s].x & 0xffffu), a1 = i8x2_bf16(mv[s].x >> 16);
            const uint32_t a2 = i8x2_bf16(mv[s].y & 0xffffu), a3 = i8x2_bf16(mv[s].y >> 16);
            const int kk = (gi * 8 + s) * 16;
#pragma unroll
            for (int n = 0; n < NT; n++) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(&xs[(n * 8 + g) * xld + kk + 2 * t]);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(&xs[(n * 8 + g) * xld + kk + 8 + 2 * t]);
                mma16816(acc[n], a0, a1, a2, a3, b0, b1);
            }
        }
#pragma unroll
        for (int s = 0; s < 8; s++) mv[s] = mn[s];
    }
    const int n0 = rg * 16, Np = n_rg * 16;
    if (a.nsplit > 1) {
        float *pp = a.part + (size_t)split * Np * MAXB;
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) pp[(size_t)(n0 + g + 8 * (e >> 1)) * MAXB + n * 8 + 2 * t + (e & 1)] = acc[n][e];
        __threadfence();
        __syncwarp();
        if (lane == 0) last_flag[warp] = atomicAdd(&a.count[rg], 1u) == (unsigned)a.nsplit - 1;
        __syncwarp();
        if (!last_flag[warp]) continue;
        __threadfence();
        // ordered sum over the ranges: per range, all of this lane's values are requested at once
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (int sp = 0; sp < a.nsplit; sp++) {
            const float *ps = a.part + (size_t)sp * Np * MAXB;
            float pv[NT][4];
#pragma unroll
            for (int n = 0; n < NT; n++)
#pragma unroll
                for (int e = 0; e < 4; e++) pv[n][e] = __ldcg(ps + (size_t)(n0 + g + 8 * (e >> 1)) * MAXB + n * 8 + 2 * t + (e & 1));
#pragma unroll
            for (int n = 0; n < NT; n++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[n][e] += pv[n][e];
        }
        if (lane == 0) a.count[rg] = 0;
    }
    const float s0v = a.scale[n0 + g], s1v = a.scale[n0 + g + 8];
#pragma unroll
    for (int n = 0; n < NT; n++) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int b = n * 8 + 2 * t + c;
            if (b >= a.B) continue;
            const float y0 = acc[n][c] * s0v, y1 = acc[n][2 + c] * s1v;
            if (a.mode == OUT_F32) {
                if (n0 + g < a.N) a.out[(size_t)b * a.ldo + n0 + g] = y0;
                if (n0 + g + 8 < a.N) a.out[(size_t)b * a.ldo + n0 + g + 8] = y1;
            } else {
                a.out_bf16[(size_t)b * a.ldo + rg * 8 + g] = (uint16_t)bf16bits(gelu_tanh(y0) * y1);
            }
        }
    }
    }
}

// RMS norm of a row held by one warp: v[i] = x[lane + 32 i], D = 32 * NPL
template <int NPL>
__device__ __forceinline__ float rms_inv(const float (&v)[NPL], int D, float eps) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NPL; i++) s += v[i] * v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return 1.0f / sqrtf(s / (float)D + eps);
}

// x[b] = embed[tok[b]] * sqrt(D); xn = bf16(rms(x) * (1 + w)); one warp per stream
template <int NPL>
__global__ void embed_norm_kernel(const int64_t *__restrict__ tok, const float *__restrict__ emb, float es, int B,
                                  const float *__restrict__ w, float eps, float *__restrict__ x,
                                  uint16_t *__restrict__ xn) {
    const int b = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    constexpr int D = 32 * NPL;
    const float *er = emb + (size_t)tok[b] * D;
    float v[NPL], wv[NPL];
#pragma unroll
    for (int i = 0; i < NPL; i++) { v[i] = er[lane + 32 * i] * es; wv[i] = w[lane + 32 * i]; }
    const float inv = rms_inv<NPL>(v, D, eps);
#pragma unroll
    for (int i = 0; i < NPL; i++) {
        x[(size_t)b * D + lane + 32 * i] = v[i];
        xn[(size_t)b * D + lane + 32 * i] = (uint16_t)bf16bits(v[i] * inv * (1.0f + wv[i]));
    }
}

// x += rms(y) * (1 + w_post); xn = bf16(rms(x) * (1 + w_next)); one warp per stream
template <int NPL>
__global__ void post_add_norm_kernel(const float *__restrict__ y, int B, const float *__restrict__ wpost,
                                     const float *__restrict__ wnext, float eps, float *__restrict__ x,
                                     uint16_t *__restrict__ xn) {
    const int b = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    constexpr int D = 32 * NPL;
    float v[NPL], xv[NPL], wp[NPL], wn[NPL];
#pragma unroll
    for (int i = 0; i < NPL; i++) {
        v[i] = y[(size_t)b * D + lane + 32 * i];
        xv[i] = x[(size_t)b * D + lane + 32 * i];
        wp[i] = wpost[lane + 32 * i];
        wn[i] = wnext[lane + 32 * i];
    }
    const float inv = rms_inv<NPL>(v, D, eps);
#pragma unroll
    for (int i = 0; i < NPL; i++) xv[i] += v[i] * inv * (1.0f + wp[i]);
    const float inv2 = rms_inv<NPL>(xv, D, eps);
#pragma unroll
    for (int i = 0; i < NPL; i++) {
        x[(size_t)b * D + lane + 32 * i] = xv[i];
        xn[(size_t)b * D + lane + 32 * i] = (uint16_t)bf16bits(xv[i] * inv2 * (1.0f + wn[i]));
    }
}

// per stream: q heads (local) and k: RMS norm over 256 + RoPE (rotate-half, theta); k, v into
// the cache slot of position pos (ring slot pos % len for local layers); q f32 out.
// qkv rows: [hq * 256 q | 256 k | 256 v]; one CTA of 256 threads per stream, thread = dim.
__global__ void __launch_bounds__(HD) qk_prep_kernel(const float *__restrict__ qkv, int hq, const int *posp,
                                                     float theta, const float *__restrict__ qn,
                                                     const float *__restrict__ kn, float eps, int cache_len,
                                                     uint16_t *__restrict__ kc, uint16_t *__restrict__ vc,
                                                     float *__restrict__ qo) {
    __shared__ float row[HD], red[8];
    const int b = blockIdx.x, d = threadIdx.x, pos = *posp;
    const int ld = (hq + 2) * HD;
    const float *r = qkv + (size_t)b * ld;
    const int h2 = HD / 2, i = d % h2;
    const float f = (float)pos * (1.0f / powf(theta, (float)(2 * i) / (float)HD));
    const float cs = cosf(f), sn = sinf(f);
    const size_t slot = (size_t)b * cache_len + pos % cache_len;
    for (int hh = 0; hh <= hq; hh++) {          // hq q heads, then k
        const float v = r[hh * HD + d];
        float s = v * v;
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if ((d & 31) == 0) red[d >> 5] = s;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) tot += red[w];
        const float inv = 1.0f / sqrtf(tot / (float)HD + eps);
        const float nv = v * inv * (1.0f + (hh < hq ? qn[d] : kn[d]));
        row[d] = nv;
        __syncthreads();
        const float o = d < h2 ? nv * cs - row[d + h2] * sn : nv * cs + row[d - h2] * sn;
        if (hh < hq) qo[((size_t)b * hq + hh) * HD + d] = o;
        else kc[slot * HD + d] = (uint16_t)bf16bits(o);
        __syncthreads();
    }
    vc[slot * HD + d] = (uint16_t)bf16bits(r[(hq + 1) * HD + d]);
}

// split attention: block (split s, stream b) takes AK cache slots; every local q head against
// the shared K/V head; writes per head (max, sum, acc[256]).  Keys visible: positions
// [lo, pos] with lo = max(0, pos - window + 1) for local layers (ring of cache_len slots).
__global__ void __launch_bounds__(256) gqa_attn_kernel(const float *__restrict__ q, int hq, const int *posp,
                                                       int window, int cache_len, const uint16_t *__restrict__ kc,
                                                       const uint16_t *__restrict__ vc, float scaling,
                                                       float *__restrict__ part, int nsplit) {
    extern __shared__ __align__(16) uint16_t kv[];           // K [AK][HD] then V [AK][HD]
    __shared__ float qs[4][HD], sc[4][AK], stat[4][2];
    const int s = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, pos = *posp;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int p0 = lo + s * AK;
    const int nk = max(0, min(AK, pos + 1 - p0));
    float *pp = part + ((size_t)b * nsplit + s) * 4 * (HD + 2);
    if (nk == 0) {
        if (tid < hq) { pp[tid * (HD + 2)] = -INFINITY; pp[tid * (HD + 2) + 1] = 0.0f; }
        for (int i = tid; i < hq * HD; i += 256) pp[(i / HD) * (HD + 2) + 2 + i % HD] = 0.0f;
        return;
    }
    uint16_t *ks = kv, *vs = kv + AK * HD;
    for (int i = tid; i < nk * (HD / 8); i += 256) {
        const int j = i / (HD / 8), c = i % (HD / 8);
        const size_t slot = (size_t)b * cache_len + (p0 + j) % cache_len;
        reinterpret_cast<uint4 *>(ks)[i] = reinterpret_cast<const uint4 *>(kc + slot * HD)[c];
        reinterpret_cast<uint4 *>(vs)[i] = reinterpret_cast<const uint4 *>(vc + slot * HD)[c];
    }
    for (int i = tid; i < hq * HD; i += 256) qs[i / HD][i % HD] = q[(size_t)b * hq * HD + i];
    __syncthreads();
    // scores: thread = (head, key)
    {
        const int hh = tid / AK, j = tid % AK;
        if (hh < hq) {
            float dot = -INFINITY;
            if (j < nk) {
                dot = 0.0f;
                const uint4 *kr = reinterpret_cast<const uint4 *>(ks + j * HD);
#pragma unroll 4
                for (int c0 = 0; c0 < HD / 8; c0++) {
                    const int c = (c0 + j) & (HD / 8 - 1);
                    const uint4 w = kr[c];
                    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) dot += qs[hh][8 * c + 2 * e] * bf16lo(u[e]) + qs[hh][8 * c + 2 * e + 1] * bf16hi(u[e]);
                }
                dot *= scaling;
            }
            sc[hh][j] = dot;
        }
    }
    __syncthreads();
    // per head max / exp / sum: warp w < hq (two keys per lane)
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < hq) {
        const float a0 = sc[warp][lane], a1 = sc[warp][lane + 32];
        float m = fmaxf(a0, a1);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float e0 = lane < nk ? expf(a0 - m) : 0.0f, e1 = lane + 32 < nk ? expf(a1 - m) : 0.0f;
        float l = e0 + e1;
#pragma unroll
        for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        sc[warp][lane] = e0;
        sc[warp][lane + 32] = e1;
        if (lane == 0) { stat[warp][0] = m; stat[warp][1] = l; }
    }
    __syncthreads();
    // acc[head][d]: thread = d, loop heads
    for (int hh = 0; hh < hq; hh++) {
        float a = 0.0f;
        for (int j = 0; j < nk; j++) a += sc[hh][j] * bf16lo(vs[j * HD + tid]);
        pp[hh * (HD + 2) + 2 + tid] = a;
    }
    if (tid < hq) { pp[tid * (HD + 2)] = stat[tid][0]; pp[tid * (HD + 2) + 1] = stat[tid][1]; }
}

// fold the splits in order -> ctx bf16 [B][hq * 256]; block = (head, stream), thread = dim
__global__ void gqa_merge_kernel(const float *__restrict__ part, int hq, int nsplit, uint16_t *__restrict__ ctx) {
    const int hh = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    float M = -INFINITY, L = 0.0f, A = 0.0f;
    for (int s0 = 0; s0 < nsplit; s0 += 8) {
        float m[8], l[8], a[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const float *pp = part + (((size_t)b * nsplit + s0 + u) * 4 + hh) * (HD + 2);
            m[u] = s0 + u < nsplit ? pp[0] : -INFINITY;
            l[u] = s0 + u < nsplit ? pp[1] : 0.0f;
            a[u] = s0 + u < nsplit ? pp[2 + d] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            if (m[u] == -INFINITY) continue;
            const float mn = fmaxf(M, m[u]);
            const float c0 = M == -INFINITY ? 0.0f : expf(M - mn), c1 = expf(m[u] - mn);
            L = L * c0 + l[u] * c1;
            A = A * c0 + a[u] * c1;
            M = mn;
        }
    }
    ctx[((size_t)b * hq + hh) * HD + d] = (uint16_t)bf16bits(A / L);
}

// per stream: the first maximum of this rank's logit slice -> (value, global index)
__global__ void __launch_bounds__(1024) argmax_local_kernel(const float *__restrict__ logits, int n, int ldl,
                                                            int base, float *__restrict__ bestv, int *__restrict__ besti) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float *lr = logits + (size_t)b * ldl;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = tid; i < n; i += blockDim.x) {
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
        for (int w = 1; w < 32; w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        bestv[b] = best;
        besti[b] = base + idx;
    }
}

// next token per stream from the P ranks' (value, index) pairs (first maximum overall), or the
// prompt while it lasts; records generated tokens; the last block advances *pos
__global__ void pick_kernel(const float *bestv, const int *besti, int P, int B, const int64_t *prompt, int n_prompt,
                            int *posp, int64_t *tok, int64_t *out, int n_new, unsigned *done) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    const int pos = *posp;
    if (b < B) {
        float best = -INFINITY;
        int idx = 0x7fffffff;
        for (int r = 0; r < P; r++) {
            const float v = bestv[r * MAXB + b];
            const int i = besti[r * MAXB + b];
            if (v > best || (v == best && i < idx)) { best = v; idx = i; }
        }
        int64_t next;
        if (pos + 1 < n_prompt) next = prompt[(size_t)b * n_prompt + pos + 1];
        else {
            next = idx;
            const int step = pos + 1 - n_prompt;
            if (step < n_new) out[(size_t)b * n_new + step] = idx;
        }
        tok[b] = next;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) { *done = 0; *posp = pos + 1; }
    }
}

// All-reduce across the tensor-parallel ranks, in rank order from every rank's published
// partial: this rank copies its partial y [n] into its own slot of its exchange buffer as
// flag-tagged 64-bit words (epoch << 32 | bits), every rank then polls the P slots (its own and
// the peers', through IPC pointers) until they carry `epoch` and sums them r = 0 .. P-1.
// The wait is bounded: after ~1 s the kernel records an error and returns.
// Two slots per rank alternate by epoch parity: a rank can be at most one exchange ahead of
// any peer (it cannot finish exchange e+1 before every peer has finished exchange e), so the
// slot it overwrites at e+2 has been read.  Slot layout: bufs[r][parity][n].
__global__ void tp_allreduce_kernel(const float *__restrict__ y, int n, uint64_t *const *bufs, int P, int rank,
                                    uint32_t epoch, float *__restrict__ out, unsigned *err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t slot = (size_t)(epoch & 1u) * n;
    if (i < n) {
        const uint64_t wv = ((uint64_t)epoch << 32) | __float_as_uint(y[i]);
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(bufs[rank] + slot + i), "l"(wv) : "memory");
    }
    if (i >= n) return;
    float sum = 0.0f;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < P; r++) {
        const uint64_t *src = bufs[r] + slot + i;
        uint64_t v;
        while (true) {
            asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            if ((uint32_t)(v >> 32) == epoch) break;
            if (globaltimer_ns() - t0 > 1000000000ull) { atomicCAS(err, 0u, 1u); return; }
        }
        sum += __uint_as_float((uint32_t)v);
    }
    out[i] = sum;
}

// gather every rank's per-stream (value, index) pairs through the same exchange slots
__global__ void tp_gather_best_kernel(int B, uint64_t *const *bufs, int P, int rank, uint32_t epoch, float *bestv,
                                      int *besti, unsigned *err) {
    const int i = threadIdx.x;                     // 2 * MAXB words: values then indices
    const int n = 2 * MAXB;
    const size_t slot = (size_t)(epoch & 1u) * n;
    if (i < n) {
        const uint32_t bits = i < MAXB ? __float_as_uint(bestv[rank * MAXB + i]) : (uint32_t)besti[rank * MAXB + i - MAXB];
        const uint64_t wv = ((uint64_t)epoch << 32) | bits;
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(bufs[rank] + slot + i), "l"(wv) : "memory");
    }
    if (i >= n) return;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < P; r++) {
        if (r == rank) continue;
        const uint64_t *src = bufs[r] + slot + i;
        uint64_t v;
        while (true) {
            asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            if ((uint32_t)(v >> 32) == epoch) break;
            if (globaltimer_ns() - t0 > 1000000000ull) { atomicCAS(err, 0u, 1u); return; }
        }
        if (i < MAXB) bestv[r * MAXB + i] = __uint_as_float((uint32_t)v);
        else besti[r * MAXB + i - MAXB] = (int)(uint32_t)v;
    }
}

}  // namespace gm

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
}  // namespace
}  // namespace xdna

using namespace xdna;

struct GmMat {
    uint8_t *w = nullptr;
    float *scale = nullptr;
    int N = 0, K = 0;
};

struct XdnaGemma {
    XdnaGemmaConfig cfg{};
    int max_batch = 0, max_ctx = 0, rank = 0, tp = 1, hq = 0, f_loc = 0, v_loc = 0, v_base = 0, k_loc = 0, k_base = 0;
    struct Layer {
        GmMat qkv, o, gu, down;
        float *norms;                      // in, q, k, post_attn, pre_ffn, post_ffn (q, k: 256)
        uint16_t *kc, *vc;
        int cache_len;
        bool global;
    };
    std::vector<Layer> layers;
    GmMat lm;
    float *emb = nullptr, *final_norm = nullptr;
    // state
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *y = nullptr, *yr = nullptr, *logits = nullptr, *part = nullptr,
          *apart = nullptr, *bestv = nullptr;
    int *besti = nullptr;
    uint16_t *xn = nullptr, *ctx = nullptr, *h = nullptr;
    unsigned *count = nullptr, *done = nullptr, *err = nullptr;
    int *pos = nullptr;
    int64_t *tok = nullptr, *prompt = nullptr, *out = nullptr;
    int n_prompt_cap = 0;
    int run_B = 0, run_prompt = 0, run_new = 0, run_done = 0;   // the staged decode
    // tensor parallel exchange: bufs[r] = rank r's exchange buffer (own or IPC-mapped)
    uint64_t *xbuf = nullptr;
    uint64_t **dbufs = nullptr;
    std::vector<void *> peer_maps;
    uint32_t epoch = 0;
    std::vector<void *> owned;
    ~XdnaGemma() {
        for (void *p : peer_maps) cudaIpcCloseMemHandle(p);
        for (void *p : owned) cudaFree(p);
    }
};

namespace {
constexpr int kD = 1152, kNPL = kD / 32;

// rows = outputs; W given [K, N] with the output columns listed in `cols` (in this order);
// pack in mma fragment order with a per-row scale (Lin::load rule, opt125m_decode.rs:41-60)
GmMat pack_i8(XdnaGemma *m, const float *w, int K, int N, const std::vector<int> &cols) {
    const int R = (int)cols.size(), nrg = (R + 15) / 16, nks = K / 16;
    std::vector<int8_t> q((size_t)nrg * 16 * K, 0);
    std::vector<float> sc((size_t)nrg * 16, 1.0f);
    for (int r = 0; r < R; r++) {
        const int n = cols[r];
        if (n < 0) continue;                       // padding row
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = std::max(amax, std::fabs(w[(size_t)k * N + n]));
        const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        sc[r] = s;
        for (int k = 0; k < K; k++) {
            float v = std::round(w[(size_t)k * N + n] / s);
            v = std::min(127.0f, std::max(-127.0f, v));
            q[(size_t)r * K + k] = (int8_t)v;
        }
    }
    std::vector<uint8_t> packed((size_t)nrg * nks * 32 * 8);
    for (int rg = 0; rg < nrg; rg++)
        for (int ks = 0; ks < nks; ks++)
            for (int lane = 0; lane < 32; lane++) {
                const int g = lane >> 2, t = lane & 3, r0 = rg * 16 + g, r1 = r0 + 8, k = ks * 16 + 2 * t;
                const int8_t v[8] = {q[(size_t)r0 * K + k], q[(size_t)r0 * K + k + 1], q[(size_t)r1 * K + k],
                                     q[(size_t)r1 * K + k + 1], q[(size_t)r0 * K + k + 8], q[(size_t)r0 * K + k + 9],
                                     q[(size_t)r1 * K + k + 8], q[(size_t)r1 * K + k + 9]};
                std::memcpy(&packed[(((size_t)rg * nks + ks) * 32 + lane) * 8], v, 8);
            }
    GmMat o;
    o.N = R;
    o.K = K;
    o.w = dupload(packed);
    o.scale = dupload(sc);
    m->owned.push_back(o.w);
    m->owned.push_back(o.scale);
    return o;
}

// K ranges of a GEMV: as few as give every SM a CTA of warps, each a multiple of 16 of K
// (and short enough that 64 streams of the range fit the GEMV's shared staging)
constexpr int kMaxChunk = 1792;
int splits_of(int N, int K) {
    const int nrg = (N + 15) / 16, ks = K / 16;
    int nsplit = std::min({ks, 8, std::max(1, (148 * gm::GW + nrg - 1) / nrg)});   // ~ a CTA of warps per SM
    while (ks % nsplit) nsplit--;
    while (K / nsplit > kMaxChunk) {
        nsplit++;
        while (ks % nsplit) nsplit++;
    }
    return nsplit;
}

cudaError_t gemv(XdnaGemma *m, const GmMat &w, const uint16_t *x, int B, int mode, float *out, uint16_t *ob, int ldo,
                 cudaStream_t st) {
    const int nrg = (w.N + 15) / 16;
    const int nsplit = splits_of(w.N, w.K);
    const int kchunk = w.K / nsplit;
    gm::GemvArgs a{w.w, w.scale, x, B, w.N, w.K, nsplit, kchunk, m->part, m->count, mode, out, ob, ldo};
    // about one CTA per SM over all K ranges; each stages its range of X once
    dim3 grid(std::max(1, std::min((nrg + gm::GW - 1) / gm::GW, 148 / nsplit)), nsplit);
    const int nt = (B + 7) / 8;
    const size_t smem = (size_t)nt * 8 * (kchunk + 8) * 2;
    switch (nt) {
    case 1: gm::i8_gemv_kernel<1><<<grid, gm::GW * 32, smem, st>>>(a); break;
    case 2: gm::i8_gemv_kernel<2><<<grid, gm::GW * 32, smem, st>>>(a); break;
    case 3: case 4: gm::i8_gemv_kernel<4><<<grid, gm::GW * 32, smem, st>>>(a); break;
    default: gm::i8_gemv_kernel<8><<<grid, gm::GW * 32, smem, st>>>(a); break;
    }
    return cudaGetLastError();
}

// sum partial vectors y [B][D] over the ranks into out (or copy when tp == 1)
cudaError_t allreduce(XdnaGemma *m, const float *y, int B, float *out, cudaStream_t st) {
    const int n = B * kD;
    if (m->tp == 1) return cudaMemcpyAsync(out, y, sizeof(float) * n, cudaMemcpyDeviceToDevice, st);
    m->epoch++;
    gm::tp_allreduce_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, n, m->dbufs, m->tp, m->rank, m->epoch, out, m->err);
    return cudaGetLastError();
}

cudaError_t step(XdnaGemma *m, int B, int n_prompt, int n_new, cudaStream_t st) {
    using namespace gm;
    const auto &c = m->cfg;
    const float eps = c.eps;
    cudaError_t e = cudaSuccess;
    embed_norm_kernel<kNPL><<<(B + 3) / 4, 128, 0, st>>>(m->tok, m->emb, sqrtf((float)kD), B, m->layers[0].norms, eps,
                                                         m->x, m->xn);
    const int hq = m->hq;
    for (int l = 0; l < c.n_layers && !e; l++) {
        const auto &L = m->layers[l];
        const float *nrm = L.norms;
        if ((e = gemv(m, L.qkv, m->xn, B, OUT_F32, m->qkv, nullptr, (hq + 2) * HD, st))) break;
        qk_prep_kernel<<<B, HD, 0, st>>>(m->qkv, hq, m->pos, L.global ? c.theta_global : c.theta_local,
                                         nrm + kD, nrm + kD + HD, eps, L.cache_len, L.kc, L.vc, m->q);
        const int span = L.global ? m->max_ctx : c.window;
        const int nsplit = (span + AK - 1) / AK;
        gqa_attn_kernel<<<dim3(nsplit, B), 256, 2 * AK * HD * 2, st>>>(m->q, hq, m->pos, L.global ? 0 : c.window,
                                                                    L.cache_len, L.kc, L.vc,
                                                                    1.0f / sqrtf(c.query_pre_attn_scalar), m->apart, nsplit);
        gqa_merge_kernel<<<dim3(hq, B), HD, 0, st>>>(m->apart, hq, nsplit, m->ctx);
        if ((e = gemv(m, L.o, m->ctx, B, OUT_F32, m->y, nullptr, kD, st))) break;
        if ((e = allreduce(m, m->y, B, m->yr, st))) break;
        post_add_norm_kernel<kNPL><<<(B + 3) / 4, 128, 0, st>>>(m->yr, B, nrm + kD + 2 * HD, nrm + 2 * kD + 2 * HD, eps,
                                                                m->x, m->xn);
        if ((e = gemv(m, L.gu, m->xn, B, OUT_GEGLU_BF16, nullptr, m->h, m->f_loc, st))) break;
        if ((e = gemv(m, L.down, m->h, B, OUT_F32, m->y, nullptr, kD, st))) break;
        if ((e = allreduce(m, m->y, B, m->yr, st))) break;
        const float *wnext = l + 1 < c.n_layers ? m->layers[l + 1].norms : m->final_norm;
        post_add_norm_kernel<kNPL><<<(B + 3) / 4, 128, 0, st>>>(m->yr, B, nrm + 3 * kD + 2 * HD, wnext, eps, m->x, m->xn);
    }
    if (e) return e;
    const int ldl = (m->v_loc + 15) / 16 * 16;
    if ((e = gemv(m, m->lm, m->xn, B, OUT_F32, m->logits, nullptr, ldl, st))) return e;
    argmax_local_kernel<<<B, 1024, 0, st>>>(m->logits, m->v_loc, ldl, m->v_base, m->bestv + m->rank * MAXB,
                                            m->besti + m->rank * MAXB);
    if (m->tp > 1) {
        m->epoch++;
        tp_gather_best_kernel<<<1, 2 * MAXB, 0, st>>>(B, m->dbufs, m->tp, m->rank, m->epoch, m->bestv, m->besti, m->err);
    }
    pick_kernel<<<1, MAXB, 0, st>>>(m->bestv, m->besti, m->tp == 1 ? 1 : m->tp, B, m->prompt, n_prompt, m->pos, m->tok,
                                    m->out, n_new, m->done);
    return cudaGetLastError();
}
}  // namespace

extern "C" {

XdnaGemma *xdna_gemma_create(XdnaDevice *dev_unused, const XdnaGemmaConfig *cfg, const XdnaGemmaWeights *w,
                             int max_batch, int max_ctx, int tp_rank, int tp_size) {
    (void)dev_unused;
    using namespace gm;
    if (!cfg || !w || !w->layers || !w->embed || !w->final_norm) {
        set_last_error_message("xdna_gemma_create: null pointer");
        return nullptr;
    }
    const XdnaGemmaConfig c = *cfg;
    if (c.d_model != kD || c.head_dim != HD || c.n_q_heads < 1 || c.n_q_heads > 4 || c.ffn % 128 || c.n_layers < 1 ||
        c.vocab < 2 || c.window < 1 || c.pattern < 1 || max_batch < 1 || max_batch > MAXB || max_ctx < 2 ||
        tp_size < 1 || tp_size > MAXTP || tp_rank < 0 || tp_rank >= tp_size || (c.n_q_heads * HD) % (tp_size * 128) ||
        c.ffn % (tp_size * 16)) {
        set_last_error_message("xdna_gemma_create: supported shape is d_model 1152, head_dim 256, 1..4 q heads, "
                               "1..64 streams, tp 1..8 with (q heads * 256) % (128 tp) == 0 and ffn % (16 tp) == 0");
        return nullptr;
    }
    auto *m = new XdnaGemma();
    try {
        m->cfg = c;
        m->max_batch = max_batch;
        m->max_ctx = max_ctx;
        m->rank = tp_rank;
        m->tp = tp_size;
        const int QD = c.n_q_heads * HD;
        // this rank's slice of the o-projection input (and the heads covering it)
        m->k_loc = QD / tp_size;
        m->k_base = tp_rank * m->k_loc;
        const int h0 = m->k_base / HD, h1 = (m->k_base + m->k_loc + HD - 1) / HD;
        m->hq = h1 - h0;
        m->f_loc = c.ffn / tp_size;
        m->v_loc = (c.vocab + tp_size - 1) / tp_size;
        m->v_base = tp_rank * m->v_loc;
        m->v_loc = std::min(m->v_loc, c.vocab - m->v_base);
        auto keep = [&](void *p) { m->owned.push_back(p); return p; };
        auto f32 = [&](std::initializer_list<std::pair<const float *, size_t>> parts) {
            std::vector<float> v;
            for (auto &pr : parts) v.insert(v.end(), pr.first, pr.first + pr.second);
            return static_cast<float *>(keep(dupload(v)));
        };
        const size_t B = (size_t)max_batch;
        for (int l = 0; l < c.n_layers; l++) {
            const XdnaGemmaLayer &L = w->layers[l];
            XdnaGemma::Layer o{};
            o.global = (l + 1) % c.pattern == 0;
            // q|k|v: [D, QD + 2*256] as one [K, N] view assembled from the three weights
            {
                const int N = QD + 2 * HD;
                std::vector<float> cat((size_t)kD * N);
                for (int k = 0; k < kD; k++) {
                    std::memcpy(&cat[(size_t)k * N], L.wq + (size_t)k * QD, sizeof(float) * QD);
                    std::memcpy(&cat[(size_t)k * N + QD], L.wk + (size_t)k * HD, sizeof(float) * HD);
                    std::memcpy(&cat[(size_t)k * N + QD + HD], L.wv + (size_t)k * HD, sizeof(float) * HD);
                }
                std::vector<int> cols;
                for (int n = h0 * HD; n < h1 * HD; n++) cols.push_back(n);
                for (int n = QD; n < N; n++) cols.push_back(n);
                o.qkv = pack_i8(m, cat.data(), kD, N, cols);
            }
            {   // o: rows = D outputs over this rank's input slice [k_base, k_base + k_loc) of ctx
                // the local ctx holds heads h0..h1; the slice starts at k_base - h0*HD
                const int off = m->k_base - h0 * HD, Kl = m->hq * HD;
                std::vector<float> sub((size_t)Kl * kD, 0.0f);
                for (int k = 0; k < m->k_loc; k++)
                    std::memcpy(&sub[(size_t)(off + k) * kD], L.wo + (size_t)(m->k_base + k) * kD, sizeof(float) * kD);
                std::vector<int> cols(kD);
                for (int n = 0; n < kD; n++) cols[n] = n;
                o.o = pack_i8(m, sub.data(), Kl, kD, cols);
            }
            {   // gate|up interleaved in groups of 8 over this rank's ffn columns
                const int F = c.ffn, f0 = tp_rank * m->f_loc;
                std::vector<float> cat((size_t)kD * 2 * F);
                for (int k = 0; k < kD; k++) {
                    std::memcpy(&cat[(size_t)k * 2 * F], L.wg + (size_t)k * F, sizeof(float) * F);
                    std::memcpy(&cat[(size_t)k * 2 * F + F], L.wu + (size_t)k * F, sizeof(float) * F);
                }
                std::vector<int> cols;
                for (int g8 = 0; g8 < m->f_loc; g8 += 8) {
                    for (int i = 0; i < 8; i++) cols.push_back(f0 + g8 + i);
                    for (int i = 0; i < 8; i++) cols.push_back(F + f0 + g8 + i);
                }
                o.gu = pack_i8(m, cat.data(), kD, 2 * F, cols);
            }
            {   // down: rows = D over this rank's ffn slice
                const int f0 = tp_rank * m->f_loc;
                std::vector<int> cols(kD);
                for (int n = 0; n < kD; n++) cols[n] = n;
                o.down = pack_i8(m, L.wd + (size_t)f0 * kD, m->f_loc, kD, cols);
            }
            o.norms = f32({{L.in_norm, (size_t)kD}, {L.q_norm, (size_t)HD}, {L.k_norm, (size_t)HD},
                           {L.post_attn_norm, (size_t)kD}, {L.pre_ffn_norm, (size_t)kD}, {L.post_ffn_norm, (size_t)kD}});
            o.cache_len = o.global ? max_ctx : std::min(c.window, max_ctx);
            o.kc = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * o.cache_len * HD)));
            o.vc = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * o.cache_len * HD)));
            m->layers.push_back(o);
        }
        {   // tied LM head over this rank's vocabulary rows: logits[v] = h . E[v] ([K = D, N = V] view)
            std::vector<float> et((size_t)kD * m->v_loc);
            for (int v = 0; v < m->v_loc; v++)
                for (int d = 0; d < kD; d++) et[(size_t)d * m->v_loc + v] = w->embed[(size_t)(m->v_base + v) * kD + d];
            std::vector<int> cols(m->v_loc);
            for (int v = 0; v < m->v_loc; v++) cols[v] = v;
            m->lm = pack_i8(m, et.data(), kD, m->v_loc, cols);
        }
        m->emb = f32({{w->embed, (size_t)c.vocab * kD}});
        m->final_norm = f32({{w->final_norm, (size_t)kD}});
        const int hqmax = 4, ldl = (m->v_loc + 15) / 16 * 16;
        m->x = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->qkv = static_cast<float *>(keep(dalloc<float>(B * (hqmax + 2) * HD)));
        m->q = static_cast<float *>(keep(dalloc<float>(B * hqmax * HD)));
        m->y = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->yr = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->logits = static_cast<float *>(keep(dalloc<float>(B * ldl)));
        size_t part = 0, rows_max = 0;
        auto acct = [&](const GmMat &g) {
            const size_t np = (size_t)(g.N + 15) / 16 * 16;
            rows_max = std::max(rows_max, np);
            const int ns = splits_of(g.N, g.K);
            if (ns > 1) part = std::max(part, (size_t)ns * np);
        };
        for (auto &L : m->layers) { acct(L.qkv); acct(L.o); acct(L.gu); acct(L.down); }
        acct(m->lm);
        m->part = static_cast<float *>(keep(dalloc<float>(std::max<size_t>(part, 1) * MAXB)));
        const int nsplit_max = (std::max(max_ctx, c.window) + AK - 1) / AK;
        m->apart = static_cast<float *>(keep(dalloc<float>(B * nsplit_max * 4 * (HD + 2))));
        m->bestv = static_cast<float *>(keep(dalloc<float>(MAXTP * MAXB)));
        m->besti = static_cast<int *>(keep(dalloc<int>(MAXTP * MAXB)));
        m->xn = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * kD)));
        m->ctx = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * hqmax * HD)));
        m->h = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * m->f_loc)));
        const size_t rg_max = rows_max / 16 + 1;
        m->count = static_cast<unsigned *>(keep(dalloc<unsigned>(rg_max)));
        m->done = static_cast<unsigned *>(keep(dalloc<unsigned>(1)));
        m->err = static_cast<unsigned *>(keep(dalloc<unsigned>(1)));
        m->pos = static_cast<int *>(keep(dalloc<int>(1)));
        m->tok = static_cast<int64_t *>(keep(dalloc<int64_t>(B)));
        m->out = static_cast<int64_t *>(keep(dalloc<int64_t>(B * max_ctx)));
        ck(cudaMemset(m->count, 0, sizeof(unsigned) * rg_max), "memset");
        ck(cudaMemset(m->done, 0, 4), "memset");
        ck(cudaMemset(m->err, 0, 4), "memset");
        ck(cudaMemset(m->bestv, 0, sizeof(float) * MAXTP * MAXB), "memset");
        ck(cudaMemset(m->besti, 0, sizeof(int) * MAXTP * MAXB), "memset");
        ck(cudaFuncSetAttribute(gqa_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * AK * HD * 2), "smem");
        const int gsm = 8 * 8 * (kMaxChunk + 8) * 2;      // the widest K range of 64 streams
        ck(cudaFuncSetAttribute(i8_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        if (tp_size > 1) {
            // exchange buffer [2 parities][MAXB * D] of 64-bit words; zero = epoch 0 (never used)
            const size_t words = (size_t)2 * MAXB * kD;
            m->xbuf = static_cast<uint64_t *>(keep(dalloc<uint64_t>(words)));
            ck(cudaMemset(m->xbuf, 0, words * 8), "memset");
            m->dbufs = static_cast<uint64_t **>(keep(dalloc<uint64_t *>(MAXTP)));
        }
        ck(cudaDeviceSynchronize(), "create sync");
        return m;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_gemma_create: ") + ex.what());
        delete m;
        return nullptr;
    }
}

void xdna_gemma_free(XdnaGemma *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    delete m;
}

// The IPC handle of this rank's exchange buffer (tensor parallel only): 64 bytes to share
int xdna_gemma_ipc_handle(XdnaGemma *m, void *handle64) {
    if (!m || !handle64 || m->tp == 1) { set_last_error_message("xdna_gemma_ipc_handle: not tensor parallel"); return -1; }
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, m->xbuf);
    if (e) { set_last_error_message(std::string("xdna_gemma_ipc_handle: ") + cudaGetErrorString(e)); return -1; }
    std::memcpy(handle64, &h, sizeof h);
    return 0;
}

// Open the peers' exchange buffers: handles [tp][64 bytes] in rank order (own entry ignored)
int xdna_gemma_connect(XdnaGemma *m, const void *handles) {
    if (!m || !handles || m->tp == 1) { set_last_error_message("xdna_gemma_connect: not tensor parallel"); return -1; }
    std::vector<uint64_t *> ptrs(gm::MAXTP, nullptr);
    for (int r = 0; r < m->tp; r++) {
        if (r == m->rank) { ptrs[r] = m->xbuf; continue; }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + 64 * r, sizeof h);
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e) { set_last_error_message(std::string("xdna_gemma_connect: ") + cudaGetErrorString(e)); return -1; }
        m->peer_maps.push_back(p);
        ptrs[r] = static_cast<uint64_t *>(p);
    }
    const cudaError_t e = cudaMemcpy(m->dbufs, ptrs.data(), sizeof(uint64_t *) * gm::MAXTP, cudaMemcpyHostToDevice);
    if (e) { set_last_error_message(std::string("xdna_gemma_connect: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

// Stage a greedy decode of B streams: prompts [B][n_prompt] (host), n_new tokens each.  The
// n_prompt - 1 + n_new steps then run through xdna_gemma_steps (the first n_prompt - 1 are the
// prefill).  Synchronous.
int xdna_gemma_begin(XdnaGemma *m, int B, const int64_t *prompts, int n_prompt, int n_new) {
    if (!m || !prompts) { set_last_error_message("xdna_gemma_begin: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch || n_prompt < 1 || n_new < 1 || n_prompt + n_new > m->max_ctx) {
        set_last_error_message("xdna_gemma_begin: bad batch or prompt + new tokens beyond max_ctx");
        return -1;
    }
    for (size_t i = 0; i < (size_t)B * n_prompt; i++)
        if (prompts[i] < 0 || prompts[i] >= m->cfg.vocab) {
            set_last_error_message("xdna_gemma_begin: prompt token out of range");
            return -1;
        }
    try {
        if (n_prompt * B > m->n_prompt_cap) {
            if (m->prompt) cudaFree(m->prompt);
            m->prompt = dalloc<int64_t>((size_t)n_prompt * B);
            m->n_prompt_cap = n_prompt * B;
        }
        std::vector<int64_t> t0(B);
        for (int b = 0; b < B; b++) t0[b] = prompts[(size_t)b * n_prompt];
        const int zero = 0;
        ck(cudaDeviceSynchronize(), "sync");
        ck(cudaMemcpy(m->prompt, prompts, sizeof(int64_t) * B * n_prompt, cudaMemcpyHostToDevice), "prompt");
        ck(cudaMemcpy(m->tok, t0.data(), sizeof(int64_t) * B, cudaMemcpyHostToDevice), "tokens");
        ck(cudaMemcpy(m->pos, &zero, sizeof(int), cudaMemcpyHostToDevice), "pos");
        m->run_B = B;
        m->run_prompt = n_prompt;
        m->run_new = n_new;
        m->run_done = 0;
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_gemma_begin: ") + ex.what());
        return -1;
    }
}

// Enqueue the next n_steps steps of the staged decode on `stream` (asynchronous; every rank of a
// tensor-parallel group makes the same calls).
int xdna_gemma_steps(XdnaGemma *m, int n_steps, void *stream) {
    if (!m || m->run_B == 0) { set_last_error_message("xdna_gemma_steps: nothing staged"); return -1; }
    if (n_steps < 0 || m->run_done + n_steps > m->run_prompt + m->run_new - 1) {
        set_last_error_message("xdna_gemma_steps: beyond the staged decode");
        return -1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int s = 0; s < n_steps; s++) {
        const cudaError_t e = step(m, m->run_B, m->run_prompt, m->run_new, st);
        if (e) { set_last_error_message(std::string("xdna_gemma_steps: ") + cudaGetErrorString(e)); return -1; }
        m->run_done++;
    }
    return 0;
}

// Wait for the staged decode and copy its tokens [B][n_new] to the host; -1 also when a peer
// exchange timed out.
int xdna_gemma_tokens(XdnaGemma *m, int64_t *tokens_host, void *stream) {
    if (!m || !tokens_host || m->run_B == 0) { set_last_error_message("xdna_gemma_tokens: nothing staged"); return -1; }
    try {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        ck(cudaMemcpyAsync(tokens_host, m->out, sizeof(int64_t) * m->run_B * m->run_new, cudaMemcpyDeviceToHost, st),
           "tokens out");
        ck(cudaStreamSynchronize(st), "sync");
        unsigned err = 0;
        ck(cudaMemcpy(&err, m->err, 4, cudaMemcpyDeviceToHost), "err");
        if (err) { set_last_error_message("xdna_gemma_tokens: a tensor-parallel exchange wait expired"); return -1; }
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_gemma_tokens: ") + ex.what());
        return -1;
    }
}

// begin + every step + tokens.  Synchronous.
int xdna_gemma_generate(XdnaGemma *m, int B, const int64_t *prompts, int n_prompt, int n_new, int64_t *tokens_host,
                        void *stream) {
    if (!tokens_host) { set_last_error_message("xdna_gemma_generate: null pointer"); return -1; }
    if (xdna_gemma_begin(m, B, prompts, n_prompt, n_new) != 0) return -1;
    if (xdna_gemma_steps(m, n_prompt + n_new - 1, stream) != 0) return -1;
    return xdna_gemma_tokens(m, tokens_host, stream);
}

}  // extern "C"
