// gemma.cu -- Gemma-3 text decoder (GEMMA3_1B shapes) on B200: B streams in lockstep, int8
// per-channel weights, optional tensor parallelism across GPUs.
//
// The reference has no Gemma decode step (rust/npu-gemma/src/lib.rs:30-43 lists what to
// reuse); this is the HF Gemma-3 text model with npu-gemma's pieces (rmsnorm_ref lib.rs:55-64,
// geglu_ref 68-77, is_global_layer config.rs:131-133).  Per token and layer:
//   in-norm (f16 out) -> int8 GEMV q | k | v (tensor cores, row scales in the epilogue)
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
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"
#include "ptx.cuh"
#include "tc.cuh"

namespace xdna {
void set_last_error_message(const std::string &m);

namespace gm {
namespace cg = cooperative_groups;

constexpr int HD = 256;              // head dim
constexpr int MAXB = 64;             // streams
constexpr int GWARPS = 8;           // warps per GEMV CTA
constexpr int AK = 64;               // keys per attention split
constexpr int MAXTP = 8;

enum { OUT_F32 = 0, OUT_GEGLU_F16 = 1, OUT_ARGMAX = 2 };
// the GeGLU output (the down projection's input) is stored divided by this power of two, so
// that large activations stay inside the f16 range; the down GEMV multiplies it back
constexpr float kHScale = 64.0f;

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816h(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// two stored weight bytes u = q + 128 -> f16x2 of q (exact): the byte becomes the low mantissa
// of 1024 + u (exponent byte 0x64), then 1152 is subtracted.  sel picks bytes 0,1 (0x5140) or
// 2,3 (0x7362) of the word.
__device__ __forceinline__ uint32_t u8x2_f16(uint32_t w, uint32_t sel) {
    const uint32_t h = __byte_perm(w, 0x64646464u, sel);
    uint32_t r;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
    return r;
}
__device__ __forceinline__ uint16_t f16bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float gelu_tanh(float x) {   // npu-gemma lib.rs:74-77
    const float C = 0.79788456f;
    return 0.5f * x * (1.0f + tanhf(C * (x + 0.044715f * x * x * x)));
}

struct GemvArgs {
    const uint8_t *w;           // [row groups][K/16][32 lanes][8] bytes q + 128 in mma fragment order
    const float *scale;         // [Np] per output row
    const uint16_t *x;          // f16 [B][K]
    int B, N, K;
    int R, Wk, nsplit;          // row groups per CTA, warps per row group (along K), K ranges = cluster size
    int red_off;                // float offset of the partial-sum area in shared memory (0: aliases X)
    int mode;
    float oscale;               // output multiplier (kHScale for the down projection, else 1)
    float *out;                 // OUT_F32: [B][ldo]
    uint16_t *out_h;            // OUT_GEGLU_F16: [B][ldo] f16, column = row group * 8 + g, divided by kHScale
    int ldo;
    unsigned long long *best;   // OUT_ARGMAX: [B] max of amax_key(y, base + row) (no logits are stored)
    int base;
};

// (value, index) -> a 64-bit key whose unsigned maximum is the largest value, and among equal
// values the smallest index (the first maximum); 0 is below every key
__device__ __forceinline__ unsigned long long amax_key(float v, int idx) {
    const uint32_t b = __float_as_uint(v), o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ void amax_unkey(unsigned long long k, float &v, int &idx) {
    const uint32_t o = (uint32_t)(k >> 32);
    v = __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
    idx = (int)(0xffffffffu - (uint32_t)k);
}


__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Y[b][n] = (X[b] . Wq[n]) * scale[n] on the f16 tensor cores (int8 weights widen exactly; f16 activations).
// Grid (row-group blocks, K ranges); the K ranges of one row-group block form a thread-block
// cluster.  CTA = GWARPS warps = R row groups x Wk warps along the CTA's K range.  The CTA
// first requests its warps' first 8 k-steps of weights (they do not depend on the previous
// kernel, which may still be running: programmatic dependent launch), then waits for the
// previous grid and stages its X range [B][kc] with cp.async in one round trip.  Partial sums
// go to shared memory, are added over the Wk warps and then over the cluster's K ranges through
// distributed shared memory, in a fixed order (results do not depend on timing).
// OUT_GEGLU_F16: row group = 8 gate rows then the 8 matching up rows; the epilogue writes
// gelu_tanh(gate) * up.
template <int NT>
__global__ void __launch_bounds__(GWARPS * 32, 2) i8_gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) uint16_t xs[];
    float *red = reinterpret_cast<float *>(xs) + a.red_off;
    const uint32_t xs_a = smem_u32(xs);
    __shared__ unsigned long long sbest[MAXB];
    if (a.mode == OUT_ARGMAX && threadIdx.x < MAXB) sbest[threadIdx.x] = 0ull;
    griddep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int n_rg = (a.N + 15) / 16, nks = a.K / 16, split = blockIdx.y;
    const int ks0 = split * nks / a.nsplit, nkc = (split + 1) * nks / a.nsplit - ks0, xld = nkc * 16 + 8;
    const int r = warp / a.Wk, wk = warp % a.Wk;
    const int w0 = wk * nkc / a.Wk, nst = (wk + 1) * nkc / a.Wk - w0, ngrp = (nst + 7) / 8;
    const int rstride = gridDim.x * a.R;
    uint2 mv[8], mn[8];
    auto fetch = [&](uint2 (&dst)[8], int rg, int s0) {
        const uint2 *mp = reinterpret_cast<const uint2 *>(a.w) + ((size_t)rg * nks + ks0 + w0 + s0) * 32 + lane;
        const bool live = rg < n_rg;
#pragma unroll
        for (int s = 0; s < 8; s++) dst[s] = live && s0 + s < nst ? __ldcs(mp + s * 32) : make_uint2(0, 0);
    };
    fetch(mv, blockIdx.x * a.R + r, 0);
    griddep_wait();
    {
        const int cpr = nkc * 2;                        // 16-byte pieces per row
        for (int i = threadIdx.x; i < NT * 8 * cpr; i += blockDim.x) {
            const int b = i / cpr, c = i - b * cpr;
            uint16_t *d = &xs[b * xld + c * 8];
            if (b < a.B) cp_async16(d, a.x + (size_t)b * a.K + ks0 * 16 + c * 8);
            else *reinterpret_cast<uint4 *>(d) = make_uint4(0, 0, 0, 0);
        }
        cp_async_commit();
        cp_async_wait_all();
    }
    __syncthreads();
    for (int rg0 = blockIdx.x * a.R; rg0 < n_rg; rg0 += rstride) {
        const int rg = rg0 + r;
        if (rg0 != (int)blockIdx.x * a.R) fetch(mv, rg, 0);
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (int gi = 0; gi < ngrp; gi++) {
            if (gi + 1 < ngrp) fetch(mn, rg, (gi + 1) * 8);
#pragma unroll
            for (int s = 0; s < 8; s++) {
                if (gi * 8 + s >= nst) break;
                const uint32_t a0 = u8x2_f16(mv[s].x, 0x5140u), a1 = u8x2_f16(mv[s].x, 0x7362u);
                const uint32_t a2 = u8x2_f16(mv[s].y, 0x5140u), a3 = u8x2_f16(mv[s].y, 0x7362u);
                const int kk = (w0 + gi * 8 + s) * 16;
                if constexpr (NT == 1) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(&xs[g * xld + kk + 2 * t]);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t *>(&xs[g * xld + kk + 8 + 2 * t]);
                    mma16816h(acc[0], a0, a1, a2, a3, b0, b1);
                } else {
#pragma unroll
                    for (int n = 0; n < NT; n += 2) {
                        uint32_t r0, r1, r2, r3;
                        ldsm_x4(xs_a + 2u * ((n * 8 + ((lane >> 4) << 3) + (lane & 7)) * xld + kk + (((lane >> 3) & 1) << 3)),
                                r0, r1, r2, r3);
                        mma16816h(acc[n], a0, a1, a2, a3, r0, r1);
                        mma16816h(acc[n + 1], a0, a1, a2, a3, r2, r3);
                    }
                }
            }
#pragma unroll
            for (int s = 0; s < 8; s++) mv[s] = mn[s];
        }
        if (a.red_off == 0) __syncthreads();            // the partials overwrite the staged X
        float *rw = red + warp * NT * 128;
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) rw[(n * 4 + e) * 32 + lane] = acc[n][e];
        __syncthreads();
        // add over the Wk warps of each row group (in place, into the wk = 0 slot)
        if (a.Wk > 1)
            for (int i = threadIdx.x; i < a.R * NT * 128; i += blockDim.x) {
                const int rr = i / (NT * 128), e = i - rr * (NT * 128);
                float sum = red[rr * a.Wk * NT * 128 + e];
                for (int k = 1; k < a.Wk; k++) sum += red[(rr * a.Wk + k) * NT * 128 + e];
                red[rr * a.Wk * NT * 128 + e] = sum;
            }
        cg::cluster_group cl = cg::this_cluster();
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
            const int orow = rg0 + rr, b = n * 8 + 2 * (ln & 3) + c, gg = ln >> 2, n0 = orow * 16;
            const bool valid = orow < n_rg && b < a.B;
            if (a.mode == OUT_ARGMAX) {
                unsigned long long k = 0ull;
                if (valid) {
                    const float y0 = v0 * a.scale[n0 + gg] * a.oscale, y1 = v1 * a.scale[n0 + gg + 8] * a.oscale;
                    if (n0 + gg < a.N) k = amax_key(y0, a.base + n0 + gg);
                    if (n0 + gg + 8 < a.N) k = max(k, amax_key(y1, a.base + n0 + gg + 8));
                }
                atomicMax(&sbest[b], k);
                continue;
            }
            if (!valid) continue;
            const float y0 = v0 * a.scale[n0 + gg] * a.oscale, y1 = v1 * a.scale[n0 + gg + 8] * a.oscale;
            if (a.mode == OUT_F32) {
                if (n0 + gg < a.N) a.out[(size_t)b * a.ldo + n0 + gg] = y0;
                if (n0 + gg + 8 < a.N) a.out[(size_t)b * a.ldo + n0 + gg + 8] = y1;
            } else {
                a.out_h[(size_t)b * a.ldo + orow * 8 + gg] = f16bits(gelu_tanh(y0) * y1 * (1.0f / kHScale));
            }
        }
        if (a.nsplit > 1) cl.sync(); else __syncthreads();   // partials stay until every CTA has read them
    }
    if (a.mode == OUT_ARGMAX && threadIdx.x < a.B && sbest[threadIdx.x]) atomicMax(&a.best[threadIdx.x], sbest[threadIdx.x]);
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

// x[b] = embed[tok[b]] * sqrt(D); xn = f16(rms(x) * (1 + w)); one warp per stream
template <int NPL>
__global__ void embed_norm_kernel(const int64_t *__restrict__ tok, const float *__restrict__ emb, float es, int B,
                                  const float *__restrict__ w, float eps, float *__restrict__ x,
                                  uint16_t *__restrict__ xn) {
    griddep_launch();                                 // the next GEMV may start its weight fetch
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
        xn[(size_t)b * D + lane + 32 * i] = f16bits(v[i] * inv * (1.0f + wv[i]));
    }
}

// x += rms(y) * (1 + w_post); xn = f16(rms(x) * (1 + w_next)); one warp per stream
template <int NPL>
__global__ void post_add_norm_kernel(const float *__restrict__ y, int B, const float *__restrict__ wpost,
                                     const float *__restrict__ wnext, float eps, float *__restrict__ x,
                                     uint16_t *__restrict__ xn) {
    griddep_launch();
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
        xn[(size_t)b * D + lane + 32 * i] = f16bits(xv[i] * inv2 * (1.0f + wn[i]));
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

// One K range (AK keys) of one stream's attention for the hq query heads that share the K/V
// head, on the tensor cores: the range's K and V rows are staged with cp.async (16-byte chunks
// XOR-swizzled by key so ldmatrix is conflict-free; K and V in separate groups, so the scores
// start while V still arrives); warp w scores keys [16w, 16w + 16) for all heads
// (mma m16n8k16, query rows padded to 16 with zeros, Q from f32 rounded to bf16); softmax
// statistics per head; then warp w accumulates P.V for dims [64w, 64w + 64) with P in bf16.
// Writes the range's (max, sum, unnormalised output) per head for the ordered merge.  Keys
// visible: positions [lo, pos] with lo = max(0, pos - window + 1) for local layers (ring of
// cache_len slots), lo = 0 for global ones.
__device__ __forceinline__ uint32_t kv_off(int key, int chunk) {      // byte offset in a K or V tile
    return (uint32_t)(key * (HD * 2) + ((chunk ^ (key & 7)) << 4));
}
__global__ void __launch_bounds__(128) gqa_attn_kernel(const float *__restrict__ q, int hq, const int *posp,
                                                       int window, int cache_len, const uint16_t *__restrict__ kc,
                                                       const uint16_t *__restrict__ vc, float scaling,
                                                       float *__restrict__ part, int nsplit) {
    extern __shared__ __align__(128) uint8_t kvs[];          // K [AK][HD] then V [AK][HD], swizzled
    __shared__ float sc[4][AK], stat[4][2];
    __shared__ __align__(16) uint16_t ps[4][AK + 8];
    const int s = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, pos = *posp;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int p0 = lo + s * AK;
    const int nk = max(0, min(AK, pos + 1 - p0));
    float *pp = part + ((size_t)b * nsplit + s) * 4 * (HD + 2);
    if (nk == 0) {
        if (tid < hq) { pp[tid * (HD + 2)] = -INFINITY; pp[tid * (HD + 2) + 1] = 0.0f; }
        for (int i = tid; i < hq * HD; i += 128) pp[(i / HD) * (HD + 2) + 2 + i % HD] = 0.0f;
        return;
    }
    uint8_t *ks = kvs, *vs = kvs + AK * HD * 2;
    const uint32_t ks_a = smem_u32(ks), vs_a = smem_u32(vs);
    for (int i = tid; i < AK * (HD / 8); i += 128) {
        const int j = i >> 5, c = i & 31;
        if (j < nk) cp_async16(ks + kv_off(j, c), kc + ((size_t)b * cache_len + (p0 + j) % cache_len) * HD + c * 8);
    }
    cp_async_commit();
    for (int i = tid; i < AK * (HD / 8); i += 128) {
        const int j = i >> 5, c = i & 31;
        if (j < nk) cp_async16(vs + kv_off(j, c), vc + ((size_t)b * cache_len + (p0 + j) % cache_len) * HD + c * 8);
        else *reinterpret_cast<uint4 *>(vs + kv_off(j, c)) = make_uint4(0, 0, 0, 0);   // P = 0 there, V must be finite
    }
    cp_async_commit();
    // query fragments (rows g < hq; rows g + 8 are padding): a0 = Q[g][16k + 2t..], a2 = Q[g][16k + 8 + 2t..]
    uint32_t qa[16][2];
    {
        const float *qr = q + ((size_t)b * hq + (g < hq ? g : 0)) * HD;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const float2 x0 = *reinterpret_cast<const float2 *>(qr + 16 * k + 2 * t);
            const float2 x1 = *reinterpret_cast<const float2 *>(qr + 16 * k + 8 + 2 * t);
            qa[k][0] = g < hq ? bf16bits(x0.x) | (bf16bits(x0.y) << 16) : 0u;
            qa[k][1] = g < hq ? bf16bits(x1.x) | (bf16bits(x1.y) << 16) : 0u;
        }
    }
    cp_async_wait_group<1>();
    __syncthreads();
    {
        float acc[2][4] = {};
#pragma unroll
        for (int k = 0; k < 16; k++) {
            uint32_t r0, r1, r2, r3;
            const int key = 16 * warp + ((lane >> 4) << 3) + (lane & 7), ch = 2 * k + ((lane >> 3) & 1);
            ldsm_x4(ks_a + kv_off(key, ch), r0, r1, r2, r3);
            mma16816(acc[0], qa[k][0], 0u, qa[k][1], 0u, r0, r1);
            mma16816(acc[1], qa[k][0], 0u, qa[k][1], 0u, r2, r3);
        }
        if (g < hq)
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int j = 16 * warp + 8 * n + 2 * t + c;
                    sc[g][j] = j < nk ? acc[n][c] * scaling : -INFINITY;
                }
    }
    __syncthreads();
    if (warp < hq) {
        const float a0 = sc[warp][lane], a1 = sc[warp][lane + 32];
        float m = fmaxf(a0, a1);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float e0 = lane < nk ? expf(a0 - m) : 0.0f, e1 = lane + 32 < nk ? expf(a1 - m) : 0.0f;
        float l = e0 + e1;
#pragma unroll
        for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        ps[warp][lane] = (uint16_t)bf16bits(e0);
        ps[warp][lane + 32] = (uint16_t)bf16bits(e1);
        if (lane == 0) { stat[warp][0] = m; stat[warp][1] = l; }
    }
    cp_async_wait_group<0>();
    __syncthreads();
    {
        float acc[8][4] = {};
#pragma unroll
        for (int k = 0; k < AK / 16; k++) {
            const uint32_t a0 = g < hq ? *reinterpret_cast<const uint32_t *>(&ps[g][16 * k + 2 * t]) : 0u;
            const uint32_t a2 = g < hq ? *reinterpret_cast<const uint32_t *>(&ps[g][16 * k + 8 + 2 * t]) : 0u;
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                uint32_t r0, r1, r2, r3;
                const int key = 16 * k + (((lane >> 3) & 1) << 3) + (lane & 7), ch = 8 * warp + n + (lane >> 4);
                ldsm_x4_t(vs_a + kv_off(key, ch), r0, r1, r2, r3);
                mma16816(acc[n], a0, 0u, a2, 0u, r0, r1);
                mma16816(acc[n + 1], a0, 0u, a2, 0u, r2, r3);
            }
        }
        if (g < hq)
#pragma unroll
            for (int n = 0; n < 8; n++)
                *reinterpret_cast<float2 *>(&pp[g * (HD + 2) + 2 + 64 * warp + 8 * n + 2 * t]) =
                    make_float2(acc[n][0], acc[n][1]);
    }
    if (tid < hq) { pp[tid * (HD + 2)] = stat[tid][0]; pp[tid * (HD + 2) + 1] = stat[tid][1]; }
}

// fold the splits in order -> ctx f16 [B][hq * 256]; block = (head, stream), thread = dim
__global__ void gqa_merge_kernel(const float *__restrict__ part, int hq, int nsplit, uint16_t *__restrict__ ctx) {
    griddep_launch();
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
    ctx[((size_t)b * hq + hh) * HD + d] = f16bits(A / L);
}

// this rank's (value, index) per stream from the LM head's keys; clears the keys for the next step
__global__ void unpack_best_kernel(unsigned long long *keys, int B, float *bestv, int *besti) {
    const int b = threadIdx.x;
    if (b >= B) return;
    amax_unkey(keys[b], bestv[b], besti[b]);
    keys[b] = 0ull;
}

// next token per stream from the P ranks' (value, index) pairs (first maximum overall), or the
// prompt while it lasts; records generated tokens; the last block advances *pos
__global__ void pick_kernel(const float *bestv, const int *besti, int P, int B, const int64_t *prompt, int n_prompt,
                            int *posp, int64_t *tok, int64_t *out, int n_new, unsigned *done, uint32_t *ebase,
                            uint32_t ex_step) {
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
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            *posp = pos + 1;
            *ebase += ex_step;                     // the next step's exchanges use fresh epochs
        }
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
                                    const uint32_t *ebase, uint32_t off, float *__restrict__ out, unsigned *err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t epoch = *ebase + off;
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
__global__ void tp_gather_best_kernel(int B, uint64_t *const *bufs, int P, int rank, const uint32_t *ebase,
                                      uint32_t off, float *bestv, int *besti, unsigned *err) {
    const int i = threadIdx.x;                     // 2 * MAXB words: values then indices
    const uint32_t epoch = *ebase + off;
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


// ---- tcgen05 GEMV for 17..64 streams ---------------------------------------------------------
// At 64 streams every weight byte carries 128 FLOP, which the mma.sync pipe cannot sustain at
// HBM rate; this kernel runs the same Y = (X . Wq^T) * scale on tcgen05.  CTA = 128 weight rows
// (one TMEM lane each) x one K range; warps 0-3 (thread r = row r) fetch the rows' int8 tiles
// (64 K: bytes q + 128, laid out so each 16-byte chunk index is one coalesced warp load) up to 4
// tiles ahead in registers, widen them to f16 exactly (byte-permute + sub.f16x2) and store them
// into a 4-slot ring of A operands in TMEM (tcgen05.st, 32 columns per tile); warp 4 issues
// tcgen05.mma (A from TMEM, B = the staged X range in shared memory, SW128 K-major; D = 128 x NB
// f32 in TMEM) and frees ring slots with tcgen05.commit.  The X range [NB streams][K range] is
// staged with cp.async once per CTA.  Partials leave TMEM by tcgen05.ld and are stored straight
// into the shared memory of the cluster CTA that owns their rows; owners add the K ranges in
// rank order; epilogues as i8_gemv_kernel.  Every mbarrier wait is bounded (1 s): on expiry the
// kernel sets *err and runs to its end without waiting (results invalid, reported by the host).
constexpr int TCK = 64;           // K per tile
constexpr int TC_SLOTS = 4;       // TMEM ring of A tiles (32 columns each)
constexpr int TC_PF = 4;          // tiles in flight per converter thread (registers)
constexpr int TC_THREADS = 160;

struct TcArgs {
    const uint8_t *w;           // [row blocks][K tiles][4 chunks][128 rows][16 B]
    const float *scale;         // [row blocks * 128]
    const uint16_t *x;          // f16 [B][K]
    int B, N, K, nkt;           // nkt = K tiles (K padded to 64 with zero weights)
    int nsplit, red_off;        // K ranges (= cluster size); float offset of the partials (0: alias X)
    int mode;
    float oscale;
    float *out;
    uint16_t *out_h;
    int ldo;
    unsigned long long *best;
    int base;
    unsigned *err;
};

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, bool &ok, unsigned *err) {
    if (!ok) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > 1000000000ull) {
            atomicCAS(err, 0u, 2u);
            ok = false;
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// kind::f16 with f16 A and B, f32 accumulate, both K-major
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int NB>
__global__ void __launch_bounds__(TC_THREADS) tc_gemv_kernel(TcArgs a) {
    extern __shared__ __align__(1024) uint8_t tsm[];
    uint8_t *xs = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tsm) + 1023) & ~uintptr_t(1023));
    float *red = reinterpret_cast<float *>(xs) + a.red_off;
    __shared__ __align__(8) uint64_t full[TC_SLOTS], empty[TC_SLOTS], done;
    __shared__ uint32_t tbase_s;
    __shared__ unsigned long long sbest[MAXB];
    griddep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int split = blockIdx.y, nrb = (a.N + 127) / 128;
    const int kt0 = split * a.nkt / a.nsplit, nkc = (split + 1) * a.nkt / a.nsplit - kt0;
    bool ok = true;
    if (tid == 0) {
        for (int i = 0; i < TC_SLOTS; i++) { mbar_init(&full[i], 128); mbar_init(&empty[i], 1); }
        mbar_init(&done, 1);
        mbar_fence_init();
    }
    if (a.mode == OUT_ARGMAX && tid < MAXB) sbest[tid] = 0ull;
    if (warp == 4) { tc::tmem_alloc(&tbase_s, 256); tc::tmem_relinquish(); }
    // converters: first TC_PF tiles of the first row block (weights only: before the grid dependency)
    uint4 pf[TC_PF][4];
    auto fetch = [&](uint4 (&d)[4], int rb, int kt) {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.w) + ((size_t)rb * a.nkt + kt) * 512 + tid;
#pragma unroll
        for (int c = 0; c < 4; c++) d[c] = __ldcs(src + c * 128);
    };
    if (warp < 4) {
#pragma unroll
        for (int j = 0; j < TC_PF; j++)
            if (j < nkc && (int)blockIdx.x < nrb) fetch(pf[j], blockIdx.x, kt0 + j);
    }
    griddep_wait();
    {   // X range -> [tile][NB rows][128 B], 16-byte chunk c of row b at chunk c ^ (b & 7)
        const int pieces = nkc * NB * 8;
        for (int i = tid; i < pieces; i += TC_THREADS) {
            const int j = i / (NB * 8), rem = i - j * (NB * 8), b = rem >> 3, c = rem & 7;
            uint8_t *dst = xs + j * (NB * 128) + b * 128 + ((c ^ (b & 7)) << 4);
            const int k = (kt0 + j) * TCK + c * 8;
            if (b < a.B && k < a.K) cp_async16(dst, a.x + (size_t)b * a.K + k);
            else *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
        }
        cp_async_commit();
        cp_async_wait_all();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    tc::fence_before_sync();
    cg::cluster_group cl = cg::this_cluster();
    if (a.nsplit > 1) cl.sync(); else __syncthreads();   // (peers store into this CTA only once it runs)
    tc::fence_after_sync();
    const uint32_t tbase = tbase_s, tD = tbase, tA = tbase + 64;
    constexpr uint32_t IDESC = idesc_f16_f32(128, NB);
    const uint32_t xs_a = smem_u32(xs);
    int it = 0;                               // ring position (continues over row blocks)
    int rbi = 0;
    for (int rb = blockIdx.x; rb < nrb; rb += gridDim.x, rbi++) {
        if (warp < 4) {
            for (int t0 = 0; t0 < nkc; t0 += TC_PF) {
#pragma unroll
                for (int j = 0; j < TC_PF; j++) {
                    const int t = t0 + j;
                    if (t >= nkc) break;
                    const int slot = (it + t) % TC_SLOTS;
                    const uint32_t ph = (uint32_t)(((it + t) / TC_SLOTS) & 1);
                    uint32_t h[32];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint32_t wv[4] = {pf[j][c].x, pf[j][c].y, pf[j][c].z, pf[j][c].w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            h[c * 8 + 2 * e] = u8x2_f16(wv[e], 0x5140u);
                            h[c * 8 + 2 * e + 1] = u8x2_f16(wv[e], 0x7362u);
                        }
                    }
                    if (t + TC_PF < nkc) fetch(pf[j], rb, kt0 + t + TC_PF);
                    tc_wait(&empty[slot], ph ^ 1u, ok, a.err);
                    tmem_st32(tA + ((uint32_t)(warp * 32) << 16) + slot * 32, h);
                    tmem_st_wait();
                    tc::fence_before_sync();
                    mbar_arrive(&full[slot]);
                }
            }
            // the next row block's first tiles, in flight during this block's epilogue
            const int rn = rb + gridDim.x;
#pragma unroll
            for (int j = 0; j < TC_PF; j++)
                if (j < nkc && rn < nrb) fetch(pf[j], rn, kt0 + j);
        } else if (lane == 0) {
            for (int t = 0; t < nkc; t++) {
                const int slot = (it + t) % TC_SLOTS;
                const uint32_t ph = (uint32_t)(((it + t) / TC_SLOTS) & 1);
                tc_wait(&full[slot], ph, ok, a.err);
                tc::fence_after_sync();
                if (ok) {
#pragma unroll
                    for (int k4 = 0; k4 < 4; k4++)
                        mma_f16_ta(tD, tA + slot * 32 + k4 * 8,
                                   tc::desc_k_sw128(xs_a + t * (NB * 128) + k4 * 32), IDESC, (t | k4) != 0);
                }
                tc::commit(&empty[slot]);
            }
            tc::commit(&done);
        }
        it += nkc;
        // partials: thread r takes row r of D from TMEM and stores it into the shared memory of the
        // CTA that owns rows [q*rpo, (q+1)*rpo) of the block (rpo = 128 / nsplit), as
        // red[src rank][stream][row - q*rpo]: remote stores, no round trips.  Each owner then adds
        // the K ranges in rank order from its own shared memory.
        const int rpo = 128 / a.nsplit;
        if (warp < 4) {
            tc_wait(&done, (uint32_t)(rbi & 1), ok, a.err);
            tc::fence_after_sync();
            const int q = tid / rpo, lr = tid - q * rpo;
            float *dst = a.nsplit > 1 ? cl.map_shared_rank(red, q) : red;
            dst += (size_t)split * NB * rpo + lr;
#pragma unroll
            for (int c0 = 0; c0 < NB; c0 += 32) {
                uint32_t r[32];
                tc::tmem_ld32(tD + ((uint32_t)(warp * 32) << 16) + c0, r);
                tc::tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 32; c++) dst[(c0 + c) * rpo] = __uint_as_float(r[c]);
            }
            tc::fence_before_sync();
        }
        if (a.nsplit > 1) cl.sync(); else __syncthreads();
        tc::fence_after_sync();
        // this CTA's rows: item = (row pair p: local rows (p/8)*16 + p%8 and +8, stream b)
        const int npair = rpo / 2, items = npair * NB;
        for (int i = tid; i < items; i += TC_THREADS) {
            const int b = i / npair, p = i - b * npair, lrow = (p >> 3) * 16 + (p & 7);
            float v0 = 0.0f, v1 = 0.0f;
            for (int q = 0; q < a.nsplit; q++) {
                const float *rp = red + ((size_t)q * NB + b) * rpo + lrow;
                v0 += rp[0];
                v1 += rp[8];
            }
            const int n0 = rb * 128 + split * rpo + lrow;
            if (a.mode == OUT_ARGMAX) {
                unsigned long long k = 0ull;
                if (b < a.B) {
                    const float y0 = v0 * a.scale[n0] * a.oscale, y1 = v1 * a.scale[n0 + 8] * a.oscale;
                    if (n0 < a.N) k = amax_key(y0, a.base + n0);
                    if (n0 + 8 < a.N) k = max(k, amax_key(y1, a.base + n0 + 8));
                }
                atomicMax(&sbest[b], k);
                continue;
            }
            if (b >= a.B) continue;
            const float y0 = v0 * a.scale[n0] * a.oscale, y1 = v1 * a.scale[n0 + 8] * a.oscale;
            if (a.mode == OUT_F32) {
                if (n0 < a.N) a.out[(size_t)b * a.ldo + n0] = y0;
                if (n0 + 8 < a.N) a.out[(size_t)b * a.ldo + n0 + 8] = y1;
            } else {
                a.out_h[(size_t)b * a.ldo + (n0 >> 4) * 8 + (n0 & 7)] = f16bits(gelu_tanh(y0) * y1 * (1.0f / kHScale));
            }
        }
        tc::fence_before_sync();
        if (a.nsplit > 1) cl.sync(); else __syncthreads();
        tc::fence_after_sync();
    }
    if (a.mode == OUT_ARGMAX && tid < a.B && sbest[tid]) atomicMax(&a.best[tid], sbest[tid]);
    __syncthreads();
    if (warp == 4) tc::tmem_dealloc(tbase, 256);
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
    float oscale = 1.0f;                  // output multiplier undoing an input prescale
    uint8_t *wt = nullptr;                // tcgen05 layout (engines created for more than 16 streams)
    int nkt = 0;
};

struct XdnaGemma {
    XdnaGemmaConfig cfg{};
    int max_batch = 0, max_ctx = 0, rank = 0, tp = 1, hq = 0, f_loc = 0, v_loc = 0, v_base = 0, k_loc = 0, k_base = 0;
    bool use_tc = false;
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
    float *x = nullptr, *qkv = nullptr, *q = nullptr, *y = nullptr, *yr = nullptr, *apart = nullptr, *bestv = nullptr;
    int *besti = nullptr;
    unsigned long long *lmbest = nullptr;  // LM head: per stream max key of (logit, vocabulary index)
    uint16_t *xn = nullptr, *ctx = nullptr, *h = nullptr;
    unsigned *done = nullptr, *err = nullptr;
    int *pos = nullptr;
    int64_t *tok = nullptr, *prompt = nullptr, *out = nullptr;
    int n_prompt_cap = 0;
    int run_B = 0, run_prompt = 0, run_new = 0, run_done = 0;   // the staged decode
    // tensor parallel exchange: bufs[r] = rank r's exchange buffer (own or IPC-mapped)
    uint64_t *xbuf = nullptr;
    uint64_t **dbufs = nullptr;
    std::vector<void *> peer_maps;
    uint32_t *ebase = nullptr;             // device: epoch base of this step's exchanges
    struct Graph {
        int B, n_prompt, n_new;
        bool lm;                          // false: a prompt step (no LM head)
        cudaGraphExec_t exec;
    };
    std::vector<Graph> graphs;            // one decode step per staged shape and step kind
    cudaStream_t cap = nullptr;
    std::vector<void *> owned;
    ~XdnaGemma() {
        for (auto &g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        if (cap) cudaStreamDestroy(cap);
        for (void *p : peer_maps) cudaIpcCloseMemHandle(p);
        for (void *p : owned) cudaFree(p);
    }
};

namespace {
constexpr int kD = 1152, kNPL = kD / 32;

// rows = outputs; W given [K, N] with the output columns listed in `cols` (in this order);
// pack in mma fragment order with a per-row scale (Lin::load rule, opt125m_decode.rs:41-60)
GmMat pack_i8(XdnaGemma *m, const float *w, int K, int N, const std::vector<int> &cols) {
    const int R = (int)cols.size(), nrg = (R + 15) / 16, nks = K / 16, nrb = (R + 127) / 128;
    std::vector<int8_t> q((size_t)nrb * 128 * K, 0);
    std::vector<float> sc((size_t)nrb * 128, 1.0f);
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
                uint8_t u[8];                  // stored as q + 128 (the kernel's f16 widening)
                for (int i = 0; i < 8; i++) u[i] = (uint8_t)(v[i] + 128);
                std::memcpy(&packed[(((size_t)rg * nks + ks) * 32 + lane) * 8], u, 8);
            }
    GmMat o;
    o.N = R;
    o.K = K;
    o.w = dupload(packed);
    o.scale = dupload(sc);
    m->owned.push_back(o.w);
    m->owned.push_back(o.scale);
    if (m->use_tc) {
        // tcgen05 layout: [row block of 128][K tile of 64][chunk c of 16 K][row][16 B], K padded
        // with zero weights (bytes 128)
        const int nkt = (K + gm::TCK - 1) / gm::TCK;
        std::vector<uint8_t> t((size_t)nrb * nkt * 8192, 128);
        for (int rb = 0; rb < nrb; rb++)
            for (int kt = 0; kt < nkt; kt++)
                for (int c = 0; c < 4; c++)
                    for (int r = 0; r < 128; r++)
                        for (int e = 0; e < 16; e++) {
                            const int k = kt * 64 + c * 16 + e, row = rb * 128 + r;
                            if (k < K)
                                t[((((size_t)rb * nkt + kt) * 4 + c) * 128 + r) * 16 + e] =
                                    (uint8_t)(q[(size_t)row * K + k] + 128);
                        }
        o.wt = dupload(t);
        o.nkt = nkt;
        m->owned.push_back(o.wt);
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
            const size_t xsb = (size_t)nt * 8 * (kc + 8) * 2, redb = (size_t)gm::GWARPS * nt * 128 * 4;
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

// tcgen05 GEMV launch shape: the fewest K ranges (cluster size 1..8) giving about one CTA per
// SM with two CTAs per SM, else the most CTAs whose staged X range fits one per SM; at least
// 80 KB of shared memory per CTA so that at most two CTAs share an SM (two x 256 TMEM columns).
struct TcPlan {
    int nsplit, gx, red_off;
    size_t smem;
};
constexpr size_t kTcSmemMax = 220 * 1024;
TcPlan tc_plan_of(int N, int nkt, int nb) {
    const int nrb = (N + 127) / 128;
    TcPlan best{0, 0, 0, 0};
    long best_ctas = -1;
    for (int ns : {1, 2, 4, 8}) {
        if (ns > nkt) break;
        const int nkc = (nkt + ns - 1) / ns;
        const size_t xsb = (size_t)nkc * nb * 128, redb = (size_t)nb * 128 * 4;
        const size_t xsa = (xsb + 1023) / 1024 * 1024;
        for (int per : {2, 1}) {                 // CTAs per SM
            const int gx = std::min(nrb, std::max(1, 148 * per / ns));
            // the partials may alias the staged X only when no other CTA writes them and the
            // CTA does not loop (peers store into a CTA's partials while its MMAs may still read X)
            const bool alias = ns == 1 && gx == nrb;
            const size_t smem = std::max<size_t>(80 * 1024, 1024 + (alias ? std::max(xsb, redb) : xsa + redb));
            if (smem > (per == 2 ? kGemvSmemCap : kTcSmemMax)) continue;
            const TcPlan p{ns, gx, alias ? 0 : (int)(xsa / 4), smem};
            const long ctas = (long)nrb * ns;
            if (per == 2 && ctas >= 140) return p;
            if (ctas > best_ctas) { best = p; best_ctas = ctas; }
            break;
        }
    }
    if (best.nsplit == 0) throw std::runtime_error("tcgen05 GEMV shape does not fit shared memory");
    return best;
}

cudaError_t gemv_tc(XdnaGemma *m, const GmMat &w, const uint16_t *x, int B, int mode, float *out, uint16_t *ob,
                    int ldo, cudaStream_t st) {
    const int nb = B <= 32 ? 32 : 64;
    TcPlan p;
    try { p = tc_plan_of(w.N, w.nkt, nb); } catch (...) { return cudaErrorInvalidValue; }
    gm::TcArgs a{w.wt, w.scale, x, B, w.N, w.K, w.nkt, p.nsplit, p.red_off, mode, w.oscale, out, ob, ldo,
                 m->lmbest, m->v_base, m->err};
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(p.gx, p.nsplit);
    lc.blockDim = dim3(gm::TC_THREADS);
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
    return nb == 32 ? cudaLaunchKernelEx(&lc, gm::tc_gemv_kernel<32>, a) : cudaLaunchKernelEx(&lc, gm::tc_gemv_kernel<64>, a);
}

cudaError_t gemv(XdnaGemma *m, const GmMat &w, const uint16_t *x, int B, int mode, float *out, uint16_t *ob, int ldo,
                 cudaStream_t st) {
    if (B > 16 && w.wt) return gemv_tc(m, w, x, B, mode, out, ob, ldo, st);
    const int nt = B <= 8 ? 1 : B <= 16 ? 2 : B <= 32 ? 4 : 8;
    GemvPlan p;
    try { p = plan_of(w.N, w.K, nt); } catch (...) { return cudaErrorInvalidValue; }
    gm::GemvArgs a{w.w, w.scale, x, B, w.N, w.K, p.R, gm::GWARPS / p.R, p.nsplit, p.red_off, mode, w.oscale, out, ob, ldo,
                   m->lmbest, m->v_base};
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(p.gx, p.nsplit);
    lc.blockDim = dim3(gm::GWARPS * 32);
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
    switch (nt) {
    case 1: return cudaLaunchKernelEx(&lc, gm::i8_gemv_kernel<1>, a);
    case 2: return cudaLaunchKernelEx(&lc, gm::i8_gemv_kernel<2>, a);
    case 4: return cudaLaunchKernelEx(&lc, gm::i8_gemv_kernel<4>, a);
    default: return cudaLaunchKernelEx(&lc, gm::i8_gemv_kernel<8>, a);
    }
}

// sum partial vectors y [B][D] over the ranks into out (nothing to do when tp == 1)
cudaError_t allreduce(XdnaGemma *m, const float *y, int B, float *out, uint32_t off, cudaStream_t st) {
    const int n = B * kD;
    if (m->tp == 1) return cudaSuccess;             // the caller reads y itself
    gm::tp_allreduce_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, n, m->dbufs, m->tp, m->rank, m->ebase, off, out, m->err);
    return cudaGetLastError();
}

// One decode step of B streams.  A step at a position before the prompt's last needs no LM head
// (the pick kernel takes the prompt's next token), so with lm == false the LM-head GEMV and the
// argmax exchange are left out.
cudaError_t step(XdnaGemma *m, int B, int n_prompt, int n_new, cudaStream_t st, bool lm = true) {
    using namespace gm;
    const auto &c = m->cfg;
    const float eps = c.eps;
    cudaError_t e = cudaSuccess;
    uint32_t ex = 0;                               // exchanges so far in this step (epoch offsets)
    const float *yin = m->tp == 1 ? m->y : m->yr;  // the (all-reduced) output of o and down
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
        gqa_attn_kernel<<<dim3(nsplit, B), 128, 2 * AK * HD * 2, st>>>(m->q, hq, m->pos, L.global ? 0 : c.window,
                                                                    L.cache_len, L.kc, L.vc,
                                                                    1.0f / sqrtf(c.query_pre_attn_scalar), m->apart, nsplit);
        gqa_merge_kernel<<<dim3(hq, B), HD, 0, st>>>(m->apart, hq, nsplit, m->ctx);
        if ((e = gemv(m, L.o, m->ctx, B, OUT_F32, m->y, nullptr, kD, st))) break;
        if ((e = allreduce(m, m->y, B, m->yr, ++ex, st))) break;
        post_add_norm_kernel<kNPL><<<(B + 3) / 4, 128, 0, st>>>(yin, B, nrm + kD + 2 * HD, nrm + 2 * kD + 2 * HD, eps,
                                                                m->x, m->xn);
        if ((e = gemv(m, L.gu, m->xn, B, OUT_GEGLU_F16, nullptr, m->h, m->f_loc, st))) break;
        if ((e = gemv(m, L.down, m->h, B, OUT_F32, m->y, nullptr, kD, st))) break;
        if ((e = allreduce(m, m->y, B, m->yr, ++ex, st))) break;
        const float *wnext = l + 1 < c.n_layers ? m->layers[l + 1].norms : m->final_norm;
        post_add_norm_kernel<kNPL><<<(B + 3) / 4, 128, 0, st>>>(yin, B, nrm + 3 * kD + 2 * HD, wnext, eps, m->x, m->xn);
    }
    if (e) return e;
    if (lm) {
        if ((e = gemv(m, m->lm, m->xn, B, OUT_ARGMAX, nullptr, nullptr, 0, st))) return e;
        unpack_best_kernel<<<1, MAXB, 0, st>>>(m->lmbest, B, m->bestv + m->rank * MAXB,
                                                m->besti + m->rank * MAXB);
        if (m->tp > 1)
            tp_gather_best_kernel<<<1, 2 * MAXB, 0, st>>>(B, m->dbufs, m->tp, m->rank, m->ebase, ++ex, m->bestv,
                                                         m->besti, m->err);
    }
    pick_kernel<<<1, MAXB, 0, st>>>(m->bestv, m->besti, m->tp == 1 ? 1 : m->tp, B, m->prompt, n_prompt, m->pos, m->tok,
                                    m->out, n_new, m->done, m->ebase, ex);
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
        // GEMVs of more than 16 streams on tcgen05 (XDNA_GEMMA_TC=0 keeps them on mma.sync)
        const char *tcv = std::getenv("XDNA_GEMMA_TC");
        m->use_tc = max_batch > 16 && !(tcv && tcv[0] == '0');
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
                o.down.oscale = gm::kHScale;   // its input is the GeGLU output divided by kHScale
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
        const int hqmax = 4;
        m->x = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->qkv = static_cast<float *>(keep(dalloc<float>(B * (hqmax + 2) * HD)));
        m->q = static_cast<float *>(keep(dalloc<float>(B * hqmax * HD)));
        m->y = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->yr = static_cast<float *>(keep(dalloc<float>(B * kD)));
        m->lmbest = static_cast<unsigned long long *>(keep(dalloc<unsigned long long>(MAXB)));
        ck(cudaMemset(m->lmbest, 0, sizeof(unsigned long long) * MAXB), "memset");
        for (int nt : {1, 2, 4, 8}) {              // every GEMV shape has a launch plan
            for (auto &L : m->layers) { plan_of(L.qkv.N, L.qkv.K, nt); plan_of(L.o.N, L.o.K, nt);
                                        plan_of(L.gu.N, L.gu.K, nt); plan_of(L.down.N, L.down.K, nt); }
            plan_of(m->lm.N, m->lm.K, nt);
        }
        if (m->use_tc)
            for (int nb : {32, 64}) {
                for (auto &L : m->layers) { tc_plan_of(L.qkv.N, L.qkv.nkt, nb); tc_plan_of(L.o.N, L.o.nkt, nb);
                                            tc_plan_of(L.gu.N, L.gu.nkt, nb); tc_plan_of(L.down.N, L.down.nkt, nb); }
                tc_plan_of(m->lm.N, m->lm.nkt, nb);
            }
        const int nsplit_max = (std::max(max_ctx, c.window) + AK - 1) / AK;
        m->apart = static_cast<float *>(keep(dalloc<float>(B * nsplit_max * 4 * (HD + 2))));
        m->bestv = static_cast<float *>(keep(dalloc<float>(MAXTP * MAXB)));
        m->besti = static_cast<int *>(keep(dalloc<int>(MAXTP * MAXB)));
        m->xn = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * kD)));
        m->ctx = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * hqmax * HD)));
        m->h = static_cast<uint16_t *>(keep(dalloc<uint16_t>(B * m->f_loc)));
        m->done = static_cast<unsigned *>(keep(dalloc<unsigned>(1)));
        m->err = static_cast<unsigned *>(keep(dalloc<unsigned>(1)));
        m->ebase = static_cast<uint32_t *>(keep(dalloc<uint32_t>(1)));
        ck(cudaMemset(m->ebase, 0, 4), "memset");
        m->pos = static_cast<int *>(keep(dalloc<int>(1)));
        m->tok = static_cast<int64_t *>(keep(dalloc<int64_t>(B)));
        m->out = static_cast<int64_t *>(keep(dalloc<int64_t>(B * max_ctx)));
        ck(cudaMemset(m->done, 0, 4), "memset");
        ck(cudaMemset(m->err, 0, 4), "memset");
        ck(cudaMemset(m->bestv, 0, sizeof(float) * MAXTP * MAXB), "memset");
        ck(cudaMemset(m->besti, 0, sizeof(int) * MAXTP * MAXB), "memset");
        ck(cudaFuncSetAttribute(gqa_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * AK * HD * 2), "smem");
        const int gsm = (int)kGemvSmemCap;
        ck(cudaFuncSetAttribute(i8_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(i8_gemv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm), "smem");
        ck(cudaFuncSetAttribute(tc_gemv_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemMax), "smem");
        ck(cudaFuncSetAttribute(tc_gemv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemMax), "smem");
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
    // the first step of a staged shape runs eagerly and is then recorded as a graph (positions,
    // tokens and exchange epochs live on the device); later steps replay the graph
    for (int s = 0; s < n_steps; s++) {
        cudaError_t e;
        // positions before the prompt's last skip the LM head (the host counts the steps)
        const bool lm = m->run_done >= m->run_prompt - 1;
        XdnaGemma::Graph *g = nullptr;
        for (auto &x : m->graphs)
            if (x.B == m->run_B && x.n_prompt == m->run_prompt && x.n_new == m->run_new && x.lm == lm) g = &x;
        if (g) {
            e = cudaGraphLaunch(g->exec, st);
        } else {
            e = step(m, m->run_B, m->run_prompt, m->run_new, st, lm);
            if (!e) {
                m->graphs.push_back({m->run_B, m->run_prompt, m->run_new, lm, nullptr});
                g = &m->graphs.back();
                if (!m->cap) e = cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking);
                cudaGraph_t graph = nullptr;
                if (!e) e = cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeThreadLocal);
                if (!e) {
                    const cudaError_t e2 = step(m, m->run_B, m->run_prompt, m->run_new, m->cap, lm);
                    e = cudaStreamEndCapture(m->cap, &graph);
                    if (!e) e = e2;
                }
                if (!e) e = cudaGraphInstantiate(&g->exec, graph, 0);
                if (graph) cudaGraphDestroy(graph);
                if (e) { m->graphs.pop_back(); g = nullptr; }
            }
        }
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
