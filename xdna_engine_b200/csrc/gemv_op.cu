// gemv_op.cu -- the op-level exact int8 GEMV behind xdna_gemv_i8 / xdna_gemv_i8_noalloc
// (the CtxDecode::gemv replacement, rust/npu-asr/src/ctx_decode.rs:325-369).
//
// y[n] = float(sum_k X_k * q[n][k]) * 2^-s * scale[n] + bias[n], where X = rint(x * 2^s) is
// the activation as a 22-bit fixed-point integer (s from max |x|).  X is split into three
// int8 limbs (X = a*2^16 + b*2^8 + c) that form three live rows of the A operand of
// mma.sync.m16n8k32.s8; the int8 weight rows are the B operand.  The int32 limb sums are
// combined exactly in int64 and rounded once, so the result equals the CPU oracle's exact
// dot (or_gemv_i8_exact) bit for bit.  One CTA per chunk: a copy warp brings the chunk in with
// one 1-D bulk copy (cp.async.bulk + mbarrier complete_tx), 8 warps split K.
#include <cuda_runtime.h>
#include <cstdint>

#include "gemv_op.h"
#include "ptx.cuh"

namespace xdna {
namespace gemvop {

struct Smem {
    static constexpr int ring = 0;
    static constexpr int limbs = ring + kStageBytes;                     // 3 x kKmax int8
    static constexpr int xf = limbs + 3 * kKmax;                         // kKmax f32
    static constexpr int part = xf + kKmax * 4;                          // partial limb sums
    static constexpr int part_ints = kWarps * kMaxTilesPerChunk * 3 * 8;
    static constexpr int red = part + part_ints * 4;                     // 32 f32
    static constexpr int bar = (red + 32 * 4 + 15) & ~15;
    static constexpr int total = bar + 16;
};

extern __shared__ __align__(1024) uint8_t gsm[];

__device__ __forceinline__ void cbar() { named_bar(1, kConsumerThreads); }

// 22-bit fixed-point exponent for a vector whose max |x| is m: X = rint(x * 2^s), |X| < 2^22
__device__ __forceinline__ int limb_exponent(float m) {
    const int E = m >= 0x1p-100f ? (int)((__float_as_uint(m) >> 23) & 0xff) - 126 : 0;   // m < 2^E
    return 22 - E;
}

// Three int8 limbs of the K-vector in xf, element i = 32*kb + lane owned by warp (kb mod 8);
// 32-byte block kb of limb row j stored at block kb ^ j (conflict-free fragment loads).
template <int K>
__device__ __forceinline__ int make_limbs(int8_t *limbs, const float *xf, float *red, int warp, int lane) {
    constexpr int PER = K / kConsumerThreads;
    float v[PER];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        v[j] = xf[32 * (warp + 8 * j) + lane];
        m = fmaxf(m, fabsf(v[j]));
    }
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    if (lane == 0) red[warp] = m;
    cbar();
#pragma unroll
    for (int w = 0; w < kWarps; w++) m = fmaxf(m, red[w]);
    const int s = limb_exponent(m);
    const float sc = exp2i(s);
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int kb = warp + 8 * j;
        const int X = __float2int_rn(v[j] * sc);
        const int c = ((X + 128) & 255) - 128;
        const int X1 = (X - c) >> 8;
        const int b = ((X1 + 128) & 255) - 128;
        const int a = (X1 - b) >> 8;
        limbs[0 * kKmax + ((kb ^ 0) << 5) + lane] = (int8_t)a;
        limbs[1 * kKmax + ((kb ^ 1) << 5) + lane] = (int8_t)b;
        limbs[2 * kKmax + ((kb ^ 2) << 5) + lane] = (int8_t)c;
    }
    return s;
}

__global__ void __launch_bounds__(kThreads, 1)
gemv_i8_kernel(const float *x, int K, const uint8_t *packed, const ChunkRef *chunks, int N, float *y) {
    int8_t *limbs = reinterpret_cast<int8_t *>(gsm + Smem::limbs);
    float *xf = reinterpret_cast<float *>(gsm + Smem::xf);
    int *part = reinterpret_cast<int *>(gsm + Smem::part);
    float *red = reinterpret_cast<float *>(gsm + Smem::red);
    uint64_t *full = reinterpret_cast<uint64_t *>(gsm + Smem::bar);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rpc = rows_per_chunk(K);
    const int row0 = blockIdx.x * rpc;
    const int rows = min(rpc, N - row0);
    if (tid == 0) {
        mbar_init(full, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == kConsumerThreads) {
        const ChunkRef ch = chunks[blockIdx.x];
        mbar_arrive_expect_tx(full, ch.bytes);
        bulk_g2s(gsm + Smem::ring, packed + ch.off, ch.bytes, full);
    }
    if (warp == kWarps) return;
    for (int i = tid; i < K; i += kConsumerThreads) xf[i] = x[i];
    cbar();
    int s = 0;
    switch (K) {
#define XDNA_GEMV_K(KK) case KK: s = make_limbs<KK>(limbs, xf, red, warp, lane); break;
        XDNA_GEMV_K(256) XDNA_GEMV_K(512) XDNA_GEMV_K(768) XDNA_GEMV_K(1024) XDNA_GEMV_K(1536)
        XDNA_GEMV_K(2048) XDNA_GEMV_K(2560) XDNA_GEMV_K(3072)
#undef XDNA_GEMV_K
        default: return;
    }
    cbar();
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(full, 0u))
        if (globaltimer_ns() - start > 1000000000ull) return;   // bounded (1 s)
    // partial limb sums: warp w covers 32-byte blocks [w*KS/8, (w+1)*KS/8) of every row
    const uint8_t *stage = gsm + Smem::ring;
    const int g = lane >> 2, tig = lane & 3;
    const int ntiles = rows >> 3;
    const int KS = K >> 5;
    const int kb0 = warp * KS / kWarps, kb1 = (warp + 1) * KS / kWarps;
    int acc[kMaxTilesPerChunk][4];
#pragma unroll
    for (int t = 0; t < kMaxTilesPerChunk; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
    const int8_t *arow = limbs + (g < 3 ? g : 0) * kKmax;
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
                int *pp = part + ((warp * kMaxTilesPerChunk + t) * 3 + g) * 8 + 2 * tig;
                pp[0] = acc[t][0];
                pp[1] = acc[t][1];
            }
        }
    }
    cbar();
    if (tid < rows) {
        const float *meta = reinterpret_cast<const float *>(stage + (size_t)rows * K);
        const int t = tid >> 3, col = tid & 7;
        long long A = 0, B = 0, C = 0;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            const int *pp = part + ((w * kMaxTilesPerChunk + t) * 3) * 8 + col;
            A += pp[0];
            B += pp[8];
            C += pp[16];
        }
        const float v = __fmul_rn(__ll2float_rn(A * 65536 + B * 256 + C), exp2i(-s));
        y[row0 + tid] = __fadd_rn(__fmul_rn(v, meta[2 * tid]), meta[2 * tid + 1]);
    }
}

cudaError_t launch_gemv_i8(const float *x, int K, const uint8_t *packed, const ChunkRef *chunks,
                           int N, float *y, cudaStream_t st) {
    // per-device attribute: set on every launch (cheap), so a second device is covered too
    cudaError_t e = cudaFuncSetAttribute(gemv_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Smem::total);
    if (e != cudaSuccess) return e;
    const int nch = (N + rows_per_chunk(K) - 1) / rows_per_chunk(K);
    gemv_i8_kernel<<<nch, kThreads, Smem::total, st>>>(x, K, packed, chunks, N, y);
    return cudaGetLastError();
}

}  // namespace gemvop
}  // namespace xdna
