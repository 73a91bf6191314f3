// gemm_tc.cu -- encoder GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's resident NPU GEMM engine for encoder projections,
// CtxAOp::forward_view (rust/npu-asr/src/ctx2.rs:674-770) with its host bias / GELU epilogue
// (bert/encoder.rs:43-57, npu-asr-host gelu lib.rs:464-495) and FfnMm2's K-split fc2
// (ctx2.rs:1195-1288): C[M, N] = epi(A[M, K] . B[N, K]^T), bf16 operands, f32 accumulation
// (in TMEM, so the K reduction is never split), fused epilogue: + bias, optional exact-erf
// GELU (the reference's Abramowitz-Stegun form), optional + residual, bf16 out.
//
// Persistent kernel, one CTA per SM, 128 x 256 output tiles: warp 0 issues TMA loads of A
// and B k-blocks (64 bf16 = 128 B per row, SWIZZLE_128B, no multicast) into a 4-stage ring;
// warp 1 allocates all 512 TMEM columns (two 256-column f32 accumulators) and issues
// tcgen05.mma (M 128, N 256, K 16) from one thread, releasing each stage with
// tcgen05.commit; warps 2-9 drain an accumulator with tcgen05.ld (two warps per 32-lane TMEM
// quarter, half the columns each) while the MMAs of the next tile fill the other one.  Every wait is bounded; TMEM
// is freed on every exit path.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/xdna_b200.h"
#include "ptx.cuh"
#include "tc.cuh"
#include "gelu.cuh"

namespace xdna {
void set_last_error_message(const std::string &m);

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
// the int8 kernel gives one ring stage to the epilogue's output staging (8 warps x 8 KB)
__host__ __device__ constexpr int stages_of(bool i8) { return i8 ? 3 : 4; }
constexpr int STG_BYTES = 8 * 8192;
__host__ __device__ constexpr int smem_of(bool i8) { return 1024 + stages_of(i8) * STAGE_BYTES + (i8 ? STG_BYTES : 0) + 4 * BN * 4 + 256; }
constexpr int THREADS = 320;
constexpr int EPI_THREADS = 256;
constexpr uint64_t TIMEOUT_NS = 2000000000ull;

static __device__ unsigned int g_gemm_error;

__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*(volatile unsigned *)&g_gemm_error) return false;
        if (globaltimer_ns() - t0 > TIMEOUT_NS) {
            atomicCAS(&g_gemm_error, 0u, code);
            return false;
        }
    }
    return true;
}


// bf16 operands, f32 accumulators: C = act(acc + bias) (+ residual), bf16 or f32 out
struct EpiBf16 {
    const float *bias;          // [N] or null
    const uint16_t *residual;   // [M, ldr] bf16 or null; row r reads residual row r % res_mod
    int ldr;
    int res_mod;                // 0: residual row = output row
    int act;                    // 0 none, 1 exact-erf GELU, 2 ReLU
    uint16_t *out;              // [M, ldc] bf16 (or null when out_f32 is set)
    float *out_f32;             // [M, ldc] f32 or null
    int ldc;

    __device__ __forceinline__ void load_cols(float *s, int n0, int j) const {
        s[j] = bias ? bias[n0 + j] : 0.0f;
    }
    // 64 accumulator columns [col, col + 64) of output row `row`; s = this tile's column params
    __device__ __forceinline__ void apply(int row, int col, const uint32_t *r, const float *s) const {
        const int rrow = res_mod ? row % res_mod : row;
        const uint4 *rp = residual ? reinterpret_cast<const uint4 *>(residual + (size_t)rrow * ldr + col) : nullptr;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float y = __uint_as_float(r[8 * u + j]) + s[8 * u + j];
                if (act == 1) y = gelu_erf_as(y);
                else if (act == 2) y = fmaxf(y, 0.0f);
                v[j] = y;
            }
            if (rp) {
                const uint4 w = rp[u];
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; e++) { v[2 * e] += bf16lo(ws[e]); v[2 * e + 1] += bf16hi(ws[e]); }
            }
            if (out_f32) {
                float4 *op = reinterpret_cast<float4 *>(out_f32 + (size_t)row * ldc + col + 8 * u);
                op[0] = make_float4(v[0], v[1], v[2], v[3]);
                op[1] = make_float4(v[4], v[5], v[6], v[7]);
            } else {
                uint4 w;
                w.x = bf16bits(v[0]) | (bf16bits(v[1]) << 16);
                w.y = bf16bits(v[2]) | (bf16bits(v[3]) << 16);
                w.z = bf16bits(v[4]) | (bf16bits(v[5]) << 16);
                w.w = bf16bits(v[6]) | (bf16bits(v[7]) << 16);
                reinterpret_cast<uint4 *>(out + (size_t)row * ldc + col)[u] = w;
            }
        }
    }
};

// int8 operands, s32 accumulators, the reference's dequant epilogue (rust/npu-asr/src/ctx2.rs
// dequant_epi 1386-1411): y = (float(acc) * s_a[clip(row)]) * ws[n] (+ bias[n]), then
// act (SiLU v * sigmoid(v), or GLU over interleaved column pairs (value, gate) ->
// value * sigmoid(gate), written at column n / 2), then out = residual + alpha * y; f32 out.
// Optionally the per-clip max |out| (the next quantisation's scale) is folded into amax[clip]
// (atomicMax on the bit pattern: order-free and exact for non-negative floats).  The kernel
// stages each warp's 32-row output slices in shared memory and writes them with TMA stores
// (the residual slice comes in by TMA the same way).
struct EpiI8 {
    const float *sa;            // [clips] activation scales
    int rows_per_clip;
    const float *ws;            // [N] weight scales
    const float *bias;          // [N] or null
    int act;                    // 0 none, 1 SiLU, 3 GLU pairs
    const float *residual;      // [M, ldr] f32 or null (may alias out)
    int ldr;
    float alpha;
    float *out;                 // [M, ldc] f32
    int ldc;
    unsigned *amax;             // [clips] or null

    __device__ __forceinline__ void load_cols(float *s, int n0, int j) const {
        s[j] = ws[n0 + j];
        s[BN + j] = bias ? bias[n0 + j] : 0.0f;
    }
    // sigmoid(g) = (1 + tanh(g / 2)) / 2 with the hardware tanh (one special-function op)
    __device__ __forceinline__ static float sigmoid(float g) {
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
        return fmaf(0.5f, t, 0.5f);
    }
    // values of row `row` for the 64 accumulator columns in r; returns how many (64, or 32 for GLU)
    __device__ __forceinline__ int compute(int row, const uint32_t *r, const float *s, float *v) const {
        const float a = sa[row / rows_per_clip];
#pragma unroll
        for (int j = 0; j < 64; j++) {
            float t = __fmul_rn(__fmul_rn((float)(int)r[j], a), s[j]);
            if (bias) t = __fadd_rn(t, s[BN + j]);
            v[j] = t;
        }
        if (act == 3) {
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = __fmul_rn(v[2 * j], sigmoid(v[2 * j + 1]));
            return 32;
        }
        if (act == 1) {
#pragma unroll
            for (int j = 0; j < 64; j++) v[j] = __fmul_rn(v[j], sigmoid(v[j]));
        }
        return 64;
    }
};

// Persistent: CTA b handles tiles b, b + grid, ...; tile t -> (m = t / n_tiles, n = t % n_tiles)
// so CTAs running together share A rows in L2.  Two TMEM accumulators of 256 columns let the
// epilogue of tile i overlap the MMAs of tile i + 1.  I8 selects kind::i8 (int8 operands, 128
// K-elements per 128-byte stage row, s32 accumulators) over kind::f16 (bf16, 64 per row).
template <bool I8, class E>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, int M, int N, int K,
            E epi) {
    constexpr int STAGES = stages_of(I8);
    constexpr int KE = I8 ? 128 : 64;            // K elements per stage (128 bytes per row)
    constexpr int KI = I8 ? 32 : 16;             // K elements per MMA instruction (32 bytes)
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *stA = smem;                            // [STAGES][BM][128 B], swizzled
    uint8_t *stB = smem + STAGES * A_BYTES;         // [STAGES][BN][128 B], swizzled
    uint8_t *stg = smem + STAGES * STAGE_BYTES;     // I8: [8 warps][2 boxes][32 rows][128 B], swizzled
    float *scol = reinterpret_cast<float *>(stg + (I8 ? STG_BYTES : 0));   // [2][2][BN] column params
    uint64_t *full = reinterpret_cast<uint64_t *>(scol + 4 * BN);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;               // [2]
    uint64_t *tempty = tfull + 2;                   // [2]
    uint64_t *rbar = tempty + 2;                    // [8] residual loads, one per epilogue warp
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rbar + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = K / KE;
    const int n_tiles = N / BN, m_tiles = (M + BM - 1) / BM;
    const int total = n_tiles * m_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; a++) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], EPI_THREADS / 32); }
        for (int a = 0; a < 8; a++) mbar_init(&rbar[a], 1);
        mbar_fence_init();
    }
    if (warp == 1) { tc::tmem_alloc(tmem_slot, 2 * BN); tc::tmem_relinquish(); }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer
        uint32_t c = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            const int m0 = (t / n_tiles) * BM, n0 = (t % n_tiles) * BN;
            for (int kb = 0; kb < nk; kb++, c++) {
                const int s = c % STAGES;
                if (c >= STAGES && !wait_bounded(&empty[s], ((c / STAGES) - 1) & 1, 1u)) { ok = false; break; }
                mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                tc::tma_load_2d(stA + s * A_BYTES, &tmA, kb * KE, m0, &full[s]);
                tc::tma_load_2d(stB + s * B_BYTES, &tmB, kb * KE, n0, &full[s]);
            }
        }
        // drain: the loads in flight must land before the CTA exits
        for (uint32_t q = c > STAGES ? c - STAGES : 0; q < c; q++) wait_bounded(&full[q % STAGES], (q / STAGES) & 1, 2u);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer (one thread)
        constexpr uint32_t idesc = I8 ? tc::idesc_s8_s32(BM, BN) : tc::idesc_bf16_f32(BM, BN);
        uint32_t c = 0;
        int i = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total; t += gridDim.x, i++) {
            const int acc = i & 1;
            if (ok && i >= 2 && !wait_bounded(&tempty[acc], ((i >> 1) - 1) & 1, 3u)) ok = false;
            tc::fence_after_sync();
            const uint32_t d = tmem + (uint32_t)(acc * BN);
            for (int kb = 0; kb < nk && ok; kb++, c++) {
                const int s = c % STAGES;
                if (!wait_bounded(&full[s], (c / STAGES) & 1, 4u)) { ok = false; break; }
                tc::fence_after_sync();
                const uint64_t da = tc::desc_k_sw128(smem_u32(stA + s * A_BYTES));
                const uint64_t db = tc::desc_k_sw128(smem_u32(stB + s * B_BYTES));
#pragma unroll
                for (int k = 0; k < KE / KI; k++) {   // 32 bytes per MMA = +2 in the start field
                    if (I8) tc::mma_s8(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    else tc::mma_bf16(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                }
                tc::commit(&empty[s]);
            }
            tc::commit(&tfull[acc]);   // always signalled, so the epilogue never waits forever
        }
    } else if (warp >= 2) {
        // ---------------- epilogue: 8 warps; TMEM lane quarter (warp & 3) holds rows
        // 32*(warp & 3) + lane, and warp half h = (warp - 2) / 4 takes columns [128h, 128h+128)
        const int q = warp & 3, h = (warp - 2) >> 2;
        const int et = threadIdx.x - 64;
        float rmax = 0.0f;
        uint32_t rph = 0;
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, i++) {
            const int acc = i & 1;
            const int m0 = (t / n_tiles) * BM, n0 = (t % n_tiles) * BN;
            const int row = m0 + 32 * q + lane;
            float *cs = scol + acc * 2 * BN;
            for (int j = et; j < BN; j += EPI_THREADS) epi.load_cols(cs, n0, j);
            named_bar(2, EPI_THREADS);
            wait_bounded(&tfull[acc], (i >> 1) & 1, 5u);
            tc::fence_after_sync();
#pragma unroll 1
            for (int c0 = 128 * h; c0 < 128 * h + 128; c0 += 64) {
                uint32_t r[64];
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN + c0);
                tc::tmem_ld32(ta, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
                tc::tmem_ld32(ta + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
                tc::tmem_ld_wait();
                if constexpr (I8) {
                    float v[64];
                    const int nc = epi.compute(row < M ? row : m0, r, cs + c0, v);
                    const int oc = epi.act == 3 ? (n0 + c0) >> 1 : n0 + c0;
                    const int r0 = m0 + 32 * q;
                    uint8_t *sb = stg + (warp - 2) * 8192;
                    if (lane == 0) tc::bulk_wait_read0();   // the previous slice's stores have read sb
                    __syncwarp();
                    if (epi.residual) {
                        if (lane == 0) {
                            mbar_arrive_expect_tx(&rbar[warp - 2], (uint32_t)nc * 128);
                            for (int b = 0; b < nc / 32; b++) tc::tma_load_2d(sb + b * 4096, &tmR, oc + 32 * b, r0, &rbar[warp - 2]);
                        }
                        wait_bounded(&rbar[warp - 2], rph, 6u);
                        rph ^= 1u;
                    }
#pragma unroll
                    for (int b = 0; b < 2; b++) {
                        if (b * 32 < nc) {
#pragma unroll
                            for (int j = 0; j < 8; j++) {
                                float4 *p = reinterpret_cast<float4 *>(sb + b * 4096 + lane * 128 + ((j ^ (lane & 7)) << 4));
                                float4 y = make_float4(v[32 * b + 4 * j], v[32 * b + 4 * j + 1], v[32 * b + 4 * j + 2],
                                                       v[32 * b + 4 * j + 3]);
                                if (epi.residual) {
                                    const float4 rq = *p;
                                    y.x = __fadd_rn(rq.x, __fmul_rn(epi.alpha, y.x));
                                    y.y = __fadd_rn(rq.y, __fmul_rn(epi.alpha, y.y));
                                    y.z = __fadd_rn(rq.z, __fmul_rn(epi.alpha, y.z));
                                    y.w = __fadd_rn(rq.w, __fmul_rn(epi.alpha, y.w));
                                }
                                *p = y;
                                rmax = fmaxf(rmax, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
                            }
                        }
                    }
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        for (int b = 0; b < nc / 32; b++) tc::tma_store_2d(&tmO, sb + b * 4096, oc + 32 * b, r0);
                        tc::bulk_commit();
                    }
                } else {
                    if (row < M) epi.apply(row, n0 + c0, r, cs + c0);
                }
            }
            if constexpr (I8) {
                if (epi.amax && row < M) atomicMax(epi.amax + row / epi.rows_per_clip, __float_as_uint(rmax));
                rmax = 0.0f;
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        if (I8 && lane == 0) tc::bulk_wait0();   // every output store has landed before the CTA exits
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, 2 * BN);
}

// ------------------------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// K-major matrix [rows, K] (row stride ld elements) as 128-byte x box_rows boxes with 128 B
// swizzle: bf16 (64 elements per box row) or int8 (128)
bool make_tmap(CUtensorMap *tm, const void *base, int rows, int K, int ld, int box_rows, bool i8) {
    auto fn = encode_fn();
    if (!fn) return false;
    const int es = i8 ? 1 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * es};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// SMs of the current device, queried per launch (cheap; no process-wide cache that another
// device or thread could see stale)
static int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// f32 matrix [rows, cols] (row stride ld) as 32 x 32 boxes (128-byte rows) with 128 B swizzle:
// the int8 epilogue's output and residual slices
bool make_tmap_f32(CUtensorMap *tm, const void *base, int rows, int cols, int ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool I8, class E>
cudaError_t launch_t(const void *A, int lda, const void *B, int ldb, int M, int N, int K, const E &epi,
                     cudaStream_t st, const CUtensorMap &to, const CUtensorMap &tr) {
    CUtensorMap ta, tb;
    if (!make_tmap(&ta, A, M, K, lda, BM, I8) || !make_tmap(&tb, B, N, K, ldb, BN, I8)) return cudaErrorInvalidValue;
    constexpr int smem = smem_of(I8);
    // the attribute is per device and cheap to set, so it is set on every launch (a
    // process-wide "done" flag would skip it on a second device)
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<I8, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int tiles = (N / BN) * ((M + BM - 1) / BM);
    const int sms = sm_count();
    gemm_kernel<I8, E><<<tiles < sms ? tiles : sms, THREADS, smem, st>>>(ta, tb, to, tr, M, N, K, epi);
    return cudaGetLastError();
}

}  // namespace gemm

cudaError_t gemm_bf16(const uint16_t *A, int lda, const uint16_t *B, int ldb, int M, int N, int K,
                      const float *bias, const uint16_t *residual, int ldr, int act, uint16_t *C, int ldc,
                      cudaStream_t st, int res_mod, float *C_f32) {
    gemm::EpiBf16 e{bias, residual, ldr, res_mod, act, C, C_f32, ldc};
    CUtensorMap unused{};
    return gemm::launch_t<false>(A, lda, B, ldb, M, N, K, e, st, unused, unused);
}

cudaError_t gemm_i8(const int8_t *A, int lda, const int8_t *B, int ldb, int M, int N, int K, const float *sa,
                    int rows_per_clip, const float *ws, const float *bias, int act, const float *residual, int ldr,
                    float alpha, float *C, int ldc, unsigned *amax, cudaStream_t st) {
    gemm::EpiI8 e{sa, rows_per_clip, ws, bias, act, residual, ldr, alpha, C, ldc, amax};
    const int ncols = act == 3 ? N / 2 : N;
    CUtensorMap to, tr;
    if (!gemm::make_tmap_f32(&to, C, M, ncols, ldc) ||
        !gemm::make_tmap_f32(&tr, residual ? residual : C, M, ncols, residual ? ldr : ldc))
        return cudaErrorInvalidValue;
    return gemm::launch_t<true>(A, lda, B, ldb, M, N, K, e, st, to, tr);
}

unsigned gemm_error_and_clear() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, gemm::g_gemm_error, sizeof v);
    cudaMemcpyToSymbol(gemm::g_gemm_error, &z, sizeof z);
    return v;
}

}  // namespace xdna

extern "C" int xdna_gemm_bf16(const uint16_t *A, const uint16_t *B, const float *bias, const uint16_t *residual,
                              uint16_t *C, int M, int N, int K, int gelu, void *stream) {
    using namespace xdna;
    if (!A || !B || !C) { set_last_error_message("xdna_gemm_bf16: null pointer"); return -1; }
    if (M <= 0 || N <= 0 || K <= 0 || N % 256 || K % 64) {
        set_last_error_message("xdna_gemm_bf16: need M > 0, N % 256 == 0, K % 64 == 0");
        return -1;
    }
    cudaError_t e = gemm_bf16(A, K, B, K, M, N, K, bias, residual, N, gelu, C, N, (cudaStream_t)stream, 0, nullptr);
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_gemm_bf16: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int xdna_gemm_i8(const int8_t *A, const int8_t *B, const float *sa, int rows_per_clip, const float *ws,
                            const float *bias, int act, const float *residual, float alpha, float *C,
                            unsigned *amax, int M, int N, int K, void *stream) {
    using namespace xdna;
    if (!A || !B || !sa || !ws || !C) { set_last_error_message("xdna_gemm_i8: null pointer"); return -1; }
    if (M <= 0 || N <= 0 || K <= 0 || N % 256 || K % 128 || rows_per_clip <= 0 || (act != 0 && act != 1 && act != 3)) {
        set_last_error_message("xdna_gemm_i8: need M > 0, N % 256 == 0, K % 128 == 0, rows_per_clip > 0, act 0/1/3");
        return -1;
    }
    const int ldc = act == 3 ? N / 2 : N;
    cudaError_t e = gemm_i8(A, K, B, K, M, N, K, sa, rows_per_clip, ws, bias, act, residual, ldc, alpha, C, ldc, amax,
                            (cudaStream_t)stream);
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_gemm_i8: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int xdna_gemm_check(void) {
    const unsigned v = xdna::gemm_error_and_clear();
    if (v) {
        xdna::set_last_error_message("tensor-core GEMM: a bounded wait expired (code " + std::to_string(v) + ")");
        return -1;
    }
    return 0;
}
