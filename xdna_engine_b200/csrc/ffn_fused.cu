// ffn_fused.cu -- the fused two-GEMM FFN with the hidden activations kept on chip:
//   out[M, N] = act(A[M, K] . W1[P, K]^T + b1) . W2[N, P]^T (+ b2) (+ residual)
// the B200 form of route_b_kernels/ffn_gemm2/ffn_gemm2_iron.py:1-30 (C = (A @ W1) @ W2 with H
// held in the NPU's MemTile), with the encoder FFN's bias and GELU / ReLU between the GEMMs.
//
// A cluster of two CTAs owns a 128-row tile.  The hidden dimension is walked in chunks of 256
// columns; CTA r computes columns [128 r, 128 r + 128) of each chunk:
//   1. GEMM1: TMEM H (128 x 128 f32) = A tile . W1 rows^T, K streamed through a TMA ring;
//   2. the epilogue warps read H from TMEM, add b1, apply the activation, round to bf16 and
//      write it into their CTA's shared-memory chunk buffer in the 128-byte-swizzled K-major
//      layout a tcgen05 operand wants (K blocks 2r and 2r+1 of the chunk's four), then one
//      bulk async copy (shared::cta -> the peer's shared::cluster, completion counted on the
//      peer's mbarrier; no multicast) gives the peer the same 32 KB, so both CTAs now hold
//      the whole 128 x 256 bf16 chunk;
//   3. GEMM2: TMEM acc (128 x N/2 f32, columns [0, 384)) += chunk . W2[rows of this CTA's
//      output half, chunk columns]^T.
// H never touches HBM.  TMEM: acc2 in columns [0, 384), H in [384, 512).  The MMA thread issues
// GEMM1 of chunk c while the epilogue is still turning chunk c-1 into bf16, then GEMM2 of
// chunk c-1; one 5-stage ring of 32 KB stages (A + W1 k-block, or one output half of a W2
// k-block) carries both GEMMs' operands in issue order.
// The chunk buffer is single: before overwriting it for chunk c, a CTA waits until both CTAs'
// GEMM2 of chunk c-1 has completed (each CTA's epilogue arrives on its own and its peer's
// "free" barrier after seeing its own GEMM2 commit).  Every wait is bounded (an error code in
// a device word, then the CTA runs to its final cluster barrier); TMEM is freed on every path.
//
// Numerics: bf16 operands, f32 accumulation in TMEM over K in order, H rounded once to bf16 --
// the rounding the unfused path (GEMM1 with the activation epilogue writing bf16, then GEMM2)
// applies to its HBM intermediate.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <string>

#include "../../include/xdna_b200.h"
#include "ptx.cuh"
#include "tc.cuh"
#include "gelu.cuh"

namespace xdna {
void set_last_error_message(const std::string &m);
namespace gemm {
bool make_tmap(CUtensorMap *tm, const void *base, int rows, int K, int ld, int box_rows, bool i8);
}

namespace ffn2 {

constexpr int BM = 128, BK = 64, PC = 256, HALF = PC / 2, STAGES = 5, STAGE_BYTES = 32 * 1024;
constexpr int A_BYTES = BM * BK * 2, W1_BYTES = HALF * BK * 2;            // 16 KB each
constexpr int HBLK = BM * 128, HBUF = 4 * HBLK;                            // 16 KB per K block, 64 KB per chunk
constexpr int H_COL = 384;                                                  // acc2 in [0, 384)
constexpr int EPI = 256;                                                   // 8 epilogue warps
constexpr int THREADS = 64 + EPI;                                          // + producer, MMA
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + HBUF + HALF * 4 + 256;
constexpr uint64_t TIMEOUT_NS = 2000000000ull;

__device__ unsigned int g_ffn_error;

__device__ __forceinline__ bool wait_b(uint64_t *bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*(volatile unsigned *)&g_ffn_error) return false;
        if (globaltimer_ns() - t0 > TIMEOUT_NS) {
            atomicCAS(&g_ffn_error, 0u, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cta address -> the same offset in CTA `rank`'s shared memory (shared::cluster)
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// bulk copy of `bytes` from this CTA's shared memory to a peer's, complete_tx on the peer's barrier
__device__ __forceinline__ void bulk_s2peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                            uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst_cluster),
        "r"(src_cta), "r"(bytes), "r"(bar_cluster)
        : "memory");
}
// barrier over the 256 epilogue threads (id 1) that also ORs a flag across them, so a decision
// taken after a bounded wait is the same in every epilogue thread
__device__ __forceinline__ bool epi_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}


struct Params {
    int M, K, P, N;
    const float *b1;            // [P] or null
    int act;                    // 0 none, 1 exact-erf GELU, 2 ReLU
    const float *b2;            // [N] or null
    const uint16_t *residual;   // [M, N] bf16 or null
    uint16_t *out_bf16;         // [M, N] or null
    float *out_f32;             // [M, N] or null
    unsigned long long *trace;  // null, or [2][1024] globaltimer stamps of cluster 0 (diagnostics)
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    ffn_fused_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *ring = smem;                                   // [STAGES][48 KB]
    uint8_t *hbuf = smem + STAGES * STAGE_BYTES;            // [4 K blocks][128 rows][128 B], swizzled
    float *sb1 = reinterpret_cast<float *>(hbuf + HBUF);       // [HALF] this chunk's b1 slice
    uint64_t *full = reinterpret_cast<uint64_t *>(sb1 + HALF);
    uint64_t *empty = full + STAGES;
    uint64_t *hacc_full = empty + STAGES;   // GEMM1 of a chunk done (MMA commit)
    uint64_t *tm_free = hacc_full + 1;      // TMEM H drained (8 epilogue warps)
    uint64_t *hready = tm_free + 1;         // chunk in shared memory: own half (1 arrival) + peer's copy (tx)
    uint64_t *g2done = hready + 1;          // GEMM2 of a chunk done (MMA commit)
    uint64_t *hfree = g2done + 1;           // both CTAs' GEMM2 of the previous chunk done (2 arrivals)
    uint64_t *acc_full = hfree + 1;         // all GEMM2 done
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = cluster_rank(), peer = r ^ 1u;
    const int m0 = (blockIdx.x >> 1) * BM;
    const int N2 = p.N / 2, nk = p.K / BK, nc = p.P / PC;
    unsigned long long *tr = (p.trace && blockIdx.x < 2) ? p.trace + blockIdx.x * 1024 : nullptr;
    auto stamp = [&](int slot) {
        if (tr && slot < 1024) tr[slot] = globaltimer_ns();
    };

    if (threadIdx.x == 0) {
        stamp(1002);
        for (int s = 0; s < STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(hacc_full, 1);
        mbar_init(tm_free, EPI / 32);
        mbar_init(hready, 1);
        mbar_init(g2done, 1);
        mbar_init(hfree, 2);
        mbar_init(acc_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) { tc::tmem_alloc(tmem_slot, 512); tc::tmem_relinquish(); }
    tc::fence_before_sync();
    __syncthreads();
    cluster_sync();                 // the peer's barriers exist before anything targets them
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        uint32_t c_ring = 0;
        bool ok = true;
        auto acquire = [&](int &s) -> bool {
            s = c_ring % STAGES;
            if (c_ring >= STAGES && !wait_b(&empty[s], ((c_ring / STAGES) - 1) & 1, 1u)) return false;
            c_ring++;
            return true;
        };
        auto gemm2_loads = [&](int c) {
            for (int j = 0; j < PC / BK && ok; j++)
                for (int h = 0; h < 2 && ok; h++) {
                    int s;
                    if (!(ok = acquire(s))) break;
                    mbar_arrive_expect_tx(&full[s], (uint32_t)(N2 / 2) * 128);
                    tc::tma_load_2d(ring + s * STAGE_BYTES, &tmW2, c * PC + BK * j, (int)r * N2 + h * (N2 / 2), &full[s]);
                }
        };
        for (int c = 0; c < nc && ok; c++) {
            for (int kb = 0; kb < nk && ok; kb++) {
                int s;
                if (!(ok = acquire(s))) break;
                uint8_t *st = ring + s * STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], A_BYTES + W1_BYTES);
                tc::tma_load_2d(st, &tmA, kb * BK, m0, &full[s]);
                tc::tma_load_2d(st + A_BYTES, &tmW1, kb * BK, c * PC + HALF * (int)r, &full[s]);
            }
            stamp(16 * c + 12);
            if (c >= 1) gemm2_loads(c - 1);
            stamp(16 * c + 13);
        }
        if (ok) gemm2_loads(nc - 1);
        // the loads in flight land before the CTA moves on
        for (uint32_t q = c_ring > STAGES ? c_ring - STAGES : 0; q < c_ring; q++)
            wait_b(&full[q % STAGES], (q / STAGES) & 1, 2u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t id1 = tc::idesc_bf16_f32(BM, HALF);
        const uint32_t id2 = tc::idesc_bf16_f32(BM, N2 / 2);
        uint32_t c_ring = 0;
        bool ok = true;
        auto gemm2 = [&](int c) {
            if (!(ok = ok && wait_b(hready, c & 1, 4u))) return;
            stamp(16 * c + 4);
            tc::fence_after_sync();
            for (int j = 0; j < PC / BK; j++)
                for (int h = 0; h < 2; h++, c_ring++) {
                    const int s = c_ring % STAGES;
                    if (!(ok = wait_b(&full[s], (c_ring / STAGES) & 1, 5u))) return;
                    tc::fence_after_sync();
                    const uint64_t da = tc::desc_k_sw128(smem_u32(hbuf + j * HBLK));
                    const uint64_t db = tc::desc_k_sw128(smem_u32(ring + s * STAGE_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc::mma_bf16(tmem + (uint32_t)(h * (N2 / 2)), da + 2 * k, db + 2 * k, id2,
                                     (c > 0 || j > 0 || k > 0) ? 1u : 0u);
                    tc::commit(&empty[s]);
                }
            tc::commit(g2done);
        };
        for (int c = 0; c < nc && ok; c++) {
            stamp(16 * c + 0);
            if (c >= 1 && !(ok = wait_b(tm_free, (c - 1) & 1, 3u))) break;
            stamp(16 * c + 1);
            tc::fence_after_sync();
            for (int kb = 0; kb < nk; kb++, c_ring++) {
                const int s = c_ring % STAGES;
                if (!(ok = wait_b(&full[s], (c_ring / STAGES) & 1, 5u))) break;
                tc::fence_after_sync();
                const uint64_t da = tc::desc_k_sw128(smem_u32(ring + s * STAGE_BYTES));
                const uint64_t db = tc::desc_k_sw128(smem_u32(ring + s * STAGE_BYTES + A_BYTES));
#pragma unroll
                for (int k = 0; k < BK / 16; k++)
                    tc::mma_bf16(tmem + H_COL, da + 2 * k, db + 2 * k, id1, (kb > 0 || k > 0) ? 1u : 0u);
                tc::commit(&empty[s]);
            }
            tc::commit(hacc_full);       // always signalled, so the epilogue never waits forever
            stamp(16 * c + 2);
            if (ok && c >= 1) gemm2(c - 1);
            stamp(16 * c + 3);
        }
        if (ok) gemm2(nc - 1);
        tc::commit(acc_full);
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue (8 warps)
        // TMEM lane quarter (warp & 3) = rows 32 (warp & 3) + lane of the tile; warp half
        // hh = (warp - 2) / 4 takes H columns [64 hh, 64 hh + 64), i.e. K block 2r + hh
        const int q = warp & 3, hh = (warp - 2) >> 2, et = threadIdx.x - 64;
        const int row_l = 32 * q + lane, row = m0 + row_l;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        // every exit from this loop is taken by all epilogue threads together (epi_bar_or), so
        // no thread is ever left waiting at a barrier the others skipped
        bool ok = true;
        for (int c = 0; c < nc; c++) {
            const int col0 = c * PC + HALF * (int)r;
            if (et < HALF) sb1[et] = p.b1 ? p.b1[col0 + et] : 0.0f;   // read after the barrier below
            if (epi_bar_or(!wait_b(hacc_full, c & 1, 6u))) { ok = false; break; }
            if (et == 0) stamp(16 * c + 8);
            tc::fence_after_sync();
            uint32_t hv[64];
            tc::tmem_ld32(tmem + lane_base + H_COL + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&hv[0]));
            tc::tmem_ld32(tmem + lane_base + H_COL + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&hv[32]));
            tc::tmem_ld_wait();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(tm_free);
            // bias + activation + bf16, packed in pairs
            const float *bb = sb1 + 64 * hh;
            uint32_t pk[32];
#pragma unroll
            for (int j = 0; j < 32; j++) {
                float a = __uint_as_float(hv[2 * j]) + bb[2 * j], b = __uint_as_float(hv[2 * j + 1]) + bb[2 * j + 1];
                if (p.act == 1) { a = gelu_erf_as(a); b = gelu_erf_as(b); }
                else if (p.act == 2) { a = fmaxf(a, 0.0f); b = fmaxf(b, 0.0f); }
                pk[j] = bf16bits(a) | (bf16bits(b) << 16);
            }
            if (et == 0) stamp(16 * c + 9);
            // the chunk buffer is free once both CTAs' GEMM2 of chunk c-1 completed
            if (c >= 1) {
                bool good = true;
                if (et == 0) {
                    good = wait_b(g2done, (c - 1) & 1, 7u);
                    if (good) {
                        mbar_arrive(hfree);
                        remote_arrive(mapa(smem_u32(hfree), peer));
                    }
                }
                good = wait_b(hfree, (c - 1) & 1, 8u) && good;
                if (epi_bar_or(!good)) { ok = false; break; }
            }
            // K block 2r + hh; row_l's 16-byte chunk j of a block sits at chunk (j ^ (row_l & 7))
            // of its 128-byte row
            uint8_t *blk = hbuf + (2 * r + hh) * HBLK + row_l * 128;
#pragma unroll
            for (int j = 0; j < 8; j++)
                *reinterpret_cast<uint4 *>(blk + ((j ^ (row_l & 7)) << 4)) =
                    make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            if (et == 0) stamp(16 * c + 10);
            tc::fence_proxy_async_smem();
            named_bar(1, EPI);
            if (et == 0) {
                stamp(16 * c + 11);
                mbar_arrive_expect_tx(hready, 2 * HBLK);                  // own half + the peer's 32 KB
                const uint32_t src = smem_u32(hbuf + 2 * r * HBLK);
                bulk_s2peer(mapa(src, peer), src, 2 * HBLK, mapa(smem_u32(hready), peer));
            }
        }
        // ---- final epilogue: acc2 columns [0, N/2) = output columns [r N/2, r N/2 + N/2)
        if (ok && !epi_bar_or(!wait_b(acc_full, 0, 9u))) {
            if (et == 0) stamp(1000);
            tc::fence_after_sync();
            for (int c0 = 32 * hh; c0 < N2; c0 += 64) {
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + c0, v);
                tc::tmem_ld_wait();
                if (row >= p.M) continue;
                const int n0 = (int)r * N2 + c0;
                float y[32];
#pragma unroll
                for (int j = 0; j < 32; j++) y[j] = __uint_as_float(v[j]) + (p.b2 ? p.b2[n0 + j] : 0.0f);
                if (p.residual) {
                    const uint4 *rp = reinterpret_cast<const uint4 *>(p.residual + (size_t)row * p.N + n0);
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const uint4 w = rp[u];
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) { y[8 * u + 2 * e] += bf16lo(ws[e]); y[8 * u + 2 * e + 1] += bf16hi(ws[e]); }
                    }
                }
                if (p.out_f32) {
                    float4 *op = reinterpret_cast<float4 *>(p.out_f32 + (size_t)row * p.N + n0);
#pragma unroll
                    for (int u = 0; u < 8; u++) op[u] = make_float4(y[4 * u], y[4 * u + 1], y[4 * u + 2], y[4 * u + 3]);
                } else {
                    uint4 *op = reinterpret_cast<uint4 *>(p.out_bf16 + (size_t)row * p.N + n0);
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        op[u] = make_uint4(bf16bits(y[8 * u]) | (bf16bits(y[8 * u + 1]) << 16),
                                           bf16bits(y[8 * u + 2]) | (bf16bits(y[8 * u + 3]) << 16),
                                           bf16bits(y[8 * u + 4]) | (bf16bits(y[8 * u + 5]) << 16),
                                           bf16bits(y[8 * u + 6]) | (bf16bits(y[8 * u + 7]) << 16));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (threadIdx.x == 0) stamp(1001);
    if (warp == 1) tc::tmem_dealloc(tmem, 512);
    cluster_sync();                 // no copy or arrive from the peer is still aimed at this CTA
}

}  // namespace ffn2
}  // namespace xdna

static unsigned long long *g_ffn_trace = nullptr;
// diagnostics: globaltimer stamps of the first cluster's CTAs into trace_dev ([2][1024] u64), or off
extern "C" void xdna_ffn_fused_set_trace(unsigned long long *trace_dev) { g_ffn_trace = trace_dev; }

extern "C" int xdna_ffn_fused_bf16(const uint16_t *A, const uint16_t *W1, const float *b1, int act, const uint16_t *W2,
                                   const float *b2, const uint16_t *residual, uint16_t *out_bf16, float *out_f32, int M,
                                   int K, int P, int N, void *stream) {
    using namespace xdna;
    if (!A || !W1 || !W2 || (!out_bf16 == !out_f32)) {
        set_last_error_message("xdna_ffn_fused_bf16: null operand, or not exactly one of out_bf16 / out_f32");
        return -1;
    }
    if (M <= 0 || K <= 0 || K % 64 || P <= 0 || P % 256 || N <= 0 || N % 64 || N > 768 || act < 0 || act > 2) {
        set_last_error_message("xdna_ffn_fused_bf16: need M > 0, K % 64 == 0, P % 256 == 0, N % 64 == 0 and "
                               "N <= 768, act 0/1/2");
        return -1;
    }
    CUtensorMap ta, t1, t2;
    if (!gemm::make_tmap(&ta, A, M, K, K, ffn2::BM, false) || !gemm::make_tmap(&t1, W1, P, K, K, ffn2::HALF, false) ||
        !gemm::make_tmap(&t2, W2, N, P, P, N / 4, false)) {
        set_last_error_message("xdna_ffn_fused_bf16: tensor map encoding failed (alignment?)");
        return -1;
    }
    cudaError_t e = cudaFuncSetAttribute(ffn2::ffn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ffn2::SMEM);
    if (e == cudaSuccess) {
        ffn2::Params prm{M, K, P, N, b1, act, b2, residual, out_bf16, out_f32, g_ffn_trace};
        const int tiles = (M + ffn2::BM - 1) / ffn2::BM;
        ffn2::ffn_fused_kernel<<<2 * tiles, ffn2::THREADS, ffn2::SMEM, static_cast<cudaStream_t>(stream)>>>(ta, t1, t2,
                                                                                                         prm);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_ffn_fused_bf16: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int xdna_ffn_fused_check(void) {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, xdna::ffn2::g_ffn_error, sizeof v);
    cudaMemcpyToSymbol(xdna::ffn2::g_ffn_error, &z, sizeof z);
    if (v) {
        xdna::set_last_error_message("fused FFN: a bounded wait expired (code " + std::to_string(v) + ")");
        return -1;
    }
    return 0;
}
