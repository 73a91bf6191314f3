// attention_tc.cu -- encoder self-attention (head dim 64) on the 5th-generation tensor cores:
// the reference's `mha` with valid_len (rust/npu-asr-host/src/lib.rs:189-326; BERT's key mask
// j >= valid_len, bert/encoder.rs:43-57), over packed variable-length sequences (BGE) or
// fixed-length clips (Whisper, 1500 positions).
//
// One CTA per (128-query tile, head, sequence); two CTAs per SM.  Warp 0 loads Q once and the
// sequence's K / V tiles of 128 keys by TMA (a 2-stage ring, no multicast); warp 1 owns TMEM
// (256 columns: S at [0, 128), O at [128, 192)) and issues, from one thread,
//   S   = Q . K_j^T      (M 128, N 128, K 64; both operands K-major in 128-byte swizzle)
//   O_j = P_j . V_j      (M 128, N 64, K 128; P K-major from shared memory, V MN-major: the
//                         [key][dim] tile exactly as TMA wrote it, no transpose)
// and S_{j+1} is issued before waiting for P_j, so it overlaps the softmax of tile j.  Warps 2-9
// (two threads per query row, each half of the keys and half of the output dims; TMEM lane
// quarter = warp % 4) read S 32 columns at a time (twice), swap partial row maxima through a
// TMEM column, mask keys at or past the sequence length, keep the running maximum and sum in f32, write
// P_j = exp2((s - m) * log2(e) / 8) as bf16 into the swizzled P buffer, and fold each O_j into
// an f32 register accumulator with the running correction, so O never needs a
// read-modify-write in TMEM.  The output row is acc / sum in bf16.  Numerics match the
// mma.sync kernel it replaces: bf16 P, f32 everything else.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <string>

#include "ptx.cuh"
#include "tc.cuh"

namespace xdna {
namespace gemm {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
}

namespace attn_tc {

constexpr int D = 768, HD = 64, LD = 3 * D;
constexpr int BQ = 128, BKV = 128, SOFTMAX = 256, THREADS = 64 + SOFTMAX;
constexpr int TILE = 128 * 128;                         // one 128-row x 128-byte swizzled tile
// 7 tiles + 128 B of barriers + up to 896 B to reach a 1024-byte boundary: 115,712 B, so two CTAs
// (plus the 1 KB each reserves) fit in an SM's 228 KB.  A base less than 128-byte aligned would
// need more padding; the kernel checks and refuses to run rather than overrun.
constexpr int PAD = 896;
constexpr int SMEM = PAD + 7 * TILE + 128;
constexpr uint32_t S_COL = 0, O_COL = 128, X_COL = 192;   // X: the row partners' exchange columns
constexpr uint64_t TIMEOUT_NS = 2000000000ull;

__device__ unsigned int g_attn_error;

__device__ __forceinline__ bool wait_b(uint64_t *bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*(volatile unsigned *)&g_attn_error) return false;
        if (globaltimer_ns() - t0 > TIMEOUT_NS) {
            atomicCAS(&g_attn_error, 0u, code);
            return false;
        }
    }
    return true;
}

// one 32-bit TMEM column of the warp's 32 lanes: store / load (thread t <-> lane base + t)
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v)) : "memory");
}
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
    return __uint_as_float(r);
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x by the hardware approximation (results below 2^-126 flush to zero: far below a bf16
// softmax weight's resolution, and exactly 0 for the masked -inf)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// two finite floats -> bf16x2 (round to nearest even) with integer ops: the same bits as
// cvt.rn.bf16x2.f32, kept off the conversion pipe that the exponentials already load
__device__ __forceinline__ uint32_t pack_bf16_rne(float a, float b) {
    const uint32_t x = __float_as_uint(a), y = __float_as_uint(b);
    const uint32_t xr = x + 0x7fffu + ((x >> 16) & 1u), yr = y + 0x7fffu + ((y >> 16) & 1u);
    return __byte_perm(xr, yr, 0x7632);
}

// barrier over the 256 softmax threads (id 1) that ORs a flag across them
__device__ __forceinline__ bool sm_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 256, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// Shared-memory descriptor of an MN-major operand in the 128-byte swizzle: rows of 128 B hold
// 64 consecutive MN elements for one K index; 8 rows (1024 B) form one swizzle atom along K.
// Both byte-offset fields are 1024 B: the atom stride along K, and (unused here, the operand
// is one atom wide in MN) the stride between 64-element MN blocks.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)(1024 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ unsigned long long *g_attn_trace;   // diagnostics: stamps of CTA (0, 0, 0), or null

__global__ void __launch_bounds__(THREADS, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const int32_t *__restrict__ cu,
                        uint16_t *__restrict__ ctx) {
    const int qt = blockIdx.x, h = blockIdx.y, sq = blockIdx.z;
    const int s0 = cu[sq], L = cu[sq + 1] - s0, q0 = qt * BQ;
    if (q0 >= L) return;                                   // the whole CTA, before any barrier
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    if (pad > (uint32_t)PAD) {                             // uniform over the CTA: nothing started yet
        if (threadIdx.x == 0) atomicCAS(&g_attn_error, 0u, 10u);
        return;
    }
    uint8_t *smem = smem_raw + pad;
    uint8_t *sQ = smem, *sKV = smem + TILE, *sP = smem + 5 * TILE;   // sKV: [stage][K | V]
    uint64_t *q_full = reinterpret_cast<uint64_t *>(smem + 7 * TILE);
    uint64_t *kv_full = q_full + 1, *kv_empty = kv_full + 2;
    uint64_t *s_full = kv_empty + 2, *s_free = s_full + 1, *p_full = s_free + 1, *o_full = p_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkv = (L + BKV - 1) / BKV;
    unsigned long long *tr = (blockIdx.x | blockIdx.y | blockIdx.z) == 0 ? g_attn_trace : nullptr;
    auto stamp = [&](int slot) {
        if (tr && slot < 512) tr[slot] = globaltimer_ns();
    };
    if (threadIdx.x == 0) stamp(511);
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; s++) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
        mbar_init(s_full, 1);
        mbar_init(s_free, SOFTMAX / 32);
        mbar_init(p_full, SOFTMAX / 32);
        mbar_init(o_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) { tc::tmem_alloc(tmem_slot, 256); tc::tmem_relinquish(); }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        mbar_arrive_expect_tx(q_full, TILE);
        tc::tma_load_2d(sQ, &tmQKV, h * HD, s0 + q0, q_full);
        for (int j = 0; j < nkv; j++) {
            const int st = j & 1;
            if (j >= 2 && !wait_b(&kv_empty[st], ((j >> 1) - 1) & 1, 1u)) break;
            uint8_t *kb = sKV + st * 2 * TILE;
            mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
            tc::tma_load_2d(kb, &tmQKV, D + h * HD, s0 + j * BKV, &kv_full[st]);
            tc::tma_load_2d(kb + TILE, &tmQKV, 2 * D + h * HD, s0 + j * BKV, &kv_full[st]);
        }
        // the loads in flight land before the CTA moves on
        wait_b(q_full, 0, 2u);
        for (int j = nkv > 2 ? nkv - 2 : 0; j < nkv; j++) wait_b(&kv_full[j & 1], (j >> 1) & 1, 2u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t id_s = tc::idesc_bf16_f32(BQ, BKV);
        constexpr uint32_t id_o = tc::idesc_bf16_f32(BQ, HD) | (1u << 16);   // B (V) MN-major
        bool ok = wait_b(q_full, 0, 3u);
        const uint64_t dq = tc::desc_k_sw128(smem_u32(sQ));
        auto issue_s = [&](int j) {
            const int st = j & 1;
            if (!(ok = ok && wait_b(&kv_full[st], (j >> 1) & 1, 4u))) return;
            if (j >= 1 && !(ok = wait_b(s_free, (j - 1) & 1, 5u))) return;
            tc::fence_after_sync();
            const uint64_t dk = tc::desc_k_sw128(smem_u32(sKV + st * 2 * TILE));
#pragma unroll
            for (int k = 0; k < HD / 16; k++) tc::mma_bf16(tmem + S_COL, dq + 2 * k, dk + 2 * k, id_s, k > 0 ? 1u : 0u);
            tc::commit(s_full);
            stamp(16 * j + 0);
        };
        if (ok) issue_s(0);
        for (int j = 0; j < nkv && ok; j++) {
            if (j + 1 < nkv) issue_s(j + 1);
            if (!ok || !(ok = wait_b(p_full, j & 1, 6u))) break;
            tc::fence_after_sync();
            const uint8_t *vb = sKV + (j & 1) * 2 * TILE + TILE;
#pragma unroll
            for (int k = 0; k < BKV / 16; k++) {
                // P: K block k / 4 (64 keys), +32 B per 16 keys inside it; V: +16 rows of 128 B
                const uint64_t dp = tc::desc_k_sw128(smem_u32(sP + (k >> 2) * TILE)) + 2 * (k & 3);
                const uint64_t dv = desc_mn_sw128(smem_u32(vb + k * 16 * 128));
                tc::mma_bf16(tmem + O_COL, dp, dv, id_o, k > 0 ? 1u : 0u);
            }
            tc::commit(o_full);
            tc::commit(&kv_empty[j & 1]);
            stamp(16 * j + 1);
        }
        // every path ends with the softmax threads released (their waits are bounded anyway)
    } else if (warp >= 2) {
        // ------------------------------------------------------------ softmax (two threads per row)
        // Warps 2-9: TMEM lane quarter q = warp % 4 holds rows 32 q + lane; warp half hf = (warp-2)/4
        // takes keys [64 hf, 64 hf + 64) of every tile (K block hf of P) and output dims
        // [32 hf, 32 hf + 32).  The two threads of a row share lane (32 q + lane), so they swap
        // their partial maxima (and, at the end, sums) through TMEM columns X_COL + hf.
        // Tile j: pass 1 (row maximum of S_j), the fold of O_{j-1} (its MMA ran meanwhile), pass 2
        // (P_j) -- so the O MMA's latency hides behind the next tile's maximum.
        const int q = warp & 3, hf = (warp - 2) >> 2, row = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const float c = 0.125f * 1.4426950408889634f;     // 1/sqrt(64) * log2(e)
        float m = -INFINITY, l = 0.0f, corr_pending = 0.0f;
        float o[32];
#pragma unroll
        for (int d = 0; d < 32; d++) o[d] = 0.0f;
        bool ok = true;
        // o = o * corr + O_t (this thread's 32 dims), t = the tile whose P.V was last committed
        auto fold = [&](int t, float corr) -> bool {
            if (sm_bar_or(!wait_b(o_full, t & 1, 8u))) return false;
            if (row == 0 && hf == 0) stamp(16 * t + 5);
            tc::fence_after_sync();
            uint32_t ov[32];
            tc::tmem_ld32(tmem + lane_base + O_COL + 32 * hf, ov);
            tc::tmem_ld_wait();
#pragma unroll
            for (int d = 0; d < 32; d++) o[d] = fmaf(o[d], corr, __uint_as_float(ov[d]));
            tc::fence_before_sync();
            if (row == 0 && hf == 0) stamp(16 * t + 6);
            return true;
        };
        for (int j = 0; j < nkv; j++) {
            if (sm_bar_or(!wait_b(s_full, j & 1, 7u))) { ok = false; break; }
            if (row == 0 && hf == 0) stamp(16 * j + 2);
            tc::fence_after_sync();
            const int kbase = j * BKV + 64 * hf;
            const bool full = j * BKV + BKV <= L;             // uniform: no key of the tile is masked
            // pass 1: the maximum over this thread's 64 keys, then over the row's 128
            float mx = -INFINITY;
#pragma unroll 1
            for (int qc = 0; qc < 2; qc++) {
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + S_COL + 64 * hf + 32 * qc, v);
                tc::tmem_ld_wait();
                if (full) {
                    float m2 = __uint_as_float(v[1]);
                    mx = fmaxf(mx, __uint_as_float(v[0]));
#pragma unroll
                    for (int i = 2; i < 32; i += 2) {
                        mx = fmaxf(mx, __uint_as_float(v[i]));
                        m2 = fmaxf(m2, __uint_as_float(v[i + 1]));
                    }
                    mx = fmaxf(mx, m2);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (kbase + 32 * qc + i < L) mx = fmaxf(mx, __uint_as_float(v[i]));
                }
            }
            tmem_st1(tmem + lane_base + X_COL + hf, mx);
            tmem_st_wait();
            tc::fence_before_sync();
            named_bar(1, SOFTMAX);
            tc::fence_after_sync();
            mx = fmaxf(mx, tmem_ld1(tmem + lane_base + X_COL + (hf ^ 1)));
            tc::tmem_ld_wait();
            if (row == 0 && hf == 0) stamp(16 * j + 3);
            const float m_new = fmaxf(m, mx);
            const float corr = exp2f((m - m_new) * c);
            const float mc = m_new * c;
            m = m_new;
            // P_{j-1} has been read by its MMA once O_{j-1} is complete: fold it, then overwrite P.
            // (A thread rewrites its X_COL only after the next tile's s_full barrier, which its
            // partner reaches after reading it.)
            if (j >= 1 && !fold(j - 1, corr_pending)) { ok = false; break; }
            corr_pending = corr;
            // pass 2: P = 2^(s c - m c) as bf16 into K block hf of the swizzled P buffer
            float ls = 0.0f;
#pragma unroll 1
            for (int qc = 0; qc < 2; qc++) {
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + S_COL + 64 * hf + 32 * qc, v);
                tc::tmem_ld_wait();
                if (qc == 1) {
                    tc::fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_free);           // S may be overwritten by S_{j+1}
                }
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    float x0 = fmaf(__uint_as_float(v[2 * i]), c, -mc);
                    float x1 = fmaf(__uint_as_float(v[2 * i + 1]), c, -mc);
                    if (!full) {
                        const int k0 = kbase + 32 * qc + 2 * i;
                        x0 = k0 < L ? x0 : -INFINITY;
                        x1 = k0 + 1 < L ? x1 : -INFINITY;
                    }
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    ls += p0 + p1;
                    pk[i] = pack_bf16_rne(p0, p1);
                }
                uint8_t *prow = sP + hf * TILE + row * 128;
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int ch = 4 * qc + u;
                    *reinterpret_cast<uint4 *>(prow + ((ch ^ (row & 7)) << 4)) =
                        make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
                }
            }
            l = l * corr + ls;
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            if (row == 0 && hf == 0) stamp(16 * j + 4);
        }
        if (ok && !fold(nkv - 1, corr_pending)) ok = false;
        if (ok) {
            // the row's sum = the two threads' partial sums (same running maximum)
            tmem_st1(tmem + lane_base + X_COL + hf, l);
            tmem_st_wait();
            tc::fence_before_sync();
            named_bar(1, SOFTMAX);
            tc::fence_after_sync();
            l += tmem_ld1(tmem + lane_base + X_COL + (hf ^ 1));
            tc::tmem_ld_wait();
        }
        if (ok && q0 + row < L) {
            const float inv = 1.0f / l;
            uint4 *dst = reinterpret_cast<uint4 *>(ctx + (size_t)(s0 + q0 + row) * D + h * HD + 32 * hf);
#pragma unroll
            for (int u = 0; u < 4; u++)
                dst[u] = make_uint4(bf16bits(o[8 * u] * inv) | (bf16bits(o[8 * u + 1] * inv) << 16),
                                    bf16bits(o[8 * u + 2] * inv) | (bf16bits(o[8 * u + 3] * inv) << 16),
                                    bf16bits(o[8 * u + 4] * inv) | (bf16bits(o[8 * u + 5] * inv) << 16),
                                    bf16bits(o[8 * u + 6] * inv) | (bf16bits(o[8 * u + 7] * inv) << 16));
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem, 256);
}

}  // namespace attn_tc

// ctx[t, h*64 .. h*64+63] = attention of the packed sequences in qkv [T_total, 2304] bf16
// (q | k | v per row, 12 heads of 64); cu [n_seqs + 1] device offsets; max_len = the longest
cudaError_t attention_tc(const uint16_t *qkv, int T_total, const int32_t *cu, int n_seqs, int max_len, uint16_t *ctx,
                         cudaStream_t st) {
    auto fn = gemm::encode_fn();
    if (!fn) return cudaErrorNotSupported;
    CUtensorMap tm;
    cuuint64_t dims[2] = {(cuuint64_t)attn_tc::LD, (cuuint64_t)T_total};
    cuuint64_t strides[1] = {(cuuint64_t)attn_tc::LD * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(qkv), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(attn_tc::attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn_tc::SMEM);
    if (e != cudaSuccess) return e;
    attn_tc::attention_tc_kernel<<<dim3((max_len + attn_tc::BQ - 1) / attn_tc::BQ, 12, n_seqs), attn_tc::THREADS,
                                   attn_tc::SMEM, st>>>(tm, cu, ctx);
    return cudaGetLastError();
}

void attention_tc_set_trace(unsigned long long *p) { cudaMemcpyToSymbol(attn_tc::g_attn_trace, &p, sizeof p); }

unsigned attention_tc_error_and_clear() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, attn_tc::g_attn_error, sizeof v);
    cudaMemcpyToSymbol(attn_tc::g_attn_error, &z, sizeof z);
    return v;
}

}  // namespace xdna

namespace xdna {
void set_last_error_message(const std::string &m);
}

extern "C" int xdna_attention_bf16(const uint16_t *qkv, int T_total, const int32_t *cu, int n_seqs, int max_len,
                                   uint16_t *ctx, void *stream) {
    if (!qkv || !cu || !ctx || T_total < 1 || n_seqs < 1 || n_seqs > 65535 || max_len < 1) {
        xdna::set_last_error_message("xdna_attention_bf16: null pointer or empty shape");
        return -1;
    }
    const cudaError_t e = xdna::attention_tc(qkv, T_total, cu, n_seqs, max_len, ctx, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        xdna::set_last_error_message(std::string("xdna_attention_bf16: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

namespace xdna {
void attention_tc_set_trace(unsigned long long *p);
}
// diagnostics: globaltimer stamps of the first CTA into trace_dev ([512] u64), or NULL for none
extern "C" void xdna_attention_set_trace(unsigned long long *trace_dev) { xdna::attention_tc_set_trace(trace_dev); }

extern "C" int xdna_attention_check(void) {
    const unsigned v = xdna::attention_tc_error_and_clear();
    if (v) {
        xdna::set_last_error_message("tensor-core attention: a bounded wait expired or the shared-memory base was "
                                     "misaligned (code " + std::to_string(v) + ")");
        return -1;
    }
    return 0;
}
