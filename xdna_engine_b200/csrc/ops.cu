// ops.cu -- op-level entry points of the device layer (the npu-xrt replacement, one call per
// reference dispatch), for hosts that drive the decode op by op the way CtxDecode does:
//
//  * device buffers        shim_bo_alloc / _write / _read / _free (rust/npu-xrt/shim/xrt_shim.h:16-40)
//  * fused arenas           FusedArena (rust/npu-xrt/src/lib.rs:641-744): input / output / scratch
//                           regions addressed by byte offset
//  * asynchronous runs      shim_run_matmul8_start / shim_run_wait / shim_run_free (xrt_shim.h:45-55):
//                           a run marks the work enqueued on a stream so far; the wait is bounded
//  * bf16 GEMV              CtxDecode::register_weight + gemv (rust/npu-asr/src/ctx_decode.rs:260-369)
//  * fused norm + GEMV      CtxDecode::register_fused + fused_norm_gemv (ctx_decode.rs:566-643): the
//                           norm's gamma folded into the weight (W'' = diag(gamma) W), LN's beta into
//                           the bias (bias' = beta . W + bias), the input statistics in f64 on the host
//  * conformer bricks       dwconv1d_glu_silu: GLU -> depthwise conv1d k 'same' -> SiLU (the conv
//                           module's middle, encoder.rs conv_module + ops.rs:92-110, the dwconv1d.cc
//                           brick); subsample_conv2d: one conv2d of the /8 subsample with bf16
//                           operands, f32 accumulation, optional ReLU, bf16 out (subsample_patch_embed.cc)
//  * paged decode attention the mha_tile kernel (route_b_kernels/mha_decode/mha_decode.cc:90-168) over
//                           the reference's packed K/V tiles (ctx_decode.rs:468-555)
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/xdna_b200.h"

namespace xdna {
void set_last_error_message(const std::string &m);
}
using xdna::set_last_error_message;

struct XdnaDevice;   // defined in engine.cu; only its ordinal is needed here
extern "C" int xdna_device_ordinal(const XdnaDevice *dev);

struct XdnaBuffer {
    int ordinal = 0;
    void *ptr = nullptr;
    size_t bytes = 0;
};
// the three resident regions of a fused dispatch: input, output, scratch (FusedArena)
struct XdnaArena {
    XdnaBuffer *part[3] = {nullptr, nullptr, nullptr};
};
struct XdnaRun {
    int ordinal = 0;
    cudaEvent_t ev = nullptr;
};
struct XdnaGemvBf16 {
    int ordinal = 0;
    int K = 0, N = 0, Kp = 0;
    int norm = 0;                   // 0 none, 1 RMSNorm, 2 LayerNorm
    float eps = 0.0f;
    uint16_t *w = nullptr;          // [N][Kp] bf16 of W'' (gamma folded), K padded to 8
    float *bias = nullptr;          // [N] bias' (folded) or bias
    float *x = nullptr, *y = nullptr;   // staging for the host-in / host-out call
};

namespace {

bool ck(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_last_error_message(std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

uint16_t bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);   // quiet NaN
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// ---- y[n] = sum_k bf16(x[k]) * W''[n][k] (f32 accumulation) + bias[n]
// One warp per output row; lane l covers k in 8-wide groups l, l + 32, ...  (fma chain, then
// the xor butterfly).  x is staged in shared memory as bf16-rounded f32.
__global__ void gemv_bf16_kernel(const uint16_t *__restrict__ w, const float *__restrict__ x,
                                 const float *__restrict__ bias, float *__restrict__ y, int N, int K, int Kp) {
    extern __shared__ float xs[];
    for (int k = threadIdx.x; k < Kp; k += blockDim.x)
        xs[k] = k < K ? __bfloat162float(__float2bfloat16_rn(x[k])) : 0.0f;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * (blockDim.x >> 5) + warp;
    if (n >= N) return;
    const uint4 *row = reinterpret_cast<const uint4 *>(w + (size_t)n * Kp);
    float acc = 0.0f;
    for (int g = lane; g < Kp / 8; g += 32) {
        const uint4 v = row[g];
        const float *xv = xs + 8 * g;
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            acc = fmaf(__uint_as_float(u[i] << 16), xv[2 * i], acc);
            acc = fmaf(__uint_as_float(u[i] & 0xffff0000u), xv[2 * i + 1], acc);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[n] = acc + (bias ? bias[n] : 0.0f);
}

// ---- mha_tile over the packed tiles of every head: one CTA of 64 threads per head.
// kv: [H][n_tiles][K 64x64 | V 64x64 | int32 header as 2 bf16] bf16; header > 0: that many keys,
// < 0: the last non-empty tile with |h| keys, 0: empty.  Per tile the scores q.k * 1/8, the tile's
// max and exp-weights update the running (max, sum, acc) in f32 (the online softmax of mha_tile,
// applied per tile); ctx = acc / sum after the last tile.
constexpr int kTkv = 64, kHd = 64;
__global__ void mha_decode_paged_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ kv,
                                        int n_tiles, float *__restrict__ ctx) {
    __shared__ float qs[kHd], ps[kTkv], red[2];
    const int h = blockIdx.x, t = threadIdx.x;
    qs[t] = __uint_as_float((uint32_t)q[h * kHd + t] << 16);
    float m = -3.0e38f, l = 0.0f, acc = 0.0f;
    __syncthreads();
    const size_t tile_elems = 2 * kTkv * kHd + 2;
    for (int ti = 0; ti < n_tiles; ti++) {
        const uint16_t *tile = kv + ((size_t)h * n_tiles + ti) * tile_elems;
        const int32_t hdr = *reinterpret_cast<const int32_t *>(tile + 2 * kTkv * kHd);   // 4-byte aligned
        const int s = hdr < 0 ? -hdr : hdr;
        if (s == 0) continue;
        float sc = -INFINITY;
        if (t < s) {
            // the packed tiles are 16,388 bytes apart, so only 4-byte alignment holds: 32-bit loads
            const uint32_t *kr = reinterpret_cast<const uint32_t *>(tile + t * kHd);
            float a = 0.0f;
#pragma unroll 8
            for (int c = 0; c < kHd / 2; c++) {
                const uint32_t u = kr[c];
                a = fmaf(qs[2 * c], __uint_as_float(u << 16), a);
                a = fmaf(qs[2 * c + 1], __uint_as_float(u & 0xffff0000u), a);
            }
            sc = a * 0.125f;
        }
        float tm = sc;
#pragma unroll
        for (int o = 16; o; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
        if ((t & 31) == 0) red[t >> 5] = tm;
        __syncthreads();
        const float m_new = fmaxf(m, fmaxf(red[0], red[1]));
        const float p = t < s ? expf(sc - m_new) : 0.0f;
        ps[t] = p;
        __syncthreads();
        const float corr = expf(m - m_new);
        float psum = 0.0f, a = 0.0f;
        const uint16_t *V = tile + kTkv * kHd;
        for (int j = 0; j < s; j++) {
            psum += ps[j];
            a = fmaf(ps[j], __uint_as_float((uint32_t)V[j * kHd + t] << 16), a);
        }
        l = l * corr + psum;
        acc = acc * corr + a;
        m = m_new;
        __syncthreads();
        if (hdr < 0) break;
    }
    ctx[h * kHd + t] = l > 0.0f ? acc / l : 0.0f;
}


// ---- conv module middle: y[b][t][c] = silu(bias[c] + sum_j taps[c][j] * glu[b][t + j - pad][c])
// with glu[t][c] = x[t][c] * sigmoid(x[t][C + c]) (x = pw1 output [B][T][2C]); taps skipped where
// t + j - pad falls outside [0, T) (ops.rs:92-110: the sum starts at the bias and adds the valid
// taps in order).  One thread per channel walks kRows rows of one clip with the last k GLU
// values in a register window; loads and stores are coalesced across channels.
constexpr int kDwRows = 32;
__device__ __forceinline__ float sigmoid_f(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }
template <int k>
__global__ void __launch_bounds__(128) dwconv1d_glu_silu_kernel(const float *__restrict__ x, int T, int C,
                                                                const float *__restrict__ taps,
                                                                const float *__restrict__ bias, float *__restrict__ y) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.z;
    if (c >= C) return;
    constexpr int pad = (k - 1) / 2;
    const int t0 = blockIdx.y * kDwRows;
    const float *xb = x + (size_t)b * T * 2 * C;
    float tp[k];
#pragma unroll
    for (int j = 0; j < k; j++) tp[j] = taps[(size_t)c * k + j];
    const float bc = bias[c];
    auto glu = [&](int s) -> float {
        const float *r = xb + (size_t)s * 2 * C;
        return __fmul_rn(r[c], sigmoid_f(r[C + c]));
    };
    float win[k];                             // win[j] = glu(t + j - pad) for the current t
#pragma unroll
    for (int j = 0; j < k - 1; j++) {
        const int s = t0 + j - pad;
        win[j + 1] = (s >= 0 && s < T) ? glu(s) : 0.0f;
    }
    const int t_end = min(T, t0 + kDwRows);
    for (int t = t0; t < t_end; t++) {
#pragma unroll
        for (int j = 0; j < k - 1; j++) win[j] = win[j + 1];
        const int s_new = t + k - 1 - pad;
        win[k - 1] = s_new < T ? glu(s_new) : 0.0f;
        float acc = bc;
#pragma unroll
        for (int j = 0; j < k; j++) {
            const int s = t + j - pad;
            if (s < 0 || s >= T) continue;
            acc = __fadd_rn(acc, __fmul_rn(tp[j], win[j]));
        }
        y[((size_t)b * T + t) * C + c] = __fmul_rn(acc, sigmoid_f(acc));
    }
}

// ---- conv2d of the subsample (ops.rs:38-89 order): out[b][o][oh][ow] = bias[o] + sum over the
// group's input channels ic and taps (i, j), in that order, of w[o][ic][i][j] * x[b][g*gci+ic][ih][iw]
// (zero-weight taps and taps outside the padded image skipped; a pointwise conv adds the bias
// after the sum, as the reference's matmul fast path does); ReLU optional; x, w bf16, the
// products exact in f32, every add rounded to f32, the result rounded once to bf16.  NCHW; one
// thread per output position, consecutive threads on consecutive ow.
__global__ void __launch_bounds__(256) conv2d_bf16_kernel(const uint16_t *__restrict__ x, int ci, int hin, int win,
                                                          const uint16_t *__restrict__ w,
                                                          const float *__restrict__ bias, int co, int kh, int kw,
                                                          int stride, int pad, int groups, int relu, int hout,
                                                          int wout, uint16_t *__restrict__ out) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x, o = blockIdx.y, b = blockIdx.z;
    if (p >= hout * wout) return;
    const int oh = p / wout, ow = p % wout;
    const int gci = ci / groups, g = o / (co / groups);
    // the pointwise case is conv2d's matmul fast path: the dot product first, then + bias
    const bool pointwise = kh == 1 && kw == 1 && groups == 1 && stride == 1 && pad == 0;
    float acc = bias && !pointwise ? bias[o] : 0.0f;
    const uint16_t *wo = w + (size_t)o * gci * kh * kw;
    for (int ic = 0; ic < gci; ic++) {
        const uint16_t *xp = x + ((size_t)b * ci + g * gci + ic) * hin * win;
        for (int i = 0; i < kh; i++) {
            const int ih = oh * stride + i - pad;
            for (int j = 0; j < kw; j++) {
                const float wv = __uint_as_float((uint32_t)wo[(ic * kh + i) * kw + j] << 16);
                const int iw = ow * stride + j - pad;
                if (wv == 0.0f || ih < 0 || ih >= hin || iw < 0 || iw >= win) continue;
                acc = __fadd_rn(acc, __fmul_rn(wv, __uint_as_float((uint32_t)xp[(size_t)ih * win + iw] << 16)));
            }
        }
    }
    if (bias && pointwise) acc = __fadd_rn(acc, bias[o]);
    if (relu) acc = fmaxf(acc, 0.0f);
    out[(((size_t)b * co + o) * hout + oh) * wout + ow] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------------------- buffers
XdnaBuffer *xdna_buffer_alloc(XdnaDevice *dev, size_t bytes) {
    if (!dev || bytes == 0) { set_last_error_message("xdna_buffer_alloc: null device or zero size"); return nullptr; }
    auto *b = new XdnaBuffer();
    b->ordinal = xdna_device_ordinal(dev);
    b->bytes = bytes;
    if (!ck(cudaSetDevice(b->ordinal), "xdna_buffer_alloc") || !ck(cudaMalloc(&b->ptr, bytes), "xdna_buffer_alloc")) {
        delete b;
        return nullptr;
    }
    return b;
}
void xdna_buffer_free(XdnaBuffer *b) {
    if (!b) return;
    cudaSetDevice(b->ordinal);
    cudaFree(b->ptr);
    delete b;
}
void *xdna_buffer_device_ptr(XdnaBuffer *b) { return b ? b->ptr : nullptr; }
int xdna_buffer_write(XdnaBuffer *b, const void *src, size_t bytes, size_t offset) {
    if (!b || (!src && bytes)) { set_last_error_message("xdna_buffer_write: null pointer"); return -1; }
    if (offset > b->bytes || bytes > b->bytes - offset) { set_last_error_message("xdna_buffer_write: range beyond the buffer"); return -1; }
    if (!ck(cudaSetDevice(b->ordinal), "xdna_buffer_write")) return -1;
    return ck(cudaMemcpy(static_cast<char *>(b->ptr) + offset, src, bytes, cudaMemcpyHostToDevice), "xdna_buffer_write") ? 0 : -1;
}
int xdna_buffer_read(XdnaBuffer *b, void *dst, size_t bytes, size_t offset) {
    if (!b || (!dst && bytes)) { set_last_error_message("xdna_buffer_read: null pointer"); return -1; }
    if (offset > b->bytes || bytes > b->bytes - offset) { set_last_error_message("xdna_buffer_read: range beyond the buffer"); return -1; }
    if (!ck(cudaSetDevice(b->ordinal), "xdna_buffer_read")) return -1;
    return ck(cudaMemcpy(dst, static_cast<const char *>(b->ptr) + offset, bytes, cudaMemcpyDeviceToHost), "xdna_buffer_read") ? 0 : -1;
}

// ----------------------------------------------------------------- arenas (FusedArena)
XdnaArena *xdna_arena_create(XdnaDevice *dev, size_t input_bytes, size_t output_bytes, size_t scratch_bytes) {
    if (!dev) { set_last_error_message("xdna_arena_create: null device"); return nullptr; }
    auto *a = new XdnaArena();
    const size_t sz[3] = {input_bytes, output_bytes, scratch_bytes};
    for (int i = 0; i < 3; i++) {
        // a zero-size region still gets an allocation (lib.rs:663-667 rounds it up to 2 bytes)
        a->part[i] = xdna_buffer_alloc(dev, std::max<size_t>(sz[i], 2));
        if (!a->part[i]) {
            xdna_arena_free(a);
            return nullptr;
        }
    }
    return a;
}
void xdna_arena_free(XdnaArena *a) {
    if (!a) return;
    for (auto *b : a->part) xdna_buffer_free(b);
    delete a;
}
XdnaBuffer *xdna_arena_region(XdnaArena *a, int which) {
    if (!a || which < 0 || which > 2) {
        set_last_error_message("xdna_arena_region: null arena or region not 0 (input), 1 (output), 2 (scratch)");
        return nullptr;
    }
    return a->part[which];
}
int xdna_arena_write(XdnaArena *a, int which, size_t offset, const void *src, size_t bytes) {
    XdnaBuffer *b = xdna_arena_region(a, which);
    return b ? xdna_buffer_write(b, src, bytes, offset) : -1;
}
int xdna_arena_read(XdnaArena *a, int which, size_t offset, void *dst, size_t bytes) {
    XdnaBuffer *b = xdna_arena_region(a, which);
    return b ? xdna_buffer_read(b, dst, bytes, offset) : -1;
}

// ---------------------------------------------------------------------------------- runs
XdnaRun *xdna_run_start(XdnaDevice *dev, void *stream) {
    if (!dev) { set_last_error_message("xdna_run_start: null device"); return nullptr; }
    auto *r = new XdnaRun();
    r->ordinal = xdna_device_ordinal(dev);
    if (!ck(cudaSetDevice(r->ordinal), "xdna_run_start") ||
        !ck(cudaEventCreateWithFlags(&r->ev, cudaEventDisableTiming), "xdna_run_start") ||
        !ck(cudaEventRecord(r->ev, static_cast<cudaStream_t>(stream)), "xdna_run_start")) {
        if (r->ev) cudaEventDestroy(r->ev);
        delete r;
        return nullptr;
    }
    return r;
}
int xdna_run_wait(XdnaRun *r, int timeout_ms) {
    if (!r) { set_last_error_message("xdna_run_wait: null run"); return -1; }
    cudaSetDevice(r->ordinal);
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t e = cudaEventQuery(r->ev);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) { ck(e, "xdna_run_wait"); return -1; }
        if (timeout_ms >= 0 && std::chrono::steady_clock::now() - t0 >= std::chrono::milliseconds(timeout_ms)) {
            set_last_error_message("xdna_run_wait: not completed within the timeout");
            return 1;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}
void xdna_run_free(XdnaRun *r) {
    if (!r) return;
    cudaSetDevice(r->ordinal);
    cudaEventDestroy(r->ev);
    delete r;
}

// ------------------------------------------------------------------------ bf16 GEMV (+ norm)
XdnaGemvBf16 *xdna_gemv_bf16_register(XdnaDevice *dev, const float *w, int K, int N, const float *bias, int norm,
                                      const float *gamma, const float *beta, float eps) {
    if (!dev || !w || K < 1 || K > 12288 || N < 1 || norm < 0 || norm > 2 || (norm && !gamma) || (norm == 2 && !beta)) {
        set_last_error_message("xdna_gemv_bf16_register: null pointer, shape outside 1 <= K <= 12288, N >= 1, or bad "
                               "norm (0 none, 1 RMS, 2 LN)");
        return nullptr;
    }
    auto *h = new XdnaGemvBf16();
    h->ordinal = xdna_device_ordinal(dev);
    h->K = K;
    h->N = N;
    h->Kp = (K + 7) & ~7;
    h->norm = norm;
    h->eps = eps;
    // fold (ctx_decode.rs:566-603): W''[k][n] = gamma[k] * W[k][n]; LN bias'[n] = sum_k beta[k] W[k][n]
    // (f32, k ascending) + bias[n]
    std::vector<uint16_t> wt((size_t)N * h->Kp, 0);
    for (int k = 0; k < K; k++) {
        const float g = norm ? gamma[k] : 1.0f;
        for (int n = 0; n < N; n++) wt[(size_t)n * h->Kp + k] = bf16_rne(g * w[(size_t)k * N + n]);
    }
    std::vector<float> bp(N, 0.0f);
    for (int n = 0; n < N; n++) {
        float s = 0.0f;
        if (norm == 2)
            for (int k = 0; k < K; k++) s += beta[k] * w[(size_t)k * N + n];
        bp[n] = s + (bias ? bias[n] : 0.0f);
    }
    bool ok = ck(cudaSetDevice(h->ordinal), "xdna_gemv_bf16_register") &&
              ck(cudaMalloc(&h->w, wt.size() * 2), "xdna_gemv_bf16_register") &&
              ck(cudaMalloc(&h->bias, (size_t)N * 4), "xdna_gemv_bf16_register") &&
              ck(cudaMalloc(&h->x, (size_t)h->Kp * 4), "xdna_gemv_bf16_register") &&
              ck(cudaMalloc(&h->y, (size_t)N * 4), "xdna_gemv_bf16_register") &&
              ck(cudaMemcpy(h->w, wt.data(), wt.size() * 2, cudaMemcpyHostToDevice), "xdna_gemv_bf16_register") &&
              ck(cudaMemcpy(h->bias, bp.data(), (size_t)N * 4, cudaMemcpyHostToDevice), "xdna_gemv_bf16_register");
    if (!ok) {
        xdna_gemv_bf16_free(h);
        return nullptr;
    }
    return h;
}

void xdna_gemv_bf16_free(XdnaGemvBf16 *h) {
    if (!h) return;
    cudaSetDevice(h->ordinal);
    cudaFree(h->w);
    cudaFree(h->bias);
    cudaFree(h->x);
    cudaFree(h->y);
    delete h;
}

int xdna_gemv_bf16_device(XdnaGemvBf16 *h, const float *x_dev, float *y_dev, void *stream) {
    if (!h || !x_dev || !y_dev) { set_last_error_message("xdna_gemv_bf16_device: null pointer"); return -1; }
    if (!ck(cudaSetDevice(h->ordinal), "xdna_gemv_bf16_device")) return -1;
    const int warps = 8;
    gemv_bf16_kernel<<<(h->N + warps - 1) / warps, warps * 32, (size_t)h->Kp * 4, static_cast<cudaStream_t>(stream)>>>(
        h->w, x_dev, h->bias, y_dev, h->N, h->K, h->Kp);
    return ck(cudaGetLastError(), "xdna_gemv_bf16_device") ? 0 : -1;
}

int xdna_gemv_bf16(XdnaGemvBf16 *h, const float *x, float *y) {
    if (!h || !x || !y) { set_last_error_message("xdna_gemv_bf16: null pointer"); return -1; }
    // the input normalisation in f64 on the host (ctx_decode.rs:617-640)
    std::vector<float> xn(h->K);
    if (h->norm == 1) {
        double ms = 0.0;
        for (int k = 0; k < h->K; k++) ms += (double)x[k] * (double)x[k];
        ms /= h->K;
        const double inv = 1.0 / std::sqrt(ms + (double)h->eps);
        for (int k = 0; k < h->K; k++) xn[k] = (float)((double)x[k] * inv);
    } else if (h->norm == 2) {
        double mean = 0.0, var = 0.0;
        for (int k = 0; k < h->K; k++) mean += (double)x[k];
        mean /= h->K;
        for (int k = 0; k < h->K; k++) var += ((double)x[k] - mean) * ((double)x[k] - mean);
        var /= h->K;
        const double inv = 1.0 / std::sqrt(var + (double)h->eps);
        for (int k = 0; k < h->K; k++) xn[k] = (float)(((double)x[k] - mean) * inv);
    } else {
        std::copy(x, x + h->K, xn.begin());
    }
    if (!ck(cudaSetDevice(h->ordinal), "xdna_gemv_bf16") ||
        !ck(cudaMemcpy(h->x, xn.data(), (size_t)h->K * 4, cudaMemcpyHostToDevice), "xdna_gemv_bf16"))
        return -1;
    if (xdna_gemv_bf16_device(h, h->x, h->y, nullptr) != 0) return -1;
    return ck(cudaMemcpy(y, h->y, (size_t)h->N * 4, cudaMemcpyDeviceToHost), "xdna_gemv_bf16") ? 0 : -1;
}

// ------------------------------------------------------------------- paged decode attention
int xdna_mha_decode_paged(const uint16_t *q_dev, const uint16_t *kv_dev, int n_heads, int n_tiles, float *ctx_dev,
                          void *stream) {
    if (!q_dev || !kv_dev || !ctx_dev || n_heads < 1 || n_tiles < 1) {
        set_last_error_message("xdna_mha_decode_paged: null pointer or empty shape");
        return -1;
    }
    mha_decode_paged_kernel<<<n_heads, kHd, 0, static_cast<cudaStream_t>(stream)>>>(q_dev, kv_dev, n_tiles, ctx_dev);
    return ck(cudaGetLastError(), "xdna_mha_decode_paged") ? 0 : -1;
}

// ------------------------------------------------------------------------- conformer bricks
int xdna_dwconv1d_glu_silu(const float *x_dev, int B, int T, int C, const float *taps_dev, int k,
                           const float *bias_dev, float *y_dev, void *stream) {
    if (!x_dev || !taps_dev || !bias_dev || !y_dev || B < 1 || B > 65535 || T < 1 || C < 1 ||
        (k != 3 && k != 5 && k != 7 && k != 9 && k != 15 && k != 31)) {
        set_last_error_message("xdna_dwconv1d_glu_silu: null pointer, empty shape, or k not one of 3 5 7 9 15 31");
        return -1;
    }
    const dim3 grid((C + 127) / 128, (T + kDwRows - 1) / kDwRows, B);
    auto st = static_cast<cudaStream_t>(stream);
    switch (k) {
    case 3: dwconv1d_glu_silu_kernel<3><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    case 5: dwconv1d_glu_silu_kernel<5><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    case 7: dwconv1d_glu_silu_kernel<7><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    case 9: dwconv1d_glu_silu_kernel<9><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    case 15: dwconv1d_glu_silu_kernel<15><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    default: dwconv1d_glu_silu_kernel<31><<<grid, 128, 0, st>>>(x_dev, T, C, taps_dev, bias_dev, y_dev); break;
    }
    return ck(cudaGetLastError(), "xdna_dwconv1d_glu_silu") ? 0 : -1;
}

int xdna_subsample_conv2d(const uint16_t *x_dev, int B, int ci, int hin, int win, const uint16_t *w_dev,
                          const float *bias_dev, int co, int kh, int kw, int stride, int pad, int groups, int relu,
                          uint16_t *out_dev, void *stream) {
    if (!x_dev || !w_dev || !out_dev || B < 1 || B > 65535 || ci < 1 || hin < 1 || win < 1 || co < 1 || co > 65535 ||
        kh < 1 || kw < 1 || stride < 1 || pad < 0 || groups < 1 || ci % groups || co % groups) {
        set_last_error_message("xdna_subsample_conv2d: null pointer, empty shape, or groups not dividing ci and co");
        return -1;
    }
    const int hout = (hin + 2 * pad - kh) / stride + 1, wout = (win + 2 * pad - kw) / stride + 1;
    if (hout < 1 || wout < 1) {
        set_last_error_message("xdna_subsample_conv2d: kernel larger than the padded image");
        return -1;
    }
    const dim3 grid((hout * wout + 255) / 256, co, B);
    conv2d_bf16_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x_dev, ci, hin, win, w_dev, bias_dev, co,
                                                                            kh, kw, stride, pad, groups, relu, hout,
                                                                            wout, out_dev);
    return ck(cudaGetLastError(), "xdna_subsample_conv2d") ? 0 : -1;
}

}  // extern "C"
