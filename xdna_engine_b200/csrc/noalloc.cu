// noalloc.cu -- xdna_gemv_i8_noalloc: the op-level int8 GEMV for callers that must not
// allocate device memory.
//
// xdna_gemv_i8 stages the caller's host arrays (activation, packed weight rows, chunk table,
// result) in buffers it cudaMallocs and frees on every call.  Some hosts cannot do that:
// a serving process whose device memory is owned by another allocator (a framework caching
// allocator or a fixed arena carved out at start-up) or an embedder that has reserved every
// byte for the model, where a stray cudaMalloc either fails or fragments the pool.  This
// entry point gives them the same computation with all staging in ONE file-scope
// __device__ array of fixed size, so a call allocates nothing, on the device or the host.
//
// Limits and caveats (for users of this entry point):
//  * the array is kNoAllocScratchBytes (8 MiB) and every GPU that loads this library keeps it
//    until the process exits; a call whose staged bytes (N*K int8 + packed copy + vectors)
//    exceed it is rejected with an error and nothing runs;
//  * the call makes `device` current for its duration and restores the calling thread's
//    previous current device before returning;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress)
//    with that device current; make that first call before any stream capture;
//  * all calls share the array, which keeps the previous call's contents: every byte the
//    kernels read is written earlier in the same call, and two calls that overlap on the
//    GPU (other threads, other host contexts on the same device) race on it -- serialise
//    them.
// It has no counterpart in the reference.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "../../include/xdna_b200.h"
#include "gemv_op.h"

namespace xdna {
void set_last_error_message(const std::string &m);
}  // namespace xdna

using namespace xdna;
using namespace xdna::gemvop;

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint8_t *g_scratch_dev[kMaxDevices] = {};   // device address of g_noalloc_scratch per device

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Repack raw output-major int8 rows [N][K] (+ scale, bias) into the chunk layout the GEMV
// kernel consumes (decode.h): per chunk rows x K bytes with 32-byte block kb of row r at
// block kb ^ (r & 3), then (scale, bias) per row; plus the chunk table.
__global__ void pack_chunks_kernel(const int8_t *q, const float *scale, const float *bias,
                                   int has_bias, int K, int N, uint8_t *packed, ChunkRef *chunks) {
    const int rpc = rows_per_chunk(K);
    const uint32_t full_bytes = chunk_bytes(rpc, K);
    const int nblk = K / 32;
    const size_t total = (size_t)N * nblk;
    for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(t / nblk), kb = (int)(t % nblk);
        const int ci = row / rpc, r = row % rpc;
        const int rows_here = min(rpc, N - ci * rpc);
        uint8_t *base = packed + (size_t)ci * full_bytes;
        const uint4 *src = reinterpret_cast<const uint4 *>(q + (size_t)row * K + kb * 32);
        uint4 *dst = reinterpret_cast<uint4 *>(base + (size_t)r * K + (kb ^ (r & 3)) * 32);
        dst[0] = src[0];
        dst[1] = src[1];
        if (kb == 0) {
            float *meta = reinterpret_cast<float *>(base + (size_t)rows_here * K);
            meta[2 * r] = scale[row];
            meta[2 * r + 1] = has_bias ? bias[row] : 0.0f;
            if (r == 0) chunks[ci] = ChunkRef{(uint32_t)((size_t)ci * full_bytes), chunk_bytes(rows_here, K)};
        }
    }
}

// One-time lookup of the array's device address for the current device.
uint8_t *scratch_for(int dev, cudaError_t *err) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (dev < 0 || dev >= kMaxDevices) { *err = cudaErrorInvalidDevice; return nullptr; }
    if (!g_scratch_dev[dev]) {
        void *ptr = nullptr;
        *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        g_scratch_dev[dev] = static_cast<uint8_t *>(ptr);
    }
    *err = cudaSuccess;
    return g_scratch_dev[dev];
}

}  // namespace

extern "C" int xdna_gemv_i8_noalloc(int device, const float *x, int K, const int8_t *q_nk,
                                    const float *scale, const float *bias, int N, float *y) {
    if (!x || !q_nk || !scale || !y) { set_last_error_message("xdna_gemv_i8_noalloc: null pointer"); return -1; }
    if (K <= 0 || K % 256 != 0 || K > kKmax || N <= 0 || N % 8 != 0) {
        set_last_error_message("xdna_gemv_i8_noalloc: K must be a multiple of 256 <= 3072 and N a multiple of 8");
        return -1;
    }
    const int rpc = rows_per_chunk(K);
    const size_t n_chunks_ = (size_t)(N + rpc - 1) / rpc;
    const size_t off_raw = 0;
    const size_t off_packed = align256(off_raw + (size_t)N * K);
    const size_t off_chunks = align256(off_packed + n_chunks_ * chunk_bytes(rpc, K));
    const size_t off_scale = align256(off_chunks + n_chunks_ * sizeof(ChunkRef));
    const size_t off_bias = align256(off_scale + (size_t)N * 4);
    const size_t off_x = align256(off_bias + (size_t)N * 4);
    const size_t off_y = align256(off_x + (size_t)K * 4);
    const size_t need = align256(off_y + (size_t)N * 4);
    if (need > kNoAllocScratchBytes) {
        set_last_error_message("xdna_gemv_i8_noalloc: N x K needs " + std::to_string(need) +
                               " bytes of staging, above the fixed 8 MiB scratch array "
                               "(use xdna_gemv_i8 for larger matrices)");
        return -1;
    }
    // the call runs with `device` current and gives the calling thread its previous current
    // device back before it returns, on every path
    int prev_device = -1;
    cudaError_t e = cudaGetDevice(&prev_device);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    struct RestoreDevice {
        int dev;
        ~RestoreDevice() { if (dev >= 0) cudaSetDevice(dev); }
    } restore{e == cudaSuccess ? prev_device : -1};
    uint8_t *s = e == cudaSuccess ? scratch_for(device, &e) : nullptr;
    if (!s) {
        set_last_error_message(std::string("xdna_gemv_i8_noalloc: scratch set-up failed: ") + cudaGetErrorString(e));
        return -1;
    }
    cudaStream_t st = nullptr;
    uint8_t *raw = s + off_raw, *packed = s + off_packed;
    ChunkRef *chunks = reinterpret_cast<ChunkRef *>(s + off_chunks);
    float *dscale = reinterpret_cast<float *>(s + off_scale), *dbias = reinterpret_cast<float *>(s + off_bias);
    float *dx = reinterpret_cast<float *>(s + off_x), *dy = reinterpret_cast<float *>(s + off_y);
    e = cudaMemcpyAsync(raw, q_nk, (size_t)N * K, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dscale, scale, (size_t)N * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && bias) e = cudaMemcpyAsync(dbias, bias, (size_t)N * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dx, x, (size_t)K * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        pack_chunks_kernel<<<148, 256, 0, st>>>(reinterpret_cast<const int8_t *>(raw), dscale, dbias,
                                                bias ? 1 : 0, K, N, packed, chunks);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = launch_gemv_i8(dx, K, packed, chunks, N, dy, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, dy, (size_t)N * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_gemv_i8_noalloc: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}
