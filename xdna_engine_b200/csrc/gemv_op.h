// gemv_op.h -- chunk format and launch entry of the op-level exact int8 GEMV
// (xdna_gemv_i8 / xdna_gemv_i8_noalloc), shared by the kernel (gemv_op.cu) and the host
// packers (engine.cu, noalloc.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace xdna {
namespace gemvop {

constexpr int kWarps = 8;
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;   // + one copy warp
constexpr int kStageBytes = 32768;                // one weight chunk
constexpr int kKmax = 3072;                       // largest reduction length
constexpr int kRowMeta = 8;                       // per-row f32 scale + f32 bias after the rows
constexpr int kMaxTilesPerChunk = kStageBytes / (768 + 8) / 8;   // 5 for K=768

struct ChunkRef {              // one weight chunk
    uint32_t off;              // byte offset
    uint32_t bytes;            // multiple of 16
};

// rows per chunk for reduction length K: whole 8-row n-tiles of (K bytes + 8 bytes meta)
__host__ __device__ inline int rows_per_chunk(int K) {
    const int r = (kStageBytes / (K + kRowMeta)) & ~7;
    return r < 8 * kMaxTilesPerChunk ? r : 8 * kMaxTilesPerChunk;
}
__host__ __device__ inline uint32_t chunk_bytes(int rows, int K) {
    return (uint32_t)(((size_t)rows * (K + kRowMeta) + 15) & ~(size_t)15);
}

// y[N] = exact-int8-GEMV(x[K]) * scale + bias over the packed chunk list (device pointers)
cudaError_t launch_gemv_i8(const float *x, int K, const uint8_t *packed, const ChunkRef *chunks,
                           int N, float *y, cudaStream_t st);

}  // namespace gemvop
}  // namespace xdna
