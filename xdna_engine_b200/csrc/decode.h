// decode.h -- device-side parameter block and layout constants of the persistent opt decode
// kernel, shared by the kernel (decode_kernel.cu) and the host packer (engine.cpp).
#pragma once
#include <cstdint>

namespace xdna {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;   // + one producer warp
constexpr int kStageBytes = 32768;                // one weight chunk (ring stage)
constexpr int kStages = 4;                        // ring depth: 128 KB of weights in flight
constexpr int kKmax = 3072;                       // largest GEMV reduction length
constexpr int kDmax = 768;                        // largest model width
constexpr int kHeadDim = 64;                      // the kernel's attention head size
constexpr int kPageTokens = 64;                   // KV page = 64 positions (the reference's TKV tile)
constexpr int kMaxTilesPerChunk = kStageBytes / (768 + 8) / 8;   // 5 for K=768
constexpr int kMaxPages = 64;                     // KV pages per sequence (4096 positions)
constexpr int kGroupPages = 3;                    // KV pages one attention item covers (192 positions)
constexpr int kRowMeta = 8;                       // per-row f32 scale + f32 bias after the rows

// Row partition and chunking shared by the host packer and the kernel.  Rows are assigned
// in units of 8 (one MMA n-tile); CTA c of `grid` owns units [c*U/grid, (c+1)*U/grid).
__host__ __device__ inline int part_row0(int c, int n_rows, int grid) {
    return 8 * (int)((long long)c * (n_rows / 8) / grid);
}
__host__ __device__ inline int part_rows(int c, int n_rows, int grid) {
    return part_row0(c + 1, n_rows, grid) - part_row0(c, n_rows, grid);
}
// rows per chunk for reduction length K: whole n-tiles of (K bytes + 8 bytes meta) per stage
__host__ __device__ inline int rows_per_chunk(int K) {
    const int r = (kStageBytes / (K + kRowMeta)) & ~7;
    return r < 8 * kMaxTilesPerChunk ? r : 8 * kMaxTilesPerChunk;
}
__host__ __device__ inline int n_chunks(int rows, int K) {
    int r = rows_per_chunk(K);
    return (rows + r - 1) / r;
}
__host__ __device__ inline uint32_t chunk_bytes(int rows, int K) {
    return (uint32_t)(((size_t)rows * (K + kRowMeta) + 15) & ~(size_t)15);
}

// GEMV phases of one token, in weight-stream order per layer, then the LM head.
enum Phase { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_FC1 = 3, PH_FC2 = 4 };
constexpr int kPhasesPerLayer = 5;

// error codes written to RunState::error
enum : uint32_t {
    ERR_NONE = 0,
    ERR_TIMEOUT_FULL = 1,      // consumer waited too long for a weight chunk
    ERR_TIMEOUT_EMPTY = 2,     // producer waited too long for a free stage
    ERR_TIMEOUT_FLAG = 3,      // a flag-tagged word never reached its epoch
    ERR_BAD_TOKEN = 4,         // token id out of range
    ERR_BAD_POS = 5,           // position beyond the KV capacity
};

struct RunState {
    uint32_t epoch_base;       // first epoch of the next launch (advanced by CTA 0 at exit)
    uint32_t error;            // first error code (0 = none)
    uint32_t error_cta;        // CTA that reported it
    uint32_t error_where;      // phase / detail
};

struct ChunkRef {              // one weight chunk of a CTA's stream
    uint32_t off;              // byte offset from DecodeParams::stream
    uint32_t bytes;            // multiple of 16
};

struct DecodeParams {
    // model
    int n_layers, d_model, n_heads, ffn, vocab, max_pos;
    float eps;
    // grid / stream
    int grid;                  // number of CTAs (all co-resident)
    const uint8_t *stream;     // packed int8 weight stream of all CTAs
    const ChunkRef *chunks;    // [grid][chunk_stride]: layer chunks, then LM chunks
    const int *n_layer_chunks; // [grid]
    const int *n_lm_chunks;    // [grid]
    int chunk_stride;
    // f32 parameters that are not streamed
    const float *emb_tok;      // [V, D]
    const float *emb_pos;      // [max_pos + 2, D]
    const float *ln;           // [L][4][D]: ln1_w ln1_b ln2_w ln2_b
    const float *lnf;          // [2][D]
    // paged KV cache: [L][n_phys_pages][2][H][page][hd] bf16
    uint16_t *kv;
    const int *page_table;     // logical page -> physical page
    int n_phys_pages;
    // flag-tagged exchange words
    uint64_t *ll_qkv;          // [3D/2]   bf16 pairs
    uint64_t *ll_att;          // [max_pages*H][2+hd]  m, l, acc[hd]
    uint64_t *ll_o;            // [D]      f32
    uint64_t *ll_h;            // [F/2]    bf16 pairs
    uint64_t *ll_f2;           // [D]      f32
    uint64_t *ll_lm;           // [grid][2] (best value, index)
    // run
    int64_t *tokens;           // [max_pos + 1]: prompt in, generated ids out at pos+1
    float *logits;             // optional [n_steps][V] (only steps with an LM head)
    int start_pos, n_steps, n_prompt;
    RunState *state;
    uint64_t timeout_ns;
    float *trace;              // optional [n_steps][2L+1][D]: residual after attention and
                               // after the FFN of each layer, then the final LN output
    unsigned long long *timing; // optional [2][grid][128] globaltimer stamps (first 2 steps)
};

}  // namespace xdna
