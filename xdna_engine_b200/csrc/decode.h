// decode.h -- parameter block, layout constants and work partition of the persistent opt
// decode kernel, shared by the kernel (decode_kernel.cu) and the host packer (engine.cu).
//
// CTA roles (grid G, clusters of 2 CTAs):
//   head pair h (CTAs 2h, 2h+1; cluster rank r): q|k|v rows of dims [32r, 32r+32) of head h,
//     single-query attention over those dims (partial scores swapped with the pair's other
//     CTA through distributed shared memory), then its K-split slice of the out projection;
//   FC CTA i (CTAs 2H + i, i < n_fc): 32-row blocks [kb0_i, kb1_i) of fc1, then the K-split
//     slice of fc2 over exactly those hidden rows;
//   spare CTAs: neither; like every CTA they keep the residual stream and take a share of the
//     LM head.
// The out projection and fc2 are summed over their K slices in exact integer arithmetic:
// every contributor adds (partial + 2^bias_shift + 2^56) into one 64-bit accumulator word per
// output with red.add.u64; the top 8 bits count contributions, so a reader knows the word is
// complete when the count reaches the number of contributors (no flags, no fences).
#pragma once
#include <cstdint>

namespace xdna {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;   // + one producer warp
constexpr int kSlotBytes = 16384;                 // one ring slot
constexpr int kSlots = 8;                         // ring depth: 128 KB of weights in flight
constexpr int kDmax = 768;                        // largest model width
constexpr int kFmax = 3072;                       // largest FFN width
constexpr int kHeadDim = 64;                      // the kernel's attention head size
constexpr int kHalfDim = 32;                      // head dims owned by one CTA of a pair
constexpr int kPageTokens = 64;                   // KV page = 64 positions (the reference's TKV tile)
constexpr int kMaxCtx = 2048;                     // positions per sequence
constexpr int kMaxPages = kMaxCtx / kPageTokens;
constexpr int kStageKeys = 256;                   // cached keys staged once per layer (fast path)
constexpr int kChunkKeys = 512;                   // keys per staged chunk beyond that
constexpr int kAccSlots = 4;                      // token ring of the accumulator words
constexpr int kMaxSubs = 8;                       // accumulator sub-words per output
constexpr int kLimbs = 4;                         // X = a*2^24 + b*2^16 + c*2^8 + d
constexpr int kLimbStride = kFmax + 16;           // bytes per limb row (bank offset 4 words)
constexpr int kTile = 16;                         // output rows of one MMA m-tile
constexpr int kFragBytes = 512;                   // one m-tile x one 32-wide k-block
constexpr int kSliceTilesPerChunk = 24;           // m-tiles of a K-split chunk (12 KB)
constexpr int kFcRows = 32;                       // fc1 rows per k-block of fc2
constexpr int kFixBits = 29;                      // |X| < 2^29
constexpr int kCountShift = 56;                   // accumulator word: count in bits 56..63
constexpr int kMaxVocabTilesPerCta = 64;

// 32-row blocks of fc1 / k-blocks of fc2 owned by FC CTA i of n
__host__ __device__ inline int fc_kb0(int i, int n_kb, int n_fc) { return (int)((long long)i * n_kb / n_fc); }
// LM-head m-tiles owned by CTA c of G
__host__ __device__ inline int lm_tile0(int c, int n_tiles, int G) { return (int)((long long)c * n_tiles / G); }

// bytes of a row-tile chunk (16 output rows x K, fragment order, then 16 x (scale, bias))
__host__ __device__ inline uint32_t row_chunk_bytes(int K) { return (uint32_t)(kTile * K + kTile * 8); }
// K-split chunks of an N-output slice (one 32-wide k-block)
__host__ __device__ inline int slice_chunks(int N) {
    return (N / kTile + kSliceTilesPerChunk - 1) / kSliceTilesPerChunk;
}
__host__ __device__ inline int slice_chunk_tiles(int N, int c) {
    const int t = N / kTile - c * kSliceTilesPerChunk;
    return t < kSliceTilesPerChunk ? t : kSliceTilesPerChunk;
}

// error codes written to RunState::error
enum : uint32_t {
    ERR_NONE = 0,
    ERR_TIMEOUT_FULL = 1,      // consumer waited too long for a weight chunk
    ERR_TIMEOUT_EMPTY = 2,     // producer waited too long for a free slot
    ERR_TIMEOUT_FLAG = 3,      // an exchange word never completed
    ERR_BAD_TOKEN = 4,         // token id out of range
    ERR_BAD_POS = 5,           // position beyond the KV capacity
    ERR_TIMEOUT_PEER = 6,      // the pair CTA's partial scores never arrived
};

struct RunState {
    uint32_t tok_base;         // tokens decoded by earlier launches (advanced by CTA 0 at exit)
    uint32_t error;            // first error code (0 = none)
    uint32_t error_cta;        // CTA that reported it
    uint32_t error_where;      // phase / detail
};

struct ChunkRef {              // one weight chunk of a CTA's stream
    uint32_t off;              // byte offset from DecodeParams::stream
    uint32_t bytes;            // multiple of 16, <= kSlotBytes
};

struct DecodeParams {
    // model
    int n_layers, d_model, n_heads, ffn, vocab, max_pos;
    float eps;
    // grid / roles
    int grid, n_fc;            // G CTAs (even, clusters of 2); FC CTAs
    int vocab_tiles;           // ceil(vocab / 16)
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
    const float *osb;          // [L][2][D]: out-proj scale, bias
    const float *f2sb;         // [L][2][D]: fc2 scale, bias
    const int *fix_ctx;        // [L] fixed-point exponent of the attention context (out-proj input)
    const int *fix_h;          // [L] fixed-point exponent of the fc1 output (fc2 input)
    const int *fix_ln1;        // [L] fixed-point exponents of the LayerNorm outputs (q|k|v input)
    const int *fix_ln2;        // [L] (fc1 input)
    int fix_lnf;               // final LayerNorm (LM-head input)
    int o_bias_shift, f2_bias_shift;
    // paged KV cache: [L][phys_page][H][2 halves][K|V][64 positions][32 dims] bf16
    uint16_t *kv;
    const int *page_table;     // logical page -> physical page
    int n_phys_pages;
    // exchange
    unsigned long long *acc;   // [kAccSlots][L][2: out-proj, fc2][kMaxSubs][D] accumulator words
    int o_subs, f2_subs;       // sub-words per output (contributor i adds into sub-word i % subs,
                               // so fewer atomics meet on one address; readers add the sub-words)
    int poll_ns;               // sleep between polls of incomplete words
    unsigned long long *lm_words; // [kAccSlots][2]: per token the max LM-head key, the CTAs counted in
    int lm_prefetch_layer;     // layer during which the LM-head rows go to L2 (< 0: never)
    // run
    int64_t *tokens;           // [max_ctx + 1]: prompt in, generated ids out at pos+1
    float *logits;             // optional [n_steps][V] (only steps with an LM head)
    int start_pos, n_steps, n_prompt;
    RunState *state;
    uint64_t timeout_ns;
    float *trace;              // optional [n_steps][2L+1][D]: residual after attention and
                               // after the FFN of each layer, then the final LN output
    unsigned long long *timing; // optional [2][grid][128] globaltimer / clock stamps (first 2 steps)
};

// ---------------------------------------------------------------- batched prompt prefill
constexpr int kPrefillTokens = 32;                // positions per prefill launch sequence
enum { PF_QKV = 0, PF_FC1 = 1, PF_RESID = 2 };

struct PrefillGemv {
    const int8_t *w;            // [N][K] row-major int8
    const float *sc, *bi;       // [N] row scale, bias
    const int8_t *limbs;        // [T][4][K] input limbs (fixed point 2^fix)
    int T, K, N, fix, mode;
    // PF_QKV: q out [T][D] (bf16 values of y / 8), K / V rows into the paged cache
    float *q;
    uint16_t *kv;
    const int *pt;
    int layer, n_phys, n_heads, pos0, D;
    // PF_FC1: limbs of bf16(relu(y)) at 2^fix_out into [T][4][N]
    int8_t *limbs_out;
    int fix_out;
    // PF_RESID: x[t][n] += y
    float *x;
    // K split: nsplit CTAs per 16-row tile add exact partials into acc[t][n] (int64, zero
    // between uses); the last of a tile's CTAs to finish (cnt[tile]) applies the epilogue and
    // clears its words and counter
    int nsplit;
    unsigned long long *acc;
    unsigned int *cnt;
};

}  // namespace xdna
