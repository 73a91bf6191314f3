// bert.cu -- the BGE-base (BERT) encoder path on B200 for batches of variable-length
// sequences, packed without padding ([T = sum of lengths, 768] bf16 activations).
//
// Replaces the reference's EmbedPipeline (rust/npu-engine/src/bert/mod.rs:24-46):
//   EmbedFrontend::run   word + position + type-0 embedding, LayerNorm eps 1e-12
//                        (bert/frontend.rs:37-61)                  -> embed_ln_kernel
//   BertBlock::forward   q/k/v/o, ffn1 (+GELU), ffn2 on the NPU GEMM engine, host MHA with
//                        the key mask j >= valid_len, post-LN (bert/encoder.rs:43-57)
//                        -> xdna_gemm_bf16 (tcgen05, fused bias/GELU/residual),
//                           attention_tc (tcgen05), ln_kernel
//   EmbedHead::run       CLS or mean pooling over valid rows, L2 with norm clamp 1e-12
//                        (bert/head.rs:20-47)                     -> pool_kernel
// Packing sequences (instead of padding each to 512 and masking keys) gives the same result
// for every valid row: a padded row can never be attended to, and only valid rows are pooled.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"
#include "ptx.cuh"

namespace xdna {
void set_last_error_message(const std::string &m);
cudaError_t gemm_bf16(const uint16_t *A, int lda, const uint16_t *B, int ldb, int M, int N, int K,
                      const float *bias, const uint16_t *residual, int ldr, int act, uint16_t *C, int ldc,
                      cudaStream_t st, int res_mod = 0, float *C_f32 = nullptr);
unsigned gemm_error_and_clear();
cudaError_t attention_tc(const uint16_t *qkv, int T_total, const int32_t *cu, int n_seqs, int max_len, uint16_t *ctx,
                         cudaStream_t st);
unsigned attention_tc_error_and_clear();

namespace bert {

constexpr int D = 768, H = 12, HD = 64, F = 3072;

__device__ __forceinline__ void unpack8(uint4 w, float *v) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; e++) { v[2 * e] = bf16lo(u[e]); v[2 * e + 1] = bf16hi(u[e]); }
}
__device__ __forceinline__ uint4 pack8(const float *v) {
    uint4 w;
    w.x = bf16bits(v[0]) | (bf16bits(v[1]) << 16);
    w.y = bf16bits(v[2]) | (bf16bits(v[3]) << 16);
    w.z = bf16bits(v[4]) | (bf16bits(v[5]) << 16);
    w.w = bf16bits(v[6]) | (bf16bits(v[7]) << 16);
    return w;
}

// LayerNorm of one 768-wide row held as 24 floats per lane (elements 8*lane + 256*j + e):
// population variance, y = (x - mean) * inv * g + b  (rust/npu-asr-host/src/lib.rs:79-110)
__device__ __forceinline__ void ln_row(float (&v)[24], const float *g, const float *b, float eps, int lane) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; i++) s += v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)D;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; i++) { const float c = v[i] - mean; q += c * c; }
#pragma unroll
    for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = 1.0f / sqrtf(q / (float)D + eps);
#pragma unroll
    for (int j = 0; j < 3; j++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int c = 8 * lane + 256 * j + e;
            v[8 * j + e] = (v[8 * j + e] - mean) * inv * g[c] + b[c];
        }
}

// x[t] = LN(word[id] + pos[t - seq_start] + type[0]); one warp per token row
__global__ void embed_ln_kernel(const int32_t *ids, const int32_t *tok_pos, int T, const uint16_t *word,
                                const uint16_t *pos, const uint16_t *type0, const float *g, const float *b,
                                float eps, uint16_t *x) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= T) return;
    const int id = ids[row], p = tok_pos[row];
    float v[24];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int c = 8 * lane + 256 * j;
        float a[8], bb[8], cc[8];
        unpack8(*reinterpret_cast<const uint4 *>(word + (size_t)id * D + c), a);
        unpack8(*reinterpret_cast<const uint4 *>(pos + (size_t)p * D + c), bb);
        unpack8(*reinterpret_cast<const uint4 *>(type0 + c), cc);
#pragma unroll
        for (int e = 0; e < 8; e++) v[8 * j + e] = a[e] + bb[e] + cc[e];
    }
    ln_row(v, g, b, eps, lane);
#pragma unroll
    for (int j = 0; j < 3; j++)
        *reinterpret_cast<uint4 *>(x + (size_t)row * D + 8 * lane + 256 * j) = pack8(v + 8 * j);
}

// y = LN(x) row-wise, bf16 in / bf16 out; one warp per row
// y = LN(x) row-wise, bf16 in / bf16 out.  Each warp walks rows w, w + W, w + 2W, ... (W = warps
// in the grid, a few per SM) and loads its next row while it normalises the current one, so
// every SM keeps ~2 rows per warp in flight; gamma and beta are staged in shared memory once
// per block.  The arithmetic is ln_row's, in the same order.
constexpr int LN_BLOCKS_PER_SM = 3;
__global__ void __launch_bounds__(256, LN_BLOCKS_PER_SM) ln_kernel(const uint16_t *__restrict__ xin, int T,
                                                                   const float *__restrict__ g,
                                                                   const float *__restrict__ b, float eps,
                                                                   uint16_t *__restrict__ y) {
    __shared__ float sg[D], sb[D];
    for (int i = threadIdx.x; i < D; i += blockDim.x) { sg[i] = g[i]; sb[i] = b[i]; }
    __syncthreads();
    const int lane = threadIdx.x & 31, nw = gridDim.x * 8;
    int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= T) return;
    uint4 cur[3];
#pragma unroll
    for (int j = 0; j < 3; j++) cur[j] = *reinterpret_cast<const uint4 *>(xin + (size_t)row * D + 8 * lane + 256 * j);
    while (row < T) {
        const int nrow = row + nw;
        uint4 nxt[3];
        if (nrow < T)
#pragma unroll
            for (int j = 0; j < 3; j++) nxt[j] = *reinterpret_cast<const uint4 *>(xin + (size_t)nrow * D + 8 * lane + 256 * j);
        float v[24];
#pragma unroll
        for (int j = 0; j < 3; j++) unpack8(cur[j], v + 8 * j);
        ln_row(v, sg, sb, eps, lane);
#pragma unroll
        for (int j = 0; j < 3; j++)
            *reinterpret_cast<uint4 *>(y + (size_t)row * D + 8 * lane + 256 * j) = pack8(v + 8 * j);
        if (nrow < T)
#pragma unroll
            for (int j = 0; j < 3; j++) cur[j] = nxt[j];
        row = nrow;
    }
}

// the row LayerNorm over T rows: a grid of LN_BLOCKS_PER_SM blocks per SM (or fewer for short inputs)
void launch_ln(const uint16_t *x, int T, const float *g, const float *b, float eps, uint16_t *y, cudaStream_t st) {
    int dev = 0, sms = 148;            // queried per call: cheap, and right on any current device
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = std::min((T + 7) / 8, sms * LN_BLOCKS_PER_SM);
    ln_kernel<<<blocks, 256, 0, st>>>(x, T, g, b, eps, y);
}

// bf16 -> f32 (exact), grid-stride
__global__ void bf16_to_f32_kernel(const uint16_t *__restrict__ x, size_t n, float *__restrict__ y) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __uint_as_float((uint32_t)x[i] << 16);
}

// ---------------------------------------------------------------------------- attention
// softmax(q k^T / 8) v per (sequence, head) over the sequence's own keys (the valid_len key
// mask of npu-asr-host mha, lib.rs:189-326): the tcgen05 kernel of attention_tc.cu.

// out[b] = l2norm(pool(x rows of sequence b)); pooling bit 0: 0 = CLS (row 0), 1 = mean;
// bit 1 set: no L2 normalisation (EmbedHead with normalize = false, bert/head.rs:20-47)
__global__ void pool_kernel(const uint16_t *x, const int32_t *cu, int pooling_flags, float *out) {
    const int pooling = pooling_flags & 1;
    const bool l2 = (pooling_flags & 2) == 0;
    const int b = blockIdx.x, lane = threadIdx.x;
    const int s0 = cu[b], L = cu[b + 1] - s0;
    float v[24];
#pragma unroll
    for (int i = 0; i < 24; i++) v[i] = 0.0f;
    const int nrows = pooling == 0 ? 1 : max(L, 1);
    for (int t = 0; t < nrows && t < max(L, 1); t++) {
#pragma unroll
        for (int j = 0; j < 3; j++) {
            float a[8];
            unpack8(*reinterpret_cast<const uint4 *>(x + (size_t)(s0 + t) * D + 8 * lane + 256 * j), a);
#pragma unroll
            for (int e = 0; e < 8; e++) v[8 * j + e] += a[e];
        }
    }
    if (pooling == 1) {
        const float inv = 1.0f / (float)max(L, 1);
#pragma unroll
        for (int i = 0; i < 24; i++) v[i] *= inv;
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; i++) s += v[i] * v[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float norm = l2 ? fmaxf(sqrtf(s), 1e-12f) : 1.0f;
#pragma unroll
    for (int j = 0; j < 3; j++)
#pragma unroll
        for (int e = 0; e < 8; e++) out[(size_t)b * D + 8 * lane + 256 * j + e] = v[8 * j + e] / norm;
}

}  // namespace bert
}  // namespace xdna

// ====================================================================================== host
namespace xdna {
namespace {

uint16_t to_bf16_bits(float f) {   // round to nearest even (rust/npu-xrt/src/lib.rs:809-818)
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// [K, N] f32 (the reference's layout) -> [N, K] bf16 rows appended to out
void append_transposed_bf16(const float *w, int K, int N, std::vector<uint16_t> &out) {
    const size_t base = out.size();
    out.resize(base + (size_t)N * K);
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) out[base + (size_t)n * K + k] = to_bf16_bits(w[(size_t)k * N + n]);
}

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

struct XdnaBert {
    XdnaBertConfig cfg{};
    int ordinal = 0, max_tokens = 0, max_seqs = 0;
    uint16_t *word = nullptr, *pos = nullptr, *type0 = nullptr;
    float *emb_ln = nullptr;                       // [2][D]
    struct Layer {
        uint16_t *wqkv, *wo, *w1, *w2;             // [N, K] bf16
        float *bqkv, *bo, *b1, *b2, *ln1, *ln2;    // ln: [2][D]
    };
    std::vector<Layer> layers;
    // activations (bf16) and packing metadata
    uint16_t *x = nullptr, *qkv = nullptr, *ctx = nullptr, *y = nullptr, *hbuf = nullptr;
    int32_t *ids = nullptr, *tokpos = nullptr, *cu = nullptr;
    float *out = nullptr;
    std::vector<void *> owned;
    ~XdnaBert() {
        for (void *p : owned) cudaFree(p);
    }
};

extern "C" {

XdnaBert *xdna_bert_create(XdnaDevice *dev_unused, const XdnaBertConfig *cfg, const XdnaBertWeights *w,
                           int max_tokens, int max_seqs) {
    (void)dev_unused;
    if (!cfg || !w || !w->layers || !w->word_emb || !w->pos_emb || !w->type_emb || !w->emb_ln_w || !w->emb_ln_b) {
        set_last_error_message("xdna_bert_create: null pointer");
        return nullptr;
    }
    const XdnaBertConfig c = *cfg;
    if (c.d_model != bert::D || c.n_heads != bert::H || c.ffn != bert::F || c.n_layers < 1 || c.vocab < 1 ||
        c.max_pos < 1 || max_tokens < 1 || max_seqs < 1 || c.pooling < 0 || c.pooling > 3) {
        set_last_error_message("xdna_bert_create: supported shape is d_model 768, 12 heads, ffn 3072 "
                               "(BERT-base / BGE-base); pooling 0 (CLS) or 1 (mean), + 2 for no L2 normalisation");
        return nullptr;
    }
    auto *m = new XdnaBert();
    try {
        int dev = 0;
        ck(cudaGetDevice(&dev), "cudaGetDevice");
        m->ordinal = dev;
        m->cfg = c;
        m->max_tokens = max_tokens;
        m->max_seqs = max_seqs;
        const int D = bert::D, F = bert::F;
        auto keep = [&](void *p) { m->owned.push_back(p); return p; };
        auto bf = [&](const float *src, size_t n) {
            std::vector<uint16_t> v(n);
            for (size_t i = 0; i < n; i++) v[i] = to_bf16_bits(src[i]);
            return static_cast<uint16_t *>(keep(dupload(v)));
        };
        auto f32 = [&](std::initializer_list<std::pair<const float *, size_t>> parts) {
            std::vector<float> v;
            for (auto &pr : parts) v.insert(v.end(), pr.first, pr.first + pr.second);
            return static_cast<float *>(keep(dupload(v)));
        };
        m->word = bf(w->word_emb, (size_t)c.vocab * D);
        m->pos = bf(w->pos_emb, (size_t)c.max_pos * D);
        m->type0 = bf(w->type_emb, D);
        m->emb_ln = f32({{w->emb_ln_w, (size_t)D}, {w->emb_ln_b, (size_t)D}});
        for (int l = 0; l < c.n_layers; l++) {
            const XdnaBertLayer &L = w->layers[l];
            XdnaBert::Layer o{};
            std::vector<uint16_t> t;
            append_transposed_bf16(L.q_w, D, D, t);
            append_transposed_bf16(L.k_w, D, D, t);
            append_transposed_bf16(L.v_w, D, D, t);
            o.wqkv = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_transposed_bf16(L.o_w, D, D, t); o.wo = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_transposed_bf16(L.ffn1_w, D, F, t); o.w1 = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_transposed_bf16(L.ffn2_w, F, D, t); o.w2 = static_cast<uint16_t *>(keep(dupload(t)));
            o.bqkv = f32({{L.q_b, (size_t)D}, {L.k_b, (size_t)D}, {L.v_b, (size_t)D}});
            o.bo = f32({{L.o_b, (size_t)D}});
            o.b1 = f32({{L.ffn1_b, (size_t)F}});
            o.b2 = f32({{L.ffn2_b, (size_t)D}});
            o.ln1 = f32({{L.attn_ln_w, (size_t)D}, {L.attn_ln_b, (size_t)D}});
            o.ln2 = f32({{L.out_ln_w, (size_t)D}, {L.out_ln_b, (size_t)D}});
            m->layers.push_back(o);
        }
        const size_t T = (size_t)max_tokens;
        m->x = static_cast<uint16_t *>(keep(dalloc<uint16_t>(T * D)));
        m->qkv = static_cast<uint16_t *>(keep(dalloc<uint16_t>(T * 3 * D)));
        m->ctx = static_cast<uint16_t *>(keep(dalloc<uint16_t>(T * D)));
        m->y = static_cast<uint16_t *>(keep(dalloc<uint16_t>(T * D)));
        m->hbuf = static_cast<uint16_t *>(keep(dalloc<uint16_t>(T * F)));
        m->ids = static_cast<int32_t *>(keep(dalloc<int32_t>(T)));
        m->tokpos = static_cast<int32_t *>(keep(dalloc<int32_t>(T)));
        m->cu = static_cast<int32_t *>(keep(dalloc<int32_t>(max_seqs + 1)));
        m->out = static_cast<float *>(keep(dalloc<float>((size_t)max_seqs * D)));
        ck(cudaDeviceSynchronize(), "create sync");
        return m;
    } catch (const std::exception &e) {
        set_last_error_message(std::string("xdna_bert_create: ") + e.what());
        delete m;
        return nullptr;
    }
}

void xdna_bert_free(XdnaBert *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    delete m;
}

// The encoder over device-resident packed inputs: ids/tok_pos [n_tokens], cu [n_seqs + 1]
// (sequence starts, cu[n_seqs] = n_tokens), max_len = longest sequence; writes the pooled,
// L2-normalised embeddings [n_seqs, 768] f32 to out_dev.  Asynchronous on `stream`.
int xdna_bert_encode_device(XdnaBert *m, const int32_t *ids, const int32_t *tok_pos, const int32_t *cu,
                            int n_tokens, int n_seqs, int max_len, float *out_dev, void *stream) {
    if (!m || !ids || !tok_pos || !cu || !out_dev) { set_last_error_message("xdna_bert_encode_device: null pointer"); return -1; }
    if (n_tokens < 1 || n_tokens > m->max_tokens || n_seqs < 1 || max_len < 1 || max_len > m->cfg.max_pos) {
        set_last_error_message("xdna_bert_encode_device: sizes beyond the model's max_tokens / max_pos");
        return -1;
    }
    using namespace bert;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int T = n_tokens;
    const float eps = m->cfg.eps;
    cudaError_t e;
    embed_ln_kernel<<<(T + 7) / 8, 256, 0, st>>>(ids, tok_pos, T, m->word, m->pos, m->type0, m->emb_ln,
                                                 m->emb_ln + D, eps, m->x);
    for (const auto &L : m->layers) {
        if ((e = gemm_bf16(m->x, D, L.wqkv, D, T, 3 * D, D, L.bqkv, nullptr, 0, 0, m->qkv, 3 * D, st))) break;
        if ((e = attention_tc(m->qkv, T, cu, n_seqs, max_len, m->ctx, st))) break;
        if ((e = gemm_bf16(m->ctx, D, L.wo, D, T, D, D, L.bo, m->x, D, 0, m->y, D, st))) break;
        launch_ln(m->y, T, L.ln1, L.ln1 + D, eps, m->x, st);
        if ((e = gemm_bf16(m->x, D, L.w1, D, T, F, D, L.b1, nullptr, 0, 1, m->hbuf, F, st))) break;
        if ((e = gemm_bf16(m->hbuf, F, L.w2, F, T, D, F, L.b2, m->x, D, 0, m->y, D, st))) break;
        launch_ln(m->y, T, L.ln2, L.ln2 + D, eps, m->x, st);
    }
    pool_kernel<<<n_seqs, 32, 0, st>>>(m->x, cu, m->cfg.pooling, out_dev);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_bert_encode_device: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int xdna_bert_embed(XdnaBert *m, const int32_t *ids, const int32_t *seq_lens, int n_seqs, float *out) {
    if (!m || !ids || !seq_lens || !out) { set_last_error_message("xdna_bert_embed: null pointer"); return -1; }
    if (n_seqs < 1 || n_seqs > m->max_seqs) { set_last_error_message("xdna_bert_embed: n_seqs beyond max_seqs"); return -1; }
    std::vector<int32_t> cu(n_seqs + 1, 0), tokpos;
    int max_len = 0;
    for (int s = 0; s < n_seqs; s++) {
        if (seq_lens[s] < 1 || seq_lens[s] > m->cfg.max_pos) {
            set_last_error_message("xdna_bert_embed: sequence length outside [1, max_pos]");
            return -1;
        }
        cu[s + 1] = cu[s] + seq_lens[s];
        max_len = std::max(max_len, seq_lens[s]);
        for (int t = 0; t < seq_lens[s]; t++) tokpos.push_back(t);
    }
    const int T = cu[n_seqs];
    if (T > m->max_tokens) { set_last_error_message("xdna_bert_embed: total tokens beyond max_tokens"); return -1; }
    for (int i = 0; i < T; i++)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab) { set_last_error_message("xdna_bert_embed: token id out of range"); return -1; }
    try {
        ck(cudaMemcpy(m->ids, ids, T * 4, cudaMemcpyHostToDevice), "copy ids");
        ck(cudaMemcpy(m->tokpos, tokpos.data(), T * 4, cudaMemcpyHostToDevice), "copy positions");
        ck(cudaMemcpy(m->cu, cu.data(), (n_seqs + 1) * 4, cudaMemcpyHostToDevice), "copy offsets");
        if (xdna_bert_encode_device(m, m->ids, m->tokpos, m->cu, T, n_seqs, max_len, m->out, nullptr) != 0) return -1;
        ck(cudaMemcpy(out, m->out, (size_t)n_seqs * bert::D * 4, cudaMemcpyDeviceToHost), "copy embeddings");
        if (gemm_error_and_clear() | attention_tc_error_and_clear()) {
            set_last_error_message("xdna_bert_embed: a tensor-core wait expired");
            return -1;
        }
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_bert_embed: ") + ex.what());
        return -1;
    }
}

}  // extern "C"

// =============================================================================== Whisper
// Whisper-small encoder (rust/npu-whisper/src/encoder.rs:183-203 conv_stem, 221-227 add_pos,
// 236-337 block, 350-375 forward_last): conv1 (k3 s1 p1) + GELU, conv2 (k3 s2 p1) + GELU,
// + embed_positions, pre-LN blocks, ln_post.  The convolutions are tcgen05 GEMMs over an
// im2col in tap-major order (column ki*Cin + ci; the weights are permuted to match), GELU and
// the positional add fused into the GEMM epilogue.  Linear weights are quantised to bfp16
// (blocks of 8 along K, route_b_kernels/ffn_bfp16/golden_ffn_gemm.py:34-49) at load; the
// block values are exactly representable in bf16, so the bf16 tensor-core GEMM computes on
// exactly the bfp16 weights.
namespace xdna {
namespace whisper {

constexpr int D = 768, F = 3072;

// cols[b*T + t][ki*C + ci] = mel[b][ci][t + ki - 1] (zero outside), columns C*3 .. ldc-1 zero
__global__ void im2col_mel_kernel(const float *mel, int B, int C, int T, int ldc, uint16_t *cols) {
    const size_t total = (size_t)B * T * ldc;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int col = (int)(i % ldc);
        const size_t row = i / ldc;
        const int b = (int)(row / T), t = (int)(row % T);
        float v = 0.0f;
        if (col < 3 * C) {
            const int ki = col / C, ci = col % C, ts = t + ki - 1;
            if (ts >= 0 && ts < T) v = mel[((size_t)b * C + ci) * T + ts];
        }
        cols[i] = (uint16_t)bf16bits(v);
    }
}

// cols[b*To + t][ki*D + c] = h[b*Ti + 2t + ki - 1][c] (zero outside): 16-byte vectors
__global__ void im2col_s2_kernel(const uint16_t *h, int B, int Ti, int To, uint16_t *cols) {
    const size_t vec_per_row = 3 * D / 8;
    const size_t total = (size_t)B * To * vec_per_row;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / vec_per_row;
        const int v = (int)(i % vec_per_row);
        const int b = (int)(row / To), t = (int)(row % To);
        const int ki = v / (D / 8), c8 = v % (D / 8);
        const int ts = 2 * t + ki - 1;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (ts >= 0 && ts < Ti) val = reinterpret_cast<const uint4 *>(h + ((size_t)b * Ti + ts) * D)[c8];
        reinterpret_cast<uint4 *>(cols)[i] = val;
    }
}

// y = LN(x) with eps, x/y [rows, 768] bf16 (pre-norm: x is kept as the residual stream)
}  // namespace whisper

namespace {
// to_bfp16_blocks along contiguous runs of 8 (golden_ffn_gemm.py:34-49): shared exponent
// e = floor(log2(max|x|)) (max 0 -> 1.0), quantum 2^(e-6), round half to even, no clamp.
void bfp16_blocks(const float *x, float *y, size_t n) {
    for (size_t b0 = 0; b0 < n; b0 += 8) {
        float m = 0.0f;
        for (int i = 0; i < 8; i++) m = std::fmax(m, std::fabs(x[b0 + i]));
        if (m == 0.0f) m = 1.0f;
        int e;
        (void)std::frexp(m, &e);
        e -= 1;
        const float q = std::ldexp(1.0f, e - 6);
        for (int i = 0; i < 8; i++) y[b0 + i] = std::nearbyint(x[b0 + i] / q) * q;
    }
}
// [K, N] f32 -> bfp16 along K for every output column -> [N, K] bf16 appended to out
void append_bfp16_transposed(const float *w, int K, int N, std::vector<uint16_t> &out) {
    const size_t base = out.size();
    out.resize(base + (size_t)N * K);
    std::vector<float> col(K), q(K);
    for (int n = 0; n < N; n++) {
        for (int k = 0; k < K; k++) col[k] = w[(size_t)k * N + n];
        bfp16_blocks(col.data(), q.data(), K);
        for (int k = 0; k < K; k++) out[base + (size_t)n * K + k] = to_bf16_bits(q[k]);
    }
}
}  // namespace
}  // namespace xdna

struct XdnaWhisperEnc {
    XdnaWhisperEncConfig cfg{};
    int max_batch = 0, K1 = 0;
    uint16_t *c1w = nullptr, *c2w = nullptr, *pos = nullptr;   // [768, K1], [768, 2304], [max_src, 768]
    float *c1b = nullptr, *c2b = nullptr, *lnpost = nullptr;
    struct Layer {
        uint16_t *wqkv, *wo, *w1, *w2;
        float *bqkv, *bo, *b1, *b2, *ln1, *ln2;
    };
    std::vector<Layer> layers;
    uint16_t *cols = nullptr, *h1 = nullptr, *x = nullptr, *y = nullptr, *qkv = nullptr, *ctx = nullptr, *hb = nullptr;
    float *mel = nullptr;
    int32_t *cu = nullptr;
    std::vector<void *> owned;
    ~XdnaWhisperEnc() {
        for (void *p : owned) cudaFree(p);
    }
};

extern "C" {

int xdna_bfp16_quantize(const float *x, size_t n, float *y) {
    if (!x || !y || n % 8) { set_last_error_message("xdna_bfp16_quantize: null pointer or n % 8 != 0"); return -1; }
    bfp16_blocks(x, y, n);
    return 0;
}

XdnaWhisperEnc *xdna_whisper_enc_create(XdnaDevice *dev_unused, const XdnaWhisperEncConfig *cfg,
                                        const XdnaWhisperEncWeights *w, int max_batch) {
    (void)dev_unused;
    if (!cfg || !w || !w->layers || !w->conv1_w || !w->conv1_b || !w->conv2_w || !w->conv2_b ||
        !w->embed_positions || !w->ln_post_w || !w->ln_post_b) {
        set_last_error_message("xdna_whisper_enc_create: null pointer");
        return nullptr;
    }
    const XdnaWhisperEncConfig c = *cfg;
    if (c.d_model != whisper::D || c.n_heads != 12 || c.ffn != whisper::F || c.n_layers < 1 || c.n_mels < 1 ||
        c.n_frames < 2 || c.n_frames % 2 || c.n_frames / 2 > c.max_src || max_batch < 1) {
        set_last_error_message("xdna_whisper_enc_create: supported shape is d_model 768, 12 heads, ffn 3072; "
                               "n_frames even with n_frames / 2 <= max_src");
        return nullptr;
    }
    auto *m = new XdnaWhisperEnc();
    try {
        const int D = whisper::D, F = whisper::F, C = c.n_mels, T = c.n_frames, To = c.n_frames / 2;
        m->cfg = c;
        m->max_batch = max_batch;
        m->K1 = (3 * C + 63) / 64 * 64;
        auto keep = [&](void *p) { m->owned.push_back(p); return p; };
        auto f32 = [&](std::initializer_list<std::pair<const float *, size_t>> parts) {
            std::vector<float> v;
            for (auto &pr : parts) {
                if (pr.first) v.insert(v.end(), pr.first, pr.first + pr.second);
                else v.insert(v.end(), pr.second, 0.0f);
            }
            return static_cast<float *>(keep(dupload(v)));
        };
        // conv weights [Cout, Cin, 3] -> tap-major [Cout, ki*Cin + ci] bf16 (K padded)
        std::vector<uint16_t> t1((size_t)D * m->K1, 0), t2((size_t)D * 3 * D, 0);
        for (int co = 0; co < D; co++)
            for (int ci = 0; ci < C; ci++)
                for (int ki = 0; ki < 3; ki++)
                    t1[(size_t)co * m->K1 + ki * C + ci] = to_bf16_bits(w->conv1_w[((size_t)co * C + ci) * 3 + ki]);
        for (int co = 0; co < D; co++)
            for (int ci = 0; ci < D; ci++)
                for (int ki = 0; ki < 3; ki++)
                    t2[(size_t)co * 3 * D + ki * D + ci] = to_bf16_bits(w->conv2_w[((size_t)co * D + ci) * 3 + ki]);
        m->c1w = static_cast<uint16_t *>(keep(dupload(t1)));
        m->c2w = static_cast<uint16_t *>(keep(dupload(t2)));
        m->c1b = f32({{w->conv1_b, (size_t)D}});
        m->c2b = f32({{w->conv2_b, (size_t)D}});
        std::vector<uint16_t> pv((size_t)To * D);
        for (size_t i = 0; i < pv.size(); i++) pv[i] = to_bf16_bits(w->embed_positions[i]);
        m->pos = static_cast<uint16_t *>(keep(dupload(pv)));
        m->lnpost = f32({{w->ln_post_w, (size_t)D}, {w->ln_post_b, (size_t)D}});
        for (int l = 0; l < c.n_layers; l++) {
            const XdnaWhisperEncLayer &L = w->layers[l];
            XdnaWhisperEnc::Layer o{};
            std::vector<uint16_t> t;
            append_bfp16_transposed(L.q_w, D, D, t);
            append_bfp16_transposed(L.k_w, D, D, t);
            append_bfp16_transposed(L.v_w, D, D, t);
            o.wqkv = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_bfp16_transposed(L.out_w, D, D, t); o.wo = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_bfp16_transposed(L.fc1_w, D, F, t); o.w1 = static_cast<uint16_t *>(keep(dupload(t)));
            t.clear(); append_bfp16_transposed(L.fc2_w, F, D, t); o.w2 = static_cast<uint16_t *>(keep(dupload(t)));
            o.bqkv = f32({{L.q_b, (size_t)D}, {L.k_b, (size_t)D}, {L.v_b, (size_t)D}});   // k_b may be null: zeros
            o.bo = f32({{L.out_b, (size_t)D}});
            o.b1 = f32({{L.fc1_b, (size_t)F}});
            o.b2 = f32({{L.fc2_b, (size_t)D}});
            o.ln1 = f32({{L.ln1_w, (size_t)D}, {L.ln1_b, (size_t)D}});
            o.ln2 = f32({{L.ln2_w, (size_t)D}, {L.ln2_b, (size_t)D}});
            m->layers.push_back(o);
        }
        const size_t B = (size_t)max_batch, R1 = B * T, R2 = B * To;
        m->mel = static_cast<float *>(keep(dalloc<float>(B * C * T)));
        m->cols = static_cast<uint16_t *>(keep(dalloc<uint16_t>(std::max(R1 * m->K1, R2 * 3 * D))));
        m->h1 = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R1 * D)));
        m->x = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R2 * D)));
        m->y = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R2 * D)));
        m->qkv = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R2 * 3 * D)));
        m->ctx = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R2 * D)));
        m->hb = static_cast<uint16_t *>(keep(dalloc<uint16_t>(R2 * F)));
        std::vector<int32_t> cu(B + 1);
        for (size_t b = 0; b <= B; b++) cu[b] = (int32_t)(b * To);
        m->cu = static_cast<int32_t *>(keep(dupload(cu)));
        ck(cudaDeviceSynchronize(), "create sync");
        return m;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_whisper_enc_create: ") + ex.what());
        delete m;
        return nullptr;
    }
}

void xdna_whisper_enc_free(XdnaWhisperEnc *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    delete m;
}

// Device-resident encoder: mel_dev [B][n_mels][n_frames] f32 -> out_dev [B][n_frames/2][768] bf16
int xdna_whisper_encode_device(XdnaWhisperEnc *m, const float *mel_dev, int B, uint16_t *out_dev, void *stream) {
    if (!m || !mel_dev || !out_dev) { set_last_error_message("xdna_whisper_encode_device: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch) { set_last_error_message("xdna_whisper_encode_device: batch beyond max_batch"); return -1; }
    using namespace whisper;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int C = m->cfg.n_mels, T = m->cfg.n_frames, To = T / 2, R1 = B * T, R2 = B * To;
    const float eps = m->cfg.eps;
    cudaError_t e = cudaSuccess;
    im2col_mel_kernel<<<1184, 256, 0, st>>>(mel_dev, B, C, T, m->K1, m->cols);
    if (!e) e = gemm_bf16(m->cols, m->K1, m->c1w, m->K1, R1, D, m->K1, m->c1b, nullptr, 0, 1, m->h1, D, st);
    im2col_s2_kernel<<<1184, 256, 0, st>>>(m->h1, B, T, To, m->cols);
    // conv2 + GELU, then + embed_positions[t] (residual row = output row mod To)
    if (!e) e = gemm_bf16(m->cols, 3 * D, m->c2w, 3 * D, R2, D, 3 * D, m->c2b, m->pos, D, 1, m->x, D, st, To);
    for (size_t li = 0; li < m->layers.size() && !e; li++) {
        const auto &L = m->layers[li];
        bert::launch_ln(m->x, R2, L.ln1, L.ln1 + D, eps, m->y, st);
        if ((e = gemm_bf16(m->y, D, L.wqkv, D, R2, 3 * D, D, L.bqkv, nullptr, 0, 0, m->qkv, 3 * D, st))) break;
        if ((e = attention_tc(m->qkv, R2, m->cu, B, To, m->ctx, st))) break;
        if ((e = gemm_bf16(m->ctx, D, L.wo, D, R2, D, D, L.bo, m->x, D, 0, m->y, D, st))) break;
        std::swap(m->x, m->y);   // x <- x + attn
        bert::launch_ln(m->x, R2, L.ln2, L.ln2 + D, eps, m->y, st);
        if ((e = gemm_bf16(m->y, D, L.w1, D, R2, F, D, L.b1, nullptr, 0, 1, m->hb, F, st))) break;
        if ((e = gemm_bf16(m->hb, F, L.w2, F, R2, D, F, L.b2, m->x, D, 0, m->y, D, st))) break;
        std::swap(m->x, m->y);   // x <- x + ffn
    }
    if (!e) bert::launch_ln(m->x, R2, m->lnpost, m->lnpost + D, eps, out_dev, st);
    if (!e) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error_message(std::string("xdna_whisper_encode_device: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// Host in / host out: mel [B][n_mels][n_frames] f32 -> encoded [B][n_frames/2][768] f32
int xdna_whisper_encode(XdnaWhisperEnc *m, const float *mel, int B, float *out) {
    if (!m || !mel || !out) { set_last_error_message("xdna_whisper_encode: null pointer"); return -1; }
    if (B < 1 || B > m->max_batch) { set_last_error_message("xdna_whisper_encode: batch beyond max_batch"); return -1; }
    const int C = m->cfg.n_mels, T = m->cfg.n_frames, To = T / 2;
    try {
        ck(cudaMemcpy(m->mel, mel, sizeof(float) * (size_t)B * C * T, cudaMemcpyHostToDevice), "copy mel");
        // the FFN buffer ([B * To][3072] bf16) holds the bf16 result and, after it, its f32 widening
        // (2 + 4 bytes per value <= 2 * 3072 / 768), which is copied straight into `out`
        const size_t n = (size_t)B * To * whisper::D;
        uint16_t *enc = m->hb;
        float *encf = reinterpret_cast<float *>(m->hb + n);
        if (xdna_whisper_encode_device(m, m->mel, B, enc, nullptr) != 0) return -1;
        bert::bf16_to_f32_kernel<<<148 * 8, 256>>>(enc, n, encf);
        ck(cudaGetLastError(), "widen");
        ck(cudaMemcpy(out, encf, n * sizeof(float), cudaMemcpyDeviceToHost), "copy encoded");
        if (gemm_error_and_clear() | attention_tc_error_and_clear()) {
            set_last_error_message("xdna_whisper_encode: a tensor-core wait expired");
            return -1;
        }
        return 0;
    } catch (const std::exception &ex) {
        set_last_error_message(std::string("xdna_whisper_encode: ") + ex.what());
        return -1;
    }
}

}  // extern "C"
