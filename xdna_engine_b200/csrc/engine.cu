// engine.cu -- host side of the B200 backend: device handle, int8 quantiser, weight-stream
// packer, decoder lifetime and the C ABI declared in include/xdna_b200.h.
//
// Replaces rust/npu-xrt (device, buffer objects, dispatch; src/lib.rs:46-158, 641-744) and
// the weight preparation of the opt-125m decode (opt125m_decode.rs Lin::load 41-60,
// Opt::load 155-181).  Error convention of the reference C ABIs: NULL / -1 plus a
// thread-local message (rust/npu-capi/src/lib.rs:11-16).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"
#include "decode.h"
#include "gemv_op.h"

namespace xdna {
int decode_smem_bytes();
cudaError_t launch_opt_decode(const DecodeParams &p, cudaStream_t st);
cudaError_t max_coresident_ctas(int d, int f, int *out);
bool decode_shape_supported(int d, int f);
cudaError_t launch_prefill_embed(const int64_t *tokens, int pos0, int T, int D, int V, const float *emb_tok,
                                 const float *emb_pos, float *x, RunState *state, cudaStream_t st);
cudaError_t launch_prefill_ln(const float *x, int T, int D, const float *g, const float *b, float eps, int fix,
                              int8_t *limbs, cudaStream_t st);
cudaError_t launch_prefill_gemv(const PrefillGemv &a, cudaStream_t st);
cudaError_t launch_prefill_attn(const float *q, const uint16_t *kv, const int *pt, int layer, int n_phys, int n_heads,
                                int pos0, int T, int D, int fix, int8_t *limbs, cudaStream_t st);
}  // namespace xdna

using namespace xdna;

namespace {

thread_local std::string g_last_error;

void set_err(const std::string &m) { g_last_error = m; }

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess)
        throw CudaError(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

template <class T>
T *dmalloc(size_t n) {
    void *p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)), "cudaMalloc");
    return static_cast<T *>(p);
}

// Lin::load (opt125m_decode.rs:41-60): per-output-column scale amax/127 (1.0 if zero),
// q = clamp(round(w / scale), -127, 127), round = half away from zero.  Output-major.
void quant_cols(const float *w, int K, int N, int8_t *q_nk, float *scale) {
    for (int c = 0; c < N; c++) {
        float amax = 0.0f;
        for (int r = 0; r < K; r++) amax = std::fmax(amax, std::fabs(w[(size_t)r * N + c]));
        scale[c] = amax > 0.0f ? amax / 127.0f : 1.0f;
    }
    for (int r = 0; r < K; r++) {
        const float *wr = w + (size_t)r * N;
        for (int c = 0; c < N; c++) {
            float v = std::round(wr[c] / scale[c]);
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            q_nk[(size_t)c * K + r] = static_cast<int8_t>(v);
        }
    }
}
// the tied LM head: output channel v = embedding row v, same rule
void quant_rows(const float *w, int M, int K, int8_t *q, float *scale) {
    for (int m = 0; m < M; m++) {
        const float *row = w + (size_t)m * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = std::fmax(amax, std::fabs(row[k]));
        const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        scale[m] = s;
        for (int k = 0; k < K; k++) {
            float v = std::round(row[k] / s);
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            q[(size_t)m * K + k] = static_cast<int8_t>(v);
        }
    }
}

// A GEMV operand in the engine's output-major int8 form.
struct QMat {
    int K = 0, N = 0;
    std::vector<int8_t> q;      // [N][K]
    std::vector<float> scale;   // [N]
    std::vector<float> bias;    // [N]
};

// Append rows [r0, r0+rows) of m as chunks of the op-level GEMV (gemv_op.h): per chunk the
// rows' K bytes with 32-byte block kb of row r stored at block kb ^ (r & 3), then (scale,
// bias) per row, padded to 16 bytes.
void pack_rows(const QMat &m, int r0, int rows, std::vector<uint8_t> &out,
               std::vector<gemvop::ChunkRef> &refs, size_t base_off) {
    using namespace gemvop;
    const int K = m.K, rpc = rows_per_chunk(K);
    for (int c0 = 0; c0 < rows; c0 += rpc) {
        const int rr = std::min(rpc, rows - c0);
        const uint32_t bytes = chunk_bytes(rr, K);
        const size_t off = out.size();
        out.resize(off + bytes, 0);
        uint8_t *dst = out.data() + off;
        for (int r = 0; r < rr; r++) {
            const int8_t *src = m.q.data() + (size_t)(r0 + c0 + r) * K;
            for (int kb = 0; kb < K / 32; kb++)
                std::memcpy(dst + (size_t)r * K + ((kb ^ (r & 3)) * 32), src + kb * 32, 32);
        }
        float *meta = reinterpret_cast<float *>(dst + (size_t)rr * K);
        for (int r = 0; r < rr; r++) {
            meta[2 * r] = m.scale[r0 + c0 + r];
            meta[2 * r + 1] = m.bias.empty() ? 0.0f : m.bias[r0 + c0 + r];
        }
        refs.push_back(gemvop::ChunkRef{static_cast<uint32_t>(base_off + off), bytes});
    }
}

// ---- the decode kernel's stream (decode.h): chunks in mma.sync m16n8k32 A-fragment order.
// Lane (g, tig) of an m-tile x 32-wide k-block holds 16 bytes: A[g][4tig..+3],
// A[g+8][4tig..+3], A[g][16+4tig..+3], A[g+8][16+4tig..+3].
template <class At>
void put_frag(uint8_t *dst, At A) {
    for (int lane = 0; lane < 32; lane++) {
        const int g = lane >> 2, tig = lane & 3;
        const int rows[4] = {g, g + 8, g, g + 8}, ks[4] = {4 * tig, 4 * tig, 16 + 4 * tig, 16 + 4 * tig};
        for (int w = 0; w < 4; w++)
            for (int i = 0; i < 4; i++) dst[lane * 16 + w * 4 + i] = (uint8_t)A(rows[w], ks[w] + i);
    }
}

struct StreamBuilder {
    std::vector<uint8_t> bytes;
    std::vector<ChunkRef> refs;
    size_t base = 0;                       // offset of this CTA's stream in the whole stream
    uint8_t *chunk(size_t n) {
        const size_t off = bytes.size();
        bytes.resize(off + ((n + 15) & ~(size_t)15), 0);
        refs.push_back(ChunkRef{static_cast<uint32_t>(base + off), static_cast<uint32_t>((n + 15) & ~(size_t)15)});
        return bytes.data() + off;
    }
};

// one 16-row tile of a GEMV whose output row r (r < 16) is row(r) of an output-major int8
// matrix with K columns (nullptr = zero row), followed by 16 x (scale, bias)
template <class RowFn>
void pack_row_tile(StreamBuilder &sb, int K, RowFn row) {
    uint8_t *dst = sb.chunk(row_chunk_bytes(K));
    for (int kb = 0; kb < K / 32; kb++)
        put_frag(dst + kb * kFragBytes, [&](int r, int k) -> int8_t {
            const int8_t *q = row(r).q;
            return q ? q[kb * 32 + k] : (int8_t)0;
        });
    float *meta = reinterpret_cast<float *>(dst + (size_t)kTile * K);
    for (int r = 0; r < kTile; r++) {
        meta[2 * r] = row(r).scale;
        meta[2 * r + 1] = row(r).bias;
    }
}
struct RowRef {
    const int8_t *q;
    float scale, bias;
};
RowRef row_of(const QMat &m, int n) {
    if (n < 0 || n >= m.N) return RowRef{nullptr, 1.0f, 0.0f};
    return RowRef{m.q.data() + (size_t)n * m.K, m.scale[n], m.bias.empty() ? 0.0f : m.bias[n]};
}
// the K-split slice of m over input columns [k0, k0 + 32) for all N outputs, as
// slice_chunks(N) chunks of up to 24 m-tiles
void pack_slice(StreamBuilder &sb, const QMat &m, int k0) {
    const int N = m.N;
    for (int c = 0; c < slice_chunks(N); c++) {
        const int nt = slice_chunk_tiles(N, c);
        uint8_t *dst = sb.chunk((size_t)nt * kFragBytes);
        for (int t = 0; t < nt; t++) {
            const int n0 = (c * kSliceTilesPerChunk + t) * kTile;
            put_frag(dst + t * kFragBytes,
                     [&](int r, int k) -> int8_t { return m.q[(size_t)(n0 + r) * m.K + k0 + k]; });
        }
    }
}

// Fixed-point exponent for values bounded by B: |x| * 2^s < 2^29.  The bounds are data
// independent (weights and LayerNorm parameters only): a LayerNorm output satisfies
// |y_k| <= sqrt(D) |gamma_k| + |beta_k|, so a linear output row n is bounded by
// sum_k |W[n][k]| * scale[n] * lnmax_k + |bias[n]|; 1% covers the bf16 and f32 roundings.
int fix_from_bound(double B) {
    if (!(B > 0.0)) return kFixBits;
    int E = 0;
    std::frexp(B, &E);                     // B < 2^E
    return kFixBits - E;
}
// a LayerNorm output: |y_k| <= sqrt(D) |g_k| + |b_k| (1% for the roundings)
double ln_bound(const float *g, const float *b, int D) {
    double B = 0.0;
    for (int k = 0; k < D; k++)
        B = std::max(B, (std::sqrt((double)D) * std::fabs((double)g[k]) + std::fabs((double)b[k])) * 1.01);
    return B;
}
double rows_bound(const QMat &m, int n0, int n1, const float *g, const float *b, int D) {
    std::vector<double> lnmax(D);
    for (int k = 0; k < D; k++)
        lnmax[k] = (std::sqrt((double)D) * std::fabs((double)g[k]) + std::fabs((double)b[k])) * 1.01;
    double B = 0.0;
    for (int n = n0; n < n1; n++) {
        const int8_t *q = m.q.data() + (size_t)n * m.K;
        double s = 0.0;
        for (int k = 0; k < m.K; k++) s += std::fabs((double)q[k]) * lnmax[k];
        s = s * (double)m.scale[n] + std::fabs((double)(m.bias.empty() ? 0.0f : m.bias[n]));
        B = std::max(B, s);
    }
    return B * 1.01;
}
// integer tuning knob from the environment (default when unset or not a number)
int env_int(const char *name, int dflt) {
    const char *v = std::getenv(name);
    if (!v || !*v) return dflt;
    char *end = nullptr;
    const long r = std::strtol(v, &end, 10);
    return (end && *end == 0 && r > 0 && r < 1000000) ? (int)r : dflt;
}
int ceil_log2(int v) {
    int e = 0;
    while ((1 << e) < v) e++;
    return e;
}

QMat quant_linear(const float *w, const float *b, int K, int N) {
    QMat m;
    m.K = K;
    m.N = N;
    m.q.resize((size_t)K * N);
    m.scale.resize(N);
    quant_cols(w, K, N, m.q.data(), m.scale.data());
    m.bias.assign(b, b + N);
    return m;
}

}  // namespace

namespace xdna {
void set_last_error_message(const std::string &m) { set_err(m); }
}  // namespace xdna

struct XdnaDevice {
    int ordinal = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
};

struct XdnaOptDecoder {
    XdnaDevice *dev = nullptr;
    XdnaOptConfig cfg{};
    int grid = 0, n_fc = 0, max_ctx = 0, n_pages = 0, vocab_tiles = 0;
    int fix_lnf = 0;
    int o_bias_shift = 0, f2_bias_shift = 0, o_subs = 2, f2_subs = 8, poll_ns = 20, lm_prefetch_layer = 0;
    size_t stream_bytes = 0, token_bytes = 0;
    uint8_t *d_stream = nullptr;
    ChunkRef *d_chunks = nullptr;
    int *d_nl = nullptr, *d_nlm = nullptr;
    int chunk_stride = 0;
    float *d_emb = nullptr, *d_pos = nullptr, *d_ln = nullptr, *d_lnf = nullptr, *d_osb = nullptr,
          *d_f2sb = nullptr;
    int *d_fix = nullptr;                  // [4][L]: context, fc1-output, LN1, LN2 exponents
    uint16_t *d_kv = nullptr;
    int *d_pt = nullptr;
    unsigned long long *d_acc = nullptr;
    size_t acc_words = 0;
    unsigned long long *d_ll = nullptr;
    int64_t *d_tokens = nullptr;
    RunState *d_state = nullptr;
    float *d_logits = nullptr;      // scratch for xdna_opt_generate
    float *trace = nullptr;         // optional residual-stream record (xdna_opt_set_trace)
    unsigned long long *timing = nullptr;  // optional phase stamps (xdna_opt_set_timing)
    size_t logits_cap = 0;
    // batched prompt prefill: row-major int8 weights per layer (q|k|v, o, fc1, fc2), the q|k|v
    // and fc1 row scale / bias, scratch for kPrefillTokens positions
    bool prefill = false;
    std::vector<int> h_fix;                // [4][L] as d_fix
    int8_t *d_pfw = nullptr;
    float *d_pfsb = nullptr;
    size_t pf_w_layer = 0, pf_sb_layer = 0;
    float *d_pfx = nullptr, *d_pfq = nullptr;
    int8_t *d_pfa = nullptr, *d_pfh = nullptr;
    unsigned long long *d_pfacc = nullptr;  // [kPrefillTokens][max(3D, F)] K-split sums (zero between uses)
    unsigned int *d_pfcnt = nullptr;        // per 16-row tile: K-slice CTAs finished
    ~XdnaOptDecoder() {
        void *ptrs[] = {d_stream, d_chunks, d_nl, d_nlm, d_emb, d_pos, d_ln, d_lnf, d_osb, d_f2sb, d_fix,
                        d_kv, d_pt, d_acc, d_ll, d_tokens, d_state, d_logits, d_pfw, d_pfsb, d_pfx, d_pfq,
                        d_pfa, d_pfh, d_pfacc, d_pfcnt};
        for (void *p : ptrs)
            if (p) cudaFree(p);
    }
};

extern "C" {

const char *xdna_last_error(void) { return g_last_error.c_str(); }

int xdna_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int usable = 0;
    for (int i = 0; i < n; i++) {
        cudaDeviceProp pr{};
        if (cudaGetDeviceProperties(&pr, i) == cudaSuccess && pr.major == 10) usable++;
    }
    return usable;
}

XdnaDevice *xdna_device_open(int ordinal) {
    try {
        int n = 0;
        ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (ordinal < 0 || ordinal >= n) {
            set_err("device ordinal " + std::to_string(ordinal) + " out of range (" + std::to_string(n) + " devices)");
            return nullptr;
        }
        cudaDeviceProp pr{};
        ck(cudaGetDeviceProperties(&pr, ordinal), "cudaGetDeviceProperties");
        if (pr.major != 10) {
            set_err(std::string("device is not sm_100 (") + pr.name + ")");
            return nullptr;
        }
        ck(cudaSetDevice(ordinal), "cudaSetDevice");
        auto *d = new XdnaDevice();
        d->ordinal = ordinal;
        d->sms = pr.multiProcessorCount;
        return d;
    } catch (const std::exception &e) {
        set_err(e.what());
        return nullptr;
    }
}

void xdna_device_close(XdnaDevice *dev) { delete dev; }
int xdna_device_ordinal(const XdnaDevice *dev) { return dev ? dev->ordinal : -1; }

int xdna_quant_i8_cols(const float *w, int K, int N, int8_t *q_nk, float *scale) {
    if (!w || !q_nk || !scale || K <= 0 || N <= 0) {
        set_err("xdna_quant_i8_cols: null pointer or empty shape");
        return -1;
    }
    quant_cols(w, K, N, q_nk, scale);
    return 0;
}

// qrow of the fused decode ELF (route_b_kernels/decode_fused/gen_decode.py:158-165): per output
// row m of an [M, K] weight, scale = max_k |W[m][k]| / 127 (1.0 for an all-zero row),
// q = clip(round half to even(W / scale), -127, 127).  The result feeds xdna_gemv_i8 directly
// (q_nk = q, y = (x . q) * scale + bias: the ELF's op_mulw scale before the bias add).
int xdna_quant_i8_rows(const float *w, int M, int K, int8_t *q, float *scale) {
    if (!w || !q || !scale || M <= 0 || K <= 0) {
        set_err("xdna_quant_i8_rows: null pointer or empty shape");
        return -1;
    }
    for (int m = 0; m < M; m++) {
        const float *row = w + (size_t)m * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = std::max(amax, std::fabs(row[k]));
        const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        scale[m] = s;
        for (int k = 0; k < K; k++) {
            const float v = std::nearbyint(row[k] / s);      // round-to-nearest-even mode
            q[(size_t)m * K + k] = (int8_t)std::min(127.0f, std::max(-127.0f, v));
        }
    }
    return 0;
}

int xdna_gemv_i8(XdnaDevice *dev, const float *x, int K, const int8_t *q_nk, const float *scale,
                 const float *bias, int N, float *y) {
    if (!dev || !x || !q_nk || !scale || !y) { set_err("xdna_gemv_i8: null pointer"); return -1; }
    if (K <= 0 || K % 256 != 0 || K > gemvop::kKmax || N <= 0 || N % 8 != 0) {
        set_err("xdna_gemv_i8: K must be a multiple of 256 <= 3072 and N a multiple of 8");
        return -1;
    }
    float *dx = nullptr, *dy = nullptr;
    uint8_t *dp = nullptr;
    gemvop::ChunkRef *dc = nullptr;
    try {
        ck(cudaSetDevice(dev->ordinal), "cudaSetDevice");
        QMat m;
        m.K = K;
        m.N = N;
        m.q.assign(q_nk, q_nk + (size_t)K * N);
        m.scale.assign(scale, scale + N);
        if (bias) m.bias.assign(bias, bias + N);
        std::vector<uint8_t> packed;
        std::vector<gemvop::ChunkRef> refs;
        pack_rows(m, 0, N, packed, refs, 0);
        dx = dmalloc<float>(K);
        dy = dmalloc<float>(N);
        dp = dmalloc<uint8_t>(packed.size());
        dc = dmalloc<gemvop::ChunkRef>(refs.size());
        ck(cudaMemcpy(dx, x, sizeof(float) * K, cudaMemcpyHostToDevice), "copy x");
        ck(cudaMemcpy(dp, packed.data(), packed.size(), cudaMemcpyHostToDevice), "copy weights");
        ck(cudaMemcpy(dc, refs.data(), refs.size() * sizeof(gemvop::ChunkRef), cudaMemcpyHostToDevice), "copy chunks");
        ck(gemvop::launch_gemv_i8(dx, K, dp, dc, N, dy, nullptr), "gemv_i8 launch");
        ck(cudaMemcpy(y, dy, sizeof(float) * N, cudaMemcpyDeviceToHost), "copy y");
        cudaFree(dx); cudaFree(dy); cudaFree(dp); cudaFree(dc);
        return 0;
    } catch (const std::exception &e) {
        set_err(e.what());
        if (dx) cudaFree(dx);
        if (dy) cudaFree(dy);
        if (dp) cudaFree(dp);
        if (dc) cudaFree(dc);
        return -1;
    }
}

XdnaOptDecoder *xdna_opt_create(XdnaDevice *dev, const XdnaOptConfig *cfg, const XdnaOptWeights *w,
                                int max_ctx, int grid) {
    if (!dev || !cfg || !w || !w->layers || !w->emb_tok || !w->emb_pos || !w->lnf_w || !w->lnf_b) {
        set_err("xdna_opt_create: null pointer");
        return nullptr;
    }
    const XdnaOptConfig c = *cfg;
    const int D = c.d_model, F = c.ffn, L = c.n_layers, V = c.vocab, H = c.n_heads;
    if (c.head_dim != kHeadDim || H * kHeadDim != D || D % 256 || D > kDmax || F % 256 || F > kFmax ||
        L < 1 || V < 8 || c.max_pos < 1 || !decode_shape_supported(D, F)) {
        set_err("xdna_opt_create: unsupported shape (head_dim 64; (d_model, ffn) one of the "
                "compiled widths (768, 3072) or (256, 512))");
        return nullptr;
    }
    if (max_ctx < 1 || max_ctx > c.max_pos || max_ctx > kMaxCtx) {
        set_err("xdna_opt_create: max_ctx must be in [1, min(max_pos, 2048)]");
        return nullptr;
    }
    auto *dec = new (std::nothrow) XdnaOptDecoder();
    if (!dec) { set_err("out of host memory"); return nullptr; }
    try {
        ck(cudaSetDevice(dev->ordinal), "cudaSetDevice");
        dec->dev = dev;
        dec->cfg = c;
        dec->max_ctx = max_ctx;
        int maxg = 0;
        ck(max_coresident_ctas(D, F, &maxg), "occupancy query");
        maxg = std::min(maxg, 256);
        int G = grid > 0 ? std::min(grid, maxg) : maxg;
        G &= ~1;
        const int KB = F / 32;
        if (G < 2 * H + 1) throw std::runtime_error("grid too small: needs 2 * n_heads CTAs plus FC CTAs");
        // FC CTAs: at most one per 32-row block of fc1; fewer CTAs each own more blocks and add
        // fewer partial sums into each fc2 accumulator word
        const int n_fc = std::min(std::min(G - 2 * H, KB), env_int("XDNA_OPT_FC_CTAS", KB));
        int max_nkb = 0;
        for (int i = 0; i < n_fc; i++) max_nkb = std::max(max_nkb, fc_kb0(i + 1, KB, n_fc) - fc_kb0(i, KB, n_fc));
        // the exact limb combination keeps a * 256 + b in 32 bits for reduction lengths up to 768
        if (max_nkb > 24) throw std::runtime_error("grid too small: an FC CTA would own more than 768 fc1 rows");
        dec->grid = G;
        dec->n_fc = n_fc;
        dec->o_bias_shift = 43;
        dec->f2_bias_shift = 43 + ceil_log2(max_nkb);
        dec->vocab_tiles = (V + kTile - 1) / kTile;

        // quantise every linear (Lin::load rule)
        std::vector<QMat> q(L), k(L), v(L), o(L), f1(L), f2(L);
        std::vector<int> fix(4 * L);
        for (int l = 0; l < L; l++) {
            const XdnaOptLayer &ly = w->layers[l];
            q[l] = quant_linear(ly.wq, ly.bq, D, D);
            k[l] = quant_linear(ly.wk, ly.bk, D, D);
            v[l] = quant_linear(ly.wv, ly.bv, D, D);
            o[l] = quant_linear(ly.wo, ly.bo, D, D);
            f1[l] = quant_linear(ly.w1, ly.b1, D, F);
            f2[l] = quant_linear(ly.w2, ly.b2, F, D);
            fix[l] = fix_from_bound(rows_bound(v[l], 0, D, ly.ln1_w, ly.ln1_b, D));
            fix[L + l] = fix_from_bound(rows_bound(f1[l], 0, F, ly.ln2_w, ly.ln2_b, D));
            fix[2 * L + l] = fix_from_bound(ln_bound(ly.ln1_w, ly.ln1_b, D));
            fix[3 * L + l] = fix_from_bound(ln_bound(ly.ln2_w, ly.ln2_b, D));
        }
        QMat lm;
        lm.K = D;
        lm.N = V;
        lm.q.resize((size_t)V * D);
        lm.scale.resize(V);
        quant_rows(w->emb_tok, V, D, lm.q.data(), lm.scale.data());

        // per-CTA streams in consumption order
        std::vector<uint8_t> all;
        std::vector<std::vector<ChunkRef>> refs(G);
        std::vector<int> nl(G), nlm(G);
        for (int cta = 0; cta < G; cta++) {
            StreamBuilder sb;
            sb.base = all.size();
            for (int l = 0; l < L; l++) {
                if (cta < 2 * H) {
                    const int h = cta / 2, r = cta % 2;
                    const QMat *qkv[3] = {&q[l], &k[l], &v[l]};
                    for (int tile = 0; tile < 6; tile++) {
                        const QMat &m = *qkv[tile / 2];
                        const int n0 = h * kHeadDim + r * kHalfDim + (tile % 2) * kTile;
                        pack_row_tile(sb, D, [&](int rr) { return row_of(m, n0 + rr); });
                    }
                    pack_slice(sb, o[l], h * kHeadDim + r * kHalfDim);
                } else if (cta - 2 * H < n_fc) {
                    const int i = cta - 2 * H;
                    const int kb0 = fc_kb0(i, KB, n_fc), kb1 = fc_kb0(i + 1, KB, n_fc);
                    for (int tile = 2 * kb0; tile < 2 * kb1; tile++)
                        pack_row_tile(sb, D, [&](int rr) { return row_of(f1[l], tile * kTile + rr); });
                    for (int kb = kb0; kb < kb1; kb++) pack_slice(sb, f2[l], kb * 32);
                }
            }
            nl[cta] = (int)sb.refs.size();
            const int t0 = lm_tile0(cta, dec->vocab_tiles, G), t1 = lm_tile0(cta + 1, dec->vocab_tiles, G);
            if (t1 - t0 > kMaxVocabTilesPerCta) throw std::runtime_error("vocabulary too large for the grid");
            for (int t = t0; t < t1; t++) pack_row_tile(sb, D, [&](int rr) { return row_of(lm, t * kTile + rr); });
            nlm[cta] = (int)sb.refs.size() - nl[cta];
            refs[cta] = sb.refs;
            all.insert(all.end(), sb.bytes.begin(), sb.bytes.end());
        }
        dec->stream_bytes = all.size();
        dec->token_bytes = all.size();
        if (all.size() >= (1ull << 32)) throw std::runtime_error("weight stream exceeds 4 GiB");
        int stride = 0;
        for (int cta = 0; cta < G; cta++) stride = std::max(stride, (int)refs[cta].size());
        dec->chunk_stride = stride;
        std::vector<ChunkRef> flat((size_t)G * stride, ChunkRef{0, 0});
        for (int cta = 0; cta < G; cta++)
            std::copy(refs[cta].begin(), refs[cta].end(), flat.begin() + (size_t)cta * stride);

        dec->d_stream = dmalloc<uint8_t>(all.size());
        ck(cudaMemcpy(dec->d_stream, all.data(), all.size(), cudaMemcpyHostToDevice), "upload stream");
        dec->d_chunks = dmalloc<ChunkRef>(flat.size());
        ck(cudaMemcpy(dec->d_chunks, flat.data(), flat.size() * sizeof(ChunkRef), cudaMemcpyHostToDevice), "upload chunks");
        dec->d_nl = dmalloc<int>(G);
        dec->d_nlm = dmalloc<int>(G);
        ck(cudaMemcpy(dec->d_nl, nl.data(), G * sizeof(int), cudaMemcpyHostToDevice), "upload nl");
        ck(cudaMemcpy(dec->d_nlm, nlm.data(), G * sizeof(int), cudaMemcpyHostToDevice), "upload nlm");

        // f32 parameters that are not streamed
        dec->d_emb = dmalloc<float>((size_t)V * D);
        ck(cudaMemcpy(dec->d_emb, w->emb_tok, sizeof(float) * V * D, cudaMemcpyHostToDevice), "upload emb");
        dec->d_pos = dmalloc<float>((size_t)(c.max_pos + 2) * D);
        ck(cudaMemcpy(dec->d_pos, w->emb_pos, sizeof(float) * (size_t)(c.max_pos + 2) * D, cudaMemcpyHostToDevice),
           "upload pos");
        std::vector<float> ln((size_t)L * 4 * D), osb((size_t)L * 2 * D), f2sb((size_t)L * 2 * D);
        for (int l = 0; l < L; l++) {
            const XdnaOptLayer &ly = w->layers[l];
            std::copy(ly.ln1_w, ly.ln1_w + D, ln.begin() + (size_t)(l * 4 + 0) * D);
            std::copy(ly.ln1_b, ly.ln1_b + D, ln.begin() + (size_t)(l * 4 + 1) * D);
            std::copy(ly.ln2_w, ly.ln2_w + D, ln.begin() + (size_t)(l * 4 + 2) * D);
            std::copy(ly.ln2_b, ly.ln2_b + D, ln.begin() + (size_t)(l * 4 + 3) * D);
            std::copy(o[l].scale.begin(), o[l].scale.end(), osb.begin() + (size_t)(l * 2 + 0) * D);
            std::copy(o[l].bias.begin(), o[l].bias.end(), osb.begin() + (size_t)(l * 2 + 1) * D);
            std::copy(f2[l].scale.begin(), f2[l].scale.end(), f2sb.begin() + (size_t)(l * 2 + 0) * D);
            std::copy(f2[l].bias.begin(), f2[l].bias.end(), f2sb.begin() + (size_t)(l * 2 + 1) * D);
        }
        auto upload = [](const std::vector<float> &h, float **d, const char *what) {
            *d = dmalloc<float>(h.size());
            ck(cudaMemcpy(*d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice), what);
        };
        upload(ln, &dec->d_ln, "upload ln");
        upload(osb, &dec->d_osb, "upload out-proj scales");
        upload(f2sb, &dec->d_f2sb, "upload fc2 scales");
        std::vector<float> lnf(2 * D);
        std::copy(w->lnf_w, w->lnf_w + D, lnf.begin());
        std::copy(w->lnf_b, w->lnf_b + D, lnf.begin() + D);
        upload(lnf, &dec->d_lnf, "upload lnf");
        dec->fix_lnf = fix_from_bound(ln_bound(w->lnf_w, w->lnf_b, D));
        dec->d_fix = dmalloc<int>(4 * L);
        ck(cudaMemcpy(dec->d_fix, fix.data(), 4 * L * sizeof(int), cudaMemcpyHostToDevice), "upload exponents");
        dec->h_fix = fix;

        // batched prompt prefill (XDNA_OPT_PREFILL=0 steps the prompt through the decode kernel)
        {
            const char *pf = std::getenv("XDNA_OPT_PREFILL");
            dec->prefill = !(pf && pf[0] == '0');
        }
        if (dec->prefill) {
            dec->pf_w_layer = (size_t)3 * D * D + (size_t)D * D + 2 * (size_t)F * D;
            dec->pf_sb_layer = (size_t)2 * 3 * D + 2 * (size_t)F;
            std::vector<int8_t> wl(dec->pf_w_layer);
            std::vector<float> sbl(dec->pf_sb_layer);
            dec->d_pfw = dmalloc<int8_t>(dec->pf_w_layer * L);
            dec->d_pfsb = dmalloc<float>(dec->pf_sb_layer * L);
            for (int l = 0; l < L; l++) {
                int8_t *o8 = wl.data();
                const QMat *qkv3[3] = {&q[l], &k[l], &v[l]};
                for (const QMat *m : qkv3) { std::copy(m->q.begin(), m->q.end(), o8); o8 += m->q.size(); }
                std::copy(o[l].q.begin(), o[l].q.end(), o8); o8 += o[l].q.size();
                std::copy(f1[l].q.begin(), f1[l].q.end(), o8); o8 += f1[l].q.size();
                std::copy(f2[l].q.begin(), f2[l].q.end(), o8);
                float *sb = sbl.data();                // qkv scale [3D], qkv bias [3D], fc1 scale [F], bias [F]
                for (int i = 0; i < 3; i++)
                    for (int n = 0; n < D; n++) {
                        const RowRef r = row_of(*qkv3[i], n);
                        sb[i * D + n] = r.scale;
                        sb[3 * D + i * D + n] = r.bias;
                    }
                for (int n = 0; n < F; n++) {
                    const RowRef r = row_of(f1[l], n);
                    sb[6 * D + n] = r.scale;
                    sb[6 * D + F + n] = r.bias;
                }
                ck(cudaMemcpy(dec->d_pfw + dec->pf_w_layer * l, wl.data(), wl.size(), cudaMemcpyHostToDevice),
                   "upload prefill weights");
                ck(cudaMemcpy(dec->d_pfsb + dec->pf_sb_layer * l, sbl.data(), sbl.size() * 4, cudaMemcpyHostToDevice),
                   "upload prefill scales");
            }
            dec->d_pfx = dmalloc<float>((size_t)kPrefillTokens * D);
            dec->d_pfq = dmalloc<float>((size_t)kPrefillTokens * D);
            dec->d_pfa = dmalloc<int8_t>((size_t)kPrefillTokens * 4 * D);
            dec->d_pfh = dmalloc<int8_t>((size_t)kPrefillTokens * 4 * F);
            const int nmax = std::max(3 * D, F);
            dec->d_pfacc = dmalloc<unsigned long long>((size_t)kPrefillTokens * nmax);
            ck(cudaMemset(dec->d_pfacc, 0, (size_t)kPrefillTokens * nmax * 8), "clear prefill sums");
            dec->d_pfcnt = dmalloc<unsigned int>(nmax / kTile);
            ck(cudaMemset(dec->d_pfcnt, 0, (size_t)(nmax / kTile) * 4), "clear prefill counters");
        }

        // paged KV: pages in reverse physical order so the page table is exercised
        dec->n_pages = (max_ctx + kPageTokens - 1) / kPageTokens;
        std::vector<int> pt(dec->n_pages);
        for (int i = 0; i < dec->n_pages; i++) pt[i] = dec->n_pages - 1 - i;
        dec->d_pt = dmalloc<int>(pt.size());
        ck(cudaMemcpy(dec->d_pt, pt.data(), pt.size() * sizeof(int), cudaMemcpyHostToDevice), "upload page table");
        const size_t kv_elems = (size_t)L * dec->n_pages * H * 2 * 2 * kPageTokens * kHalfDim;
        dec->d_kv = dmalloc<uint16_t>(kv_elems);
        ck(cudaMemset(dec->d_kv, 0, kv_elems * 2), "clear kv");

        // exchange: accumulator words (zero) and the LM-head key words (epoch 0)
        dec->o_subs = std::min(kMaxSubs, env_int("XDNA_OPT_O_SUBS", 2));
        dec->f2_subs = std::min(kMaxSubs, env_int("XDNA_OPT_F2_SUBS", 8));
        dec->poll_ns = env_int("XDNA_OPT_POLL_NS", 20);
        dec->lm_prefetch_layer = std::max(0, L - 4);
        if (const char *e = std::getenv("XDNA_OPT_LM_PREFETCH_LAYER")) dec->lm_prefetch_layer = std::atoi(e);
        dec->acc_words = (size_t)kAccSlots * L * 2 * D * kMaxSubs;
        dec->d_acc = dmalloc<unsigned long long>(dec->acc_words);
        ck(cudaMemset(dec->d_acc, 0, dec->acc_words * 8), "clear accumulators");
        dec->d_ll = dmalloc<unsigned long long>(2 * kAccSlots);
        ck(cudaMemset(dec->d_ll, 0, 2 * kAccSlots * 8), "clear LM-head words");

        dec->d_tokens = dmalloc<int64_t>(max_ctx + 1);
        ck(cudaMemset(dec->d_tokens, 0, (max_ctx + 1) * sizeof(int64_t)), "clear tokens");
        dec->d_state = dmalloc<RunState>(1);
        RunState rs{0u, 0u, 0u, 0u};
        ck(cudaMemcpy(dec->d_state, &rs, sizeof(rs), cudaMemcpyHostToDevice), "init state");
        ck(cudaDeviceSynchronize(), "create sync");
        return dec;
    } catch (const std::exception &e) {
        set_err(std::string("xdna_opt_create: ") + e.what());
        delete dec;
        return nullptr;
    }
}

void xdna_opt_free(XdnaOptDecoder *dec) {
    if (!dec) return;
    cudaSetDevice(dec->dev->ordinal);
    cudaDeviceSynchronize();
    delete dec;
}

int64_t *xdna_opt_tokens_device(XdnaOptDecoder *dec) { return dec ? dec->d_tokens : nullptr; }

static int copy_tokens(XdnaOptDecoder *dec, void *host, size_t off, size_t n, void *stream, bool up) {
    if (!dec || (!host && n)) { set_err("xdna_opt_*_tokens: null pointer"); return -1; }
    if (off + n > (size_t)dec->max_ctx + 1) { set_err("xdna_opt_*_tokens: range beyond max_ctx + 1"); return -1; }
    cudaError_t e = cudaSetDevice(dec->dev->ordinal);
    if (e == cudaSuccess && n)
        e = up ? cudaMemcpyAsync(dec->d_tokens + off, host, n * 8, cudaMemcpyHostToDevice, (cudaStream_t)stream)
               : cudaMemcpyAsync(host, dec->d_tokens + off, n * 8, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e != cudaSuccess) { set_err(std::string("xdna_opt_*_tokens: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}
int xdna_opt_set_tokens(XdnaOptDecoder *dec, const int64_t *host, size_t off, size_t n, void *stream) {
    return copy_tokens(dec, const_cast<int64_t *>(host), off, n, stream, true);
}
int xdna_opt_get_tokens(XdnaOptDecoder *dec, int64_t *host, size_t off, size_t n, void *stream) {
    return copy_tokens(dec, host, off, n, stream, false);
}
int xdna_opt_grid(const XdnaOptDecoder *dec) { return dec ? dec->grid : 0; }
int xdna_opt_config(const XdnaOptDecoder *dec, XdnaOptConfig *out) {
    if (!dec || !out) { set_err("xdna_opt_config: null decoder or output"); return -1; }
    *out = dec->cfg;
    return 0;
}
int xdna_opt_set_timing(XdnaOptDecoder *dec, unsigned long long *timing_dev) {
    if (!dec) { set_err("xdna_opt_set_timing: decoder is null"); return -1; }
    dec->timing = timing_dev;
    return 0;
}
int xdna_opt_set_trace(XdnaOptDecoder *dec, float *trace_dev) {
    if (!dec) { set_err("xdna_opt_set_trace: decoder is null"); return -1; }
    dec->trace = trace_dev;
    return 0;
}
size_t xdna_opt_stream_bytes_per_token(const XdnaOptDecoder *dec) { return dec ? dec->token_bytes : 0; }

int xdna_opt_launch(XdnaOptDecoder *dec, int start_pos, int n_steps, int n_prompt, float *logits_dev,
                    void *stream) {
    if (!dec) { set_err("xdna_opt_launch: decoder is null"); return -1; }
    if (start_pos < 0 || n_steps < 1 || n_prompt < 1 || start_pos + n_steps > dec->max_ctx) {
        set_err("xdna_opt_launch: positions out of range (start_pos + n_steps must be <= max_ctx)");
        return -1;
    }
    const XdnaOptConfig &c = dec->cfg;
    DecodeParams p{};
    p.n_layers = c.n_layers;
    p.d_model = c.d_model;
    p.n_heads = c.n_heads;
    p.ffn = c.ffn;
    p.vocab = c.vocab;
    p.max_pos = c.max_pos;
    p.eps = c.eps;
    p.grid = dec->grid;
    p.n_fc = dec->n_fc;
    p.vocab_tiles = dec->vocab_tiles;
    p.stream = dec->d_stream;
    p.chunks = dec->d_chunks;
    p.n_layer_chunks = dec->d_nl;
    p.n_lm_chunks = dec->d_nlm;
    p.chunk_stride = dec->chunk_stride;
    p.emb_tok = dec->d_emb;
    p.emb_pos = dec->d_pos;
    p.ln = dec->d_ln;
    p.lnf = dec->d_lnf;
    p.osb = dec->d_osb;
    p.f2sb = dec->d_f2sb;
    p.fix_ctx = dec->d_fix;
    p.fix_h = dec->d_fix + c.n_layers;
    p.fix_ln1 = dec->d_fix + 2 * c.n_layers;
    p.fix_ln2 = dec->d_fix + 3 * c.n_layers;
    p.fix_lnf = dec->fix_lnf;
    p.o_bias_shift = dec->o_bias_shift;
    p.f2_bias_shift = dec->f2_bias_shift;
    p.kv = dec->d_kv;
    p.page_table = dec->d_pt;
    p.n_phys_pages = dec->n_pages;
    p.acc = dec->d_acc;
    p.o_subs = dec->o_subs;
    p.f2_subs = dec->f2_subs;
    p.poll_ns = dec->poll_ns;
    p.lm_words = dec->d_ll;
    p.lm_prefetch_layer = dec->lm_prefetch_layer;
    p.tokens = dec->d_tokens;
    p.logits = logits_dev;
    p.start_pos = start_pos;
    p.n_steps = n_steps;
    p.n_prompt = n_prompt;
    p.state = dec->d_state;
    p.timeout_ns = 1000000000ull;   // 1 s per wait; normal waits are microseconds
    p.trace = dec->trace;
    p.timing = dec->timing;
    cudaError_t e = cudaSetDevice(dec->dev->ordinal);
    if (e == cudaSuccess) e = launch_opt_decode(p, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        set_err(std::string("xdna_opt_launch: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// K slices (CTAs) per 16-row tile: about 256 CTAs per GEMV, a slice at most 32 k-blocks (4 per
// warp) and, where the shape allows, at least 16 (two per warp)
static PrefillGemv with_split(PrefillGemv g) {
    const int tiles = g.N / kTile, nkb = g.K / 32;
    const int lo = (nkb + 31) / 32;
    g.nsplit = std::max(lo, std::min(std::max(1, nkb / 16), 256 / tiles));
    return g;
}

int xdna_opt_prefill(XdnaOptDecoder *dec, int start_pos, int n, void *stream) {
    if (!dec) { set_err("xdna_opt_prefill: decoder is null"); return -1; }
    if (!dec->prefill) { set_err("xdna_opt_prefill: the decoder was created with XDNA_OPT_PREFILL=0"); return -1; }
    if (start_pos < 0 || n < 0 || start_pos + n > dec->max_ctx) {
        set_err("xdna_opt_prefill: positions out of range (start_pos + n must be <= max_ctx)");
        return -1;
    }
    const XdnaOptConfig &c = dec->cfg;
    const int D = c.d_model, F = c.ffn, L = c.n_layers, H = c.n_heads;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSetDevice(dec->dev->ordinal);
    for (int p0 = start_pos; e == cudaSuccess && p0 < start_pos + n; p0 += kPrefillTokens) {
        const int T = std::min(kPrefillTokens, start_pos + n - p0);
        e = launch_prefill_embed(dec->d_tokens, p0, T, D, c.vocab, dec->d_emb, dec->d_pos, dec->d_pfx, dec->d_state, st);
        for (int l = 0; l < L && e == cudaSuccess; l++) {
            const int8_t *wl = dec->d_pfw + dec->pf_w_layer * l;
            const float *sb = dec->d_pfsb + dec->pf_sb_layer * l;
            const float *ln = dec->d_ln + (size_t)l * 4 * D;
            PrefillGemv g{};
            g.acc = dec->d_pfacc;
            g.cnt = dec->d_pfcnt;
            g.T = T;
            g.x = dec->d_pfx;
            g.q = dec->d_pfq;
            g.kv = dec->d_kv;
            g.pt = dec->d_pt;
            g.layer = l;
            g.n_phys = dec->n_pages;
            g.n_heads = H;
            g.pos0 = p0;
            g.D = D;
            // LN1 -> q | k | v (K / V rows into the cache)
            e = launch_prefill_ln(dec->d_pfx, T, D, ln, ln + D, c.eps, dec->h_fix[2 * L + l], dec->d_pfa, st);
            g.w = wl; g.sc = sb; g.bi = sb + 3 * D; g.limbs = dec->d_pfa;
            g.K = D; g.N = 3 * D; g.fix = dec->h_fix[2 * L + l]; g.mode = PF_QKV;
            if (e == cudaSuccess) e = launch_prefill_gemv(with_split(g), st);
            // attention -> context limbs -> x += out projection
            if (e == cudaSuccess)
                e = launch_prefill_attn(dec->d_pfq, dec->d_kv, dec->d_pt, l, dec->n_pages, H, p0, T, D, dec->h_fix[l],
                                        dec->d_pfa, st);
            g.w = wl + (size_t)3 * D * D; g.sc = dec->d_osb + (size_t)l * 2 * D; g.bi = g.sc + D;
            g.K = D; g.N = D; g.fix = dec->h_fix[l]; g.mode = PF_RESID;
            if (e == cudaSuccess) e = launch_prefill_gemv(with_split(g), st);
            // LN2 -> fc1 + ReLU -> x += fc2
            if (e == cudaSuccess)
                e = launch_prefill_ln(dec->d_pfx, T, D, ln + 2 * D, ln + 3 * D, c.eps, dec->h_fix[3 * L + l],
                                      dec->d_pfa, st);
            g.w = wl + (size_t)4 * D * D; g.sc = sb + 6 * D; g.bi = sb + 6 * D + F; g.limbs = dec->d_pfa;
            g.K = D; g.N = F; g.fix = dec->h_fix[3 * L + l]; g.mode = PF_FC1;
            g.limbs_out = dec->d_pfh; g.fix_out = dec->h_fix[L + l];
            if (e == cudaSuccess) e = launch_prefill_gemv(with_split(g), st);
            g.w = wl + (size_t)4 * D * D + (size_t)F * D; g.sc = dec->d_f2sb + (size_t)l * 2 * D; g.bi = g.sc + D;
            g.limbs = dec->d_pfh; g.K = F; g.N = D; g.fix = dec->h_fix[L + l]; g.mode = PF_RESID;
            if (e == cudaSuccess) e = launch_prefill_gemv(with_split(g), st);
        }
    }
    if (e != cudaSuccess) {
        set_err(std::string("xdna_opt_prefill: ") + cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int xdna_opt_sync(XdnaOptDecoder *dec, void *stream) {
    if (!dec) { set_err("xdna_opt_sync: decoder is null"); return -1; }
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        set_err(std::string("xdna_opt_sync: ") + cudaGetErrorString(e));
        return -1;
    }
    RunState rs{};
    e = cudaMemcpy(&rs, dec->d_state, sizeof(rs), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        set_err(std::string("xdna_opt_sync: ") + cudaGetErrorString(e));
        return -1;
    }
    if (rs.error != ERR_NONE) {
        static const char *names[] = {"none", "timeout waiting for a weight chunk",
                                      "timeout waiting for a free ring slot",
                                      "timeout waiting for an exchange word", "token id out of range",
                                      "position out of range", "timeout waiting for the pair CTA"};
        char buf[256];
        std::snprintf(buf, sizeof buf, "decode kernel error: %s (cta %u, where 0x%x)",
                      rs.error < 7 ? names[rs.error] : "unknown", rs.error_cta, rs.error_where);
        set_err(buf);
        // the failed launch may have left partial sums and key words behind: clear the
        // accumulators and skip the LM-key epochs far past the failed ones
        rs.tok_base += 1u << 20;
        rs.error = rs.error_cta = rs.error_where = 0;
        cudaMemset(dec->d_acc, 0, dec->acc_words * 8);
        cudaMemset(dec->d_ll, 0, 2 * kAccSlots * 8);
        cudaMemcpy(dec->d_state, &rs, sizeof(rs), cudaMemcpyHostToDevice);
        return -1;
    }
    return 0;
}

int xdna_opt_generate(XdnaOptDecoder *dec, const int64_t *prompt, size_t n_prompt, size_t n_new,
                      int64_t *out_ids, float *out_logits) {
    if (!dec || !prompt || !out_ids) { set_err("xdna_opt_generate: null pointer"); return -1; }
    if (n_prompt < 1 || n_new < 1 || n_prompt + n_new > (size_t)dec->max_ctx + 1) {
        set_err("xdna_opt_generate: n_prompt + n_new - 1 must be <= max_ctx");
        return -1;
    }
    const int V = dec->cfg.vocab;
    try {
        ck(cudaSetDevice(dec->dev->ordinal), "cudaSetDevice");
        for (size_t i = 0; i < n_prompt; i++)
            if (prompt[i] < 0 || prompt[i] >= V) throw std::runtime_error("prompt token id out of range");
        if (out_logits && dec->logits_cap < n_new) {
            if (dec->d_logits) cudaFree(dec->d_logits);
            dec->d_logits = dmalloc<float>(n_new * (size_t)V);
            dec->logits_cap = n_new;
        }
        cudaStream_t st = nullptr;
        ck(cudaMemcpyAsync(dec->d_tokens, prompt, n_prompt * sizeof(int64_t), cudaMemcpyHostToDevice, st),
           "copy prompt");
        // the prompt's positions before the last one as a batch (their K / V rows only), then the
        // decode kernel from the last prompt position; without the batched path every position
        // is a decode step
        const int start = dec->prefill ? (int)n_prompt - 1 : 0;
        if (start > 0 && xdna_opt_prefill(dec, 0, start, st) != 0) return -1;
        const int n_steps = (int)(n_prompt + n_new - 1) - start;
        if (xdna_opt_launch(dec, start, n_steps, (int)n_prompt, out_logits ? dec->d_logits : nullptr, st) != 0)
            return -1;
        ck(cudaMemcpyAsync(out_ids, dec->d_tokens + n_prompt, n_new * sizeof(int64_t), cudaMemcpyDeviceToHost, st),
           "copy ids");
        if (out_logits)
            ck(cudaMemcpyAsync(out_logits, dec->d_logits, n_new * (size_t)V * sizeof(float),
                               cudaMemcpyDeviceToHost, st),
               "copy logits");
        return xdna_opt_sync(dec, st);
    } catch (const std::exception &e) {
        set_err(std::string("xdna_opt_generate: ") + e.what());
        return -1;
    }
}

}  // extern "C"
