/*
 * numerics.c -- scalar/vector primitives of the oracle (TEST INFRASTRUCTURE ONLY; see
 * oracle.h).  Built with -ffp-contract=off so that every f32 multiply and add rounds
 * separately, as the reference's Rust code does.
 */
#include "oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* rust/npu-xrt/src/lib.rs:809-818 (f32_to_bf16_bits): NaN stays a quiet NaN, everything
 * else rounds to nearest even by adding 0x7fff + lsb and truncating. */
uint16_t or_f32_to_bf16_bits(float x) {
    uint32_t bits = f2u(x);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + bias) >> 16);
}
float or_bf16_bits_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* rust/npu-asr-host/src/lib.rs:12-19 (bf16_round) -- same bits as the pack above. */
float or_bf16_round(float x) {
    uint32_t bits = f2u(x);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return u2f(((bits >> 16) | 0x0040u) << 16);
    uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
    return u2f((bits + bias) & 0xffff0000u);
}
void or_bf16_round_n(const float *x, float *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = or_bf16_round(x[i]);
}
void or_f32_to_bf16_n(const float *x, uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = or_f32_to_bf16_bits(x[i]);
}

/* rust/npu-whisper/src/bin/opt125m_decode.rs:41-60 (Lin::load, OPT_INT8):
 * scale[c] = amax_k |W[k,c]| / 127 (1.0 if the column is all zero);
 * q = clamp(round(W / scale), -127, 127) with f32::round = half away from zero. */
void or_quant_i8_cols(const float *w, int K, int N, int8_t *q, float *scale) {
    for (int c = 0; c < N; c++) {
        float amax = 0.0f;
        for (int r = 0; r < K; r++) amax = fmaxf(amax, fabsf(w[(size_t)r * N + c]));
        scale[c] = amax > 0.0f ? amax / 127.0f : 1.0f;
    }
    for (int r = 0; r < K; r++)
        for (int c = 0; c < N; c++) {
            float v = roundf(w[(size_t)r * N + c] / scale[c]);
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            q[(size_t)r * N + c] = (int8_t)v;
        }
}

/* route_b_kernels/decode_fused/gen_decode.py:158-165 (qrow): per-row scale
 * max_k|W[m,k]|/127 (1.0 if zero), np.round = round half to even, clip +-127. */
void or_quant_i8_rows(const float *w, int M, int K, int8_t *q, float *scale) {
    for (int m = 0; m < M; m++) {
        const float *row = w + (size_t)m * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) amax = fmaxf(amax, fabsf(row[k]));
        float s = amax / 127.0f;
        s = s > 0.0f ? s : 1.0f;
        scale[m] = s;
        for (int k = 0; k < K; k++) {
            float v = rintf(row[k] / s);          /* default rounding mode: half to even */
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            q[(size_t)m * K + k] = (int8_t)v;
        }
    }
}

/* rust/npu-whisper/src/bin/opt125m_decode.rs:106-124 (Lin::fwd, int8 branch):
 * y[n] += a * w_i8[k,n] over k in order (f32 multiply, then f32 add), then
 * y = y * scale[n] + b[n]. */
void or_lin_i8_fwd(const float *x, const int8_t *q, const float *scale, const float *bias,
                   int K, int N, float *y) {
    for (int n = 0; n < N; n++) y[n] = 0.0f;
    for (int k = 0; k < K; k++) {
        float a = x[k];
        const int8_t *wr = q + (size_t)k * N;
        for (int n = 0; n < N; n++) { float p = a * (float)wr[n]; y[n] = y[n] + p; }
    }
    for (int n = 0; n < N; n++) { float t = y[n] * scale[n]; y[n] = t + (bias ? bias[n] : 0.0f); }
}

/* route_b_kernels/ffn_bfp16/golden_ffn_gemm.py:34-49 (to_bfp16_blocks): blocks of 8
 * share e = floor(log2(max|x|)) (max 0 -> 1.0, so e = 0); quantum 2^(e-6); values are
 * rounded half-to-even onto the grid (np.round) with no clamp. */
void or_bfp16_blocks(const float *x, float *y, size_t n) {
    for (size_t b0 = 0; b0 < n; b0 += 8) {
        float m = 0.0f;
        for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(x[b0 + i]));
        if (m == 0.0f) m = 1.0f;
        int e; (void)frexpf(m, &e); e -= 1;          /* floor(log2(m)) for normal m */
        float q = ldexpf(1.0f, e - 6);
        for (int i = 0; i < 8; i++) y[b0 + i] = rintf(x[b0 + i] / q) * q;
    }
}
void or_bfp16_pack(const float *x, size_t n, int16_t *mant, int8_t *exp) {
    for (size_t b0 = 0; b0 < n; b0 += 8) {
        float m = 0.0f;
        for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(x[b0 + i]));
        if (m == 0.0f) m = 1.0f;
        int e; (void)frexpf(m, &e); e -= 1;
        exp[b0 / 8] = (int8_t)e;
        float q = ldexpf(1.0f, e - 6);
        for (int i = 0; i < 8; i++) mant[b0 + i] = (int16_t)rintf(x[b0 + i] / q);
    }
}

/* rust/npu-asr-host/src/lib.rs:79-110 (layer_norm): f32 sums in index order,
 * population variance, y = (x - mean) * inv * g + b. */
void or_layer_norm(const float *x, const float *g, const float *b, int T, int D, float eps,
                   float *y) {
    for (int t = 0; t < T; t++) {
        const float *r = x + (size_t)t * D;
        float *o = y + (size_t)t * D;
        float sum = 0.0f;
        for (int j = 0; j < D; j++) sum += r[j];
        float mean = sum / (float)D;
        float vs = 0.0f;
        for (int j = 0; j < D; j++) { float c = r[j] - mean; vs += c * c; }
        float inv = 1.0f / sqrtf(vs / (float)D + eps);
        for (int j = 0; j < D; j++) {
            float t0 = (r[j] - mean) * inv;
            float t1 = t0 * (g ? g[j] : 1.0f);
            o[j] = t1 + (b ? b[j] : 0.0f);
        }
    }
}

/* rust/npu-asr/src/ctx_decode.rs:617-640 (fused_norm_gemv input normalisation, f64). */
void or_ln_normalize_f64(const float *x, int K, float eps, float *y) {
    double mean = 0.0, var = 0.0;
    for (int i = 0; i < K; i++) mean += (double)x[i];
    mean /= (double)K;
    for (int i = 0; i < K; i++) { double c = (double)x[i] - mean; var += c * c; }
    var /= (double)K;
    double inv = 1.0 / sqrt(var + (double)eps);
    for (int i = 0; i < K; i++) y[i] = (float)(((double)x[i] - mean) * inv);
}
void or_rms_normalize_f64(const float *x, int K, float eps, float *y) {
    double ms = 0.0;
    for (int i = 0; i < K; i++) ms += (double)x[i] * (double)x[i];
    ms /= (double)K;
    double inv = 1.0 / sqrt(ms + (double)eps);
    for (int i = 0; i < K; i++) y[i] = (float)((double)x[i] * inv);
}

/* rust/npu-gemma/src/lib.rs:55-64 (rmsnorm_ref). */
void or_gemma_rmsnorm(const float *x, const float *w, int D, float eps, float *y) {
    float ms = 0.0f;
    for (int i = 0; i < D; i++) ms += x[i] * x[i];
    ms = ms / (float)D;
    float inv = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < D; i++) y[i] = x[i] * inv * (1.0f + w[i]);
}

/* rust/npu-asr-host/src/lib.rs:38-58 (fast_exp_nonpos): the reference's own
 * 2^floor * degree-5 polynomial for x <= 0. */
float or_fast_exp_nonpos(float x) {
    if (x < -87.0f) x = -87.0f;
    const float LOG2E = 1.442695040888963f;
    float yv = x * LOG2E;
    float yf = floorf(yv);
    float f = yv - yf;
    float p = 1.0f + f * (0.6931471805599453f
              + f * (0.2402265069591007f
              + f * (0.05550410866482158f
              + f * (0.009618129107628477f + f * 0.0013333558146428443f))));
    uint32_t e = (uint32_t)((int32_t)yf + 127);
    return p * u2f(e << 23);
}

/* rust/npu-asr-host/src/lib.rs:401-410 (sigmoid_scalar). */
float or_sigmoid(float g) {
    if (g >= 0.0f) return 1.0f / (1.0f + or_fast_exp_nonpos(-g));
    float e = or_fast_exp_nonpos(g);
    return e / (1.0f + e);
}
float or_silu(float v) { return v * or_sigmoid(v); }

/* rust/npu-asr-host/src/lib.rs:464-476: Abramowitz & Stegun 7.1.26 erf. */
static float erf_as(float x) {
    float sign = x < 0.0f ? -1.0f : 1.0f;
    x = fabsf(x);
    float t = 1.0f / (1.0f + 0.3275911f * x);
    float y = 1.0f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t
                       - 0.284496736f) * t + 0.254829592f) * t * expf(-x * x);
    return sign * y;
}
/* rust/npu-asr-host/src/lib.rs:477-495 (gelu, exact-erf form). */
float or_gelu_erf(float v) {
    const float INV_SQRT2 = 0.70710678118654752440f;
    return 0.5f * v * (1.0f + erf_as(v * INV_SQRT2));
}
/* rust/npu-gemma/src/lib.rs:74-77 (gelu_pytorch_tanh). */
float or_gelu_tanh(float x) {
    const float C = 0.79788456f;
    return 0.5f * x * (1.0f + tanhf(C * (x + 0.044715f * x * x * x)));
}

/* rust/npu-asr-host/src/lib.rs:189-326 (mha): per head, scores = q k^T, max over the
 * valid keys, e = fast_exp(s*scale - max*scale), sum with 8 lane accumulators, probs =
 * e * (1/sum) (optionally bf16-rounded), padded keys 0, ctx = probs v. */
void or_mha(const float *q, const float *k, const float *v, int T, int H, int hd,
            int round_probs, int valid_len, float *out) {
    int D = H * hd;
    int vl = valid_len < T ? valid_len : T;
    float scale = 1.0f / sqrtf((float)hd);
    float *sc = (float *)malloc(sizeof(float) * (size_t)T);
    for (int h = 0; h < H; h++) {
        int base = h * hd;
        for (int i = 0; i < T; i++) {
            for (int j = 0; j < T; j++) {
                float s = 0.0f;
                for (int d = 0; d < hd; d++) s += q[(size_t)i * D + base + d] * k[(size_t)j * D + base + d];
                sc[j] = s;
            }
            float maxv = -INFINITY;
            for (int j = 0; j < vl; j++) maxv = fmaxf(maxv, sc[j]);
            float off = maxv * scale;
            for (int j = 0; j < vl; j++) sc[j] = or_fast_exp_nonpos(sc[j] * scale - off);
            float acc[8] = {0};
            int nfull = vl / 8 * 8;
            for (int j = 0; j < nfull; j += 8)
                for (int l = 0; l < 8; l++) acc[l] += sc[j + l];
            for (int j = nfull; j < vl; j++) acc[j - nfull] += sc[j];
            float sum = 0.0f;
            for (int l = 0; l < 8; l++) sum += acc[l];
            for (int j = vl; j < T; j++) sc[j] = 0.0f;
            float inv = 1.0f / sum;
            for (int j = 0; j < vl; j++) {
                float p = sc[j] * inv;
                sc[j] = round_probs ? or_bf16_round(p) : p;
            }
            for (int d = 0; d < hd; d++) {
                float s = 0.0f;
                for (int j = 0; j < T; j++) s += sc[j] * v[(size_t)j * D + base + d];
                out[(size_t)i * D + base + d] = s;
            }
        }
    }
    free(sc);
}

/* route_b_kernels/mha_decode/mha_decode.cc:90-168 (mha_tile): per key, score = q.k *
 * scale; m_new = max(m, score); corr = exp(m - m_new); p = exp(score - m_new);
 * l = l*corr + p; acc = acc*corr + p*v; ctx = acc / l.  (exp in f32.) */
void or_mha_tile_online(const float *q, const float *k, const float *v, int s, int hd,
                        float scale, float *ctx) {
    float m = -3.0e38f, l = 0.0f;
    float *acc = (float *)calloc((size_t)hd, sizeof(float));
    for (int j = 0; j < s; j++) {
        float sc = 0.0f;
        for (int d = 0; d < hd; d++) sc += q[d] * k[(size_t)j * hd + d];
        sc *= scale;
        float mn = sc > m ? sc : m;
        float corr = expf(m - mn);
        float p = expf(sc - mn);
        l = l * corr + p;
        m = mn;
        for (int d = 0; d < hd; d++) acc[d] = acc[d] * corr + p * v[(size_t)j * hd + d];
    }
    float inv = 1.0f / l;
    for (int d = 0; d < hd; d++) ctx[d] = acc[d] * inv;
    free(acc);
}

/* rust/npu-whisper/src/bin/opt125m_decode.rs:303: Iterator::max_by(partial_cmp) returns
 * the LAST of several equal maxima. */
int64_t or_argmax_last(const float *x, size_t n) {
    size_t bi = 0;
    for (size_t i = 1; i < n; i++) if (x[i] >= x[bi]) bi = i;
    return (int64_t)bi;
}
/* rust/npu-engine/src/asr/whisper.rs:749-757 and argmax_slice.cc:14-29: strict '>' so
 * the FIRST maximum wins. */
int64_t or_argmax_first(const float *x, size_t n) {
    float best = -3.0e38f; size_t bi = 0;
    for (size_t i = 0; i < n; i++) if (x[i] > best) { best = x[i]; bi = i; }
    return (int64_t)bi;
}

/* rust/npu-xrt/src/lib.rs:992-1004 (FusedElfPatcher::patch): KV site <- base +
 * n_preceding*head_dim*2 (bf16 bytes), softmax length <- n_preceding + 1. */
uint32_t or_kv_byte_offset(uint32_t base, uint32_t n_preceding, uint32_t head_dim) {
    return base + n_preceding * head_dim * 2u;
}
uint32_t or_softmax_len(uint32_t n_preceding) { return n_preceding + 1u; }

/* The engine's paged cache: page table entry p covers positions [p*pt, (p+1)*pt); a
 * physical page holds [K|V][H][pt][hd] bf16.  Element index of (kv, head, pos, d). */
size_t or_paged_kv_index(const int32_t *page_table, int pt, int H, int hd, int kv, int head,
                         int pos, int d) {
    size_t page = (size_t)page_table[pos / pt];
    size_t page_elems = (size_t)2 * H * pt * hd;
    return page * page_elems + (((size_t)kv * H + head) * pt + (size_t)(pos % pt)) * hd + d;
}

/* Fixed-point activation limbs (the engine's GEMV numerics, see oracle.h). */
int or_limbs(const float *x, int K, int8_t *a, int8_t *b, int8_t *c) {
    float mx = 0.0f;
    for (int i = 0; i < K; i++) mx = fmaxf(mx, fabsf(x[i]));
    int E = 0;
    if (mx > 0.0f) (void)frexpf(mx, &E);
    int s = 22 - E;
    for (int i = 0; i < K; i++) {
        int32_t X = (int32_t)rintf(ldexpf(x[i], s));
        int32_t cc = ((X + 128) & 255) - 128;
        int32_t X1 = (X - cc) >> 8;
        int32_t bb = ((X1 + 128) & 255) - 128;
        int32_t aa = (X1 - bb) >> 8;
        a[i] = (int8_t)aa; b[i] = (int8_t)bb; c[i] = (int8_t)cc;
    }
    return s;
}

void or_gemv_i8_exact(const float *x, const int8_t *wq_nk, const float *scale,
                      const float *bias, int K, int N, float *y) {
    int8_t *a = (int8_t *)malloc((size_t)K * 3);
    int8_t *b = a + K, *c = b + K;
    int s = or_limbs(x, K, a, b, c);
    for (int n = 0; n < N; n++) {
        const int8_t *w = wq_nk + (size_t)n * K;
        int64_t A = 0, B = 0, C = 0;
        for (int k = 0; k < K; k++) { A += a[k] * w[k]; B += b[k] * w[k]; C += c[k] * w[k]; }
        int64_t S = A * 65536 + B * 256 + C;
        float t = ldexpf((float)S, -s);
        t = t * scale[n];
        y[n] = t + (bias ? bias[n] : 0.0f);
    }
    free(a);
}
