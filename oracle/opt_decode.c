/*
 * opt_decode.c -- oracle for the opt-125m greedy decode (TEST INFRASTRUCTURE ONLY; see
 * oracle.h).  Restates rust/npu-whisper/src/bin/opt125m_decode.rs:
 *   Lin::load (41-60) / Lin::fwd (106-124), Opt::step (252-293), Opt::generate (296-315).
 *
 * Two numerics modes:
 *  OR_MODE_REF_F32  the reference host path run with OPT_INT8: f32 activations, the six
 *                   Lin layers int8 (per-output-column scale), f32 LM head, f32 KV.
 *  OR_MODE_DEVICE   the B200 engine's numerics: LN outputs / attention context / FFN hidden
 *                   rounded to bf16 before each GEMV, K and V stored as bf16, q scaled then
 *                   rounded to bf16, every int8 GEMV computed as the exact integer dot of the
 *                   activation in 29-bit fixed point (exponent from the vector's max for the
 *                   LayerNorm outputs; a weight-derived bound per layer for the attention
 *                   context and the fc1 output, whose GEMVs the engine splits over K), rounded
 *                   once to f32, int8 LM head (same quantiser, per vocab row), residual stream
 *                   f32.  LayerNorm sums and the softmax follow the engine's reduction trees
 *                   and use the reference's fast_exp_nonpos, so this mode is bit-exact with
 *                   the GPU (ln_dev_bf16, attn_dev_head, gemv_fix).
 *
 * The GEMVs are parallelised over output columns with OpenMP; each output keeps the
 * reference's k-ascending summation order, so results do not depend on the thread count.
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
    const float *w;  /* F32 mode: the unquantised [K,N] weight */
    int8_t *q;       /* REF: [K,N] (reference layout); DEVICE: [N,K] (output-major) */
    float *scale;    /* [N] */
    const float *bias;
    int K, N;
} lin_t;

struct or_opt {
    or_opt_cfg cfg;
    or_opt_weights w;
    int mode, nthreads;
    lin_t *lins;           /* [L][6]: q k v o fc1 fc2 */
    int8_t *lm_q;          /* DEVICE: [V,D] */
    float *lm_scale;       /* DEVICE: [V] */
    float *kc, *vc;        /* [L][max_ctx][D] (DEVICE: values already bf16-rounded) */
    int max_ctx;
    float *trace;          /* optional [pos][2L+1][D] residual-stream record */
    int *fix_ctx, *fix_h;  /* DEVICE: [L] fixed-point exponents of the K-split GEMV inputs */
};

void or_opt_set_trace(or_opt *m, float *trace) { m->trace = trace; }
static void trace_x(or_opt *m, int pos, int slot, const float *v) {
    if (!m->trace) return;
    int D = m->cfg.d_model;
    memcpy(m->trace + ((size_t)pos * (2 * m->cfg.n_layers + 1) + slot) * D, v, sizeof(float) * D);
}

static int fix_of_bound(const lin_t *l, int n0, int n1, const float *g, const float *b, int D);

static void lin_init(lin_t *l, const float *w, const float *b, int K, int N, int mode) {
    l->K = K; l->N = N; l->bias = b; l->w = w;
    if (mode == OR_MODE_F32) return;
    l->q = (int8_t *)malloc((size_t)K * N);
    l->scale = (float *)malloc(sizeof(float) * (size_t)N);
    or_quant_i8_cols(w, K, N, l->q, l->scale);
    if (mode == OR_MODE_DEVICE) {       /* transpose to [N,K] for the exact dot */
        int8_t *t = (int8_t *)malloc((size_t)K * N);
        for (int k = 0; k < K; k++)
            for (int n = 0; n < N; n++) t[(size_t)n * K + k] = l->q[(size_t)k * N + n];
        free(l->q);
        l->q = t;
    }
}

or_opt *or_opt_create(const or_opt_cfg *cfg, const or_opt_weights *w, int mode, int nthreads) {
    or_opt *m = (or_opt *)calloc(1, sizeof(or_opt));
    m->cfg = *cfg; m->w = *w; m->mode = mode; m->nthreads = nthreads > 0 ? nthreads : 1;
    int L = cfg->n_layers, D = cfg->d_model, F = cfg->ffn;
    m->lins = (lin_t *)calloc((size_t)L * 6, sizeof(lin_t));
    for (int l = 0; l < L; l++) {
        const or_opt_layer *ly = &w->layers[l];
        lin_t *p = m->lins + l * 6;
        lin_init(p + 0, ly->wq, ly->bq, D, D, mode);
        lin_init(p + 1, ly->wk, ly->bk, D, D, mode);
        lin_init(p + 2, ly->wv, ly->bv, D, D, mode);
        lin_init(p + 3, ly->wo, ly->bo, D, D, mode);
        lin_init(p + 4, ly->w1, ly->b1, D, F, mode);
        lin_init(p + 5, ly->w2, ly->b2, F, D, mode);
    }
    if (mode == OR_MODE_DEVICE) {
        /* The tied LM head as an int8 linear [D -> V]: output channel v is embedding row v,
         * quantised with the Lin::load rule (per output channel, half away from zero). */
        int V = cfg->vocab;
        m->lm_q = (int8_t *)malloc((size_t)V * D);
        m->lm_scale = (float *)malloc(sizeof(float) * (size_t)V);
        for (int v = 0; v < V; v++) {
            const float *row = w->emb_tok + (size_t)v * D;
            float amax = 0.0f;
            for (int d = 0; d < D; d++) amax = fmaxf(amax, fabsf(row[d]));
            float s = amax > 0.0f ? amax / 127.0f : 1.0f;
            m->lm_scale[v] = s;
            for (int d = 0; d < D; d++) {
                float q = roundf(row[d] / s);
                q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
                m->lm_q[(size_t)v * D + d] = (int8_t)q;
            }
        }
    }
    if (mode == OR_MODE_DEVICE) {
        m->fix_ctx = (int *)malloc(sizeof(int) * (size_t)L);
        m->fix_h = (int *)malloc(sizeof(int) * (size_t)L);
        for (int l = 0; l < L; l++) {
            const or_opt_layer *ly = &w->layers[l];
            m->fix_ctx[l] = fix_of_bound(&m->lins[l * 6 + 2], 0, D, ly->ln1_w, ly->ln1_b, D);
            m->fix_h[l] = fix_of_bound(&m->lins[l * 6 + 4], 0, F, ly->ln2_w, ly->ln2_b, D);
        }
    }
    m->max_ctx = cfg->max_pos;
    m->kc = (float *)malloc(sizeof(float) * (size_t)L * m->max_ctx * D);
    m->vc = (float *)malloc(sizeof(float) * (size_t)L * m->max_ctx * D);
    return m;
}

void or_opt_free(or_opt *m) {
    if (!m) return;
    for (int i = 0; i < m->cfg.n_layers * 6; i++) { free(m->lins[i].q); free(m->lins[i].scale); }
    free(m->lins); free(m->lm_q); free(m->lm_scale); free(m->kc); free(m->vc);
    free(m->fix_ctx); free(m->fix_h); free(m);
}

const int8_t *or_opt_qweight(const or_opt *m, int layer, int which, float const **scale) {
    if (which == 6) { if (scale) *scale = m->lm_scale; return m->lm_q; }
    const lin_t *l = &m->lins[layer * 6 + which];
    if (scale) *scale = l->scale;
    return l->q;
}

/* ---- the engine's reduction trees (device numerics) --------------------------------
 * A GPU warp reduces 32 lane partials with an xor butterfly (v = v + v[lane ^ o] for o = 16,
 * 8, 4, 2, 1).  Float addition is commutative, so the butterfly yields one well-defined
 * value, replayed here. */
static float warp_tree(const float *v32) {
    float v[32], t[32];
    memcpy(v, v32, sizeof v);
    for (int o = 16; o; o >>= 1) {
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ o];
        memcpy(v, t, sizeof v);
    }
    return v[0];
}
/* LayerNorm as the engine's 8 consumer warps compute it: warp w owns the 32-wide blocks
 * [w*nkb/8, (w+1)*nkb/8) (nkb = D/32: the engine's split for D = 256 and 768, and a defined
 * tree for the narrower models the HuggingFace goldens use); lane l adds its elements
 * 32*kb + l in kb order (sum and sum of squares in the same pass), each warp adds its lanes
 * with the butterfly, and the 8 warp totals are added in warp order; mean = S1 / D,
 * var = max(S2 / D - mean^2, 0), y = bf16((x - mean) * (1 / sqrt(var + eps)) * g + b)
 * (rust/npu-asr-host/src/lib.rs:79-110 in single-pass form). */
static float lane_tree(const float *x, int D, int squares) {
    int nkb = D / 32;
    float tot = 0.0f;
    for (int w = 0; w < 8; w++) {
        float part[32];
        for (int l = 0; l < 32; l++) {
            float s = 0.0f;
            for (int kb = w * nkb / 8; kb < (w + 1) * nkb / 8; kb++) {
                float v = x[32 * kb + l];
                s = squares ? s + v * v : s + v;
            }
            part[l] = s;
        }
        tot = tot + warp_tree(part);
    }
    return tot;
}
static void ln_dev_bf16(const float *x, const float *g, const float *b, int D, float eps, float *y) {
    float mean = lane_tree(x, D, 0) / (float)D;
    float var = lane_tree(x, D, 1) / (float)D - mean * mean;
    var = fmaxf(var, 0.0f);
    float inv = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < D; i++) {
        float t0 = (x[i] - mean) * inv;
        t0 = t0 * g[i];
        y[i] = or_bf16_round(t0 + b[i]);
    }
}

/* ---- 29-bit fixed point (the engine's GEMV input) ---------------------------------- */
#define FIX_BITS 29
/* data-independent exponent of a LayerNorm output: |y_k| <= sqrt(D) |g_k| + |b_k| (1% margin);
 * the same double arithmetic as the engine */
static int fix_of_ln(const float *g, const float *b, int D) {
    double B = 0.0;
    for (int k = 0; k < D; k++) {
        double v = (sqrt((double)D) * fabs((double)g[k]) + fabs((double)b[k])) * 1.01;
        if (v > B) B = v;
    }
    if (!(B > 0.0)) return FIX_BITS;
    int E = 0;
    frexp(B, &E);
    return FIX_BITS - E;
}
/* X = rint(x * 2^s), clamped to +-(2^30 - 64) */
static int32_t to_fix(float x, int s) {
    float v = x * ldexpf(1.0f, s);
    v = fminf(fmaxf(v, -1073741760.0f), 1073741760.0f);
    return (int32_t)nearbyintf(v);
}
/* Data-independent exponent for a linear's output rows [n0, n1) fed by a LayerNorm with
 * parameters (g, b): |y_n| <= sum_k |q[n][k]| scale[n] (sqrt(D)|g_k| + |b_k|) + |bias_n|;
 * 1% margins cover the bf16 / f32 roundings.  The same double arithmetic as the engine. */
static int fix_of_bound(const lin_t *l, int n0, int n1, const float *g, const float *b, int D) {
    double *lnmax = (double *)malloc(sizeof(double) * (size_t)D);
    for (int k = 0; k < D; k++) lnmax[k] = (sqrt((double)D) * fabs((double)g[k]) + fabs((double)b[k])) * 1.01;
    double B = 0.0;
    for (int n = n0; n < n1; n++) {
        const int8_t *q = l->q + (size_t)n * l->K;
        double s = 0.0;
        for (int k = 0; k < l->K; k++) s += fabs((double)q[k]) * lnmax[k];
        s = s * (double)l->scale[n] + fabs((double)(l->bias ? l->bias[n] : 0.0f));
        if (s > B) B = s;
    }
    free(lnmax);
    B *= 1.01;
    if (!(B > 0.0)) return FIX_BITS;
    int E = 0;
    frexp(B, &E);
    return FIX_BITS - E;
}
/* exact int8 GEMV on an output-major [N,K] weight with the activation in fixed point 2^s:
 * y = ((float)sum X_k q_nk * 2^-s) * scale + bias */
static void gemv_fix(const or_opt *m, const int8_t *wq, const float *scale, const float *bias, int K, int N,
                     const float *x, int s, float *y) {
    int32_t *X = (int32_t *)malloc(sizeof(int32_t) * (size_t)K);
    for (int k = 0; k < K; k++) X[k] = to_fix(x[k], s);
    float inv = ldexpf(1.0f, -s);
#pragma omp parallel for num_threads(m->nthreads) schedule(static)
    for (int n = 0; n < N; n++) {
        const int8_t *w = wq + (size_t)n * K;
        int64_t S = 0;
        for (int k = 0; k < K; k++) S += (int64_t)X[k] * w[k];
        float t = (float)S * inv;
        t = t * scale[n];
        y[n] = t + (bias ? bias[n] : 0.0f);
    }
    free(X);
}

/* Single-query attention of one head as an engine head pair computes it: CTA r owns dims
 * [32r, 32r+32); its partial score of key j is 4 fma chains of 8 dims, (c0 + c1) + (c2 + c3);
 * s_j = part_0 + part_1; M = max s; p_j = fast_exp_nonpos(s_j - M) (rust/npu-asr-host/src/
 * lib.rs:38-58); l = sum over 256 lanes of keys j = t mod 256 in order, butterfly per warp of
 * 32, the 8 warp sums in order; ctx_d = (sum over groups g = 0..7, in order, of the fma chain
 * over keys j = g mod 8) / l, rounded to bf16.  mha_tile (route_b_kernels/mha_decode/
 * mha_decode.cc:90-168) with one softmax over the whole context. */
static void attn_dev_head(const float *q, const float *kc, const float *vc, int stride, int tk,
                          float *sc, float *ctx) {
    float M = -INFINITY;
    for (int j = 0; j < tk; j++) {
        const float *kr = kc + (size_t)j * stride;
        float part[2];
        for (int r = 0; r < 2; r++) {
            float c4[4];
            for (int i = 0; i < 4; i++) {
                float a = 0.0f;
                for (int d = 0; d < 8; d++) a = fmaf(q[32 * r + 8 * i + d], kr[32 * r + 8 * i + d], a);
                c4[i] = a;
            }
            part[r] = (c4[0] + c4[1]) + (c4[2] + c4[3]);
        }
        sc[j] = part[0] + part[1];
        M = fmaxf(M, sc[j]);
    }
    for (int j = 0; j < tk; j++) sc[j] = or_fast_exp_nonpos(sc[j] - M);
    float L = 0.0f;
    for (int w = 0; w < 8; w++) {
        float v32[32];
        for (int l = 0; l < 32; l++) {
            float a = 0.0f;
            for (int j = 32 * w + l; j < tk; j += 256) a = a + sc[j];
            v32[l] = a;
        }
        L = L + warp_tree(v32);
    }
    for (int d = 0; d < 64; d++) {
        float tot = 0.0f;
        for (int g = 0; g < 8; g++) {
            float a = 0.0f;
            for (int j = g; j < tk; j += 8) a = fmaf(sc[j], vc[(size_t)j * stride + d], a);
            tot = tot + a;
        }
        ctx[d] = or_bf16_round(tot / L);
    }
}

/* Lin::fwd (int8 branch) parallel over blocks of output columns, k-outer inside a block. */
static void lin_fwd_ref(const or_opt *m, const lin_t *l, const float *x, float *y) {
    int K = l->K, N = l->N;
    const int BLK = 256;
    int nblk = (N + BLK - 1) / BLK;
#pragma omp parallel for num_threads(m->nthreads) schedule(static)
    for (int bi = 0; bi < nblk; bi++) {
        int n0 = bi * BLK, n1 = n0 + BLK < N ? n0 + BLK : N;
        for (int n = n0; n < n1; n++) y[n] = 0.0f;
        for (int k = 0; k < K; k++) {
            float a = x[k];
            const int8_t *wr = l->q + (size_t)k * N;
            for (int n = n0; n < n1; n++) { float p = a * (float)wr[n]; y[n] = y[n] + p; }
        }
        for (int n = n0; n < n1; n++) { float t = y[n] * l->scale[n]; y[n] = t + l->bias[n]; }
    }
}

/* Lin::fwd f32 branch (opt125m_decode.rs:125-128): y = x.W + b, k ascending. */
static void lin_fwd_f32(const or_opt *m, const lin_t *l, const float *x, float *y) {
    int K = l->K, N = l->N;
#pragma omp parallel for num_threads(m->nthreads) schedule(static)
    for (int n = 0; n < N; n++) {
        float s = 0.0f;
        for (int k = 0; k < K; k++) s += x[k] * l->w[(size_t)k * N + n];
        y[n] = s + l->bias[n];
    }
}

/* s_fix: the device mode's fixed-point exponent (ignored by the other modes) */
static void lin_apply(const or_opt *m, const lin_t *l, const float *x, int s_fix, float *y) {
    if (m->mode == OR_MODE_F32) lin_fwd_f32(m, l, x, y);
    else if (m->mode == OR_MODE_DEVICE) gemv_fix(m, l->q, l->scale, l->bias, l->K, l->N, x, s_fix, y);
    else lin_fwd_ref(m, l, x, y);
}

/* Opt::step (opt125m_decode.rs:252-293) for one token at position `pos`. */
static void opt_step(or_opt *m, int64_t id, int pos, float *logits, int want_logits) {
    const or_opt_cfg *c = &m->cfg;
    int D = c->d_model, H = c->n_heads, HD = c->head_dim, F = c->ffn, V = c->vocab;
    int dev = m->mode == OR_MODE_DEVICE;
    float *x = (float *)malloc(sizeof(float) * (size_t)(8 * D + F + pos + 1));
    float *h = x + D, *q = h + D, *kn = q + D, *vn = kn + D, *ctx = vn + D, *o = ctx + D,
          *xr = o + D, *f = xr + D, *sc = f + F;
    const float scale = 0.125f;   /* (HD as f32).powf(-0.5) for HD = 64 */
    for (int d = 0; d < D; d++)
        x[d] = m->w.emb_tok[(size_t)id * D + d] + m->w.emb_pos[(size_t)(pos + 2) * D + d];
    for (int l = 0; l < c->n_layers; l++) {
        const or_opt_layer *ly = &m->w.layers[l];
        lin_t *lin = m->lins + l * 6;
        if (dev) ln_dev_bf16(x, ly->ln1_w, ly->ln1_b, D, c->eps, h);
        else or_layer_norm(x, ly->ln1_w, ly->ln1_b, 1, D, c->eps, h);
        int sx = dev ? fix_of_ln(ly->ln1_w, ly->ln1_b, D) : 0;
        lin_apply(m, &lin[0], h, sx, q);
        lin_apply(m, &lin[1], h, sx, kn);
        lin_apply(m, &lin[2], h, sx, vn);
        for (int d = 0; d < D; d++) q[d] = q[d] * scale;
        if (dev) { or_bf16_round_n(q, q, D); or_bf16_round_n(kn, kn, D); or_bf16_round_n(vn, vn, D); }
        float *kc = m->kc + (size_t)l * m->max_ctx * D, *vc = m->vc + (size_t)l * m->max_ctx * D;
        memcpy(kc + (size_t)pos * D, kn, sizeof(float) * D);
        memcpy(vc + (size_t)pos * D, vn, sizeof(float) * D);
        int tk = pos + 1;
        for (int hh = 0; hh < H; hh++) {
            int c0 = hh * HD;
            if (!dev) {
                /* reference: sc = q.k^T; mx; e = exp(sc - mx); sum; sc /= sum; ctx = sc.v */
                float mx = -INFINITY;
                for (int j = 0; j < tk; j++) {
                    float s = 0.0f;
                    for (int d = 0; d < HD; d++) s += q[c0 + d] * kc[(size_t)j * D + c0 + d];
                    sc[j] = s; mx = fmaxf(mx, s);
                }
                float sum = 0.0f;
                for (int j = 0; j < tk; j++) { float e = expf(sc[j] - mx); sc[j] = e; sum += e; }
                for (int j = 0; j < tk; j++) sc[j] = sc[j] / sum;
                for (int d = 0; d < HD; d++) {
                    float s = 0.0f;
                    for (int j = 0; j < tk; j++) s += sc[j] * vc[(size_t)j * D + c0 + d];
                    ctx[c0 + d] = s;
                }
            } else {
                attn_dev_head(q + c0, kc + c0, vc + c0, D, tk, sc, ctx + c0);
            }
        }
        lin_apply(m, &lin[3], ctx, dev ? m->fix_ctx[l] : 0, o);
        for (int d = 0; d < D; d++) xr[d] = x[d] + o[d];
        trace_x(m, pos, 2 * l, xr);
        if (dev) ln_dev_bf16(xr, ly->ln2_w, ly->ln2_b, D, c->eps, h);
        else or_layer_norm(xr, ly->ln2_w, ly->ln2_b, 1, D, c->eps, h);
        lin_apply(m, &lin[4], h, dev ? fix_of_ln(ly->ln2_w, ly->ln2_b, D) : 0, f);
        for (int i = 0; i < F; i++) f[i] = f[i] > 0.0f ? f[i] : 0.0f;
        if (dev) or_bf16_round_n(f, f, (size_t)F);
        lin_apply(m, &lin[5], f, dev ? m->fix_h[l] : 0, o);
        for (int d = 0; d < D; d++) x[d] = xr[d] + o[d];
        trace_x(m, pos, 2 * l + 1, x);
    }
    if (want_logits) {
        if (dev) ln_dev_bf16(x, m->w.lnf_w, m->w.lnf_b, D, c->eps, h);
        else or_layer_norm(x, m->w.lnf_w, m->w.lnf_b, 1, D, c->eps, h);
        if (dev) {
            trace_x(m, pos, 2 * c->n_layers, h);
            gemv_fix(m, m->lm_q, m->lm_scale, NULL, D, V, h, fix_of_ln(m->w.lnf_w, m->w.lnf_b, D), logits);
        } else {
#pragma omp parallel for num_threads(m->nthreads) schedule(static)
            for (int v = 0; v < V; v++) {
                const float *e = m->w.emb_tok + (size_t)v * D;
                float s = 0.0f;
                for (int d = 0; d < D; d++) s += h[d] * e[d];
                logits[v] = s;
            }
        }
    }
    free(x);
}

/* One Opt::step with the LM head: feed `id` at `pos` (positions before pos must already be
 * in the cache), return the greedy id (last max wins); logits optional. */
int64_t or_opt_step(or_opt *m, int64_t id, int pos, float *logits_out) {
    float *lg = logits_out ? logits_out : (float *)malloc(sizeof(float) * (size_t)m->cfg.vocab);
    opt_step(m, id, pos, lg, 1);
    int64_t r = or_argmax_last(lg, (size_t)m->cfg.vocab);
    if (!logits_out) free(lg);
    return r;
}

/* Opt::generate (opt125m_decode.rs:296-315): prefill token by token, then greedy with
 * max_by(partial_cmp) (last maximum wins).  With force_ids, step g feeds force_ids[g]
 * instead of the argmax (teacher forcing, so logits stay comparable across numerics
 * modes after a near-tie flips a token).  Logits are only needed for the last prompt
 * token and each decoded token, so earlier prompt steps skip the LM head. */
int or_opt_generate(or_opt *m, const int64_t *prompt, int n_prompt, int n_new,
                    const int64_t *force_ids, int64_t *out_ids, float *logits_out) {
    int V = m->cfg.vocab;
    if (n_prompt < 1 || n_prompt + n_new > m->max_ctx) return -1;
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    for (int p = 0; p < n_prompt; p++) opt_step(m, prompt[p], p, logits, p == n_prompt - 1);
    int pos = n_prompt;
    for (int g = 0; g < n_new; g++) {
        int64_t next = or_argmax_last(logits, (size_t)V);
        out_ids[g] = next;
        if (logits_out) memcpy(logits_out + (size_t)g * V, logits, sizeof(float) * V);
        if (g + 1 == n_new) break;
        opt_step(m, force_ids ? force_ids[g] : next, pos, logits, 1);
        pos++;
    }
    free(logits);
    return 0;
}
