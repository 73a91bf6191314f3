/*
 * gemma.c -- oracle for the Gemma-3 text decoder (TEST INFRASTRUCTURE ONLY; see oracle.h).
 * The reference has no Gemma decoder step (rust/npu-gemma/src/lib.rs:30-43 lists the pieces
 * to reuse); this restates the HuggingFace Gemma-3 text model it ports, with the reference's
 * own pieces where they exist:
 *   rmsnorm_ref  npu-gemma/src/lib.rs:55-64   x * 1/sqrt(mean(x^2) + eps) * (1 + w)
 *   geglu_ref    npu-gemma/src/lib.rs:68-77   gelu_tanh(gate) * up
 *   is_global_layer npu-gemma/src/config.rs:131-133 ((i + 1) % 6 == 0); the other layers
 *                attend within a sliding window of 512 positions
 *   config       npu-gemma/src/config.rs:156-170 (GEMMA3_1B)
 *   and HF Gemma3: embeddings * sqrt(d_model); per layer input norm -> q, k, v (no biases) ->
 *   per-head q_norm / k_norm -> RoPE (rotate-half; theta 10k local, 1M global) -> GQA attention
 *   scaled by query_pre_attn_scalar^-1/2 -> o -> post-attention norm -> + residual;
 *   pre-FFN norm -> GeGLU -> post-FFN norm -> + residual; final norm; logits = h . E^T (tied).
 * With int8 != 0 every linear and the tied LM head follow the reference's Lin rule
 * (opt125m_decode.rs:41-60, 106-124): per-output-channel int8 weights, f32 activations,
 * y[n] = (sum_k x[k] q[k][n]) * scale[n].  Greedy selection: first maximum.
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    const float *w;      /* [K, N] */
    int8_t *q;           /* int8: [K, N] */
    float *scale;
    int K, N;
} glin;

static void glin_init(glin *l, const float *w, int K, int N, int int8) {
    l->w = w; l->K = K; l->N = N; l->q = NULL; l->scale = NULL;
    if (!int8) return;
    l->q = (int8_t *)malloc((size_t)K * N);
    l->scale = (float *)malloc(sizeof(float) * N);
    or_quant_i8_cols(w, K, N, l->q, l->scale);
}
static void glin_free(glin *l) { free(l->q); free(l->scale); }

static void glin_fwd(const glin *l, const float *x, float *y, int nt) {
    const int K = l->K, N = l->N, BLK = 256, nblk = (N + BLK - 1) / BLK;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int bi = 0; bi < nblk; bi++) {
        const int n0 = bi * BLK, n1 = n0 + BLK < N ? n0 + BLK : N;
        for (int n = n0; n < n1; n++) y[n] = 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = x[k];
            if (l->q) {
                const int8_t *wr = l->q + (size_t)k * N;
                for (int n = n0; n < n1; n++) y[n] += a * (float)wr[n];
            } else {
                const float *wr = l->w + (size_t)k * N;
                for (int n = n0; n < n1; n++) y[n] += a * wr[n];
            }
        }
        if (l->q)
            for (int n = n0; n < n1; n++) y[n] = y[n] * l->scale[n];
    }
}

static void rms(const float *x, const float *w, int n, float eps, float *y) {
    float ms = 0.0f;
    for (int i = 0; i < n; i++) ms += x[i] * x[i];
    ms = ms / (float)n;
    const float inv = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * inv * (1.0f + w[i]);
}

float or_gelu_tanh_gemma(float x) {
    const float C = 0.79788456f;
    return 0.5f * x * (1.0f + tanhf(C * (x + 0.044715f * x * x * x)));
}

static void rope(float *x, int hd, int pos, float theta) {
    const int h = hd / 2;
    for (int i = 0; i < h; i++) {
        const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
        const float f = (float)pos * inv;
        const float c = cosf(f), s = sinf(f);
        const float a = x[i], b = x[i + h];
        x[i] = a * c - b * s;
        x[i + h] = b * c + a * s;
    }
}

int or_gemma_decode(const or_gemma_cfg *c, const or_gemma_weights *w, const int64_t *prompt, int n_prompt, int n_new,
                    int64_t *out_tokens, float *logits, int nt, const int64_t *force) {
    const int D = c->d_model, HQ = c->n_q_heads, HD = c->head_dim, F = c->ffn, V = c->vocab, L = c->n_layers;
    const int S = n_prompt + n_new, QD = HQ * HD;
    if (nt < 1) nt = 1;
    glin *lins = (glin *)calloc((size_t)L * 7, sizeof(glin));
    for (int l = 0; l < L; l++) {
        const or_gemma_layer *ly = &w->layers[l];
        glin_init(&lins[l * 7 + 0], ly->wq, D, QD, c->int8);
        glin_init(&lins[l * 7 + 1], ly->wk, D, HD, c->int8);
        glin_init(&lins[l * 7 + 2], ly->wv, D, HD, c->int8);
        glin_init(&lins[l * 7 + 3], ly->wo, QD, D, c->int8);
        glin_init(&lins[l * 7 + 4], ly->wg, D, F, c->int8);
        glin_init(&lins[l * 7 + 5], ly->wu, D, F, c->int8);
        glin_init(&lins[l * 7 + 6], ly->wd, F, D, c->int8);
    }
    /* tied LM head: logits[v] = h . E[v]; as a [K = D, N = V] linear over E^T */
    float *et = (float *)malloc(sizeof(float) * (size_t)D * V);
    for (int v = 0; v < V; v++)
        for (int d = 0; d < D; d++) et[(size_t)d * V + v] = w->embed[(size_t)v * D + d];
    glin lm;
    glin_init(&lm, et, D, V, c->int8);
    float *kc = (float *)malloc(sizeof(float) * (size_t)L * S * HD), *vc = (float *)malloc(sizeof(float) * (size_t)L * S * HD);
    float *x = (float *)malloc(sizeof(float) * D), *h = (float *)malloc(sizeof(float) * D);
    float *q = (float *)malloc(sizeof(float) * QD), *ctx = (float *)malloc(sizeof(float) * QD);
    float *kk = (float *)malloc(sizeof(float) * HD), *vv = (float *)malloc(sizeof(float) * HD);
    float *o = (float *)malloc(sizeof(float) * D), *g = (float *)malloc(sizeof(float) * F), *u = (float *)malloc(sizeof(float) * F);
    float *lg = (float *)malloc(sizeof(float) * V), *sc = (float *)malloc(sizeof(float) * S);
    const float es = sqrtf((float)D), scaling = 1.0f / sqrtf(c->query_pre_attn_scalar);
    int64_t tok = prompt[0];
    for (int pos = 0; pos < S - 1; pos++) {
        for (int d = 0; d < D; d++) x[d] = w->embed[(size_t)tok * D + d] * es;
        for (int l = 0; l < L; l++) {
            const or_gemma_layer *ly = &w->layers[l];
            const int global = (l + 1) % c->pattern == 0;
            const float theta = global ? c->theta_global : c->theta_local;
            rms(x, ly->in_norm, D, c->eps, h);
            glin_fwd(&lins[l * 7 + 0], h, q, nt);
            glin_fwd(&lins[l * 7 + 1], h, kk, nt);
            glin_fwd(&lins[l * 7 + 2], h, vv, nt);
            for (int hh = 0; hh < HQ; hh++) {
                rms(q + hh * HD, ly->q_norm, HD, c->eps, q + hh * HD);
                rope(q + hh * HD, HD, pos, theta);
            }
            rms(kk, ly->k_norm, HD, c->eps, kk);
            rope(kk, HD, pos, theta);
            memcpy(kc + ((size_t)l * S + pos) * HD, kk, sizeof(float) * HD);
            memcpy(vc + ((size_t)l * S + pos) * HD, vv, sizeof(float) * HD);
            const int j0 = global ? 0 : (pos - c->window + 1 > 0 ? pos - c->window + 1 : 0);
            for (int hh = 0; hh < HQ; hh++) {
                float mx = -INFINITY;
                for (int j = j0; j <= pos; j++) {
                    float dot = 0.0f;
                    for (int d = 0; d < HD; d++) dot += q[hh * HD + d] * kc[((size_t)l * S + j) * HD + d];
                    sc[j] = dot * scaling;
                    mx = fmaxf(mx, sc[j]);
                }
                float sum = 0.0f;
                for (int j = j0; j <= pos; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                for (int d = 0; d < HD; d++) ctx[hh * HD + d] = 0.0f;
                for (int j = j0; j <= pos; j++) {
                    const float p = sc[j] / sum;
                    for (int d = 0; d < HD; d++) ctx[hh * HD + d] += p * vc[((size_t)l * S + j) * HD + d];
                }
            }
            glin_fwd(&lins[l * 7 + 3], ctx, o, nt);
            rms(o, ly->post_attn_norm, D, c->eps, o);
            for (int d = 0; d < D; d++) x[d] += o[d];
            rms(x, ly->pre_ffn_norm, D, c->eps, h);
            glin_fwd(&lins[l * 7 + 4], h, g, nt);
            glin_fwd(&lins[l * 7 + 5], h, u, nt);
            for (int i = 0; i < F; i++) g[i] = or_gelu_tanh_gemma(g[i]) * u[i];
            glin_fwd(&lins[l * 7 + 6], g, o, nt);
            rms(o, ly->post_ffn_norm, D, c->eps, o);
            for (int d = 0; d < D; d++) x[d] += o[d];
        }
        if (pos + 1 < n_prompt) { tok = prompt[pos + 1]; continue; }
        rms(x, w->final_norm, D, c->eps, h);
        glin_fwd(&lm, h, lg, nt);
        int best = 0;
        for (int i = 1; i < V; i++)
            if (lg[i] > lg[best]) best = i;
        const int step = pos + 1 - n_prompt;
        out_tokens[step] = best;
        if (logits) memcpy(logits + (size_t)step * V, lg, sizeof(float) * V);
        tok = force ? force[step] : best;       /* teacher forcing */
    }
    for (int i = 0; i < L * 7; i++) glin_free(&lins[i]);
    glin_free(&lm);
    free(lins); free(et); free(kc); free(vc); free(x); free(h); free(q); free(ctx); free(kk); free(vv); free(o);
    free(g); free(u); free(lg); free(sc);
    return 0;
}
