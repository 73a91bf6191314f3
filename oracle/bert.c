/*
 * bert.c -- oracle for the BGE/BERT embedder (TEST INFRASTRUCTURE ONLY; see oracle.h).
 * Restates the reference's host path in f32:
 *   EmbedFrontend::run  rust/npu-engine/src/bert/frontend.rs:37-61
 *   BertBlock::forward  rust/npu-engine/src/bert/encoder.rs:43-57 (its GEMMs run on the NPU
 *                       in the reference; here x.W + b with f32 accumulation in k order)
 *   mha                 rust/npu-asr-host/src/lib.rs:189-326 (or_mha, valid_len = L)
 *   gelu                rust/npu-asr-host/src/lib.rs:464-495 (or_gelu_erf)
 *   EmbedHead::run      rust/npu-engine/src/bert/head.rs:20-47
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* y[T, N] = x[T, K] . W[K, N] + b, W given transposed as wt[N, K] */
static void linear(const float *x, int T, int K, const float *wt, const float *b, int N, float *y,
                   int nthreads) {
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
    for (int t = 0; t < T; t++)
        for (int n = 0; n < N; n++) {
            const float *xr = x + (size_t)t * K, *wr = wt + (size_t)n * K;
            float s = 0.0f;
            for (int k = 0; k < K; k++) s += xr[k] * wr[k];
            y[(size_t)t * N + n] = s + (b ? b[n] : 0.0f);
        }
}

static float *transpose(const float *w, int K, int N) {
    float *t = (float *)malloc(sizeof(float) * (size_t)K * N);
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) t[(size_t)n * K + k] = w[(size_t)k * N + n];
    return t;
}

int or_bert_embed(const or_bert_cfg *c, const or_bert_weights *w, const int32_t *ids,
                  const int32_t *seq_lens, int n_seqs, float *out, int nthreads) {
    const int D = c->d_model, F = c->ffn, H = c->n_heads, hd = D / H;
    if (nthreads < 1) nthreads = 1;
    /* transposed weights, once */
    float **wt = (float **)calloc((size_t)c->n_layers * 6, sizeof(float *));
    for (int l = 0; l < c->n_layers; l++) {
        const or_bert_layer *L = &w->layers[l];
        wt[l * 6 + 0] = transpose(L->q_w, D, D);
        wt[l * 6 + 1] = transpose(L->k_w, D, D);
        wt[l * 6 + 2] = transpose(L->v_w, D, D);
        wt[l * 6 + 3] = transpose(L->o_w, D, D);
        wt[l * 6 + 4] = transpose(L->ffn1_w, D, F);
        wt[l * 6 + 5] = transpose(L->ffn2_w, F, D);
    }
    int off = 0;
    for (int s = 0; s < n_seqs; s++) {
        const int T = seq_lens[s];
        float *x = (float *)malloc(sizeof(float) * (size_t)T * D);
        float *q = (float *)malloc(sizeof(float) * (size_t)T * D);
        float *k = (float *)malloc(sizeof(float) * (size_t)T * D);
        float *v = (float *)malloc(sizeof(float) * (size_t)T * D);
        float *ctx = (float *)malloc(sizeof(float) * (size_t)T * D);
        float *h = (float *)malloc(sizeof(float) * (size_t)T * F);
        /* frontend: word + position + type 0, then LayerNorm */
        for (int t = 0; t < T; t++)
            for (int j = 0; j < D; j++) {
                float e = w->word_emb[(size_t)ids[off + t] * D + j] + w->pos_emb[(size_t)t * D + j];
                x[(size_t)t * D + j] = e + w->type_emb[j];
            }
        or_layer_norm(x, w->emb_ln_w, w->emb_ln_b, T, D, c->eps, x);
        for (int l = 0; l < c->n_layers; l++) {
            const or_bert_layer *L = &w->layers[l];
            linear(x, T, D, wt[l * 6 + 0], L->q_b, D, q, nthreads);
            linear(x, T, D, wt[l * 6 + 1], L->k_b, D, k, nthreads);
            linear(x, T, D, wt[l * 6 + 2], L->v_b, D, v, nthreads);
            or_mha(q, k, v, T, H, hd, 0, T, ctx);
            linear(ctx, T, D, wt[l * 6 + 3], L->o_b, D, q, nthreads);     /* q <- attn out */
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + q[i];
            or_layer_norm(x, L->attn_ln_w, L->attn_ln_b, T, D, c->eps, x);
            linear(x, T, D, wt[l * 6 + 4], L->ffn1_b, F, h, nthreads);
            for (size_t i = 0; i < (size_t)T * F; i++) h[i] = or_gelu_erf(h[i]);
            linear(h, T, F, wt[l * 6 + 5], L->ffn2_b, D, q, nthreads);
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + q[i];
            or_layer_norm(x, L->out_ln_w, L->out_ln_b, T, D, c->eps, x);
        }
        /* head: CLS or mean over the valid rows, then L2 with the norm clamped at 1e-12 */
        float *o = out + (size_t)s * D;
        for (int j = 0; j < D; j++) o[j] = 0.0f;
        if (c->pooling == 0) {
            for (int j = 0; j < D; j++) o[j] = x[j];
        } else {
            for (int t = 0; t < T; t++)
                for (int j = 0; j < D; j++) o[j] += x[(size_t)t * D + j];
            float inv = 1.0f / (float)T;
            for (int j = 0; j < D; j++) o[j] *= inv;
        }
        float ss = 0.0f;
        for (int j = 0; j < D; j++) ss += o[j] * o[j];
        float norm = fmaxf(sqrtf(ss), 1e-12f);
        for (int j = 0; j < D; j++) o[j] /= norm;
        free(x); free(q); free(k); free(v); free(ctx); free(h);
        off += T;
    }
    for (int i = 0; i < c->n_layers * 6; i++) free(wt[i]);
    free(wt);
    return 0;
}
