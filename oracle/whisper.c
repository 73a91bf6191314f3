/*
 * whisper.c -- oracle for the Whisper-small encoder (TEST INFRASTRUCTURE ONLY; see oracle.h).
 * Restates rust/npu-whisper/src/encoder.rs (host path) in f32:
 *   conv_stem 183-203 (im2col_conv1d, npu-asr-host/src/lib.rs:523-553, + exact-erf GELU),
 *   add_pos 221-227, block 236-337 (pre-LN, full attention via mha with valid_len = T),
 *   forward_last 350-375 (ln_post).
 * Linear weights are used as given (the test passes the bfp16-quantised values the engine
 * also computes with).
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

static void lin(const float *x, int T, int K, const float *w, const float *b, int N, float *y, int nt) {
    /* y[T,N] = x[T,K] . w[K,N] + b, k ascending */
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int t = 0; t < T; t++) {
        float *yr = y + (size_t)t * N;
        for (int n = 0; n < N; n++) yr[n] = 0.0f;
        for (int k = 0; k < K; k++) {
            float a = x[(size_t)t * K + k];
            const float *wr = w + (size_t)k * N;
            for (int n = 0; n < N; n++) yr[n] += a * wr[n];
        }
        for (int n = 0; n < N; n++) yr[n] = yr[n] + (b ? b[n] : 0.0f);
    }
}

/* conv1d k=3, pad 1: x [Cin, L] -> y [Cout, Lout] (im2col_conv1d order: col = ci*3 + ki) */
static void conv1d(const float *x, int Cin, int L, const float *w, const float *b, int Cout, int stride,
                   float *y, int Lout, int nt) {
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int co = 0; co < Cout; co++)
        for (int t = 0; t < Lout; t++) {
            float s = 0.0f;
            for (int ci = 0; ci < Cin; ci++)
                for (int ki = 0; ki < 3; ki++) {
                    int ts = t * stride + ki - 1;
                    float v = (ts >= 0 && ts < L) ? x[(size_t)ci * L + ts] : 0.0f;
                    s += v * w[((size_t)co * Cin + ci) * 3 + ki];
                }
            y[(size_t)co * Lout + t] = s + b[co];
        }
}

int or_whisper_encode(const or_whisper_enc_cfg *c, const or_whisper_enc_weights *w, const float *mel,
                      int B, float *out, int nt) {
    const int D = c->d_model, F = c->ffn, C = c->n_mels, T = c->n_frames, To = T / 2, H = c->n_heads;
    if (nt < 1) nt = 1;
    float *h1 = (float *)malloc(sizeof(float) * (size_t)D * T);
    float *h2 = (float *)malloc(sizeof(float) * (size_t)D * To);
    float *x = (float *)malloc(sizeof(float) * (size_t)To * D);
    float *ln = (float *)malloc(sizeof(float) * (size_t)To * D);
    float *q = (float *)malloc(sizeof(float) * (size_t)To * D), *k = (float *)malloc(sizeof(float) * (size_t)To * D);
    float *v = (float *)malloc(sizeof(float) * (size_t)To * D), *ctx = (float *)malloc(sizeof(float) * (size_t)To * D);
    float *f = (float *)malloc(sizeof(float) * (size_t)To * F);
    for (int b = 0; b < B; b++) {
        conv1d(mel + (size_t)b * C * T, C, T, w->conv1_w, w->conv1_b, D, 1, h1, T, nt);
        for (size_t i = 0; i < (size_t)D * T; i++) h1[i] = or_gelu_erf(h1[i]);
        conv1d(h1, D, T, w->conv2_w, w->conv2_b, D, 2, h2, To, nt);
        for (int t = 0; t < To; t++)
            for (int d = 0; d < D; d++)
                x[(size_t)t * D + d] = or_gelu_erf(h2[(size_t)d * To + t]) + w->embed_positions[(size_t)t * D + d];
        for (int l = 0; l < c->n_layers; l++) {
            const or_whisper_enc_layer *L = &w->layers[l];
            or_layer_norm(x, L->ln1_w, L->ln1_b, To, D, c->eps, ln);
            lin(ln, To, D, L->q_w, L->q_b, D, q, nt);
            lin(ln, To, D, L->k_w, L->k_b, D, k, nt);
            lin(ln, To, D, L->v_w, L->v_b, D, v, nt);
            or_mha(q, k, v, To, H, D / H, 0, To, ctx);
            lin(ctx, To, D, L->out_w, L->out_b, D, q, nt);
            for (size_t i = 0; i < (size_t)To * D; i++) x[i] = x[i] + q[i];
            or_layer_norm(x, L->ln2_w, L->ln2_b, To, D, c->eps, ln);
            lin(ln, To, D, L->fc1_w, L->fc1_b, F, f, nt);
            for (size_t i = 0; i < (size_t)To * F; i++) f[i] = or_gelu_erf(f[i]);
            lin(f, To, F, L->fc2_w, L->fc2_b, D, q, nt);
            for (size_t i = 0; i < (size_t)To * D; i++) x[i] = x[i] + q[i];
        }
        or_layer_norm(x, w->ln_post_w, w->ln_post_b, To, D, c->eps, out + (size_t)b * To * D);
    }
    free(h1); free(h2); free(x); free(ln); free(q); free(k); free(v); free(ctx); free(f);
    return 0;
}
