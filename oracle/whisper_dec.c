/*
 * whisper_dec.c -- oracle for the Whisper-small greedy decoder (TEST INFRASTRUCTURE ONLY; see
 * oracle.h).  Restates the reference's host f32 decoder, rust/npu-engine/src/asr/
 * whisper_decoder.rs:
 *   precompute_cross 388-399   K_enc = enc . cross_k (+0), V_enc = enc . cross_v + b
 *   HostDecoder::step 401-560  x = embed_tokens[t] + embed_positions[pos]; per layer: pre-LN
 *                              self-attention over the cache (attend_one 242-278, scale
 *                              1/sqrt(64), exact softmax), pre-LN cross-attention over the
 *                              encoder positions, pre-LN FFN with exact GELU (gelu_row 1903-1906
 *                              = the A&S erf form), residual adds; ln_post; logits = ln . proj_out
 *   linear_row 214-229         out = b, then out[j] += x[i] W[i][j] for i ascending
 *   ln_row 1894-1901           population variance, eps 1e-5
 * Greedy selection is whisper.rs argmax (749-757): strict >, the first maximum wins.
 * Weights are used as given (the tests pass the bfp16-quantised values the engine computes
 * with).
 */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

static void lrow(const float *x, int K, const float *w, const float *b, int N, float *y, int nt) {
    const int BLK = 256, nblk = (N + BLK - 1) / BLK;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int bi = 0; bi < nblk; bi++) {
        const int n0 = bi * BLK, n1 = n0 + BLK < N ? n0 + BLK : N;
        for (int n = n0; n < n1; n++) y[n] = b ? b[n] : 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = x[k];
            const float *wr = w + (size_t)k * N;
            for (int n = n0; n < n1; n++) y[n] += a * wr[n];
        }
    }
}

static void attend(const float *q, const float *kf, const float *vf, int s, int H, int hd, float *ctx, float *sc) {
    const int D = H * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = 0; i < D; i++) ctx[i] = 0.0f;
    for (int h = 0; h < H; h++) {
        const int base = h * hd;
        for (int j = 0; j < s; j++) {
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot += q[base + d] * kf[(size_t)j * D + base + d];
            sc[j] = dot * scale;
        }
        float mx = -INFINITY;
        for (int j = 0; j < s; j++) mx = fmaxf(mx, sc[j]);
        float sum = 0.0f;
        for (int j = 0; j < s; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
        const float inv = 1.0f / sum;
        for (int j = 0; j < s; j++) {
            const float p = sc[j] * inv;
            for (int d = 0; d < hd; d++) ctx[base + d] += p * vf[(size_t)j * D + base + d];
        }
    }
}

int or_whisper_decode(const or_whisper_dec_cfg *c, const or_whisper_dec_weights *w, const float *enc, int B,
                      const int64_t *prompt, int n_prompt, int n_new, int64_t *out_tokens, float *logits, int nt,
                      const int64_t *force) {
    const int D = c->d_model, H = c->n_heads, hd = D / H, F = c->ffn, V = c->vocab, L = c->n_layers, TE = c->n_enc;
    const int S = n_prompt + n_new;
    if (nt < 1) nt = 1;
    if (S > c->max_tgt) return -1;
    float *ck = (float *)malloc(sizeof(float) * (size_t)L * TE * D), *cv = (float *)malloc(sizeof(float) * (size_t)L * TE * D);
    float *sk = (float *)malloc(sizeof(float) * (size_t)L * S * D), *sv = (float *)malloc(sizeof(float) * (size_t)L * S * D);
    float *x = (float *)malloc(sizeof(float) * D), *ln = (float *)malloc(sizeof(float) * D);
    float *q = (float *)malloc(sizeof(float) * D), *ctx = (float *)malloc(sizeof(float) * D);
    float *a = (float *)malloc(sizeof(float) * D), *h1 = (float *)malloc(sizeof(float) * F);
    float *lg = (float *)malloc(sizeof(float) * V), *sc = (float *)malloc(sizeof(float) * (TE > S ? TE : S));
    for (int b = 0; b < B; b++) {
        const float *e = enc + (size_t)b * TE * D;
        for (int l = 0; l < L; l++) {
            const or_whisper_dec_layer *lw = &w->layers[l];
#pragma omp parallel for num_threads(nt) schedule(static)
            for (int t = 0; t < TE; t++) {
                lrow(e + (size_t)t * D, D, lw->cross_k_w, lw->cross_k_b, D, ck + ((size_t)l * TE + t) * D, 1);
                lrow(e + (size_t)t * D, D, lw->cross_v_w, lw->cross_v_b, D, cv + ((size_t)l * TE + t) * D, 1);
            }
        }
        int64_t tok = prompt[0];
        for (int pos = 0; pos < S - 1; pos++) {
            for (int d = 0; d < D; d++)
                x[d] = w->embed_tokens[(size_t)tok * D + d] + w->embed_positions[(size_t)pos * D + d];
            for (int l = 0; l < L; l++) {
                const or_whisper_dec_layer *lw = &w->layers[l];
                or_layer_norm(x, lw->ln_self_w, lw->ln_self_b, 1, D, 1e-5f, ln);
                lrow(ln, D, lw->q_w, lw->q_b, D, q, nt);
                lrow(ln, D, lw->k_w, lw->k_b, D, sk + ((size_t)l * S + pos) * D, nt);
                lrow(ln, D, lw->v_w, lw->v_b, D, sv + ((size_t)l * S + pos) * D, nt);
                attend(q, sk + (size_t)l * S * D, sv + (size_t)l * S * D, pos + 1, H, hd, ctx, sc);
                lrow(ctx, D, lw->out_w, lw->out_b, D, a, nt);
                for (int d = 0; d < D; d++) x[d] += a[d];
                or_layer_norm(x, lw->ln_cross_w, lw->ln_cross_b, 1, D, 1e-5f, ln);
                lrow(ln, D, lw->cross_q_w, lw->cross_q_b, D, q, nt);
                attend(q, ck + (size_t)l * TE * D, cv + (size_t)l * TE * D, TE, H, hd, ctx, sc);
                lrow(ctx, D, lw->cross_out_w, lw->cross_out_b, D, a, nt);
                for (int d = 0; d < D; d++) x[d] += a[d];
                or_layer_norm(x, lw->ln_final_w, lw->ln_final_b, 1, D, 1e-5f, ln);
                lrow(ln, D, lw->fc1_w, lw->fc1_b, F, h1, nt);
                for (int i = 0; i < F; i++) h1[i] = or_gelu_erf(h1[i]);
                lrow(h1, F, lw->fc2_w, lw->fc2_b, D, a, nt);
                for (int d = 0; d < D; d++) x[d] += a[d];
            }
            if (pos + 1 < n_prompt) { tok = prompt[pos + 1]; continue; }
            or_layer_norm(x, w->ln_post_w, w->ln_post_b, 1, D, 1e-5f, ln);
            lrow(ln, D, w->proj_out, NULL, V, lg, nt);
            int best = 0;
            for (int i = 1; i < V; i++)
                if (lg[i] > lg[best]) best = i;
            const int step = pos + 1 - n_prompt;
            out_tokens[(size_t)b * n_new + step] = best;
            if (logits) memcpy(logits + ((size_t)b * n_new + step) * V, lg, sizeof(float) * V);
            tok = force ? force[(size_t)b * n_new + step] : best;   /* teacher forcing */
        }
    }
    free(ck); free(cv); free(sk); free(sv); free(x); free(ln); free(q); free(ctx); free(a); free(h1); free(lg); free(sc);
    return 0;
}
