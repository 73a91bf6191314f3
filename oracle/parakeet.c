/*
 * parakeet.c -- oracle for the Parakeet FastConformer encoder (TEST INFRASTRUCTURE ONLY; see
 * oracle.h).  Restates the reference's host f32 encoder, rust/npu-parakeet/src/:
 *   subsample        encoder.rs:200-237 with conv2d (ops.rs:38-89): conv.0 (1->C, k3 s2 p1)
 *                    + ReLU, conv.2 depthwise k3 s2 p1, conv.3 pointwise + ReLU, conv.5
 *                    depthwise, conv.6 pointwise + ReLU, flatten [t, c*F + f], out linear
 *   feed_forward     encoder.rs:102-168 (LN -> linear1 -> SiLU -> linear2, no biases)
 *   mhsa             encoder.rs:238-253 + attention_core 285-414 (rel-pos MHA: q + u, q + v,
 *                    AC = qu k^T, BD = qv p^T, rel_shift (ops.rs:113-133), /sqrt(dk),
 *                    exact softmax, P V)
 *   conv_module      encoder.rs:416-570 (LN -> pw1 -> GLU -> depthwise k9 'same' + bias
 *                    (ops.rs:92-110) -> SiLU -> pw2)
 *   block            encoder.rs:572-654 (macaron: x + 0.5 ff1, + mhsa, + conv, + 0.5 ff2, LN)
 *   rel_pos_encoding pos.rs:7-47 (f64 sinusoids, positions T-1 .. -(T-1))
 * With cfg->int8 every weight linear (everything but the subsample stem) follows the
 * reference's int8 GEMM engine (rust/npu-asr/src/ctx2.rs): per-output-channel weight scale
 * max|W[:,n]|/127 (549-584), dynamic per-tensor activation scale max|A|/127 over the call's
 * [T, K] input (quant_scale 1361-1377), quant_i8 = round-half-away(x / s) clamped to +-127
 * (1352-1354), exact i32 accumulation, dequant (acc * s_a) * ws[n] (dequant_epi 1386-1411).
 * Each clip of a batch is its own call, as in the reference (one utterance per encode).
 */
#include "oracle.h"
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float q_i8(float x, float s) {
    float v = roundf(x / s);
    return v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
}

/* y[T, N] = x[T, K] . W[K, N] (+ bias): f32 (k ascending) or the int8 engine rule */
static void lin(const float *x, int T, int K, const float *w, const float *bias, int N, int int8, float *y,
                int nt) {
    if (!int8) {
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int t = 0; t < T; t++) {
            float *yr = y + (size_t)t * N;
            for (int n = 0; n < N; n++) yr[n] = 0.0f;
            for (int k = 0; k < K; k++) {
                const float a = x[(size_t)t * K + k];
                const float *wr = w + (size_t)k * N;
                for (int n = 0; n < N; n++) yr[n] += a * wr[n];
            }
            if (bias)
                for (int n = 0; n < N; n++) yr[n] = yr[n] + bias[n];
        }
        return;
    }
    int8_t *wq = (int8_t *)malloc((size_t)K * N), *wt = (int8_t *)malloc((size_t)K * N);
    float *ws = (float *)malloc(sizeof(float) * N);
    or_quant_i8_cols(w, K, N, wq, ws);
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) wt[(size_t)n * K + k] = wq[(size_t)k * N + n];
    float amax = 0.0f;
    for (size_t i = 0; i < (size_t)T * K; i++) amax = fmaxf(amax, fabsf(x[i]));
    const float sa = amax > 0.0f ? amax / 127.0f : 1.0f;
    int8_t *xq = (int8_t *)malloc((size_t)T * K);
    for (size_t i = 0; i < (size_t)T * K; i++) xq[i] = (int8_t)q_i8(x[i], sa);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int t = 0; t < T; t++)
        for (int n = 0; n < N; n++) {
            const int8_t *a = xq + (size_t)t * K, *b = wt + (size_t)n * K;
            int32_t acc = 0;
            for (int k = 0; k < K; k++) acc += (int32_t)a[k] * (int32_t)b[k];
            float v = (float)acc * sa;
            v = v * ws[n];
            y[(size_t)t * N + n] = bias ? v + bias[n] : v;
        }
    free(wq); free(wt); free(ws); free(xq);
}

void or_parakeet_quant_lin(const float *x, int T, int K, const float *w, const float *bias, int N, float *y,
                           int nt) {
    lin(x, T, K, w, bias, N, 1, y, nt > 0 ? nt : 1);
}

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* conv2d of ops.rs:38-89 on [Ci, H, W]: output plane starts at the bias, then for each input
 * channel and tap (i, j) in order, plane += w * shifted input (taps with w == 0 skipped) */
void or_conv2d(const float *x, int ci, int hin, int win, const float *w, const float *b, int co, int kh, int kw,
               int stride, int pad, int groups, float *y, int nt) {
    const int hout = (hin + 2 * pad - kh) / stride + 1, wout = (win + 2 * pad - kw) / stride + 1;
    const int gci = ci / groups, gco = co / groups;
    if (kh == 1 && kw == 1 && groups == 1 && stride == 1 && pad == 0) {
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int o = 0; o < co; o++) {
            float *yp = y + (size_t)o * hin * win;
            for (int p = 0; p < hin * win; p++) yp[p] = 0.0f;
            for (int c = 0; c < ci; c++) {
                const float wv = w[(size_t)o * ci + c];
                const float *xp = x + (size_t)c * hin * win;
                for (int p = 0; p < hin * win; p++) yp[p] += wv * xp[p];
            }
            for (int p = 0; p < hin * win; p++) yp[p] = yp[p] + b[o];
        }
        return;
    }
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int o = 0; o < co; o++) {
        const int g = o / gco;
        float *yp = y + (size_t)o * hout * wout;
        for (int p = 0; p < hout * wout; p++) yp[p] = b[o];
        for (int ic = 0; ic < gci; ic++) {
            const float *xp = x + (size_t)(g * gci + ic) * hin * win;
            for (int i = 0; i < kh; i++)
                for (int j = 0; j < kw; j++) {
                    const float wv = w[(((size_t)o * gci + ic) * kh + i) * kw + j];
                    if (wv == 0.0f) continue;
                    for (int oh = 0; oh < hout; oh++) {
                        const int ih = oh * stride + i - pad;
                        if (ih < 0 || ih >= hin) continue;
                        for (int ow = 0; ow < wout; ow++) {
                            const int iw = ow * stride + j - pad;
                            if (iw < 0 || iw >= win) continue;
                            yp[(size_t)oh * wout + ow] += wv * xp[(size_t)ih * win + iw];
                        }
                    }
                }
        }
    }
}

/* ops.rs:92-110: out[c][t] = bias[c] + sum_j taps[c][j] * x[c][t + j - pad] (valid j only) */
void or_dwconv1d(const float *x, int C, int T, const float *taps, const float *bias, int k, float *y) {
    const int pad = (k - 1) / 2;
    for (int c = 0; c < C; c++)
        for (int t = 0; t < T; t++) {
            float acc = bias[c];
            for (int j = 0; j < k; j++) {
                const int s = t + j - pad;
                if (s >= 0 && s < T) acc += taps[(size_t)c * k + j] * x[(size_t)c * T + s];
            }
            y[(size_t)c * T + t] = acc;
        }
}

/* ops.rs:113-133: bd [H, T, 2T-1] -> [H, T, T] through NeMo's pad / reshape / slice */
void or_rel_shift(const float *bd, int H, int T, float *out) {
    const int P = 2 * T - 1;
    for (int h = 0; h < H; h++)
        for (int i = 0; i < T; i++)
            for (int j = 0; j < T; j++) {
                const size_t f = (size_t)T + (size_t)i * P + j;       /* flat index into [T, P+1] */
                const size_t r = f / (P + 1), c = f % (P + 1);
                out[((size_t)h * T + i) * T + j] = c == 0 ? 0.0f : bd[((size_t)h * T + r) * P + (c - 1)];
            }
}

/* pos.rs:7-47 */
void or_rel_pos_encoding(int T, int D, float *pe) {
    const int half = D / 2;
    for (int k = 0; k < 2 * T - 1; k++) {
        const double pos = k < T ? (double)(T - 1 - k) : -(double)(k - T + 1);
        for (int i = 0; i < half; i++) {
            const double dv = exp(-log(10000.0) * (double)(2 * i) / (double)D);
            const double a = pos * dv;
            pe[(size_t)k * D + 2 * i] = (float)sin(a);
            pe[(size_t)k * D + 2 * i + 1] = (float)cos(a);
        }
    }
}

static void ffn(const or_parakeet_cfg *c, const float *x, int T, const float *g, const float *b, const float *w1,
                const float *w2, float *y, float *ln, float *h, int nt) {
    or_layer_norm(x, g, b, T, c->d_model, 1e-5f, ln);
    lin(ln, T, c->d_model, w1, NULL, c->ffn, c->int8, h, nt);
    for (size_t i = 0; i < (size_t)T * c->ffn; i++) h[i] = h[i] * (1.0f / (1.0f + expf(-h[i])));
    lin(h, T, c->ffn, w2, NULL, c->d_model, c->int8, y, nt);
}

int or_parakeet_encode(const or_parakeet_cfg *c, const or_parakeet_weights *w, const float *mel, int B,
                       float *out, int nt) {
    const int D = c->d_model, F = c->ffn, H = c->n_heads, dk = D / H, C = c->sub_ch, KC = c->kconv;
    const int NM = c->n_mels, T0 = c->n_frames;
    if (nt < 1) nt = 1;
    const int H1 = (T0 - 1) / 2 + 1, W1 = (NM - 1) / 2 + 1, H2 = (H1 - 1) / 2 + 1, W2 = (W1 - 1) / 2 + 1;
    const int T = (H2 - 1) / 2 + 1, W3 = (W2 - 1) / 2 + 1, P = 2 * T - 1;
    float *img = (float *)malloc(sizeof(float) * (size_t)T0 * NM);
    float *a1 = (float *)malloc(sizeof(float) * (size_t)C * H1 * W1);
    float *a2 = (float *)malloc(sizeof(float) * (size_t)C * H2 * W2);
    float *a3 = (float *)malloc(sizeof(float) * (size_t)C * H2 * W2);
    float *a5 = (float *)malloc(sizeof(float) * (size_t)C * T * W3);
    float *a6 = (float *)malloc(sizeof(float) * (size_t)C * T * W3);
    float *flat = (float *)malloc(sizeof(float) * (size_t)T * C * W3);
    float *x = (float *)malloc(sizeof(float) * (size_t)T * D), *y = (float *)malloc(sizeof(float) * (size_t)T * D);
    float *ln = (float *)malloc(sizeof(float) * (size_t)T * D);
    float *hbuf = (float *)malloc(sizeof(float) * (size_t)T * (F > 2 * D ? F : 2 * D));
    float *q = (float *)malloc(sizeof(float) * (size_t)T * D), *k = (float *)malloc(sizeof(float) * (size_t)T * D);
    float *v = (float *)malloc(sizeof(float) * (size_t)T * D), *ctx = (float *)malloc(sizeof(float) * (size_t)T * D);
    float *pe = (float *)malloc(sizeof(float) * (size_t)P * D), *pm = (float *)malloc(sizeof(float) * (size_t)P * D);
    float *bd = (float *)malloc(sizeof(float) * (size_t)H * T * P), *bds = (float *)malloc(sizeof(float) * (size_t)H * T * T);
    float *ac = (float *)malloc(sizeof(float) * (size_t)T * T), *sc = (float *)malloc(sizeof(float) * (size_t)T);
    float *gt = (float *)malloc(sizeof(float) * (size_t)D * T), *dw = (float *)malloc(sizeof(float) * (size_t)D * T);
    or_rel_pos_encoding(T, D, pe);
    const float scale = sqrtf((float)dk);
    for (int bi = 0; bi < B; bi++) {
        /* ---- subsample: image [1, time, freq] */
        const float *m = mel + (size_t)bi * NM * T0;
        for (int t = 0; t < T0; t++)
            for (int f = 0; f < NM; f++) img[(size_t)t * NM + f] = m[(size_t)f * T0 + t];
        or_conv2d(img, 1, T0, NM, w->c0_w, w->c0_b, C, 3, 3, 2, 1, 1, a1, nt);
        for (size_t i = 0; i < (size_t)C * H1 * W1; i++) a1[i] = fmaxf(a1[i], 0.0f);
        or_conv2d(a1, C, H1, W1, w->c2_w, w->c2_b, C, 3, 3, 2, 1, C, a2, nt);
        or_conv2d(a2, C, H2, W2, w->c3_w, w->c3_b, C, 1, 1, 1, 0, 1, a3, nt);
        for (size_t i = 0; i < (size_t)C * H2 * W2; i++) a3[i] = fmaxf(a3[i], 0.0f);
        or_conv2d(a3, C, H2, W2, w->c5_w, w->c5_b, C, 3, 3, 2, 1, C, a5, nt);
        or_conv2d(a5, C, T, W3, w->c6_w, w->c6_b, C, 1, 1, 1, 0, 1, a6, nt);
        for (size_t i = 0; i < (size_t)C * T * W3; i++) a6[i] = fmaxf(a6[i], 0.0f);
        for (int t = 0; t < T; t++)
            for (int ci = 0; ci < C; ci++)
                for (int f = 0; f < W3; f++) flat[(size_t)t * C * W3 + ci * W3 + f] = a6[((size_t)ci * T + t) * W3 + f];
        lin(flat, T, C * W3, w->out_w, w->out_b, D, 0, x, nt);
        /* ---- blocks */
        for (int l = 0; l < c->n_layers; l++) {
            const or_parakeet_layer *L = &w->layers[l];
            ffn(c, x, T, L->ff1_ln_w, L->ff1_ln_b, L->ff1_w1, L->ff1_w2, y, ln, hbuf, nt);
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + 0.5f * y[i];
            /* rel-pos MHSA */
            or_layer_norm(x, L->att_ln_w, L->att_ln_b, T, D, 1e-5f, ln);
            lin(ln, T, D, L->wq, NULL, D, c->int8, q, nt);
            lin(ln, T, D, L->wk, NULL, D, c->int8, k, nt);
            lin(ln, T, D, L->wv, NULL, D, c->int8, v, nt);
            lin(pe, P, D, L->wpos, NULL, D, c->int8, pm, nt);
            for (int h = 0; h < H; h++)
                for (int i = 0; i < T; i++)
                    for (int p = 0; p < P; p++) {
                        float s = 0.0f;
                        for (int d = 0; d < dk; d++)
                            s += (q[(size_t)i * D + h * dk + d] + L->pos_v[h * dk + d]) * pm[(size_t)p * D + h * dk + d];
                        bd[((size_t)h * T + i) * P + p] = s;
                    }
            or_rel_shift(bd, H, T, bds);
            for (int h = 0; h < H; h++) {
                for (int i = 0; i < T; i++)
                    for (int j = 0; j < T; j++) {
                        float s = 0.0f;
                        for (int d = 0; d < dk; d++)
                            s += (q[(size_t)i * D + h * dk + d] + L->pos_u[h * dk + d]) * k[(size_t)j * D + h * dk + d];
                        ac[(size_t)i * T + j] = s;
                    }
                for (int i = 0; i < T; i++) {
                    float mx = -INFINITY;
                    for (int j = 0; j < T; j++) {
                        sc[j] = (ac[(size_t)i * T + j] + bds[((size_t)h * T + i) * T + j]) / scale;
                        mx = fmaxf(mx, sc[j]);
                    }
                    float sum = 0.0f;
                    for (int j = 0; j < T; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                    for (int j = 0; j < T; j++) sc[j] /= sum;
                    for (int d = 0; d < dk; d++) {
                        float o = 0.0f;
                        for (int j = 0; j < T; j++) o += sc[j] * v[(size_t)j * D + h * dk + d];
                        ctx[(size_t)i * D + h * dk + d] = o;
                    }
                }
            }
            lin(ctx, T, D, L->wout, NULL, D, c->int8, y, nt);
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + y[i];
            /* conv module */
            or_layer_norm(x, L->conv_ln_w, L->conv_ln_b, T, D, 1e-5f, ln);
            lin(ln, T, D, L->pw1, NULL, 2 * D, c->int8, hbuf, nt);
            for (int t = 0; t < T; t++)
                for (int ch = 0; ch < D; ch++)
                    gt[(size_t)ch * T + t] = hbuf[(size_t)t * 2 * D + ch] * sigm(hbuf[(size_t)t * 2 * D + D + ch]);
            or_dwconv1d(gt, D, T, L->dw_w, L->dw_b, KC, dw);
            for (size_t i = 0; i < (size_t)D * T; i++) dw[i] = dw[i] * (1.0f / (1.0f + expf(-dw[i])));
            for (int t = 0; t < T; t++)
                for (int ch = 0; ch < D; ch++) ln[(size_t)t * D + ch] = dw[(size_t)ch * T + t];
            lin(ln, T, D, L->pw2, NULL, D, c->int8, y, nt);
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + y[i];
            ffn(c, x, T, L->ff2_ln_w, L->ff2_ln_b, L->ff2_w1, L->ff2_w2, y, ln, hbuf, nt);
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] = x[i] + 0.5f * y[i];
            or_layer_norm(x, L->out_ln_w, L->out_ln_b, T, D, 1e-5f, x);
        }
        memcpy(out + (size_t)bi * T * D, x, sizeof(float) * (size_t)T * D);
    }
    free(img); free(a1); free(a2); free(a3); free(a5); free(a6); free(flat); free(x); free(y); free(ln);
    free(hbuf); free(q); free(k); free(v); free(ctx); free(pe); free(pm); free(bd); free(bds); free(ac);
    free(sc); free(gt); free(dw);
    return 0;
}
