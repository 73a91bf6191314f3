/*
 * oracle.h -- CPU restatement of xdna-engine's host math for the fused transformer
 * hot path.  TEST INFRASTRUCTURE ONLY: the parity tests, `__graft_entry__.smoke()` and
 * the `cpu_baseline` / `--impl reference` legs of bench.py link this library as the
 * checker.  The product (libxdna_b200.so) never links, loads or calls it.
 *
 * Every function names the reference file:line it restates (paths are relative to the
 * xdna-engine source tree).  The reference is Rust (no toolchain here) plus numpy
 * goldens, so this is a restatement, not a build of the reference; it is pinned against
 * the reference's own known-answer tests and numpy goldens (tests/golden/).
 */
#ifndef XDNA_ORACLE_H
#define XDNA_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 (rust/npu-xrt/src/lib.rs:809-818, rust/npu-asr-host/src/lib.rs:12-19) ---- */
uint16_t or_f32_to_bf16_bits(float x);
float or_bf16_bits_to_f32(uint16_t b);
float or_bf16_round(float x);
void or_bf16_round_n(const float *x, float *y, size_t n);
void or_f32_to_bf16_n(const float *x, uint16_t *y, size_t n);

/* ---- int8 weight quantisation ---------------------------------------------------- */
/* per-output-column symmetric int8 of a [K,N] row-major weight, f32::round (half away
 * from zero): rust/npu-whisper/src/bin/opt125m_decode.rs:41-60 */
void or_quant_i8_cols(const float *w, int K, int N, int8_t *q, float *scale);
/* per-output-row int8 of an [M,K] weight with np.round (half to even):
 * route_b_kernels/decode_fused/gen_decode.py:158-165 (qrow) */
void or_quant_i8_rows(const float *w, int M, int K, int8_t *q, float *scale);
/* int8 GEMV exactly as Lin::fwd (opt125m_decode.rs:106-124): k-outer, f32 mul+add */
void or_lin_i8_fwd(const float *x, const int8_t *q, const float *scale, const float *bias,
                   int K, int N, float *y);

/* ---- bfp16ebs8 block format (route_b_kernels/ffn_bfp16/golden_ffn_gemm.py:25-60) ---- */
/* quantise `n` values in blocks of 8 (n % 8 == 0) -> fp32 values on the block grid */
void or_bfp16_blocks(const float *x, float *y, size_t n);
/* storage split: shared exponent e (quantum 2^(e-6)) and signed mantissa m (int16:
 * the reference does not clamp, so |m| can reach 128) */
void or_bfp16_pack(const float *x, size_t n, int16_t *mant, int8_t *exp);

/* ---- norms -------------------------------------------------------------------------- */
/* rust/npu-asr-host/src/lib.rs:79-110 (population var, f32 index-order sums) */
void or_layer_norm(const float *x, const float *g, const float *b, int T, int D, float eps,
                   float *y);
/* rust/npu-asr/src/ctx_decode.rs:617-640: the f64 input normalisation of fused_norm_gemv */
void or_ln_normalize_f64(const float *x, int K, float eps, float *y);
void or_rms_normalize_f64(const float *x, int K, float eps, float *y);
/* rust/npu-gemma/src/lib.rs:55-64: x * rsqrt(mean(x^2)+eps) * (1+w) */
void or_gemma_rmsnorm(const float *x, const float *w, int D, float eps, float *y);

/* ---- activations ---------------------------------------------------------------------- */
float or_fast_exp_nonpos(float x);                 /* npu-asr-host/src/lib.rs:38-58 */
float or_gelu_erf(float x);                        /* npu-asr-host/src/lib.rs:464-495 */
float or_gelu_tanh(float x);                       /* gen_decode.py:509, npu-gemma lib.rs:68-77 */
float or_sigmoid(float x);                         /* npu-asr-host/src/lib.rs:401-409 */
float or_silu(float x);

/* ---- attention ------------------------------------------------------------------------ */
/* npu-asr-host/src/lib.rs:189-326: q,k,v [T, H*hd]; keys j >= valid_len masked */
void or_mha(const float *q, const float *k, const float *v, int T, int H, int hd,
            int round_probs, int valid_len, float *out);
/* route_b_kernels/mha_decode/mha_decode.cc:90-168: single-query online softmax over
 * a head's keys in tiles of `tkv` (the tile order the device kernel also follows) */
void or_mha_tile_online(const float *q, const float *k, const float *v, int s, int hd,
                        float scale, float *ctx);

/* ---- greedy selection (rust/npu-whisper/src/bin/opt125m_decode.rs:303; whisper.rs:749-757) */
int64_t or_argmax_last(const float *x, size_t n);   /* max_by(partial_cmp): last max wins */
int64_t or_argmax_first(const float *x, size_t n);  /* strict '>': first max wins */

/* ---- KV indexing (rust/npu-xrt/src/lib.rs:992-1004; whisper_decoder.rs:550-570) ---- */
uint32_t or_kv_byte_offset(uint32_t base, uint32_t n_preceding, uint32_t head_dim);
uint32_t or_softmax_len(uint32_t n_preceding);
/* paged layout used by the device: page = [K|V][H][page_tokens][hd] bf16 */
size_t or_paged_kv_index(const int32_t *page_table, int page_tokens, int H, int hd,
                         int kv, int head, int pos, int d);

/* ---- fixed-point activation limbs (device GEMV numerics; defined by this engine) ---- */
/* x -> X = rint(x * 2^s) with s = 22 - E, max|x| < 2^E; X = a*2^16 + b*2^8 + c,
 * a,b,c in [-128,127].  Returns s. */
int or_limbs(const float *x, int K, int8_t *a, int8_t *b, int8_t *c);
/* exact int8 dot of a limbed activation with an int8 weight column, rounded once to f32,
 * then * scale + bias (separate f32 multiply and add). */
void or_gemv_i8_exact(const float *x, const int8_t *wq_nk, const float *scale,
                      const float *bias, int K, int N, float *y);

/* ---- opt-125m greedy decode (rust/npu-whisper/src/bin/opt125m_decode.rs:252-315) ---- */
typedef struct {
    int n_layers, d_model, n_heads, head_dim, ffn, vocab, max_pos;
    float eps;
} or_opt_cfg;

typedef struct {               /* layouts follow the reference's npy arrays */
    const float *ln1_w, *ln1_b;          /* [D] */
    const float *wq, *wk, *wv, *wo;      /* [D, D] as [K, N] */
    const float *bq, *bk, *bv, *bo;      /* [D] */
    const float *ln2_w, *ln2_b;          /* [D] */
    const float *w1, *b1;                /* [D, F], [F] */
    const float *w2, *b2;                /* [F, D], [D] */
} or_opt_layer;

typedef struct {
    const float *emb_tok;      /* [V, D]; the LM head is tied: logits = x . emb_tok[v] */
    const float *emb_pos;      /* [max_pos + 2, D] (position offset +2) */
    const float *lnf_w, *lnf_b;
    const or_opt_layer *layers;
} or_opt_weights;

enum {
    OR_MODE_REF_F32 = 0,  /* the reference host path with OPT_INT8: f32 activations, int8
                             Lin layers, f32 LM head (opt125m_decode.rs:106-124, 252-293) */
    OR_MODE_DEVICE = 1,   /* the B200 engine's numerics: bf16 activations into every GEMV,
                             bf16 KV cache, exact limbed int8 GEMV, int8 LM head */
    OR_MODE_F32 = 2       /* the reference host path without OPT_INT8: every Lin is the f32
                             x.W + b (opt125m_decode.rs:125-128); used to pin the model
                             composition against the HF OPT implementation */
};

typedef struct or_opt or_opt;
or_opt *or_opt_create(const or_opt_cfg *cfg, const or_opt_weights *w, int mode, int nthreads);
void or_opt_free(or_opt *m);
/* prefill prompt token by token, then greedy-decode n_new tokens (Opt::generate).
 * force_ids (optional, [n_new]) replaces the fed-back argmax by force_ids[g] (teacher
 * forcing); out_ids still receives each step's argmax.  logits_out (optional) receives
 * the logits of each step, [n_new, V].  Returns 0, or -1 on bad sizes. */
int or_opt_generate(or_opt *m, const int64_t *prompt, int n_prompt, int n_new,
                    const int64_t *force_ids, int64_t *out_ids, float *logits_out);
/* debugging aid: record x after each attention / FFN residual add and the final LN output
 * (device mode) per position into trace[pos][2L+1][D]; NULL turns it off */
void or_opt_set_trace(or_opt *m, float *trace);
/* one Opt::step (opt125m_decode.rs:252-293) with the LM head at `pos`; returns the argmax */
int64_t or_opt_step(or_opt *m, int64_t id, int pos, float *logits_out);
/* quantised weights as the engine sees them (for bit-exact checks) */
const int8_t *or_opt_qweight(const or_opt *m, int layer, int which, float const **scale);

/* ---- BGE / BERT embedder (rust/npu-engine/src/bert/{frontend,encoder,head}.rs) ---- */
typedef struct {
    int n_layers, d_model, n_heads, ffn, vocab, max_pos;
    float eps;
    int pooling;               /* 0 CLS, 1 mean */
} or_bert_cfg;
typedef struct {               /* linear weights [K, N] */
    const float *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *o_w, *o_b;
    const float *attn_ln_w, *attn_ln_b;
    const float *ffn1_w, *ffn1_b, *ffn2_w, *ffn2_b;
    const float *out_ln_w, *out_ln_b;
} or_bert_layer;
typedef struct {
    const float *word_emb, *pos_emb, *type_emb, *emb_ln_w, *emb_ln_b;
    const or_bert_layer *layers;
} or_bert_weights;
/* embeddings [n_seqs, D] of the token-id sequences (concatenated ids, seq_lens each) */
int or_bert_embed(const or_bert_cfg *c, const or_bert_weights *w, const int32_t *ids,
                  const int32_t *seq_lens, int n_seqs, float *out, int nthreads);

/* ---- Whisper-small encoder (rust/npu-whisper/src/encoder.rs:183-375) ---- */
typedef struct {
    int n_layers, d_model, n_heads, ffn, n_mels, n_frames, max_src;
    float eps;
} or_whisper_enc_cfg;
typedef struct {
    const float *ln1_w, *ln1_b, *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *out_w, *out_b;
    const float *ln2_w, *ln2_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
} or_whisper_enc_layer;
typedef struct {
    const float *conv1_w, *conv1_b, *conv2_w, *conv2_b, *embed_positions, *ln_post_w, *ln_post_b;
    const or_whisper_enc_layer *layers;
} or_whisper_enc_weights;
/* mel [B][n_mels][n_frames] -> out [B][n_frames/2][d_model] */
int or_whisper_encode(const or_whisper_enc_cfg *c, const or_whisper_enc_weights *w, const float *mel,
                      int B, float *out, int nthreads);

/* ---- Parakeet FastConformer encoder (rust/npu-parakeet/src/encoder.rs, ops.rs, pos.rs) ---- */
typedef struct {
    int n_layers, d_model, n_heads, ffn, n_mels, n_frames, sub_ch, kconv;
    int int8;   /* 1: the int8 GEMM engine rule for every weight linear; 0: f32 host path */
} or_parakeet_cfg;
typedef struct {
    const float *ff1_ln_w, *ff1_ln_b, *ff1_w1, *ff1_w2;             /* w1 [D, F], w2 [F, D] ([in, out]) */
    const float *att_ln_w, *att_ln_b, *wq, *wk, *wv, *wpos, *wout;  /* [D, D] */
    const float *pos_u, *pos_v;                                     /* [H, dk] */
    const float *conv_ln_w, *conv_ln_b, *pw1, *dw_w, *dw_b, *pw2;   /* pw1 [D, 2D], dw_w [D, k], pw2 [D, D] */
    const float *ff2_ln_w, *ff2_ln_b, *ff2_w1, *ff2_w2;
    const float *out_ln_w, *out_ln_b;
} or_parakeet_layer;
typedef struct {
    const float *c0_w, *c0_b, *c2_w, *c2_b, *c3_w, *c3_b, *c5_w, *c5_b, *c6_w, *c6_b;  /* conv [Co, Ci/g, kh, kw] */
    const float *out_w, *out_b;                                     /* [C * F/8, D], [D] */
    const or_parakeet_layer *layers;
} or_parakeet_weights;
/* mel [B][n_mels][n_frames] -> out [B][T'][d_model], T' = n_frames subsampled 8x */
int or_parakeet_encode(const or_parakeet_cfg *c, const or_parakeet_weights *w, const float *mel, int B,
                       float *out, int nthreads);
void or_parakeet_quant_lin(const float *x, int T, int K, const float *w, const float *bias, int N, float *y,
                           int nthreads);
void or_conv2d(const float *x, int ci, int hin, int win, const float *w, const float *b, int co, int kh, int kw,
               int stride, int pad, int groups, float *y, int nthreads);
void or_dwconv1d(const float *x, int C, int T, const float *taps, const float *bias, int k, float *y);
void or_rel_shift(const float *bd, int H, int T, float *out);
void or_rel_pos_encoding(int T, int D, float *pe);

/* ---- Whisper-small greedy decoder (rust/npu-engine/src/asr/whisper_decoder.rs:388-560) ---- */
typedef struct {
    int n_layers, d_model, n_heads, ffn, vocab, max_tgt, n_enc;
} or_whisper_dec_cfg;
typedef struct {               /* linear weights [K, N] = [in, out] */
    const float *ln_self_w, *ln_self_b, *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *out_w, *out_b;
    const float *ln_cross_w, *ln_cross_b, *cross_q_w, *cross_q_b, *cross_k_w, *cross_k_b;
    const float *cross_v_w, *cross_v_b, *cross_out_w, *cross_out_b;
    const float *ln_final_w, *ln_final_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
} or_whisper_dec_layer;
typedef struct {
    const float *embed_tokens, *embed_positions, *proj_out, *ln_post_w, *ln_post_b;  /* proj_out [D, V] */
    const or_whisper_dec_layer *layers;
} or_whisper_dec_weights;
/* enc [B][n_enc][d_model]; the same prompt for every stream; out_tokens [B][n_new],
 * logits (nullable) [B][n_new][vocab]; force (nullable, [B][n_new]): feed force[b][g] after
 * step g instead of the argmax (teacher forcing), so logits stay comparable across numerics */
int or_whisper_decode(const or_whisper_dec_cfg *c, const or_whisper_dec_weights *w, const float *enc, int B,
                      const int64_t *prompt, int n_prompt, int n_new, int64_t *out_tokens, float *logits,
                      int nthreads, const int64_t *force);

/* ---- Gemma-3 text decoder (npu-gemma pieces + the HF Gemma-3 model they port) ---- */
typedef struct {
    int n_layers, d_model, n_q_heads, head_dim, ffn, vocab, window, pattern;
    float theta_local, theta_global, query_pre_attn_scalar, eps;
    int int8;            /* 1: int8 per-channel linears + LM head (Lin rule) */
} or_gemma_cfg;
typedef struct {         /* [K, N] = [in, out]; one KV head */
    const float *in_norm, *wq, *wk, *wv, *q_norm, *k_norm, *wo, *post_attn_norm;
    const float *pre_ffn_norm, *wg, *wu, *wd, *post_ffn_norm;
} or_gemma_layer;
typedef struct {
    const float *embed, *final_norm;      /* embed [V, D], tied LM head */
    const or_gemma_layer *layers;
} or_gemma_weights;
/* force (nullable, [n_new]): teacher forcing as for or_whisper_decode */
int or_gemma_decode(const or_gemma_cfg *c, const or_gemma_weights *w, const int64_t *prompt, int n_prompt,
                    int n_new, int64_t *out_tokens, float *logits, int nthreads, const int64_t *force);
float or_gelu_tanh_gemma(float x);

#ifdef __cplusplus
}
#endif
#endif
