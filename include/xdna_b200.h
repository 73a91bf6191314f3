/*
 * xdna_b200.h -- C ABI of the B200 backend for xdna-engine's fused transformer hot path.
 *
 * This library replaces the reference's device layer (rust/npu-xrt: shim/xrt_shim.h:16-113,
 * src/lib.rs:46-158, 641-744) for the decode hot path.  Conventions follow the reference's C
 * ABIs (rust/npu-capi/src/lib.rs:11-16, rust/npu-xrt/shim/xrt_shim.h:1-3): opaque handles,
 * NULL / nonzero return on failure, and a thread-local message readable with
 * xdna_last_error() until the next call on the same thread.  No entry point throws across
 * the boundary.  Plain pointers and sizes only.
 *
 * Pointers documented as "device" must be CUDA device pointers; all others are host memory.
 * `stream` arguments are cudaStream_t values passed as void* (NULL = the legacy stream).
 */
#ifndef XDNA_B200_H
#define XDNA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- device (npu-xrt Device) */
typedef struct XdnaDevice XdnaDevice;

/* Number of usable sm_100 devices (0 if none).  Replaces shim_device_open's probe and
 * npu_available (rust/npu-capi/src/lib.rs:22-25). */
int xdna_device_count(void);
/* Open device `ordinal`; NULL on error.  Replaces shim_device_open (xrt_shim.h:16). */
XdnaDevice *xdna_device_open(int ordinal);
void xdna_device_close(XdnaDevice *dev);
/* Thread-local last error ("" if none).  Replaces shim_last_error (xrt_shim.h:113). */
const char *xdna_last_error(void);

/* ------------------------------------------------- weight quantisation (npu-weights / Lin) */
/* Per-output-column symmetric int8 of a [K,N] row-major f32 weight, exactly Lin::load with
 * OPT_INT8 (rust/npu-whisper/src/bin/opt125m_decode.rs:41-60): scale[n] = max_k|W[k,n]|/127
 * (1.0 for an all-zero column), q = clamp(round_half_away(W/scale), -127, 127).  The result is
 * written output-major, q_nk[n*K + k].  Returns 0. */
int xdna_quant_i8_cols(const float *w, int K, int N, int8_t *q_nk, float *scale);
/* qrow, the fused decode ELF's per-output-row int8 rule (route_b_kernels/decode_fused/
 * gen_decode.py:158-165): w [M, K] -> q [M, K], scale [M]; max|row|/127 (1.0 if zero), round
 * half to even, clip +-127.  q and scale feed xdna_gemv_i8 as q_nk / scale.  Host only. */
int xdna_quant_i8_rows(const float *w, int M, int K, int8_t *q, float *scale);

/* ------------------------------------------------------------- op level (CtxDecode::gemv) */
/* y[N] = dot(x, W[:,n]) * scale[n] + bias[n] on the GPU with the engine's exact int8 GEMV
 * (activation as a 22-bit fixed-point vector split into int8 limbs, int8 tensor-core MMA,
 * exact integer accumulation, one rounding).  Replaces CtxDecode::gemv / fused_norm_gemv's
 * device dispatch (rust/npu-asr/src/ctx_decode.rs:325-369, 617-643).  x, q_nk, scale, bias
 * (nullable) and y are host arrays; K must be a multiple of 256 and <= 3072, N a multiple
 * of 8.  Returns 0, or -1 with xdna_last_error() set. */
int xdna_gemv_i8(XdnaDevice *dev, const float *x, int K, const int8_t *q_nk, const float *scale,
                 const float *bias, int N, float *y);

/* The same GEMV for callers that cannot allocate device memory -- a host whose device
 * memory belongs to another allocator (a framework's caching allocator, an arena reserved at
 * start-up) where a cudaMalloc would fail or fragment the pool.  It has no counterpart in the
 * reference.  Arguments and result are those of xdna_gemv_i8, on device ordinal `device`;
 * instead of cudaMalloc'd staging it uses one fixed 8 MiB __device__ array that every GPU
 * loading this library keeps until exit, so the call allocates nothing.  Calls whose staging
 * (about 2*N*K + 12*N + 4*K bytes) exceeds 8 MiB are rejected with an error.  The first call
 * on a device looks up the array's address and should come before any stream capture.  All
 * calls share the array: calls that overlap on the GPU race and must be serialised.
 * Synchronous; returns 0, or -1 with xdna_last_error() set. */
int xdna_gemv_i8_noalloc(int device, const float *x, int K, const int8_t *q_nk,
                         const float *scale, const float *bias, int N, float *y);

/* ------------------------------------------- encoder GEMM (CtxAOp::forward / FfnMm2) */
/* C[M, N] = epi(A[M, K] . B[N, K]^T) on the tcgen05 tensor cores: bf16 operands (device, row
 * major, A rows = tokens, B = weight [out, in]), f32 accumulation, epilogue + bias[N] (f32,
 * nullable), then the exact-erf GELU if gelu != 0 (the reference's form,
 * npu-asr-host/src/lib.rs:464-495), then + residual[M, N] (bf16, nullable); C bf16 [M, N].
 * Replaces the reference's resident-GEMM dispatch + host epilogue (rust/npu-asr/src/
 * ctx2.rs:674-770, 1195-1288; npu-engine/src/bert/encoder.rs:43-57).  Needs N % 256 == 0,
 * K % 64 == 0 and 16-byte aligned rows.  Asynchronous on `stream`; 0 or -1. */
int xdna_gemm_bf16(const uint16_t *A, const uint16_t *B, const float *bias, const uint16_t *residual,
                   uint16_t *C, int M, int N, int K, int gelu, void *stream);
/* The int8 encoder GEMM on the tcgen05 tensor cores (kind::i8, exact s32 accumulation in
 * TMEM) with the reference's dequant epilogue (rust/npu-asr/src/ctx2.rs forward_view_int8
 * 771-829, dequant_epi 1386-1411): A int8 [M, K] quantised per clip with scale sa[clip]
 * (clip = row / rows_per_clip), B int8 weight [N, K] with per-output-channel scales ws[N];
 * y = (float(acc) * sa) * ws[n] (+ bias[n], nullable); act 0 none, 1 SiLU
 * (v * (1 / (1 + e^-v))), 3 GLU over interleaved column pairs (2c value, 2c + 1 gate) ->
 * y[2c] * sigmoid(y[2c + 1]) at column c; then C = residual + alpha * y (residual f32,
 * nullable, may equal C); C f32 [M, N] (N / 2 columns for GLU).  amax (nullable, [clips]
 * uint32): atomically raised to the bit pattern of each clip's max |C|, the next layer's
 * activation scale.  Needs N % 256 == 0, K % 128 == 0.  Asynchronous on `stream`; 0 or -1. */
int xdna_gemm_i8(const int8_t *A, const int8_t *B, const float *sa, int rows_per_clip, const float *ws,
                 const float *bias, int act, const float *residual, float alpha, float *C,
                 unsigned *amax, int M, int N, int K, void *stream);
/* After the stream has finished: -1 (with xdna_last_error) if a GEMM's bounded wait expired
 * since the last check, else 0. */
int xdna_gemm_check(void);
/* The fused two-GEMM FFN with the hidden activations kept on chip (ffn_gemm2,
 * route_b_kernels/ffn_gemm2/ffn_gemm2_iron.py:1-30, with the encoder FFN's bias and activation
 * between the GEMMs): out[M, N] = act(A[M, K] . W1[P, K]^T + b1) . W2[N, P]^T (+ b2) (+ residual).
 * bf16 operands (row-major, K-major weights as nn.Linear stores them), f32 accumulation, the
 * hidden rounded to bf16 on chip (as the unfused path rounds it in HBM).  act: 0 none, 1
 * exact-erf GELU (the reference's Abramowitz-Stegun form), 2 ReLU.  b1, b2, residual ([M, N]
 * bf16) nullable; exactly one of out_bf16 / out_f32.  K % 64 == 0, P % 256 == 0, N % 64 == 0,
 * N <= 768.  Asynchronous on `stream`; xdna_ffn_fused_check reports a bounded wait that expired. */
int xdna_ffn_fused_bf16(const uint16_t *A, const uint16_t *W1, const float *b1, int act, const uint16_t *W2,
                        const float *b2, const uint16_t *residual, uint16_t *out_bf16, float *out_f32, int M, int K,
                        int P, int N, void *stream);
int xdna_ffn_fused_check(void);
/* Encoder self-attention, 12 heads of 64, on the tcgen05 tensor cores: the reference's `mha`
 * with valid_len (rust/npu-asr-host/src/lib.rs:189-326) over packed sequences.  qkv
 * [T_total, 2304] bf16 (q | k | v per row, head h at columns 64 h of each), cu [n_seqs + 1]
 * int32 device offsets of the sequences, max_len >= the longest; ctx [T_total, 768] bf16 =
 * softmax(q k^T / 8) v over each sequence's own keys.  Asynchronous on `stream`;
 * xdna_attention_check reports a bounded wait that expired. */
int xdna_attention_bf16(const uint16_t *qkv, int T_total, const int32_t *cu, int n_seqs, int max_len, uint16_t *ctx,
                        void *stream);
int xdna_attention_check(void);
/* diagnostics: globaltimer stamps of the first CTA into trace_dev ([512] u64), NULL for none */
void xdna_attention_set_trace(unsigned long long *trace_dev);
/* diagnostics: globaltimer stamps of the first cluster's two CTAs into trace_dev ([2][1024] u64,
 * slot 16 c + k for chunk c), or NULL (the default) for none */
void xdna_ffn_fused_set_trace(unsigned long long *trace_dev);

/* ------------------------------------------------ BGE / BERT embeddings (EmbedPipeline) */
typedef struct {
    int n_layers, d_model, n_heads, ffn, vocab, max_pos;
    float eps;                 /* LayerNorm eps (BERT: 1e-12) */
    int pooling;               /* 0 = CLS row, 1 = mean over valid rows (bert/head.rs:20-47);
                                  + 2: skip the L2 normalisation (EmbedHead normalize = false) */
} XdnaBertConfig;

typedef struct {               /* f32, linear weights [K, N] = [in, out] */
    const float *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *o_w, *o_b;
    const float *attn_ln_w, *attn_ln_b;
    const float *ffn1_w, *ffn1_b, *ffn2_w, *ffn2_b;
    const float *out_ln_w, *out_ln_b;
} XdnaBertLayer;

typedef struct {
    const float *word_emb;     /* [vocab, D] */
    const float *pos_emb;      /* [max_pos, D] */
    const float *type_emb;     /* [>= 1, D]; row 0 is used (single segment) */
    const float *emb_ln_w, *emb_ln_b;
    const XdnaBertLayer *layers;
} XdnaBertWeights;

typedef struct XdnaBert XdnaBert;

/* Load a BERT-base-shaped embedder (d_model 768, 12 heads, ffn 3072): weights are rounded to
 * bf16 and kept resident on the current device; buffers hold up to max_tokens packed tokens
 * and max_seqs sequences.  Replaces Model::load for an embed scenario (rust/npu-engine/src/
 * api.rs:44-100, bert/mod.rs:24-46).  NULL on error. */
XdnaBert *xdna_bert_create(XdnaDevice *dev, const XdnaBertConfig *cfg, const XdnaBertWeights *w,
                           int max_tokens, int max_seqs);
void xdna_bert_free(XdnaBert *m);
/* Embed n_seqs token-id sequences (ids concatenated, seq_lens[s] tokens each, [CLS] first):
 * frontend (word + position + type-0, LayerNorm), the encoder blocks, then pooling + L2 --
 * EmbedPipeline::embed without the tokenizer (bert/frontend.rs:37-61, encoder.rs:43-57,
 * head.rs:20-47).  Host in, host out ([n_seqs, 768] f32).  Returns 0 or -1. */
int xdna_bert_embed(XdnaBert *m, const int32_t *ids, const int32_t *seq_lens, int n_seqs, float *out);
/* Device-resident form: ids / tok_pos [n_tokens] (position of each token in its sequence),
 * cu [n_seqs + 1] sequence starts, out_dev [n_seqs, 768]; asynchronous on `stream`. */
int xdna_bert_encode_device(XdnaBert *m, const int32_t *ids, const int32_t *tok_pos, const int32_t *cu,
                            int n_tokens, int n_seqs, int max_len, float *out_dev, void *stream);

/* The embedding front end on its own, host only: the token ids npu_embed (include/npu_engine.h)
 * feeds the encoder for `text` -- BERT uncased WordPiece over the vocabulary of tokenizer_path
 * (HuggingFace tokenizer.json with a WordPiece model, or vocab.txt), [CLS] ... [SEP], truncated
 * to max_len (rust/npu-engine/src/bert/frontend.rs:29-35).  Writes min(count, cap) ids and
 * returns the count, or -1 with npu_last_error() set. */
int xdna_wordpiece_encode(const char *tokenizer_path, const char *text, int max_len, int32_t *ids, int cap);

/* ------------------------------------------------------------- bfp16 block format */
/* to_bfp16_blocks of the reference's golden (route_b_kernels/ffn_bfp16/golden_ffn_gemm.py:
 * 34-49) over contiguous blocks of 8: shared exponent floor(log2(max|x|)), quantum 2^(e-6),
 * round half to even, no clamp.  n % 8 == 0.  Returns 0 or -1. */
int xdna_bfp16_quantize(const float *x, size_t n, float *y);

/* -------------------------------------------- Whisper-small encoder (WhisperEncoder) */
typedef struct {
    int n_layers, d_model, n_heads, ffn;
    int n_mels, n_frames;      /* input mel [n_mels, n_frames]; output n_frames / 2 rows */
    int max_src;               /* rows of embed_positions */
    float eps;                 /* LayerNorm eps (Whisper: 1e-5) */
} XdnaWhisperEncConfig;

typedef struct {               /* f32; linear weights [K, N] = [in, out]; k_b may be NULL */
    const float *ln1_w, *ln1_b;
    const float *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *out_w, *out_b;
    const float *ln2_w, *ln2_b;
    const float *fc1_w, *fc1_b, *fc2_w, *fc2_b;
} XdnaWhisperEncLayer;

typedef struct {
    const float *conv1_w, *conv1_b;   /* [d_model, n_mels, 3], [d_model] */
    const float *conv2_w, *conv2_b;   /* [d_model, d_model, 3] */
    const float *embed_positions;     /* [max_src, d_model] */
    const float *ln_post_w, *ln_post_b;
    const XdnaWhisperEncLayer *layers;
} XdnaWhisperEncWeights;

typedef struct XdnaWhisperEnc XdnaWhisperEnc;

/* Load the encoder (d_model 768, 12 heads, ffn 3072): linear weights quantised to bfp16
 * along K, conv weights and positions bf16; up to max_batch clips per call.  Replaces
 * WhisperEncoder's weights + conv_stem / block / forward_last (rust/npu-whisper/src/
 * encoder.rs:183-375).  NULL on error. */
XdnaWhisperEnc *xdna_whisper_enc_create(XdnaDevice *dev, const XdnaWhisperEncConfig *cfg,
                                        const XdnaWhisperEncWeights *w, int max_batch);
void xdna_whisper_enc_free(XdnaWhisperEnc *m);
/* mel [B][n_mels][n_frames] f32 (host) -> encoder states [B][n_frames/2][768] f32 (host). */
int xdna_whisper_encode(XdnaWhisperEnc *m, const float *mel, int B, float *out);
/* Device-resident form: mel_dev f32, out_dev bf16 [B][n_frames/2][768]; async on `stream`. */
int xdna_whisper_encode_device(XdnaWhisperEnc *m, const float *mel_dev, int B, uint16_t *out_dev,
                               void *stream);

/* ------------------------------------------------ opt-125m greedy decode (Opt::generate) */
typedef struct {
    int n_layers, d_model, n_heads, head_dim, ffn, vocab, max_pos;
    float eps;
} XdnaOptConfig;

typedef struct {               /* f32, the reference's npy layouts: linear weights [K, N] */
    const float *ln1_w, *ln1_b;
    const float *wq, *wk, *wv, *wo;
    const float *bq, *bk, *bv, *bo;
    const float *ln2_w, *ln2_b;
    const float *w1, *b1;      /* [D, F], [F] */
    const float *w2, *b2;      /* [F, D], [D] */
} XdnaOptLayer;

typedef struct {
    const float *emb_tok;      /* [V, D]; tied LM head */
    const float *emb_pos;      /* [max_pos + 2, D]; position offset +2 */
    const float *lnf_w, *lnf_b;
    const XdnaOptLayer *layers;
} XdnaOptWeights;

typedef struct XdnaOptDecoder XdnaOptDecoder;

/* Quantise (int8, per output channel, LM head included), pack and upload the model; the
 * replacement of Opt::load + Lin::load (opt125m_decode.rs:41-60, 158-186).  max_ctx bounds
 * prompt + generated tokens (<= max_pos); grid = CTAs of the persistent kernel (0 = one per
 * SM).  Requires head_dim 64, d_model <= 1024 and a multiple of 256, ffn <= 3072 and a
 * multiple of 256.  NULL on error. */
XdnaOptDecoder *xdna_opt_create(XdnaDevice *dev, const XdnaOptConfig *cfg,
                                const XdnaOptWeights *w, int max_ctx, int grid);
void xdna_opt_free(XdnaOptDecoder *dec);

/* Opt::generate (opt125m_decode.rs:296-315): prefill `prompt` token by token, then greedily
 * decode n_new tokens (ties -> the last maximal logit, as max_by(partial_cmp)).  Host in,
 * host out, synchronous.  out_logits (nullable) receives [n_new, V] f32: the logits that
 * chose each generated token.  Returns 0, or -1 with xdna_last_error() set. */
int xdna_opt_generate(XdnaOptDecoder *dec, const int64_t *prompt, size_t n_prompt, size_t n_new,
                      int64_t *out_ids, float *out_logits);

/* Asynchronous, device-resident form used for streaming decode and timing.
 * The decoder owns a device token array `tokens[max_ctx + 1]` (xdna_opt_tokens_device).
 * xdna_opt_launch runs positions start_pos .. start_pos + n_steps - 1 in ONE kernel launch:
 * position p feeds tokens[p] when p < n_prompt or when it is the first step of the launch,
 * otherwise the id it generated itself; every step at p >= n_prompt - 1 writes its greedy
 * id to tokens[p + 1] and, if logits_dev is non-NULL, its logits to
 * logits_dev[(p - max(start_pos, n_prompt - 1)) * V ...].  Positions must be launched in
 * order: the KV cache of positions < start_pos must come from earlier launches. */
int64_t *xdna_opt_tokens_device(XdnaOptDecoder *dec);
/* Copy n token ids between host memory and tokens[off .. off+n) on `stream` (asynchronous
 * when the host buffer is pinned).  Returns 0, or -1 on a bad range. */
int xdna_opt_set_tokens(XdnaOptDecoder *dec, const int64_t *host, size_t off, size_t n,
                        void *stream);
int xdna_opt_get_tokens(XdnaOptDecoder *dec, int64_t *host, size_t off, size_t n, void *stream);
int xdna_opt_launch(XdnaOptDecoder *dec, int start_pos, int n_steps, int n_prompt,
                    float *logits_dev, void *stream);
/* Prompt prefill as a batch (replaces stepping the prompt through Opt::step,
 * rust/npu-whisper/src/bin/opt125m_decode.rs:296-315): writes the K / V rows of positions
 * start_pos .. start_pos + n - 1 for tokens[] already on the device, up to 32 positions per
 * launch sequence, with exactly the decode kernel's arithmetic (the cache, and every later
 * token, are bit-identical to launching those positions).  No LM head: follow with
 * xdna_opt_launch from start_pos + n.  Asynchronous on `stream`; bad token ids are reported by
 * xdna_opt_sync.  xdna_opt_generate uses it for all prompt positions but the last.  It uses the
 * decoder's own scratch (split-K sums, counters), so a decoder takes one prefill or launch at a
 * time, on one stream.  Returns 0, or -1 (also when the decoder was created with
 * XDNA_OPT_PREFILL=0). */
int xdna_opt_prefill(XdnaOptDecoder *dec, int start_pos, int n, void *stream);
/* Wait for the decoder's launches on `stream` and report a device-side failure (bounded
 * waits that expired).  Returns 0, or -1 with xdna_last_error() set. */
int xdna_opt_sync(XdnaOptDecoder *dec, void *stream);
/* Bytes of weights one decoded token streams from HBM (int8 rows + per-row scale/bias). */
size_t xdna_opt_stream_bytes_per_token(const XdnaOptDecoder *dec);
int xdna_opt_grid(const XdnaOptDecoder *dec);
/* the configuration the decoder was created with (for one made by xdna_opt_load) */
int xdna_opt_config(const XdnaOptDecoder *dec, XdnaOptConfig *out);
/* Debugging aid: when trace_dev (device, [n_steps][2*n_layers+1][d_model] f32) is non-NULL,
 * later launches record the residual stream after each attention and each FFN residual add,
 * then the final LayerNorm output, per step of the launch.  NULL turns it off. */
int xdna_opt_set_trace(XdnaOptDecoder *dec, float *trace_dev);
/* Profiling aid: when timing_dev (device, [2][grid][128] u64) is non-NULL, the first two steps
 * of later launches record the global nanosecond timer per CTA at each phase boundary (slot 0
 * token start, 1 + 5*layer + {0 qkv, 1 attention, 2 out-proj, 3 fc1, 4 fc2} after the phase's
 * outputs are published, 5*n_layers + 1 after the LM head, + 2 once the greedy id is known). */
int xdna_opt_set_timing(XdnaOptDecoder *dec, unsigned long long *timing_dev);

/* ------------------------------------------- Whisper-small greedy decoder (HostDecoder) */
/* Replaces rust/npu-engine/src/asr/whisper_decoder.rs HostDecoder (precompute_cross 388-399,
 * step 401-560) and the fused per-token decode ELF (route_b_kernels/decode_fused/gen_decode.py)
 * with the device lm-head + argmax (gen_projout.py, argmax_slice.cc; whisper.rs:749-757 first
 * maximum).  Linear weights and proj_out are quantised to the reference's bfp16 blocks
 * (golden_ffn_gemm.py:34-49) along K.  1..32 streams decode in lockstep after one shared
 * prompt.  Shapes: d_model 768, 12 heads, ffn 3072, max_tgt <= 448. */
typedef struct {
    int n_layers, d_model, n_heads, ffn, vocab, max_tgt, n_enc;
} XdnaWhisperDecConfig;
typedef struct {               /* f32; linear weights [K, N] = [in, out]; k biases may be NULL */
    const float *ln_self_w, *ln_self_b, *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *out_w, *out_b;
    const float *ln_cross_w, *ln_cross_b, *cross_q_w, *cross_q_b, *cross_k_w, *cross_k_b;
    const float *cross_v_w, *cross_v_b, *cross_out_w, *cross_out_b;
    const float *ln_final_w, *ln_final_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
} XdnaWhisperDecLayer;
typedef struct {
    const float *embed_tokens, *embed_positions, *proj_out, *ln_post_w, *ln_post_b;  /* proj_out [D, vocab] */
    const XdnaWhisperDecLayer *layers;
} XdnaWhisperDecWeights;
typedef struct XdnaWhisperDec XdnaWhisperDec;
XdnaWhisperDec *xdna_whisper_dec_create(XdnaDevice *dev, const XdnaWhisperDecConfig *cfg,
                                        const XdnaWhisperDecWeights *w, int max_batch);
void xdna_whisper_dec_free(XdnaWhisperDec *m);
/* bfp16 blocks that held both mantissa +128 and -128 (stored with +128 as 127): 251 of the
 * ~15.6 million blocks of the random-init N(0, 0.02) Whisper-small decoder */
long long xdna_whisper_dec_clamped_blocks(const XdnaWhisperDec *m);
/* cross K/V of every layer from encoder states enc_dev [B][n_enc][768] f32 (device); async */
int xdna_whisper_dec_set_encoder(XdnaWhisperDec *m, const float *enc_dev, int B, void *stream);
/* greedy decode of n_new tokens per stream after the prompt (host array); tokens_dev [B][n_new],
 * logits_dev [B][n_new][vocab] (nullable), both device; async on `stream` after a short
 * synchronous staging of the prompt.  The first run of a shape records a CUDA graph of one
 * token, later runs replay it per token. */
int xdna_whisper_dec_run(XdnaWhisperDec *m, int B, const int64_t *prompt_host, int n_prompt, int n_new,
                         int64_t *tokens_dev, float *logits_dev, void *stream);
/* host in / host out: encoder states enc [B][n_enc][768] f32 -> tokens [B][n_new] (+ logits,
 * nullable, [B][n_new][vocab]).  Synchronous. */
int xdna_whisper_dec_generate(XdnaWhisperDec *m, const float *enc_host, int B, const int64_t *prompt, int n_prompt,
                              int n_new, int64_t *tokens_host, float *logits_host);
/* Continuous batching (per-stream positions; the batched decode with per-stream positions and
 * masks that gen_decode_batched.py:3-12 defers): the decoder holds max_batch slots, each with its
 * own cross K/V and self-attention cache.  A stream joins by loading its encoder states into a
 * free slot (set_encoder_slot: enc_dev [n_enc][768] f32 device, asynchronous on `stream`) and
 * feeding its prompt from position 0; every step_slots call runs one decoder step for slots
 * 0 .. n_slots-1, slot b feeding tokens[b] at positions[b] (its own K/V row is written there and
 * its self-attention spans positions 0 .. positions[b]; a negative position marks an empty slot)
 * and returning its greedy next token (first maximum; -1 for an empty slot) in next[b], with the
 * logits rows in logits [n_slots][vocab] when not NULL.  Host arrays; synchronous; the first step
 * of each width is recorded as a CUDA graph.  A stream leaves by simply not being fed. */
int xdna_whisper_dec_set_encoder_slot(XdnaWhisperDec *m, int slot, const float *enc_dev, void *stream);
int xdna_whisper_dec_step_slots(XdnaWhisperDec *m, int n_slots, const int64_t *tokens, const int *positions,
                                int64_t *next, float *logits);

/* ------------------------------------------------------------ Gemma-3 text decoder */
/* The reference has no Gemma decode step (rust/npu-gemma/src/lib.rs:30-43 maps what to reuse:
 * rmsnorm_ref 55-64, geglu_ref 68-77, config.rs GEMMA3_1B, is_global_layer 131-133); this is
 * the HF Gemma-3 text model on those pieces, with the reference's int8 Lin rule
 * (opt125m_decode.rs:41-60) for every linear and the tied LM head.  1..64 streams decode in
 * lockstep; tensor parallel over tp_size GPUs (one process per GPU, same calls on every
 * rank): q heads, FFN columns and LM-head vocabulary rows are split, partial sums are
 * all-reduced in rank order over peer memory (xdna_gemma_ipc_handle / xdna_gemma_connect). */
typedef struct {
    int n_layers, d_model, n_q_heads, head_dim, ffn, vocab, window, pattern;
    float theta_local, theta_global, query_pre_attn_scalar, eps;
} XdnaGemmaConfig;
typedef struct {               /* f32, [K, N] = [in, out]; norm weights are the (1 + w) offsets */
    const float *in_norm, *wq, *wk, *wv, *q_norm, *k_norm, *wo, *post_attn_norm;
    const float *pre_ffn_norm, *wg, *wu, *wd, *post_ffn_norm;
} XdnaGemmaLayer;
typedef struct {
    const float *embed, *final_norm;           /* embed [vocab, d_model], tied LM head */
    const XdnaGemmaLayer *layers;
} XdnaGemmaWeights;
typedef struct XdnaGemma XdnaGemma;
XdnaGemma *xdna_gemma_create(XdnaDevice *dev, const XdnaGemmaConfig *cfg, const XdnaGemmaWeights *w, int max_batch,
                             int max_ctx, int tp_rank, int tp_size);
void xdna_gemma_free(XdnaGemma *m);
/* tensor parallel set-up: this rank's 64-byte IPC handle; then every rank passes all handles
 * (tp_size x 64 bytes, rank order) to xdna_gemma_connect */
int xdna_gemma_ipc_handle(XdnaGemma *m, void *handle64);
int xdna_gemma_connect(XdnaGemma *m, const void *handles);
/* greedy decode: prompts [B][n_prompt] (host) -> tokens [B][n_new] (host); the prompt is run
 * through the decode step (prefill); synchronous; -1 also when a peer exchange timed out */
int xdna_gemma_generate(XdnaGemma *m, int B, const int64_t *prompts, int n_prompt, int n_new, int64_t *tokens_host,
                        void *stream);
/* the same in parts: stage (synchronous), enqueue steps (asynchronous on `stream`; the first
 * n_prompt - 1 of the n_prompt + n_new - 1 steps are the prefill), collect the tokens */
int xdna_gemma_begin(XdnaGemma *m, int B, const int64_t *prompts, int n_prompt, int n_new);
int xdna_gemma_steps(XdnaGemma *m, int n_steps, void *stream);
int xdna_gemma_tokens(XdnaGemma *m, int64_t *tokens_host, void *stream);

/* ------------------------------------ Parakeet FastConformer encoder (FastConformerEncoder) */
/* Replaces rust/npu-parakeet/src/encoder.rs FastConformerEncoder::subsample (200-237) +
 * forward_last (657-665) with every weight linear on the int8 GEMM engine (the reference's
 * NPU_PRECISION=int8 rule, rust/npu-asr/src/ctx2.rs).  Shapes: d_model 1024, 8 heads x 128,
 * ffn 4096, 256 subsample channels, conv kernel 9, at most 128 frames after the 8x
 * subsampling (n_frames <= 1017). */
typedef struct {
    int n_layers, d_model, n_heads, ffn, n_mels, n_frames, sub_ch, kconv;
} XdnaParakeetConfig;
typedef struct {               /* f32; linear weights [K, N] = [in, out], no biases */
    const float *ff1_ln_w, *ff1_ln_b, *ff1_w1, *ff1_w2;
    const float *att_ln_w, *att_ln_b, *wq, *wk, *wv, *wpos, *wout;
    const float *pos_u, *pos_v;                       /* [heads, 128] */
    const float *conv_ln_w, *conv_ln_b, *pw1, *dw_w, *dw_b, *pw2;   /* pw1 [D, 2D] (value | gate), dw_w [D, 9] */
    const float *ff2_ln_w, *ff2_ln_b, *ff2_w1, *ff2_w2;
    const float *out_ln_w, *out_ln_b;
} XdnaParakeetLayer;
typedef struct {
    const float *c0_w, *c0_b, *c2_w, *c2_b, *c3_w, *c3_b, *c5_w, *c5_b, *c6_w, *c6_b;  /* conv [Co, Ci/g, kh, kw] */
    const float *out_w, *out_b;                       /* [256 * F/8, D] ([in, out]), [D] */
    const XdnaParakeetLayer *layers;
} XdnaParakeetWeights;
typedef struct XdnaParakeet XdnaParakeet;
XdnaParakeet *xdna_parakeet_create(XdnaDevice *dev, const XdnaParakeetConfig *cfg, const XdnaParakeetWeights *w,
                                   int max_batch);
void xdna_parakeet_free(XdnaParakeet *m);
/* frames per clip after subsampling (T') */
int xdna_parakeet_frames_out(const XdnaParakeet *m);
/* host mel [B][n_mels][n_frames] f32 -> host encodings [B][T'][1024] f32.  Synchronous. */
int xdna_parakeet_encode(XdnaParakeet *m, const float *mel, int B, float *out);
/* device-resident form: asynchronous on `stream` */
int xdna_parakeet_encode_device(XdnaParakeet *m, const float *mel_dev, int B, float *out_dev, void *stream);


/* ------------------------------------------- device layer, op by op (npu-xrt shim + CtxDecode) */
/* The ordinal an open device was opened with (-1 for NULL). */
int xdna_device_ordinal(const XdnaDevice *dev);

/* Device buffers.  Replace shim_bo_alloc / shim_bo_free / shim_bo_write / shim_bo_read
 * (rust/npu-xrt/shim/xrt_shim.h:26-30): device memory has no host mirror, so the reference's
 * sync_to/from_device pair (xrt_shim.h:31-32) is folded into write / read.  write and read
 * return 0, or -1 with xdna_last_error() set (a NULL pointer, or a range past the end). */
typedef struct XdnaBuffer XdnaBuffer;
XdnaBuffer *xdna_buffer_alloc(XdnaDevice *dev, size_t bytes);
void xdna_buffer_free(XdnaBuffer *b);
void *xdna_buffer_device_ptr(XdnaBuffer *b);
int xdna_buffer_write(XdnaBuffer *b, const void *src, size_t bytes, size_t offset);
int xdna_buffer_read(XdnaBuffer *b, void *dst, size_t bytes, size_t offset);

/* Fused arenas: FusedArena (rust/npu-xrt/src/lib.rs:641-744), the three resident regions a
 * fused dispatch reads and writes -- 0 input (written per call), 1 output (read back), 2
 * scratch (weights, KV caches, intermediates) -- each a device buffer addressed by byte offset
 * (write_at / read_at).  A zero-size region is allocated with 2 bytes, as the reference does.
 * xdna_arena_region hands out a region as an XdnaBuffer (owned by the arena) for its device
 * pointer.  write/read return 0, or -1 with xdna_last_error() set. */
typedef struct XdnaArena XdnaArena;
XdnaArena *xdna_arena_create(XdnaDevice *dev, size_t input_bytes, size_t output_bytes, size_t scratch_bytes);
void xdna_arena_free(XdnaArena *a);
XdnaBuffer *xdna_arena_region(XdnaArena *a, int which);
int xdna_arena_write(XdnaArena *a, int which, size_t offset, const void *src, size_t bytes);
int xdna_arena_read(XdnaArena *a, int which, size_t offset, void *dst, size_t bytes);

/* Asynchronous runs.  Replace shim_run_matmul8_start / shim_run_elf_start + shim_run_wait +
 * shim_run_free (xrt_shim.h:51-54, 75): a run marks all work enqueued on `stream` (a
 * cudaStream_t; NULL = the legacy default stream) so far; xdna_run_wait returns 0 when it has
 * completed, 1 if it has not within timeout_ms (< 0: wait without limit), -1 on a device
 * error.  The reference's wait has no limit and folds "not completed" into -1. */
typedef struct XdnaRun XdnaRun;
XdnaRun *xdna_run_start(XdnaDevice *dev, void *stream);
int xdna_run_wait(XdnaRun *r, int timeout_ms);
void xdna_run_free(XdnaRun *r);

/* Resident bf16 GEMV with an optional fused pre-norm.  Replaces CtxDecode::register_weight +
 * gemv (rust/npu-asr/src/ctx_decode.rs:269-369) for norm = 0 and register_fused +
 * fused_norm_gemv (ctx_decode.rs:566-643) for norm = 1 (RMSNorm, gamma) and norm = 2
 * (LayerNorm, gamma and beta).  w is [K, N] f32 row-major, bias length N or NULL.  The
 * fold: W'' = bf16(gamma[k] * W[k][n]); LayerNorm's bias' = sum_k beta[k] W[k][n] (f32, k
 * ascending) + bias[n].  1 <= K <= 12288. */
typedef struct XdnaGemvBf16 XdnaGemvBf16;
XdnaGemvBf16 *xdna_gemv_bf16_register(XdnaDevice *dev, const float *w, int K, int N, const float *bias, int norm,
                                      const float *gamma, const float *beta, float eps);
void xdna_gemv_bf16_free(XdnaGemvBf16 *h);
/* Handles with staging buffers (XdnaGemvBf16, XdnaLogMel) serve one call at a time: calls on
 * one handle from several threads must be serialised by the caller (as the reference's device
 * objects, which are neither Send nor Sync).
 * Host x[K] -> host y[N]: the input statistics in f64 on the host (RMS: x / sqrt(mean(x^2)
 * + eps); LN: (x - mean) / sqrt(var + eps)), x rounded to bf16, f32 accumulation over
 * bf16 products on the GPU, + bias'.  Synchronous; 0 or -1. */
int xdna_gemv_bf16(XdnaGemvBf16 *h, const float *x, float *y);
/* Device form of the dot product alone (x already normalised): y_dev = bf16(x_dev) . W'' +
 * bias', asynchronous on `stream`. */
int xdna_gemv_bf16_device(XdnaGemvBf16 *h, const float *x_dev, float *y_dev, void *stream);

/* Single-query multi-head decode attention over the reference's packed K/V tiles.  Replaces
 * the mha_decode kernel (route_b_kernels/mha_decode/mha_decode.cc:90-168) as CtxDecode
 * dispatches it (ctx_decode.rs:464-555).  q_dev: [n_heads][64] bf16; kv_dev: per head
 * n_tiles tiles of [K 64x64 | V 64x64 | int32 key count as 2 bf16] bf16 (16,388 bytes); the
 * count is > 0 for a full or partial tile, < 0 (-count) for the last non-empty tile, 0 for an
 * empty one.  ctx_dev: [n_heads][64] f32 = softmax(q.K^T / 8) V over the real keys.  Device
 * pointers on the current device; asynchronous on `stream`. */
int xdna_mha_decode_paged(const uint16_t *q_dev, const uint16_t *kv_dev, int n_heads, int n_tiles, float *ctx_dev,
                          void *stream);


/* Conformer bricks, op by op (the on-NPU kernels NpuMatmul dispatches, npu-parakeet/src/npu.rs).
 * All pointers are device pointers on the current device; asynchronous on `stream`.
 *
 * Rel-pos multi-head attention, Parakeet shapes (H = 8, d_k = 128, D = 1024, T <= 128): the
 * relpos_mha brick (route_b_kernels/relpos_mha/relpos_mha.cc:1-60, 193-280) with attention_core's
 * math (rust/npu-parakeet/src/encoder.rs:285-414): per head AC = (q + u) k^T, BD = (q + v) p^T
 * read at the rel_shift index BD[i][T - 1 - i + j] (ops.rs:113-133), softmax((AC + BD) / sqrt(128))
 * over the T keys, ctx = P V.  qkv: [B][T][3 * 1024] f32 (q | k | v per row); pm: the projected
 * positions [2T - 1][1024] f32, row p for relative position T - 1 - p; pos_u, pos_v: [1024] f32;
 * ctx: [B][T][1024] f32.  Operands are rounded to bf16 for the tensor cores, f32 accumulation. */
int xdna_relpos_mha(const float *qkv_dev, const float *pm_dev, const float *pos_u_dev, const float *pos_v_dev, int T,
                    int B, float *ctx_dev, void *stream);
/* The conv module's middle (encoder.rs conv_module; ops.rs:92-110; dwconv1d.cc): x = the
 * pointwise-1 output [B][T][2C] f32 (values in channels 0..C-1, gates in C..2C-1);
 * g = x_val * sigmoid(x_gate); y[b][t][c] = silu(bias[c] + sum_j taps[c][j] g[t + j - (k-1)/2][c])
 * over the taps inside [0, T) ('same' zero padding, BatchNorm folded into taps and bias);
 * y: [B][T][C] f32, ready for pointwise-2.  taps: [C][k] f32, k one of 3, 5, 7, 9, 15, 31. */
int xdna_dwconv1d_glu_silu(const float *x_dev, int B, int T, int C, const float *taps_dev, int k,
                           const float *bias_dev, float *y_dev, void *stream);
/* One conv2d of the /8 subsample front end (route_b_kernels/subsample_conv2d/
 * subsample_patch_embed.cc: bf16 operands, f32 accumulation, optional ReLU, bf16 out):
 * x [B][ci][hin][win] bf16, w [co][ci/groups][kh][kw] bf16, bias [co] f32 (nullable) ->
 * out [B][co][hout][wout] bf16, hout = (hin + 2 pad - kh) / stride + 1 (likewise wout).
 * Covers conv.0 (1 -> 256, k3 s2 p1, ReLU), the depthwise conv.2/.5 (groups = ci) and the
 * pointwise conv.3/.6 (k1, ReLU).  The accumulation starts at the bias and adds the taps in
 * (input channel, row, column) order, as conv2d of ops.rs:38-89; a pointwise conv (k1 s1 p0,
 * groups 1) sums the taps first and adds the bias last, as that function's matmul path. */
int xdna_subsample_conv2d(const uint16_t *x_dev, int B, int ci, int hin, int win, const uint16_t *w_dev,
                          const float *bias_dev, int co, int kh, int kw, int stride, int pad, int groups, int relu,
                          uint16_t *out_dev, void *stream);


/* ------------------------------------------------- weight stores (npu-weights arena, npy dirs) */
/* A baked weight arena: one safetensors file (rust/npu-weights/src/arena.rs:13-100) --
 * tensors BF16 or F32, "__metadata__" {format_version, arch, source_ref, source_fingerprint}.
 * xdna_weights_open memory-maps it and checks arch == expect_arch (NULL: any) and
 * format_version == 1, failing with the reference's messages ("arena arch ... != expected ...",
 * "arena format_version N != 1 (rebake)").  NULL on error. */
typedef struct XdnaWeightArena XdnaWeightArena;
XdnaWeightArena *xdna_weights_open(const char *path, const char *expect_arch);
void xdna_weights_close(XdnaWeightArena *a);
/* number of tensors; name i in sorted order (NULL out of range) */
int xdna_weights_count(const XdnaWeightArena *a);
const char *xdna_weights_name(const XdnaWeightArena *a, int i);
/* a metadata string, or NULL */
const char *xdna_weights_meta(const XdnaWeightArena *a, const char *key);
/* dtype (0 F32, 1 BF16) and up to max_dims extents of tensor `name`; returns its rank, -1 if absent */
int xdna_weights_info(const XdnaWeightArena *a, const char *name, int *dtype, int64_t *shape, int max_dims);
/* tensor_f32 (arena.rs:62-78): n values upcast to f32; 0, or -1 (absent, or n not its size) */
int xdna_weights_read_f32(const XdnaWeightArena *a, const char *name, float *out, size_t n);
/* tensor_bf16 (arena.rs:86-100): the raw bf16 bits; 0, 1 for an F32 tensor (nothing copied), -1 */
int xdna_weights_read_bf16(const XdnaWeightArena *a, const char *name, uint16_t *out, size_t n);

/* Opt::load (opt125m_decode.rs:155-180) from a baked arena of arch "opt" (a file) or from the
 * npy directory it was baked from (a directory; names + ".npy"), with the names of
 * rust/npu-weights/src/arch/opt.rs:7-16; the configuration comes from the shapes (head_dim 64,
 * eps 1e-5).  lm_head.weight must be embed_tokens transposed (OPT ties them).  Then as
 * xdna_opt_create (max_ctx <= 0: min(max_pos, 2048)).  NULL on error. */
XdnaOptDecoder *xdna_opt_load(XdnaDevice *dev, const char *path, int max_ctx, int grid);


/* ------------------------------------------------------------ Whisper log-mel front end */
/* What the reference runs through preprocessor.onnx (rust/npu-engine/src/asr/whisper.rs:686-705),
 * the Whisper feature extractor: 480,000 samples (30 s at 16 kHz) -> input_features [80][3000]:
 * reflect-padded 400-sample frames every 160 samples, periodic Hann window, power spectrum, 80
 * Slaney mel filters over 0..8 kHz, log10(max(., 1e-10)), clamped below at the clip maximum - 8,
 * then (x + 4) / 4. */
typedef struct XdnaLogMel XdnaLogMel;
XdnaLogMel *xdna_log_mel_create(XdnaDevice *dev);
void xdna_log_mel_free(XdnaLogMel *h);
/* wav_dev [B][480000] f32 -> mel_dev [B][80][3000] f32, asynchronous on `stream` */
int xdna_log_mel_device(XdnaLogMel *h, const float *wav_dev, int B, float *mel_dev, void *stream);
/* the reference's host step: pcm i16 / 32768, zero-padded or truncated to 480,000 samples ->
 * mel [80][3000] f32 (host).  Synchronous. */
int xdna_log_mel(XdnaLogMel *h, const int16_t *pcm, size_t n, float *mel);

/* Detokenizer of the ASR front end: ids -> text with a byte-level BPE tokenizer.json (Whisper's),
 * as the HuggingFace tokenizers library decodes (whisper.rs:671-679): added tokens, then the BPE
 * vocabulary; special tokens dropped when skip_special; bytes through the inverse GPT-2
 * byte-to-unicode table; invalid UTF-8 replaced by U+FFFD.  Writes up to cap - 1 bytes + NUL to
 * out (nullable); returns the full length, or -1 with xdna_last_error() set. */
int xdna_bpe_decode(const char *tokenizer_path, const int64_t *ids, size_t n, int skip_special, char *out, size_t cap);

#ifdef __cplusplus
}
#endif
#endif
