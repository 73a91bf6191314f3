"""Seeded synthetic models: the "synthetic" weight source of this engine.

The reference loads baked checkpoints (rust/npu-weights/src/arena.rs:13-60,
rust/npu-weights/src/arch/opt.rs).  No checkpoints exist on this machine, so the engine
also accepts random-init weights drawn here from a seeded generator: every weight matrix
N(0, 0.02), biases 0, LayerNorm gamma 1 / beta 0 (the opt-125m config), with optional
non-zero biases / norm parameters so that tests exercise every epilogue term.

Arrays use the reference's npy layouts: linear weights are [K, N] = [in, out]
(rust/npu-whisper/src/bin/opt125m_decode.rs:30-40), the token embedding is [V, D] and is
tied to the LM head, the learned positions are [max_pos + 2, D] (offset +2).
"""
from __future__ import annotations

from dataclasses import dataclass, asdict

import numpy as np


@dataclass(frozen=True)
class OptConfig:
    n_layers: int = 12
    d_model: int = 768
    n_heads: int = 12
    head_dim: int = 64
    ffn: int = 3072
    vocab: int = 50272
    max_pos: int = 2048
    eps: float = 1e-5

    def as_dict(self):
        return asdict(self)


OPT_125M = OptConfig()
LAYER_KEYS = ("ln1_w", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
              "ln2_w", "ln2_b", "w1", "b1", "w2", "b2")


def make_opt_weights(cfg: OptConfig = OPT_125M, seed: int = 0, std: float = 0.02,
                     bias_std: float = 0.0, ln_std: float = 0.0) -> dict:
    """Random-init OPT weights.  Returns {"emb_tok", "emb_pos", "lnf_w", "lnf_b",
    "layers": [dict per layer]} of float32 arrays."""
    rng = np.random.default_rng(seed)
    D, F, V = cfg.d_model, cfg.ffn, cfg.vocab

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return a

    def vec(n, base, s):
        if s == 0.0:
            return np.full(n, base, np.float32)
        return (np.float32(base) + normal(n, s)).astype(np.float32)

    w = {"emb_tok": normal((V, D), std), "emb_pos": normal((cfg.max_pos + 2, D), std)}
    layers = []
    for _ in range(cfg.n_layers):
        ly = {
            "ln1_w": vec(D, 1.0, ln_std), "ln1_b": vec(D, 0.0, ln_std),
            "wq": normal((D, D), std), "bq": vec(D, 0.0, bias_std),
            "wk": normal((D, D), std), "bk": vec(D, 0.0, bias_std),
            "wv": normal((D, D), std), "bv": vec(D, 0.0, bias_std),
            "wo": normal((D, D), std), "bo": vec(D, 0.0, bias_std),
            "ln2_w": vec(D, 1.0, ln_std), "ln2_b": vec(D, 0.0, ln_std),
            "w1": normal((D, F), std), "b1": vec(F, 0.0, bias_std),
            "w2": normal((F, D), std), "b2": vec(D, 0.0, bias_std),
        }
        layers.append(ly)
    w["layers"] = layers
    w["lnf_w"] = vec(D, 1.0, ln_std)
    w["lnf_b"] = vec(D, 0.0, ln_std)
    return w


def make_prompt(cfg: OptConfig = OPT_125M, n: int = 32, seed: int = 0) -> np.ndarray:
    """Prompt ids uniform in [2, vocab) (the opt-125m config's synthetic prompt)."""
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.integers(2, cfg.vocab, size=n, dtype=np.int64)


# ------------------------------------------------------------------------- BGE-base / BERT
@dataclass(frozen=True)
class BertConfig:
    n_layers: int = 12
    d_model: int = 768
    n_heads: int = 12
    ffn: int = 3072
    vocab: int = 30522
    max_pos: int = 512
    eps: float = 1e-12
    pooling: int = 0          # 0 = CLS (BGE), 1 = mean


BGE_BASE = BertConfig()
BERT_LAYER_KEYS = ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "attn_ln_w", "attn_ln_b",
                   "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b", "out_ln_w", "out_ln_b")


def _bf16(a):
    """Round float32 to bf16-representable float32 (nearest even), so the f32 oracle and the
    engine's bf16 weights hold the same values."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def make_bert_weights(cfg: BertConfig = BGE_BASE, seed: int = 0, std: float = 0.02,
                      bias_std: float = 0.0, ln_std: float = 0.0) -> dict:
    """Random-init BERT weights, bf16-valued float32: matrices N(0, std), biases N(0,
    bias_std), LayerNorm gamma 1 + N(0, ln_std), beta N(0, ln_std).  Linear weights are
    [K, N] = [in, out]."""
    rng = np.random.default_rng(seed)
    D, F = cfg.d_model, cfg.ffn

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return _bf16(a)

    def vec(n, base, s):
        if s == 0.0:
            return np.full(n, base, np.float32)
        return (np.float32(base) + rng.standard_normal(n, dtype=np.float32) * np.float32(s)).astype(np.float32)

    w = {"word_emb": normal((cfg.vocab, D), std), "pos_emb": normal((cfg.max_pos, D), std),
         "type_emb": normal((2, D), std), "emb_ln_w": vec(D, 1.0, ln_std), "emb_ln_b": vec(D, 0.0, ln_std)}
    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "q_w": normal((D, D), std), "q_b": vec(D, 0.0, bias_std),
            "k_w": normal((D, D), std), "k_b": vec(D, 0.0, bias_std),
            "v_w": normal((D, D), std), "v_b": vec(D, 0.0, bias_std),
            "o_w": normal((D, D), std), "o_b": vec(D, 0.0, bias_std),
            "attn_ln_w": vec(D, 1.0, ln_std), "attn_ln_b": vec(D, 0.0, ln_std),
            "ffn1_w": normal((D, F), std), "ffn1_b": vec(F, 0.0, bias_std),
            "ffn2_w": normal((F, D), std), "ffn2_b": vec(D, 0.0, bias_std),
            "out_ln_w": vec(D, 1.0, ln_std), "out_ln_b": vec(D, 0.0, ln_std),
        })
    w["layers"] = layers
    return w


def make_bge_batch(n_seqs: int = 256, seed: int = 0, lo: int = 32, hi: int = 512):
    """The BGE config's synthetic batch: lengths uniform in [lo, hi], ids uniform in
    [1000, 30000).  Returns (ids concatenated int32, seq_lens int32)."""
    rng = np.random.default_rng(seed + 7_000_003)
    lens = rng.integers(lo, hi + 1, size=n_seqs).astype(np.int32)
    ids = rng.integers(1000, 30000, size=int(lens.sum())).astype(np.int32)
    return ids, lens


# --------------------------------------------------------------------- Whisper-small encoder
@dataclass(frozen=True)
class WhisperEncConfig:
    n_layers: int = 12
    d_model: int = 768
    n_heads: int = 12
    ffn: int = 3072
    n_mels: int = 80
    n_frames: int = 3000
    max_src: int = 1500
    eps: float = 1e-5


WHISPER_SMALL_ENC = WhisperEncConfig()
WHISPER_ENC_LAYER_KEYS = ("ln1_w", "ln1_b", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "out_w", "out_b",
                          "ln2_w", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")


def make_whisper_enc_weights(cfg: WhisperEncConfig = WHISPER_SMALL_ENC, seed: int = 0, std: float = 0.02,
                             bias_std: float = 0.0, ln_std: float = 0.0) -> dict:
    """Random-init Whisper encoder weights (f32; linear weights [K, N]); k has no bias (zeros),
    as in Whisper."""
    rng = np.random.default_rng(seed)
    D, F = cfg.d_model, cfg.ffn

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return a

    def vec(n, base, s):
        if s == 0.0:
            return np.full(n, base, np.float32)
        return (np.float32(base) + rng.standard_normal(n, dtype=np.float32) * np.float32(s)).astype(np.float32)

    w = {"conv1_w": normal((D, cfg.n_mels, 3), std), "conv1_b": vec(D, 0.0, bias_std),
         "conv2_w": normal((D, D, 3), std), "conv2_b": vec(D, 0.0, bias_std),
         "embed_positions": normal((cfg.max_src, D), std),
         "ln_post_w": vec(D, 1.0, ln_std), "ln_post_b": vec(D, 0.0, ln_std)}
    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "ln1_w": vec(D, 1.0, ln_std), "ln1_b": vec(D, 0.0, ln_std),
            "q_w": normal((D, D), std), "q_b": vec(D, 0.0, bias_std),
            "k_w": normal((D, D), std), "k_b": np.zeros(D, np.float32),
            "v_w": normal((D, D), std), "v_b": vec(D, 0.0, bias_std),
            "out_w": normal((D, D), std), "out_b": vec(D, 0.0, bias_std),
            "ln2_w": vec(D, 1.0, ln_std), "ln2_b": vec(D, 0.0, ln_std),
            "fc1_w": normal((D, F), std), "fc1_b": vec(F, 0.0, bias_std),
            "fc2_w": normal((F, D), std), "fc2_b": vec(D, 0.0, bias_std),
        })
    w["layers"] = layers
    return w


def make_mel(cfg: WhisperEncConfig = WHISPER_SMALL_ENC, batch: int = 1, seed: int = 0) -> np.ndarray:
    """Synthetic log-mel input ~N(0, 1), [batch, n_mels, n_frames]."""
    rng = np.random.default_rng(seed + 9_000_011)
    return rng.standard_normal((batch, cfg.n_mels, cfg.n_frames), dtype=np.float32)


# --------------------------------------------------------------- Parakeet FastConformer encoder
@dataclass(frozen=True)
class ParakeetConfig:
    n_layers: int = 24
    d_model: int = 1024
    n_heads: int = 8
    ffn: int = 4096
    n_mels: int = 128
    n_frames: int = 1000
    sub_ch: int = 256
    kconv: int = 9

    @property
    def frames_out(self) -> int:
        t = self.n_frames
        for _ in range(3):
            t = (t - 1) // 2 + 1
        return t

    @property
    def freq_out(self) -> int:
        f = self.n_mels
        for _ in range(3):
            f = (f - 1) // 2 + 1
        return f


PARAKEET_V3 = ParakeetConfig()


def make_parakeet_weights(cfg: ParakeetConfig = PARAKEET_V3, seed: int = 0, std: float = 0.02,
                          ln_std: float = 0.0, n_layers: int | None = None) -> dict:
    """Random-init FastConformer weights (f32).  Linear weights N(0, std) in [in, out] layout
    (no linear biases, as in the checkpoint the reference bakes); the subsample convolutions
    use N(0, 1/sqrt(fan_in)) so the stem's activations stay O(1); depthwise taps and bias are
    the BatchNorm-folded values the reference loads."""
    rng = np.random.default_rng(seed)
    D, F, C, H = cfg.d_model, cfg.ffn, cfg.sub_ch, cfg.n_heads
    dk = D // H

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return a

    def vec(n, base, s):
        if s == 0.0:
            return np.full(n, base, np.float32)
        return (np.float32(base) + rng.standard_normal(n, dtype=np.float32) * np.float32(s)).astype(np.float32)

    fo = cfg.freq_out
    w = {"c0_w": normal((C, 1, 3, 3), 1 / 3), "c0_b": normal((C,), 0.1),
         "c2_w": normal((C, 1, 3, 3), 1 / 3), "c2_b": normal((C,), 0.1),
         "c3_w": normal((C, C, 1, 1), 1 / 16), "c3_b": normal((C,), 0.1),
         "c5_w": normal((C, 1, 3, 3), 1 / 3), "c5_b": normal((C,), 0.1),
         "c6_w": normal((C, C, 1, 1), 1 / 16), "c6_b": normal((C,), 0.1),
         "out_w": normal((C * fo, D), 1 / np.sqrt(C * fo)), "out_b": normal((D,), 0.02)}
    layers = []
    for _ in range(cfg.n_layers if n_layers is None else n_layers):
        ly = {}
        for p in ("ff1", "ff2"):
            ly[p + "_ln_w"], ly[p + "_ln_b"] = vec(D, 1.0, ln_std), vec(D, 0.0, ln_std)
            ly[p + "_w1"], ly[p + "_w2"] = normal((D, F), std), normal((F, D), std)
        ly["att_ln_w"], ly["att_ln_b"] = vec(D, 1.0, ln_std), vec(D, 0.0, ln_std)
        for n in ("wq", "wk", "wv", "wpos", "wout"):
            ly[n] = normal((D, D), std)
        ly["pos_u"], ly["pos_v"] = normal((H, dk), 0.02), normal((H, dk), 0.02)
        ly["conv_ln_w"], ly["conv_ln_b"] = vec(D, 1.0, ln_std), vec(D, 0.0, ln_std)
        ly["pw1"], ly["pw2"] = normal((D, 2 * D), std), normal((D, D), std)
        ly["dw_w"], ly["dw_b"] = normal((D, cfg.kconv), 1 / 3), normal((D,), 0.02)
        ly["out_ln_w"], ly["out_ln_b"] = vec(D, 1.0, ln_std), vec(D, 0.0, ln_std)
        layers.append(ly)
    w["layers"] = layers
    return w


def make_parakeet_mel(cfg: ParakeetConfig = PARAKEET_V3, batch: int = 1, seed: int = 0) -> np.ndarray:
    """Synthetic log-mel input ~N(0, 1), [batch, n_mels, n_frames]."""
    rng = np.random.default_rng(seed + 7_000_003)
    return rng.standard_normal((batch, cfg.n_mels, cfg.n_frames), dtype=np.float32)


# ------------------------------------------------------------------- Whisper-small decoder
@dataclass(frozen=True)
class WhisperDecConfig:
    n_layers: int = 12
    d_model: int = 768
    n_heads: int = 12
    ffn: int = 3072
    vocab: int = 51865
    max_tgt: int = 448
    n_enc: int = 1500


WHISPER_SMALL_DEC = WhisperDecConfig()
# start-of-transcript, language (en), transcribe, no-timestamps: the greedy decode's forced prefix
WHISPER_PROMPT = (50258, 50259, 50359, 50363)


def make_whisper_dec_weights(cfg: WhisperDecConfig = WHISPER_SMALL_DEC, seed: int = 0, std: float = 0.02,
                             bias_std: float = 0.0, ln_std: float = 0.0) -> dict:
    """Random-init Whisper decoder weights (f32; linear weights [K, N] = [in, out]; k biases 0;
    proj_out tied to embed_tokens as in the checkpoint)."""
    rng = np.random.default_rng(seed)
    D, F, V = cfg.d_model, cfg.ffn, cfg.vocab

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return a

    def vec(n, base, s):
        if s == 0.0:
            return np.full(n, base, np.float32)
        return (np.float32(base) + rng.standard_normal(n, dtype=np.float32) * np.float32(s)).astype(np.float32)

    emb = normal((V, D), std)
    w = {"embed_tokens": emb, "embed_positions": normal((cfg.max_tgt, D), std),
         "proj_out": np.ascontiguousarray(emb.T), "ln_post_w": vec(D, 1.0, ln_std), "ln_post_b": vec(D, 0.0, ln_std)}
    layers = []
    for _ in range(cfg.n_layers):
        ly = {}
        for p in ("ln_self", "ln_cross", "ln_final"):
            ly[p + "_w"], ly[p + "_b"] = vec(D, 1.0, ln_std), vec(D, 0.0, ln_std)
        for n in ("q", "k", "v", "out", "cross_q", "cross_k", "cross_v", "cross_out"):
            ly[n + "_w"] = normal((D, D), std)
            ly[n + "_b"] = np.zeros(D, np.float32) if n in ("k", "cross_k") else vec(D, 0.0, bias_std)
        ly["fc1_w"], ly["fc1_b"] = normal((D, F), std), vec(F, 0.0, bias_std)
        ly["fc2_w"], ly["fc2_b"] = normal((F, D), std), vec(D, 0.0, bias_std)
        layers.append(ly)
    w["layers"] = layers
    return w


def make_encoder_states(cfg: WhisperDecConfig = WHISPER_SMALL_DEC, batch: int = 1, seed: int = 0) -> np.ndarray:
    """Synthetic encoder output (the decoder's cross-attention input) ~N(0, 1), [batch, n_enc, D]."""
    rng = np.random.default_rng(seed + 5_000_017)
    return rng.standard_normal((batch, cfg.n_enc, cfg.d_model), dtype=np.float32)


# --------------------------------------------------------------------- Gemma-3 text decoder
@dataclass(frozen=True)
class GemmaConfig:
    """rust/npu-gemma/src/config.rs GEMMA3_1B (one KV head; every 6th layer global)."""
    n_layers: int = 26
    d_model: int = 1152
    n_q_heads: int = 4
    head_dim: int = 256
    ffn: int = 6912
    vocab: int = 262144
    window: int = 512
    pattern: int = 6
    theta_local: float = 10_000.0
    theta_global: float = 1_000_000.0
    query_pre_attn_scalar: float = 256.0
    eps: float = 1e-6


GEMMA3_1B = GemmaConfig()


def make_gemma_weights(cfg: GemmaConfig = GEMMA3_1B, seed: int = 0, std: float = 0.02, norm_std: float = 0.0,
                       n_layers: int | None = None, embed_std: float | None = None) -> dict:
    """Random-init Gemma-3 weights (f32, linear weights [K, N] = [in, out]); norm weights are
    the (1 + w) offsets, 0 by default.  The embedding (tied LM head) uses embed_std (default
    std)."""
    rng = np.random.default_rng(seed)
    D, F, HQ, HD = cfg.d_model, cfg.ffn, cfg.n_q_heads, cfg.head_dim

    def normal(shape, s):
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(s)
        return a

    def nrm(n):
        return normal((n,), norm_std) if norm_std else np.zeros(n, np.float32)

    w = {"embed": normal((cfg.vocab, D), std if embed_std is None else embed_std), "final_norm": nrm(D)}
    layers = []
    for _ in range(cfg.n_layers if n_layers is None else n_layers):
        layers.append({"in_norm": nrm(D), "wq": normal((D, HQ * HD), std), "wk": normal((D, HD), std),
                       "wv": normal((D, HD), std), "q_norm": nrm(HD), "k_norm": nrm(HD),
                       "wo": normal((HQ * HD, D), std), "post_attn_norm": nrm(D), "pre_ffn_norm": nrm(D),
                       "wg": normal((D, F), std), "wu": normal((D, F), std), "wd": normal((F, D), std),
                       "post_ffn_norm": nrm(D)})
    w["layers"] = layers
    return w
