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
