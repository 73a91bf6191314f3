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
