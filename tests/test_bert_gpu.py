"""BGE/BERT embedder on B200 (tcgen05 GEMMs, tensor-core attention, fused LN) against the
CPU oracle's restatement of the reference's f32 host path, through the C ABI.

Bar (the north-star's embedding bar): every embedding's cosine to the oracle's >= 0.999.
The engine keeps activations in bf16 between kernels (the oracle is f32 throughout), so exact
equality is not expected; the measured gap is ~1e-3 relative."""
import dataclasses

import numpy as np
import pytest

from oracle import oracle as O
from xdna_engine_b200.synth import BGE_BASE, make_bert_weights, make_bge_batch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def cosines(a, b):
    return (a * b).sum(1) / np.linalg.norm(a, axis=1) / np.linalg.norm(b, axis=1)


@pytest.mark.parametrize("pooling", [0, 1])
def test_bert_small_edges(X, pooling):
    """2 layers; lengths on both sides of the 64-key attention tile, a single-token
    sequence, and non-zero biases / LayerNorm parameters."""
    cfg = dataclasses.replace(BGE_BASE, n_layers=2, pooling=pooling)
    w = make_bert_weights(cfg, seed=2, bias_std=0.02, ln_std=0.05)
    lens = np.array([1, 63, 64, 65, 130, 7], np.int32)
    rng = np.random.default_rng(4)
    ids = rng.integers(1000, 30000, size=int(lens.sum())).astype(np.int32)
    dev = X.Device(0)
    m = X.BertEmbedder(dev, cfg, w, max_tokens=1024, max_seqs=16)
    got = m.embed(ids, lens)
    again = m.embed(ids, lens)
    m.close()
    np.testing.assert_array_equal(got, again)
    ref = O.bert_embed(cfg, w, ids, lens)
    c = cosines(got, ref)
    assert c.min() >= 0.999, c


def test_bge_base_config(X):
    """The BGE-base config (12 layers, N(0,0.02) weights, CLS + L2) on a few sequences."""
    w = make_bert_weights(BGE_BASE, seed=0)
    ids, lens = make_bge_batch(3, seed=0, lo=32, hi=160)
    dev = X.Device(0)
    m = X.BertEmbedder(dev, BGE_BASE, w, max_tokens=4096, max_seqs=8)
    got = m.embed(ids, lens)
    m.close()
    ref = O.bert_embed(BGE_BASE, w, ids, lens)
    c = cosines(got, ref)
    assert c.min() >= 0.999, c
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)


def test_bert_rejects_bad_input(X):
    cfg = dataclasses.replace(BGE_BASE, n_layers=1)
    w = make_bert_weights(cfg, seed=3)
    dev = X.Device(0)
    m = X.BertEmbedder(dev, cfg, w, max_tokens=64, max_seqs=2)
    with pytest.raises(X.XdnaError):
        m.embed(np.array([5, 99999], np.int32), np.array([2], np.int32))   # id >= vocab
    with pytest.raises(X.XdnaError):
        m.embed(np.zeros(100, np.int32), np.array([100], np.int32))        # > max_tokens
    out = m.embed(np.array([1500, 2000], np.int32), np.array([2], np.int32))
    assert out.shape == (1, 768)
    m.close()


def test_bge_base_config_long_sequences(X):
    """The BGE-base config at its length range: a batch of 6 drawn from U[32, 512] plus a
    512-token and a 511-token sequence (all 8 key tiles of the attention, ragged tails), cos >=
    0.999 against the oracle (bert/encoder.rs:43-57, head.rs:20-47)."""
    w = make_bert_weights(BGE_BASE, seed=1)
    ids, lens = make_bge_batch(6, seed=1)
    rng = np.random.default_rng(11)
    lens = np.concatenate([lens, np.array([512, 511], np.int32)])
    ids = np.concatenate([ids, rng.integers(1000, 30000, 1023).astype(np.int32)])
    m = X.BertEmbedder(X.Device(0), BGE_BASE, w, max_tokens=int(lens.sum()), max_seqs=8)
    got = m.embed(ids, lens)
    m.close()
    c = cosines(got, O.bert_embed(BGE_BASE, w, ids, lens))
    assert c.min() >= 0.999, c
