"""Whisper-small encoder (xdna_whisper_encode) against the oracle's restatement of the
reference's encoder.rs (conv stem, pre-LN blocks, ln_post).

The oracle is fed the weights the engine computes with: linear weights bfp16-quantised along K
(the reference's NPU weight format), conv weights and positions rounded to bf16. What remains is
bf16 activations between kernels on the GPU vs f32 in the oracle, so rows are compared by cosine
(>= 0.999) and by max error relative to the row's rms (<= 0.08)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def bf16(a):
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def engine_weights(w):
    from oracle import oracle as O
    q = dict(w)
    for k in ("conv1_w", "conv2_w", "embed_positions"):
        q[k] = bf16(w[k])
    q["layers"] = []
    for ly in w["layers"]:
        d = dict(ly)
        for k in ("q_w", "k_w", "v_w", "out_w", "fc1_w", "fc2_w"):
            d[k] = np.ascontiguousarray(O.bfp16_blocks(np.ascontiguousarray(ly[k].T)).T)
        q["layers"].append(d)
    return q


def compare(got, want):
    g = got.reshape(-1, got.shape[-1]).astype(np.float64)
    r = want.reshape(-1, want.shape[-1]).astype(np.float64)
    cos = (g * r).sum(1) / np.linalg.norm(g, axis=1) / np.linalg.norm(r, axis=1)
    rms = np.sqrt((r * r).mean(1))
    rel = np.abs(g - r).max(1) / rms
    assert cos.min() >= 0.999, cos.min()
    assert rel.max() <= 0.08, rel.max()


def test_whisper_encoder_small_frames(X):
    from oracle import oracle as O
    cfg = X.WhisperEncConfig(n_layers=2, n_frames=200, max_src=100)
    w = X.make_whisper_enc_weights(cfg, seed=1, bias_std=0.02, ln_std=0.05)
    mel = X.make_mel(cfg, batch=3, seed=1)
    enc = X.WhisperEncoder(X.Device(0), cfg, w, max_batch=4)
    got = enc.encode(mel)
    want = O.whisper_encode(cfg, engine_weights(w), mel)
    compare(got, want)
    # batch invariance: each clip alone gives the same bits as inside the batch
    for b in range(3):
        one = enc.encode(mel[b:b + 1])
        assert np.array_equal(one[0], got[b])
    enc.close()


def test_whisper_encoder_full_clip_one_layer(X):
    """A full 30 s clip (3000 frames -> 1500 positions): the attention spans 12 key tiles."""
    from oracle import oracle as O
    cfg = X.WhisperEncConfig(n_layers=1)
    w = X.make_whisper_enc_weights(cfg, seed=2)
    mel = X.make_mel(cfg, batch=1, seed=2)
    enc = X.WhisperEncoder(X.Device(0), cfg, w, max_batch=1)
    got = enc.encode(mel)
    compare(got, O.whisper_encode(cfg, engine_weights(w), mel))
    enc.close()


def test_whisper_encoder_rejects_bad_shapes(X):
    with pytest.raises(X.XdnaError):
        bad = X.WhisperEncConfig(n_layers=1, d_model=512, n_frames=64, max_src=32)
        X.WhisperEncoder(X.Device(0), bad, X.make_whisper_enc_weights(bad), max_batch=1)
    cfg = X.WhisperEncConfig(n_layers=1, n_frames=64, max_src=32)
    enc = X.WhisperEncoder(X.Device(0), cfg, X.make_whisper_enc_weights(cfg), max_batch=1)
    with pytest.raises(X.XdnaError):
        enc.encode(X.make_mel(cfg, batch=2))
    enc.close()


def test_whisper_encoder_baseline_config(X):
    """The BASELINE config: all 12 layers over a full 30 s clip (80 x 3000 mel -> 1500 x 768),
    one clip, against the oracle's restatement of encoder.rs:236-337 at cos >= 0.999."""
    from oracle import oracle as O
    cfg = X.WhisperEncConfig()
    w = X.make_whisper_enc_weights(cfg, seed=3)
    mel = X.make_mel(cfg, batch=1, seed=3)
    enc = X.WhisperEncoder(X.Device(0), cfg, w, max_batch=1)
    got = enc.encode(mel)
    enc.close()
    compare(got, O.whisper_encode(cfg, engine_weights(w), mel))
