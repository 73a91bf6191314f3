"""The Whisper log-mel front end (preprocessor.onnx in the reference, whisper.rs:686-705).

The oracle (oracle/logmel.py, float64) is pinned to HuggingFace's WhisperFeatureExtractor --
the feature extractor the ONNX graph exports -- through the committed golden frames and, where
transformers is importable, live.  The GPU path computes the DFT in f32, so it is held to the
oracle within 2e-3 (max) and 5e-5 (mean) on the normalised features, whose range is about 2:
the f32 DFT's error is relative to the frame's loudest bins, and log10 magnifies it only in
bins far below them (the clamp at max - 8 bounds how far)."""
import os
import sys

import numpy as np
import pytest

from oracle import logmel as LM

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_logmel_golden import clip_pcm  # noqa: E402


def _signals():
    rng = np.random.default_rng(7)
    t = np.arange(16000 * 9) / 16000.0
    speechy = (5000 * np.sin(2 * np.pi * 180 * t) * (1 + np.sin(2 * np.pi * 3 * t))
               + 1500 * rng.standard_normal(t.size)).astype(np.int16)
    return {
        "golden_clip": clip_pcm(),
        "short_tones": speechy,
        "silence": np.zeros(16000, np.int16),
        "long_noise": (3000 * rng.standard_normal(16000 * 31)).astype(np.int16),   # > 30 s: truncated
        "one_sample": np.array([12345], np.int16),
    }


def test_oracle_matches_golden_frames():
    g = np.load(os.path.join(HERE, "golden", "whisper_logmel.npz"))
    f = LM.log_mel(LM.pcm_to_wave(clip_pcm()))
    np.testing.assert_allclose(f[:, g["frames"]], g["features"], atol=1e-4, rtol=0)


def test_oracle_matches_transformers_live():
    tr = pytest.importorskip("transformers")
    fe = tr.WhisperFeatureExtractor()
    np.testing.assert_array_equal(LM.mel_filters(), fe.mel_filters)
    for name, pcm in _signals().items():
        w = LM.pcm_to_wave(pcm)
        ref = fe(w, sampling_rate=16000, return_tensors="np")["input_features"][0]
        np.testing.assert_allclose(LM.log_mel(w), ref, atol=1e-4, rtol=0, err_msg=name)


def test_silence_is_the_floor():
    f = LM.log_mel(LM.pcm_to_wave(np.zeros(10, np.int16)))
    np.testing.assert_array_equal(f, np.full((80, 3000), -1.5, np.float32))


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


@pytest.mark.gpu
def test_gpu_log_mel_matches_oracle(X):
    dev = X.Device(0)
    L = X.lib()
    h = L.xdna_log_mel_create(dev.handle)
    assert h, X.last_error()
    try:
        for name, pcm in _signals().items():
            out = np.zeros((80, 3000), np.float32)
            pcm = np.ascontiguousarray(pcm)
            assert L.xdna_log_mel(h, pcm.ctypes.data, pcm.size, out.ctypes.data) == 0, X.last_error()
            ref = LM.log_mel(LM.pcm_to_wave(pcm))
            err = np.abs(out - ref)
            assert err.max() <= 2e-3 and err.mean() <= 5e-5, (name, float(err.max()), float(err.mean()))
            if name == "silence":
                np.testing.assert_array_equal(out, ref)
    finally:
        L.xdna_log_mel_free(h)


@pytest.mark.gpu
def test_gpu_log_mel_batch_equals_single(X):
    """The device form over a batch of 3 clips equals clip-by-clip calls bit for bit (each clip
    has its own maximum)."""
    import torch
    dev = X.Device(0)
    L = X.lib()
    h = L.xdna_log_mel_create(dev.handle)
    try:
        sig = _signals()
        waves = np.stack([LM.pcm_to_wave(sig[k]) for k in ("golden_clip", "silence", "short_tones")])
        wd = torch.from_numpy(waves).cuda()
        md = torch.empty((3, 80, 3000), dtype=torch.float32, device="cuda")
        assert L.xdna_log_mel_device(h, wd.data_ptr(), 3, md.data_ptr(), None) == 0
        got = md.cpu().numpy()
        for b, k in enumerate(("golden_clip", "silence", "short_tones")):
            one = np.zeros((80, 3000), np.float32)
            pcm = np.ascontiguousarray(sig[k])
            assert L.xdna_log_mel(h, pcm.ctypes.data, pcm.size, one.ctypes.data) == 0
            np.testing.assert_array_equal(got[b], one, err_msg=k)
    finally:
        L.xdna_log_mel_free(h)
