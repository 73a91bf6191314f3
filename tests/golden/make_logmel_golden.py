"""Generates whisper_logmel.npz: input_features of HuggingFace's WhisperFeatureExtractor (the
algorithm behind the reference's preprocessor.onnx, rust/npu-engine/src/asr/whisper.rs:686-705)
for one seeded synthetic clip, frames 0..63 and 2936..2999 (the reflect-padded edges included).
Run in an environment with transformers: python tests/golden/make_logmel_golden.py"""
import os

import numpy as np


def clip_pcm():
    rng = np.random.default_rng(1234)
    t = np.arange(16000 * 30) / 16000.0
    x = (6000 * np.sin(2 * np.pi * 220 * t) + 2500 * np.sin(2 * np.pi * (900 + 300 * np.sin(t)) * t)
         + 800 * rng.standard_normal(t.size))
    x *= np.clip(np.sin(np.pi * t / 30.0) * 1.5, 0.0, 1.0)      # fade in and out
    return np.clip(x, -32768, 32767).astype(np.int16)


if __name__ == "__main__":
    from transformers import WhisperFeatureExtractor
    pcm = clip_pcm()
    wav = pcm.astype(np.float32) / np.float32(32768.0)
    f = WhisperFeatureExtractor()(wav, sampling_rate=16000, return_tensors="np")["input_features"][0]
    frames = np.r_[0:64, 2936:3000]
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "whisper_logmel.npz")
    np.savez_compressed(out, frames=frames, features=f[:, frames].astype(np.float32))
    print(out, f.shape)
