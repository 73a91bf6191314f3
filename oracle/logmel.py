"""CPU oracle (test infrastructure only: imported by tests/, never by the product path) for the
Whisper log-mel front end.

The reference computes it with `preprocessor.onnx` (rust/npu-engine/src/asr/whisper.rs:686-705:
i16 / 32768, padded or truncated to 480,000 samples, then input_features [80, 3000]).  That ONNX
graph is an export of HuggingFace's WhisperFeatureExtractor, a third-party dependency absent
from the reference tree; this is a restatement of its published algorithm (the one OpenAI's
whisper.audio.log_mel_spectrogram defines), in float64:

* reflect-pad the 480,000 samples by n_fft / 2 = 200 on each side (STFT center=True);
* frames of 400 samples every 160, times the periodic Hann window 0.5 - 0.5 cos(2 pi n / 400);
* power spectrum |rfft|^2 (201 bins), the last of the 3,001 frames dropped;
* 80 Slaney mel filters over 0..8000 Hz (Slaney mel scale: linear 3 f / 200 below 1 kHz,
  15 + 27 ln(f / 1000) / ln 6.4 above; triangular filters between consecutive centre
  frequencies, scaled by 2 / (f[m+2] - f[m]));
* log10(max(mel, 1e-10)); clamp below at the clip maximum - 8; (x + 4) / 4.

Pinned by tests/test_logmel.py against transformers' WhisperFeatureExtractor in this image and
against the committed golden frames tests/golden/whisper_logmel.npz."""
import numpy as np

N_FFT, HOP, N_MELS, SR, N_SAMPLES = 400, 160, 80, 16000, 480000


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-300) / 1000.0) * (27.0 / np.log(6.4)), 3.0 * f / 200.0)


def _mel_to_hz(m):
    m = np.asarray(m, np.float64)
    return np.where(m >= 15.0, 1000.0 * np.exp((m - 15.0) * (np.log(6.4) / 27.0)), 200.0 * m / 3.0)


def mel_filters():
    """[201, 80] float64 Slaney filter bank."""
    fft_f = np.linspace(0.0, SR // 2, N_FFT // 2 + 1)
    f = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(8000.0), N_MELS + 2))
    diff = np.diff(f)
    slopes = f[None, :] - fft_f[:, None]
    fb = np.maximum(0.0, np.minimum(-slopes[:, :-2] / diff[:-1], slopes[:, 2:] / diff[1:]))
    return fb * (2.0 / (f[2:N_MELS + 2] - f[:N_MELS]))[None, :]


def pcm_to_wave(pcm):
    """whisper.rs:686-693: i16 / 32768 into a zeroed 480,000-sample buffer (truncating)."""
    wav = np.zeros(N_SAMPLES, np.float32)
    m = min(len(pcm), N_SAMPLES)
    wav[:m] = np.asarray(pcm[:m], np.int16).astype(np.float32) / np.float32(32768.0)
    return wav


def log_mel(wav):
    """[480000] f32 -> [80, 3000] f32 input_features."""
    x = np.asarray(wav, np.float64)
    x = np.pad(x, N_FFT // 2, mode="reflect")
    n_frames = 1 + (len(x) - N_FFT) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(n_frames)[:, None]
    win = 0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(N_FFT) / N_FFT)
    spec = np.abs(np.fft.rfft(x[idx] * win, axis=1)) ** 2           # [frames, 201]
    mel = spec @ mel_filters()                                         # [frames, 80]
    lg = np.log10(np.maximum(mel, 1e-10)).T[:, :-1]
    lg = np.maximum(lg, lg.max() - 8.0)
    return ((lg + 4.0) / 4.0).astype(np.float32)
