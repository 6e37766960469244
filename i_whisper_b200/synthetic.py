"""Seeded synthetic inputs standing in for LibriSpeech (absent here).

``synthetic_audio`` makes the 30 s, 16 kHz test window the benchmark
configurations describe (a sum of five sine tones, 100-4000 Hz, random
amplitudes and phases, plus Gaussian noise of sigma 0.05).
``log_mel_int8`` turns it into the INT8 mel the integer encoder consumes:
the float log-mel of i_whisper/audio.py:216-265 (n_fft 512, hop 160, Hann
window, power spectrum without the last frame, Slaney mel filterbank,
log10 clamped at max-8, /4+1) followed by the input quantisation of
AudioEncoder_int.forward (model_int.py:1265-1267), in float64 numpy. The
mel filterbank is the published Slaney construction (the reference gets it
from librosa, which is not installed). The GPU frontend (frontend.py)
computes the same in float32; the benchmark feeds this INT8 mel so the
oracle and the GPU encoder consume the same bytes.
"""
from __future__ import annotations

import numpy as np

from .frontend import HOP, N_FFT, SAMPLE_RATE, mel_filterbank

N_SAMPLES = 30 * SAMPLE_RATE


def synthetic_audio(seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    t = np.arange(N_SAMPLES, dtype=np.float64) / SAMPLE_RATE
    x = np.zeros(N_SAMPLES, np.float64)
    for _ in range(5):
        f = rng.uniform(100.0, 4000.0)
        a = rng.uniform(0.05, 0.3)
        ph = rng.uniform(0, 2 * np.pi)
        x += a * np.sin(2 * np.pi * f * t + ph)
    x += rng.normal(0.0, 0.05, N_SAMPLES)
    return x.astype(np.float32)


def log_mel(audio: np.ndarray, n_mels: int) -> np.ndarray:
    pad = N_FFT // 2
    x = np.pad(audio.astype(np.float64), (pad, pad), mode="reflect")
    n_frames = 1 + (len(x) - N_FFT) // HOP
    idx = np.arange(N_FFT)[None, :] + HOP * np.arange(n_frames)[:, None]
    win = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(N_FFT) / N_FFT)
    spec = np.fft.rfft(x[idx] * win, axis=-1)
    mag = (np.abs(spec) ** 2)[:-1].T  # [freq, frames-1]
    mel = mel_filterbank(n_mels).astype(np.float64) @ mag
    lg = np.log10(np.maximum(mel, 1e-10))
    lg = np.maximum(lg, lg.max() - 8.0)
    return (lg / 4.0 + 1.0).astype(np.float32)


def log_mel_int8(audio: np.ndarray, n_mels: int, input_alpha: float) -> np.ndarray:
    """[n_mels, 3000] INT8: round(mel * input_alpha) clamped to +-127."""
    m = log_mel(audio, n_mels) * np.float32(input_alpha)
    return np.clip(np.rint(m), -127, 127).astype(np.int8)


def synthetic_mel_batch(n_mels: int, seeds, input_alpha: float = 100.0) -> np.ndarray:
    return np.stack([log_mel_int8(synthetic_audio(s), n_mels, input_alpha) for s in seeds])
