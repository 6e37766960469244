"""Seeded synthetic inputs standing in for LibriSpeech (absent here).

``synthetic_audio`` makes the 30 s, 16 kHz test window the benchmark
configurations describe (a sum of five sine tones, 100-4000 Hz, random
amplitudes and phases, plus Gaussian noise of sigma 0.05).
``log_mel_int8`` turns it into the INT8 mel the integer encoder consumes:
the float log-mel of i_whisper/audio.py:216-265 (n_fft 512, hop 160, Hann
window, power spectrum without the last frame, Slaney mel filterbank,
log10 clamped at max-8, /4+1) followed by the input quantisation of
AudioEncoder_int.forward (model_int.py:1265-1267). The mel filterbank is
the published Slaney construction (the reference gets it from librosa,
which is not installed); frontend parity is therefore not claimed -- both
the oracle and the GPU path consume the same INT8 bytes.
"""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000
N_FFT = 512
HOP = 160
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


def _hz_to_mel(f):
    f = np.asarray(f, np.float64)
    f_sp = 200.0 / 3
    mels = f / f_sp
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, 1e-10) / min_log_hz) / logstep, mels)


def _mel_to_hz(m):
    m = np.asarray(m, np.float64)
    f_sp = 200.0 / 3
    freqs = f_sp * m
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), freqs)


def mel_filterbank(n_mels: int, n_fft: int = N_FFT, sr: int = SAMPLE_RATE) -> np.ndarray:
    """Slaney-scale triangular filters with area normalisation."""
    fft_freqs = np.linspace(0, sr / 2, 1 + n_fft // 2)
    mel_pts = np.linspace(_hz_to_mel(0.0), _hz_to_mel(sr / 2), n_mels + 2)
    hz = _mel_to_hz(mel_pts)
    fdiff = np.diff(hz)
    ramps = hz[:, None] - fft_freqs[None, :]
    w = np.zeros((n_mels, len(fft_freqs)))
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        w[i] = np.maximum(0, np.minimum(lower, upper))
    w *= (2.0 / (hz[2:n_mels + 2] - hz[:n_mels]))[:, None]
    return w.astype(np.float32)


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
