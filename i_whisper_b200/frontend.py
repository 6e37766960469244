"""Audio frontend on the GPU: float32 16 kHz audio -> the INT8 mel the
integer encoder consumes, without a host round trip.

``log_mel_int8_cuda`` runs ``iw_log_mel_int8``: the log-Mel spectrogram of
i_whisper/audio.py:216-265 (n_fft 512, hop 160, periodic Hann window,
reflect padding, power spectrum without the last frame, mel filterbank,
log10 clamped at the window max - 8, /4 + 1) and the input quantisation of
AudioEncoder_int.forward (model_int.py:1265-1267). The mel filterbank is the
published Slaney construction (``mel_filterbank``; the reference takes it
from librosa, which is not available here).
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch

from . import _lib

SAMPLE_RATE = 16000
N_FFT = 512
HOP = 160


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
    """Slaney-scale triangular filters with area normalisation, [n_mels, n_fft/2+1]."""
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


_FILTERS: Dict[Tuple[int, str], torch.Tensor] = {}


def mel_filters_device(n_mels: int, device) -> torch.Tensor:
    key = (n_mels, str(torch.device(device)))
    if key not in _FILTERS:
        _FILTERS[key] = torch.from_numpy(mel_filterbank(n_mels)).to(device)
    return _FILTERS[key]


def log_mel_int8_cuda(audio: torch.Tensor, n_mels: int, input_alpha: float) -> torch.Tensor:
    """INT8 mel [B, n_mels, n_samples/160] of float32 CUDA audio [B, n_samples]
    (or [n_samples]); the log-mel max is taken per window."""
    if audio.dtype != torch.float32 or not audio.is_cuda:
        raise RuntimeError("audio must be a float32 CUDA tensor")
    squeeze = audio.dim() == 1
    a = audio.reshape(1, -1) if squeeze else audio
    if a.dim() != 2 or a.stride(1) != 1:
        raise RuntimeError("audio must be [B, n_samples] with contiguous rows")
    B, n = a.shape
    out = torch.empty(B, n_mels, n // HOP, dtype=torch.int8, device=a.device)
    filt = mel_filters_device(n_mels, a.device)
    _lib.call("iw_log_mel_int8", a.data_ptr(), B, n, a.stride(0), filt.data_ptr(), n_mels, float(input_alpha),
              out.data_ptr(), torch.cuda.current_stream(a.device).cuda_stream)
    return out[0] if squeeze else out
