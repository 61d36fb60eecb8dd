"""Whisper log-mel features on the GPU (the data side of the train step).

The reference computes the encoder input per sample on the host, in its
DataLoader workers: ``processor.feature_extractor(audio, sampling_rate=16000)``
(echo/train_echo_opus1.py:126), i.e. transformers' WhisperFeatureExtractor:

  * pad / truncate the waveform to 30 s (480000 samples at 16 kHz);
  * frames of 400 samples every 160, centred (reflect padding of 200 at both
    ends), periodic Hann window, power spectrum of bins 0..200;
  * 80 triangular mel filters (Slaney mel scale, 0..8000 Hz, Slaney area
    normalisation), log10 of max(mel, 1e-10); the last of the 3001 frames is
    dropped;
  * per sample: max(x, max(x) - 8), then (x + 4) / 4.

``log_mel_spectrogram`` does the same for a batch of waveforms already on the
GPU with the ``whisper_log_mel`` kernels of libtau_dxb.so (fp32 throughout);
``mel_filters`` restates the filter bank (transformers' mel_filter_bank with
Slaney scale and normalisation, which the extractor uses).
"""
from __future__ import annotations

import math
from functools import lru_cache

import numpy as np
import torch

from . import _capi as C

SAMPLE_RATE = 16000
N_FFT = 400
HOP = 160
N_MELS = 80
N_SAMPLES = 30 * SAMPLE_RATE
N_FRAMES = N_SAMPLES // HOP
N_BINS = N_FFT // 2 + 1


def _hz_to_mel(f):
    """Slaney mel scale: linear below 1 kHz (3 mels per 200 Hz), logarithmic above."""
    f = np.asarray(f, dtype=np.float64)
    mel = 3.0 * f / 200.0
    logstep = 27.0 / math.log(6.4)
    return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-30) / 1000.0) * logstep, mel)


def _mel_to_hz(m):
    m = np.asarray(m, dtype=np.float64)
    f = 200.0 * m / 3.0
    return np.where(m >= 15.0, 1000.0 * np.exp(math.log(6.4) / 27.0 * (m - 15.0)), f)


def mel_filters(n_mels: int = N_MELS, n_bins: int = N_BINS, sample_rate: int = SAMPLE_RATE,
                f_min: float = 0.0, f_max: float = 8000.0) -> np.ndarray:
    """[n_bins, n_mels] triangular filters between n_mels + 2 points equally
    spaced on the Slaney mel scale, each scaled by 2 / (its bandwidth in Hz)."""
    mel_pts = np.linspace(_hz_to_mel(f_min), _hz_to_mel(f_max), n_mels + 2)
    hz_pts = _mel_to_hz(mel_pts)
    fft_hz = np.linspace(0.0, sample_rate / 2.0, n_bins)
    width = np.diff(hz_pts)
    slopes = hz_pts[None, :] - fft_hz[:, None]
    down = -slopes[:, :-2] / width[:-1]
    up = slopes[:, 2:] / width[1:]
    fb = np.maximum(0.0, np.minimum(down, up))
    fb *= (2.0 / (hz_pts[2:n_mels + 2] - hz_pts[:n_mels]))[None, :]
    return fb


@lru_cache(maxsize=8)
def _filters_on(device_index: int) -> torch.Tensor:
    return torch.tensor(mel_filters(), dtype=torch.float32, device=torch.device("cuda", device_index))


def log_mel_spectrogram(audio: torch.Tensor) -> torch.Tensor:
    """[B, T] (or [T]) fp32 waveforms at 16 kHz on a CUDA device -> [B, 80, 3000]
    fp32 log-mel features, as WhisperFeatureExtractor computes them."""
    if not audio.is_cuda:
        raise RuntimeError("tau_dxb_b200: log_mel_spectrogram runs on CUDA tensors only "
                           "(this build has no CPU implementation)")
    squeeze = audio.dim() == 1
    x = audio.reshape(1, -1) if squeeze else audio
    x = x.float()
    if x.shape[1] != N_SAMPLES:                  # 30 s: zero padding or truncation
        x = torch.nn.functional.pad(x[:, :N_SAMPLES], (0, max(0, N_SAMPLES - x.shape[1])))
    x = x.contiguous()
    B = x.shape[0]
    out = torch.empty(B, N_MELS, N_FRAMES, dtype=torch.float32, device=x.device)
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    lib = C.lib()
    ws = torch.empty(lib.whisper_log_mel_workspace_bytes(B), dtype=torch.uint8, device=x.device)
    rc = lib.whisper_log_mel(x.data_ptr(), B, N_SAMPLES, _filters_on(dev).data_ptr(), out.data_ptr(),
                             ws.data_ptr(), ws.numel(), C.stream_ptr(x.device))
    C.check("whisper_log_mel", rc)
    return out[0] if squeeze else out
