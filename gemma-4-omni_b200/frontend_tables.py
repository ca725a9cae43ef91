"""Constant tables of the log-mel frontend, computed on the host once.

The reference takes them from transformers 5.5.0 Gemma4AudioFeatureExtractor
(models/gemma4/feature_extraction_gemma4.py:95-160): frame 320 samples (20 ms),
hop 160, FFT 512, periodic Hann window, 128 HTK mel filters over 0-8 kHz with
no normalisation.  They are restated here from the published definitions:

- periodic Hann: w[n] = 0.5 - 0.5 cos(2 pi n / N), n < N (float64, then float32)
- HTK mel scale: mel(f) = 2595 log10(1 + f / 700)
- triangular filters between consecutive mel-spaced corner frequencies,
  evaluated at the FFT bin centre frequencies linspace(0, sr/2, 257).
"""
from __future__ import annotations

import numpy as np

FRAME_LENGTH = 320
HOP_LENGTH = 160
FFT_LENGTH = 512
NUM_BINS = FFT_LENGTH // 2 + 1
NUM_MEL = 128
SAMPLE_RATE = 16_000
MEL_FLOOR = 1e-3


def hann_window(n: int = FRAME_LENGTH) -> np.ndarray:
    k = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2.0 * np.pi * k / n)).astype(np.float32)


def _hz_to_mel(f):
    return 2595.0 * np.log10(1.0 + np.asarray(f, dtype=np.float64) / 700.0)


def _mel_to_hz(m):
    return 700.0 * (10.0 ** (np.asarray(m, dtype=np.float64) / 2595.0) - 1.0)


def mel_filterbank(num_bins: int = NUM_BINS, num_mel: int = NUM_MEL, fmin: float = 0.0,
                   fmax: float = 8000.0, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    """[num_bins, num_mel] float64 triangular HTK filters (norm=None)."""
    bin_freqs = np.linspace(0.0, sample_rate / 2.0, num_bins)
    corners = _mel_to_hz(np.linspace(_hz_to_mel(fmin), _hz_to_mel(fmax), num_mel + 2))
    widths = np.diff(corners)
    offset = corners[None, :] - bin_freqs[:, None]
    rising = -offset[:, :-2] / widths[:-1]
    falling = offset[:, 2:] / widths[1:]
    return np.maximum(0.0, np.minimum(rising, falling))
