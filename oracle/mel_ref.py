"""NumPy restatement of the incremental 80 ms log-mel step (test oracle).

``extract_single_frame`` follows GemmaAudioTowerBackend._extract_single_frame
(duplex_kernel/listener.py:1807-1850): ``[160-sample tail | 1280 PCM | 0]`` ->
eight 321-sample windows at hop 160 -> first 320 samples x periodic Hann ->
rfft(n=512) -> |X| -> x mel filterbank (257 x 128, float64) -> log(x + 1e-3).
The window and filterbank come from the reference's own dependency,
transformers 5.5.0 ``Gemma4AudioFeatureExtractor`` (feature_extraction_gemma4.py:95-160):
frame_length 320, hop 160, fft 512, HTK mel scale 0-8 kHz, norm None,
preemphasis 0, mel_floor 1e-3, no per-bin normalisation.

TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import functools

import numpy as np

PCM_SAMPLES = 1280
TAIL = 160


@functools.lru_cache(maxsize=1)
def reference_tables() -> tuple[np.ndarray, np.ndarray]:
    """(window float32 [320], mel_filters float64 [257, 128]) from the extractor."""
    from transformers.models.gemma4.feature_extraction_gemma4 import Gemma4AudioFeatureExtractor

    fe = Gemma4AudioFeatureExtractor()
    assert fe.frame_length == 320 and fe.hop_length == 160 and fe.fft_length == 512
    assert fe.preemphasis == 0.0 and fe.per_bin_mean is None and fe.per_bin_stddev is None
    return np.asarray(fe.window, dtype=np.float32), np.asarray(fe.mel_filters, dtype=np.float64)


def extract_single_frame(pcm: np.ndarray, tail: np.ndarray | None) -> tuple[np.ndarray, np.ndarray]:
    """One session's tick: returns (mel [8,128] float32, next tail [160] float32)."""
    window, filters = reference_tables()
    curr = np.asarray(pcm, dtype=np.float32)
    if tail is None or len(tail) == 0:
        past = np.zeros(TAIL, dtype=np.float32)
    else:
        past = np.asarray(tail, dtype=np.float32)
        if len(past) < TAIL:
            past = np.pad(past, (TAIL - len(past), 0))
        elif len(past) > TAIL:
            past = past[-TAIL:]
    padded = np.concatenate((past, curr, np.zeros(1, dtype=np.float32)))
    frames = np.lib.stride_tricks.sliding_window_view(padded, window_shape=321)[::160][..., :-1]
    frames = frames * window
    mag = np.abs(np.fft.rfft(frames, n=512, axis=-1))
    log_mel = np.log(mag @ filters + 1e-3)
    return log_mel.astype(np.float32), curr[-TAIL:].copy()


def extract_batch(pcm: np.ndarray, tails: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Row-wise ``extract_single_frame`` over [N,1280] PCM and [N,160] tails."""
    mels, new_tails = zip(*(extract_single_frame(p, t) for p, t in zip(pcm, tails)))
    return np.stack(mels), np.stack(new_tails)
