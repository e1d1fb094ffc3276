"""CPU ORACLE for the ASR front end (test infrastructure, never the product).

* `log_mel` restates MelExtractor.__call__ and _stft_numpy
  (examples/qwen3_asr/mel.py:6-27, :52-67 of suharvest/rknn-matmul-parallel):
  reflect padding by 200, periodic Hann window, 400-point real DFT (computed
  here in float64), power, mel = filters^T . power, log10(max(., 1e-10)),
  clamp at (max over all frames) - 8, (x + 4) / 4, last frame dropped.
* `build_embed` restates the row assembly of build_embed
  (examples/qwen3_asr/engine.py:255-314) for given token ids.
* `mel_filters` makes a triangular mel filter bank [201][128] (HTK mel scale,
  area-normalized) for tests; the reference loads Whisper's mel_filters.npy,
  which is not in the repository.
Only tests/ use it.
"""
from __future__ import annotations

import numpy as np

N_FFT, HOP, N_MELS = 400, 160, 128


def mel_filters(sr: int = 16000, n_fft: int = N_FFT, n_mels: int = N_MELS) -> np.ndarray:
    def hz_to_mel(f):
        return 2595.0 * np.log10(1.0 + f / 700.0)

    def mel_to_hz(m):
        return 700.0 * (10.0 ** (m / 2595.0) - 1.0)

    freqs = np.arange(n_fft // 2 + 1) * sr / n_fft
    pts = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(sr / 2), n_mels + 2))
    fb = np.zeros((n_fft // 2 + 1, n_mels))
    for m in range(n_mels):
        lo, c, hi = pts[m], pts[m + 1], pts[m + 2]
        up = (freqs - lo) / (c - lo)
        down = (hi - freqs) / (hi - c)
        fb[:, m] = np.maximum(0.0, np.minimum(up, down)) * (2.0 / (hi - lo))
    return fb.astype(np.float32)


def log_mel(audio: np.ndarray, filters: np.ndarray) -> np.ndarray:
    x = np.asarray(audio, np.float32)
    n = x.size
    padded = np.concatenate([x[1:N_FFT // 2 + 1][::-1], x, x[-N_FFT // 2 - 1:-1][::-1]])  # numpy 'reflect'
    window = (0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(N_FFT) / N_FFT)).astype(np.float32)
    n_frames = 1 + (padded.size - N_FFT) // HOP
    frames = np.stack([padded[f * HOP:f * HOP + N_FFT] for f in range(n_frames)]) * window  # float32
    spec = np.fft.rfft(frames.astype(np.float64), axis=1)
    power = (spec.real ** 2 + spec.imag ** 2).T  # [201][frames]
    mel = filters.astype(np.float64).T @ power
    lg = np.log10(np.maximum(mel, 1e-10))
    lg = np.maximum(lg, lg.max() - 8.0)
    lg = (lg + 4.0) / 4.0
    return lg[:, :n // HOP].astype(np.float32)


def build_embed(table: np.ndarray, prefix_ids, audio_embd: np.ndarray, suffix_ids) -> np.ndarray:
    rows = [table[list(prefix_ids)]] if len(prefix_ids) else []
    rows.append(np.asarray(audio_embd, np.float32))
    if len(suffix_ids):
        rows.append(table[list(suffix_ids)])
    return np.concatenate(rows).astype(np.float32)
