"""ASR front end on the GPU, mirroring the reference example's interface
(examples/qwen3_asr/mel.py: MelExtractor; examples/qwen3_asr/engine.py:
_build_prefix_tokens / build_embed).

* MelExtractor(filter_path)(audio) -> (128, T) log-mel features, computed by
  the CUDA kernel b2_log_mel through matmul_log_mel.
* asr_prompt_ids(encode, ids, ...) -> (prefix ids, suffix ids): the prompt
  around the audio, as the reference assembles it (engine.py:243-306), for a
  caller-supplied tokenizer `encode(text) -> list[int]` and special-token ids.
* build_embed(decoder, audio_embd, prefix_ids, suffix_ids) -> (rows, n): the
  decoder input rows [prefix | audio | suffix], gathered on the device from
  the decoder's embedding table (matmul_decoder_build_embed).
"""
from __future__ import annotations

import ctypes

import numpy as np

import b200_decoder as bd

N_FFT, HOP, N_MELS = 400, 160, 128


class MelExtractor:
    """Whisper-style log-mel features (n_fft 400, hop 160, Hann, center)."""

    def __init__(self, filter_path=None, filters: np.ndarray | None = None):
        f = np.load(filter_path) if filters is None else filters
        self.filters = np.ascontiguousarray(f, np.float32)
        if self.filters.shape != (N_FFT // 2 + 1, N_MELS):
            raise ValueError(f"mel filters must be [{N_FFT // 2 + 1}, {N_MELS}], got {self.filters.shape}")

    def __call__(self, audio: np.ndarray, dtype=np.float32) -> np.ndarray:
        a = np.ascontiguousarray(audio, np.float32).reshape(-1)
        out = np.empty((N_MELS, a.size // HOP), np.float32)
        rc = bd.capi().matmul_log_mel(a.ctypes.data, a.size, self.filters.ctypes.data, out.ctypes.data)
        if rc < 0:
            raise RuntimeError(f"matmul_log_mel failed ({rc}): {bd.capi().b2_last_error().decode()}")
        return out.astype(dtype, copy=False)


def asr_prompt_ids(encode, ids: dict, language: str | None = None, context: str = "", prefix_text: str = "",
                   compact_suffix: bool = True, skip_prefix: bool = False):
    """(prefix ids, suffix ids) of the ASR prompt.  ids holds the special
    tokens: im_start, im_end, audio_start, audio_end, asr_text."""
    system_text = "You are a helpful assistant. " + (context or "")
    prefix = [] if skip_prefix else (
        [ids["im_start"]] + list(encode(f"system\n{system_text}")) + [ids["im_end"]]
        + [ids["im_start"]] + list(encode("user\n")) + [ids["audio_start"]])
    assistant = "assistant\nlanguage " + (language or "")
    instruction = "\u8f6c\u5f55\uff1a" if compact_suffix else "\u6570\u5b57\u75280123456789\uff0c\u8bed\u97f3\u8f6c\u5f55\uff1a"
    suffix = ([ids["audio_end"]] + list(encode(instruction)) + [ids["im_end"]] + [ids["im_start"]]
              + list(encode(assistant)) + [ids["asr_text"]])
    if prefix_text:
        suffix += list(encode(prefix_text))
    return prefix, suffix


def build_embed(decoder, audio_embd: np.ndarray, prefix_ids, suffix_ids):
    """(rows [n, hidden], n): [prefix token rows | audio rows | suffix token
    rows] from the decoder's device embedding table."""
    ctx = decoder.ctx if hasattr(decoder, "ctx") else decoder
    a = np.ascontiguousarray(audio_embd, np.float32)
    pre = np.ascontiguousarray(prefix_ids, np.int32)
    suf = np.ascontiguousarray(suffix_ids, np.int32)
    H = a.shape[1] if a.ndim == 2 and a.size else decoder.cfg.hidden_dim
    total = pre.size + (a.shape[0] if a.ndim == 2 else 0) + suf.size
    out = np.empty((total, H), np.float32)
    n = bd.capi().matmul_decoder_build_embed(ctx, pre.ctypes.data, pre.size, a.ctypes.data,
                                             a.shape[0] if a.ndim == 2 else 0, suf.ctypes.data, suf.size,
                                             out.ctypes.data)
    if n < 0:
        raise RuntimeError(f"matmul_decoder_build_embed failed ({n})")
    return out, n
