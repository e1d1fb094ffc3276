"""RKLLM-compatible Python wrapper over the `matmul_decoder` module.

Mirror of the reference wrapper python/matmul_decoder.py of
suharvest/rknn-matmul-parallel: classes MatmulDecoder (RKLLMDecoder-style
run_embed), MatmulDecoderWrapper and the factory create_decoder, with the same
constructor arguments.  Named matmul_decoder_wrapper so it does not shadow the
compiled `matmul_decoder` module it imports.

Behaviour differences, each fixing a reference defect:
  * run_embed prefills the first n-1 embeddings with one batch prefill and
    runs the lm_head only on the last one, then feeds every generated token
    back (the reference wrapper passes token -1 after the prompt,
    python/matmul_decoder.py:202, which the C step rejects);
  * the default config uses head_dim 128 (the reference writes 64, :95);
  * weights count as present with either embeddings.npy or embeddings.bin
    (the C loader reads embeddings.bin; the reference checks only .npy, :147);
  * the result dict also carries "token_ids", the generated ids (additive key).
"""
from __future__ import annotations

import json
import logging
import os
import sys
import time
from pathlib import Path
from typing import Callable

import numpy as np

logger = logging.getLogger(__name__)

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG_DIR not in sys.path:
    sys.path.insert(0, _PKG_DIR)


class MatmulDecoder:
    """Decoder with the RKLLMDecoder-style interface (run_embed)."""

    def __init__(self, model_path: str, model_dir: str | None = None, tokenizer=None,
                 max_context_len: int = 4096, max_new_tokens: int = 500, top_k: int = 1,
                 top_p: float = 1.0, temperature: float = 1.0, repeat_penalty: float = 1.0,
                 frequency_penalty: float = 0.0, presence_penalty: float = 0.0, enabled_cpus: int = 2,
                 exec_mode: str = "dual_core", callback_fn: Callable | None = None,
                 quant_type: str = "int4"):
        try:
            import matmul_decoder as md
        except ImportError as e:  # the compiled module is the only implementation
            raise ImportError("matmul_decoder extension not found; build it with "
                              f"`make -C {_PKG_DIR}`") from e
        self._md = md
        if model_dir:
            model_path = model_dir
        self.model_path = Path(model_path)
        cfg_path = self.model_path / "config.json"
        if cfg_path.exists():
            with open(cfg_path) as f:
                self._config = json.load(f)
        else:
            self._config = dict(name="qwen3-asr-0.6b", hidden_dim=1024, num_q_heads=16, num_kv_heads=8,
                                head_dim=128, ffn_dim=3072, num_layers=28, vocab_size=151936,
                                rms_eps=1e-6, rope_theta=1000000.0)
        self.max_context_len = max_context_len
        self.max_new_tokens = max_new_tokens
        self.top_k, self.top_p, self.temperature = top_k, top_p, temperature
        self.repeat_penalty = repeat_penalty
        self.callback_fn = callback_fn
        self._tokenizer = tokenizer
        self._eos_token_id = 151645
        self._seq_len = 0
        t0 = time.time()
        if self._check_weights_ready():
            self._decoder = md.MatmulDecoder(model_dir=str(self.model_path), max_seq_len=max_context_len,
                                             quant_type=quant_type, exec_mode=exec_mode)
            logger.info("MatmulDecoder loaded in %.1fs (mode=%s)", time.time() - t0, exec_mode)
        else:
            self._decoder = None
            logger.warning("MatmulDecoder weights not found at %s", self.model_path)

    def _check_weights_ready(self) -> bool:
        p = self.model_path
        emb = (p / "embeddings.bin").exists() or (p / "embeddings.npy").exists()
        return emb and (p / "config.json").exists() and (
            (p / "layers").exists() or (p / "layer_00").exists())

    @property
    def seq_len(self) -> int:
        return self._seq_len

    def clear_kv_cache(self):
        if self._decoder:
            self._decoder.clear_kv_cache()
        self._seq_len = 0

    def run_embed(self, embed_array: np.ndarray, n_tokens: int, keep_history: int = 0,
                  keep_prefix: bool = False) -> dict:
        """Prefill n_tokens embeddings [n, hidden], then generate greedily until EOS."""
        if self._decoder is None:
            raise RuntimeError("MatmulDecoder not initialized: weights are missing")
        if keep_history == 0:
            self.clear_kv_cache()
        emb = np.ascontiguousarray(embed_array[:n_tokens], dtype=np.float32)
        t0 = time.time()
        if n_tokens > 1:
            self._decoder.prefill_batch(emb[:-1])
        t_pre = time.time()
        tokens = []
        token = self._decoder.step_get_token(0, emb[-1])
        while True:
            if token < 0:
                raise RuntimeError(f"decode step failed ({token})")
            tokens.append(token)
            if token == self._eos_token_id or len(tokens) >= self.max_new_tokens:
                break
            if self.callback_fn and self._tokenizer:
                self.callback_fn(self._tokenizer.decode([token]), False)
            token = self._decoder.step_get_token(token)
        t_gen = time.time()
        if self.callback_fn:
            self.callback_fn("", True)
        if self._tokenizer:
            text = self._tokenizer.decode(tokens)
            for tag in ("<|im_end|>", "<|endoftext|>", "<|im_start|>"):
                text = text.replace(tag, "")
        else:
            text = "".join(chr(t) if 32 <= t < 127 else "" for t in tokens)
        self._seq_len = self._decoder.seq_len
        return {"text": text,
                "perf": {"prefill_time_ms": (t_pre - t0) * 1e3, "generate_time_ms": (t_gen - t_pre) * 1e3,
                         "generate_tokens": len(tokens)},
                "n_tokens_generated": len(tokens), "ret_code": 0, "aborted": False,
                "token_ids": tokens}

    def release(self):
        self._decoder = None

    def __del__(self):
        self.release()


class MatmulDecoderWrapper:
    """RKLLMDecoder-compatible facade (run_embed / clear_kv_cache / release / seq_len)."""

    def __init__(self, **kwargs):
        self._impl = MatmulDecoder(**kwargs)

    def run_embed(self, *args, **kwargs):
        return self._impl.run_embed(*args, **kwargs)

    def clear_kv_cache(self):
        return self._impl.clear_kv_cache()

    def release(self):
        return self._impl.release()

    @property
    def seq_len(self):
        return self._impl.seq_len


def create_decoder(model_path: str, use_matmul: bool = True, exec_mode: str = "dual_core",
                   **kwargs) -> MatmulDecoderWrapper:
    """Factory of the reference wrapper; only the matmul decoder exists here."""
    if not use_matmul:
        raise ValueError("the RKLLM decoder is not part of this runtime")
    kwargs["exec_mode"] = exec_mode
    return MatmulDecoderWrapper(model_path=model_path, **kwargs)
