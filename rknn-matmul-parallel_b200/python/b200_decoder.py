"""ctypes access to libmatmul_decoder.so (the C-ABI of include/*.h).

This is how Python code that is not the pybind module (tests, bench.py) calls
the runtime: `capi()` returns the loaded library with argument/return types
declared for every exported function, `Decoder` wraps a
MatmulDecoderContext*, and `BatchDecoder` a MatmulDecoderBatch*.  Device
pointers are plain integers (e.g. torch tensor data_ptr()); no torch type
crosses the boundary.  Importing this module never falls back to anything:
if the library is missing, it raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libmatmul_decoder.so")

c_int, c_float, c_vp, c_size = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
QUANT = {"fp16": 0, "int8": 1, "int4": 2, "int4_g128": 3}
W_F16, W_I8, W_I4, W_F32 = 0, 1, 2, 3
EPI_STORE, EPI_ADD, EPI_SILU_PAIR, EPI_ARGMAX = 0, 1, 2, 3


class MatmulDecoderConfig(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("hidden_dim", c_int), ("num_q_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int), ("ffn_dim", c_int),
                ("num_layers", c_int), ("vocab_size", c_int), ("max_seq_len", c_int),
                ("rms_eps", c_float), ("rope_theta", c_float), ("tie_word_embeddings", c_int),
                ("rope_scaling_factor", c_float), ("rope_scaling_type", c_int),
                ("norm_type", c_int), ("rope_style", c_int), ("ffn_act_type", c_int),
                ("has_qk_norm", c_int), ("num_lm_heads", c_int), ("lm_head_vocab_size", c_int),
                ("context_pool_mode", c_int), ("iommu_domain_id", c_int), ("exec_mode", c_int),
                ("disable_npu_lm_head", c_int), ("max_batch_prefill", c_int)]


class MatmulDecoderStats(ctypes.Structure):
    _fields_ = [("total_ms", c_float), ("matmul_ms", c_float), ("rebind_ms", c_float),
                ("convert_ms", c_float), ("cpu_ops_ms", c_float), ("lm_head_ms", c_float),
                ("n_steps", c_int)]


class ProjectionWeight(ctypes.Structure):
    _fields_ = [("data", c_vp), ("scales", c_vp), ("K", c_int), ("N", c_int), ("quant_type", c_int)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("q_proj", ProjectionWeight), ("k_proj", ProjectionWeight), ("v_proj", ProjectionWeight),
                ("o_proj", ProjectionWeight), ("gate_proj", ProjectionWeight), ("up_proj", ProjectionWeight),
                ("down_proj", ProjectionWeight), ("input_norm_weight", c_vp), ("post_attn_norm_weight", c_vp),
                ("q_norm_weight", c_vp), ("k_norm_weight", c_vp)]


class B2GemvArgs(ctypes.Structure):
    _fields_ = [("y", c_vp), ("ldy", c_int), ("x", c_vp), ("ldx", c_int), ("M", c_int),
                ("K", c_int), ("N", c_int), ("w", c_vp), ("scales", c_vp), ("wtype", c_int),
                ("norm_w", c_vp), ("eps", c_float), ("epilogue", c_int)]


class SamplingParams(ctypes.Structure):
    """SamplingParams of include/matmul_decoder.h (the reference's layout)."""
    _fields_ = [("top_k", c_int), ("top_p", ctypes.c_float), ("temperature", ctypes.c_float),
                ("repeat_penalty", ctypes.c_float), ("repeat_tokens", c_vp), ("n_repeat_tokens", c_int)]


class B2GemmArgs(ctypes.Structure):
    _fields_ = [("y", c_vp), ("ldy", c_int), ("x16", c_vp), ("ldx", c_int), ("M", c_int),
                ("K", c_int), ("N", c_int), ("w", c_vp), ("scales", c_vp), ("wtype", c_int),
                ("epilogue", c_int), ("keys", c_vp), ("tokens", c_vp), ("y16", c_vp),
                ("split_k", c_int)]


class B2KVRef(ctypes.Structure):
    _fields_ = [("k_base", c_vp), ("v_base", c_vp), ("seq_stride", ctypes.c_longlong),
                ("layer_stride", ctypes.c_longlong), ("layer", c_int), ("max_seq", c_int),
                ("rows_seq", c_vp), ("pos", c_vp), ("n_seqs", c_int)]


# name -> (restype, argtypes); every symbol of include/matmul_decoder.h and
# include/b2_kernels.h that has a non-inline definition.
SIGNATURES = {
    # matmul_decoder.h
    "matmul_kv_cache_create": (c_vp, [c_int, c_int, c_int, c_int]),
    "matmul_kv_cache_clear": (None, [c_vp]),
    "matmul_kv_cache_get_seq_len": (c_int, [c_vp]),
    "matmul_kv_cache_destroy": (None, [c_vp]),
    "matmul_decoder_create": (c_vp, [ctypes.c_char_p, c_vp, c_int, c_int]),
    "matmul_decoder_create_from_weights": (c_vp, [c_vp, c_vp, c_vp, c_vp, c_int, c_int]),
    "matmul_decoder_step": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "matmul_decoder_step_get_logits": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "matmul_decoder_step_head": (c_int, [c_vp, c_int, c_vp, c_int, c_vp]),
    "matmul_decoder_prefill_batch": (c_int, [c_vp, c_vp, c_int]),
    "matmul_decoder_clear_kv_cache": (None, [c_vp]),
    "matmul_decoder_get_seq_len": (c_int, [c_vp]),
    "matmul_decoder_get_config": (c_vp, [c_vp]),
    "matmul_decoder_get_stats": (None, [c_vp, c_vp]),
    "matmul_decoder_destroy": (None, [c_vp]),
    "matmul_sample_token": (c_int, [c_vp, c_int, c_vp]),
    "matmul_decoder_generate": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "matmul_decoder_load_config": (c_int, [ctypes.c_char_p, c_vp]),
    "matmul_decoder_export_hf_model": (c_int, [ctypes.c_char_p, ctypes.c_char_p, c_int]),
    "matmul_decoder_step_token": (c_int, [c_vp, c_int, c_vp]),
    "matmul_decoder_decode_greedy": (c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_step_sample": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "matmul_decoder_set_seed": (c_int, [c_vp, ctypes.c_ulonglong]),
    "matmul_log_mel": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "matmul_decoder_build_embed": (c_int, [c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp]),
    "matmul_decoder_set_kv": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_get_kv": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_set_seq_len": (c_int, [c_vp, c_int]),
    "matmul_decoder_get_hidden": (c_int, [c_vp, c_vp]),
    "matmul_decoder_uses_persistent_kernel": (c_int, [c_vp]),
    "matmul_decoder_step_kernel": (c_int, [c_vp, c_int]),
    "matmul_decoder_quantize_weight": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_quantize_lm_head": (c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_batch_create": (c_vp, [ctypes.c_char_p, c_vp, c_int, c_int, c_int]),
    "matmul_decoder_batch_set_kv": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "matmul_decoder_batch_set_seq_len": (c_int, [c_vp, c_int, c_int]),
    "matmul_decoder_batch_get_seq_len": (c_int, [c_vp, c_int]),
    "matmul_decoder_batch_step": (c_int, [c_vp, c_vp, c_vp, c_vp]),
    "matmul_decoder_batch_get_stats": (None, [c_vp, c_vp]),
    "matmul_decoder_batch_destroy": (None, [c_vp]),
    "matmul_decoder_nccl_unique_id": (c_int, [c_vp]),
    "matmul_decoder_batch_shard_vocab": (c_int, [c_vp, c_int, c_int, c_vp, c_int]),
    # b2_kernels.h
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_sample_max_vocab": (c_size, []),
    "b2_log_mel_workspace": (c_size, [c_int]),
    "b2_log_mel": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    "b2_build_embed": (c_int, [c_vp, c_int, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_vp]),
    "b2_sample_token": (c_int, [c_vp, c_int, c_vp, c_int, ctypes.c_float, c_int, ctypes.c_float, ctypes.c_float,
                                ctypes.c_ulonglong, ctypes.c_ulonglong, c_vp, c_vp, c_vp]),
    "b2_device_count": (c_int, [c_vp]),
    "b2_set_device": (c_int, [c_int]),
    "b2_get_device": (c_int, [c_vp]),
    "b2_sm_count": (c_int, [c_vp]),
    "b2_malloc": (c_int, [c_vp, c_size]),
    "b2_free": (c_int, [c_vp]),
    "b2_host_alloc": (c_int, [c_vp, c_size]),
    "b2_host_free": (c_int, [c_vp]),
    "b2_mem_get_info": (c_int, [c_vp, c_vp]),
    "b2_memcpy_h2d": (c_int, [c_vp, c_vp, c_size, c_vp]),
    "b2_memcpy_d2h": (c_int, [c_vp, c_vp, c_size, c_vp]),
    "b2_memcpy_d2d": (c_int, [c_vp, c_vp, c_size, c_vp]),
    "b2_memset": (c_int, [c_vp, c_int, c_size, c_vp]),
    "b2_stream_create": (c_int, [c_vp]),
    "b2_stream_destroy": (c_int, [c_vp]),
    "b2_stream_sync": (c_int, [c_vp]),
    "b2_stream_query": (c_int, [c_vp]),
    "b2_event_create": (c_int, [c_vp]),
    "b2_event_destroy": (c_int, [c_vp]),
    "b2_event_record": (c_int, [c_vp, c_vp]),
    "b2_event_elapsed_ms": (c_int, [c_vp, c_vp, c_vp]),
    "b2_graph_begin": (c_int, [c_vp]),
    "b2_graph_end": (c_int, [c_vp, c_vp]),
    "b2_graph_launch": (c_int, [c_vp, c_vp]),
    "b2_graph_destroy": (c_int, [c_vp]),
    "b2_gemv": (c_int, [c_vp, c_vp]),
    "b2_gemm": (c_int, [c_vp, c_vp]),
    "b2_attention_prefill": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_int, c_vp]),
    "b2_gemm_argmax_keys": (ctypes.c_size_t, [c_int, c_int]),
    "b2_rows_to_f16": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_int, c_vp, c_float, c_vp]),
    "b2_embed": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_vp]),
    "b2_qk_rope_kv": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_float,
                              c_vp, c_vp, c_int, c_vp, c_vp]),
    "b2_attention_workspace": (c_size, [c_int, c_int, c_int, c_int]),
    "b2_attention": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp]),
    "b2_attention_f16": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp]),
    "b2_attention_blocks_split": (c_int, [c_int, c_int]),
    "b2_attention_blocks": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp,
                                    c_vp]),
    "b2_lm_head_workspace": (c_size, [c_int, c_int]),
    "b2_loop_advance": (c_int, [c_vp, c_vp, c_int, c_vp]),
    "b2_lm_head_noalloc_max_keys": (c_size, []),
    "b2_lm_head_argmax_noalloc": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp, c_float,
                                          c_vp, c_int, c_vp, c_vp]),
    "b2_mk_check": (c_int, [c_vp]),
    "b2_mk_scratch_bytes": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "b2_mk_decode": (c_int, [c_vp, c_vp]),
    "b2_mk_final_hidden": (c_vp, [c_vp]),
    "b2_mk_smem_bytes": (c_size, []),
    "b2_mk2_check": (c_int, [c_vp]),
    "b2_mk2_max_context": (c_int, []),
    "b2_mk2_scratch_bytes": (c_size, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "b2_mk2_decode": (c_int, [c_vp, c_vp]),
    "b2_mk2_final_hidden": (c_vp, [c_vp]),
    "b2_tile_relayout": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    "b2_argmax_keys_merge": (c_int, [c_vp, c_int, c_int, ctypes.c_uint, c_vp, c_vp]),
    "b2_keys_tokens": (c_int, [c_vp, c_int, c_vp, c_vp]),
    "b2_lm_head_argmax": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int, c_vp, c_float,
                                  c_vp, c_int, c_vp, c_vp, c_vp]),
}

_lib = None


def capi(path: str = LIB_PATH):
    """Load libmatmul_decoder.so and declare every exported signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with `make -C {PKG_DIR}`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def nccl_unique_id() -> bytes:
    """128-byte NCCL unique id (matmul_decoder_nccl_unique_id)."""
    buf = ctypes.create_string_buffer(128)
    rc = capi().matmul_decoder_nccl_unique_id(buf)
    if rc != 0:
        raise RuntimeError(f"matmul_decoder_nccl_unique_id failed ({rc})")
    return buf.raw


def check(rc: int, what: str = "call"):
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {capi().b2_last_error().decode(errors='replace')}")


def _ptr(a: np.ndarray):
    return a.ctypes.data if a is not None else None


class Decoder:
    """MatmulDecoderContext* over the C API (host buffers in, host results out)."""

    def __init__(self, model_dir: str, quant: str = "fp16", max_seq_len: int = 4096,
                 disable_npu_lm_head: bool = False):
        L = capi()
        cfg = MatmulDecoderConfig()
        check(L.matmul_decoder_load_config(os.path.join(model_dir, "config.json").encode(),
                                           ctypes.byref(cfg)), "load_config")
        cfg.max_seq_len = max_seq_len
        cfg.disable_npu_lm_head = int(disable_npu_lm_head)
        self.cfg = cfg
        self.ctx = L.matmul_decoder_create(model_dir.encode(), ctypes.byref(cfg), QUANT[quant], max_seq_len)
        if not self.ctx:
            raise RuntimeError(f"matmul_decoder_create failed for {model_dir}")
        self.V, self.H = cfg.vocab_size, cfg.hidden_dim

    @classmethod
    def from_weights(cls, cfg: MatmulDecoderConfig, embeddings: np.ndarray, layers: list[dict],
                     lm_head: np.ndarray | None, quant: str = "fp16", max_seq_len: int = 4096):
        """matmul_decoder_create_from_weights over host arrays.  Each layer dict
        holds the seven projections as (data, scales|None) in the on-disk layout
        and the four FP32 norm vectors."""
        self = cls.__new__(cls)
        keep = [np.ascontiguousarray(embeddings, np.float32)]
        lw = (LayerWeights * len(layers))()
        qt = QUANT[quant]
        H, qd, kvd, F = cfg.hidden_dim, cfg.num_q_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim, cfg.ffn_dim
        dims = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
                "gate_proj": (H, F), "up_proj": (H, F), "down_proj": (F, H)}
        for i, L in enumerate(layers):
            for name, (K, N) in dims.items():
                data, sc = L[name]
                data = np.ascontiguousarray(data)
                keep.append(data)
                pw = getattr(lw[i], name)
                pw.data, pw.K, pw.N, pw.quant_type = data.ctypes.data, K, N, qt
                if sc is not None:
                    sc = np.ascontiguousarray(sc, np.float32)
                    keep.append(sc)
                    pw.scales = sc.ctypes.data
            for f in ("input_norm_weight", "post_attn_norm_weight", "q_norm_weight", "k_norm_weight"):
                a = np.ascontiguousarray(L[f], np.float32)
                keep.append(a)
                setattr(lw[i], f, a.ctypes.data)
        lm = None if lm_head is None else np.ascontiguousarray(lm_head, np.float32)
        cfg.max_seq_len = max_seq_len
        self.cfg = cfg
        self.ctx = capi().matmul_decoder_create_from_weights(ctypes.byref(cfg), keep[0].ctypes.data, lw,
                                                             _ptr(lm), qt, max_seq_len)
        if not self.ctx:
            raise RuntimeError("matmul_decoder_create_from_weights failed")
        self.V, self.H = cfg.vocab_size, cfg.hidden_dim
        return self

    def close(self):
        if getattr(self, "ctx", None):
            capi().matmul_decoder_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        self.close()

    def step(self, token_id=-1, embedding=None, logits=None):
        """matmul_decoder_step; logits: np.float32[V] to fill, or None for prefill mode."""
        emb = None if embedding is None else np.ascontiguousarray(embedding, np.float32)
        return capi().matmul_decoder_step(self.ctx, token_id, _ptr(emb), _ptr(logits))

    def step_logits(self, token_id=-1, embedding=None):
        logits = np.empty(self.V, np.float32)
        tok = self.step(token_id, embedding, logits)
        if tok < 0:
            raise RuntimeError(f"step failed ({tok})")
        return tok, logits

    def step_head(self, token_id=-1, lm_head_idx=0, embedding=None):
        """matmul_decoder_step_head; returns (token, logits[lm_head_vocab])."""
        n = self.cfg.lm_head_vocab_size if self.cfg.num_lm_heads > 1 and self.cfg.lm_head_vocab_size > 0 \
            else self.V
        logits = np.empty(n, np.float32)
        emb = None if embedding is None else np.ascontiguousarray(embedding, np.float32)
        tok = capi().matmul_decoder_step_head(self.ctx, token_id, _ptr(emb), lm_head_idx, logits.ctypes.data)
        return tok, logits

    def step_token(self, token_id=-1, embedding=None):
        emb = None if embedding is None else np.ascontiguousarray(embedding, np.float32)
        return capi().matmul_decoder_step_token(self.ctx, token_id, _ptr(emb))

    def step_sample(self, token_id=-1, params=None, embedding=None):
        """matmul_decoder_step_sample: the step's token drawn on the device."""
        emb = None if embedding is None else np.ascontiguousarray(embedding, np.float32)
        keep = params  # the repeat list stays alive for the call
        tok = capi().matmul_decoder_step_sample(self.ctx, token_id, _ptr(emb),
                                                ctypes.byref(params) if params is not None else None)
        del keep
        return tok

    def set_seed(self, seed):
        check(capi().matmul_decoder_set_seed(self.ctx, seed), "set_seed")

    def decode_greedy(self, first_token, n_tokens):
        """Device-resident greedy loop; returns (tokens, device_ms)."""
        out = np.empty(n_tokens, np.int32)
        ms = ctypes.c_float(0.0)
        rc = capi().matmul_decoder_decode_greedy(self.ctx, first_token, n_tokens, out.ctypes.data,
                                                 ctypes.byref(ms))
        if rc != n_tokens:
            raise RuntimeError(f"decode_greedy failed ({rc}): {capi().b2_last_error().decode()}")
        return out, ms.value

    def prefill_batch(self, embeds):
        e = np.ascontiguousarray(embeds, np.float32)
        check(capi().matmul_decoder_prefill_batch(self.ctx, e.ctypes.data, e.shape[0]), "prefill_batch")

    def set_kv(self, layer, start, k_f16, v_f16):
        k = np.ascontiguousarray(k_f16, np.float16)
        v = np.ascontiguousarray(v_f16, np.float16)
        check(capi().matmul_decoder_set_kv(self.ctx, layer, start, k.shape[0], k.ctypes.data, v.ctypes.data),
              "set_kv")

    def get_kv(self, layer, start, length):
        shape = (length, self.cfg.num_kv_heads, self.cfg.head_dim)
        k = np.empty(shape, np.float16)
        v = np.empty(shape, np.float16)
        check(capi().matmul_decoder_get_kv(self.ctx, layer, start, length, k.ctypes.data, v.ctypes.data),
              "get_kv")
        return k, v

    def set_seq_len(self, n):
        check(capi().matmul_decoder_set_seq_len(self.ctx, n), "set_seq_len")

    @property
    def seq_len(self):
        return capi().matmul_decoder_get_seq_len(self.ctx)

    def hidden(self):
        h = np.empty(self.H, np.float32)
        check(capi().matmul_decoder_get_hidden(self.ctx, h.ctypes.data), "get_hidden")
        return h

    def uses_persistent_kernel(self):
        return bool(capi().matmul_decoder_uses_persistent_kernel(self.ctx))

    def step_kernel(self, n_cached):
        """2: tile-stream persistent kernel, 1: first persistent kernel, 0: graph."""
        return capi().matmul_decoder_step_kernel(self.ctx, n_cached)

    def stats(self):
        s = MatmulDecoderStats()
        capi().matmul_decoder_get_stats(self.ctx, ctypes.byref(s))
        return {f: getattr(s, f) for f, _ in MatmulDecoderStats._fields_}


class BatchDecoder:
    """MatmulDecoderBatch* over the C API."""

    def __init__(self, model_dir: str, n_seqs: int, quant: str = "int4", max_seq_len: int = 4096):
        L = capi()
        cfg = MatmulDecoderConfig()
        check(L.matmul_decoder_load_config(os.path.join(model_dir, "config.json").encode(),
                                           ctypes.byref(cfg)), "load_config")
        cfg.max_seq_len = max_seq_len
        self.cfg, self.n = cfg, n_seqs
        self.b = L.matmul_decoder_batch_create(model_dir.encode(), ctypes.byref(cfg), QUANT[quant],
                                               max_seq_len, n_seqs)
        if not self.b:
            raise RuntimeError(f"matmul_decoder_batch_create failed for {model_dir}")

    def close(self):
        if self.b:
            capi().matmul_decoder_batch_destroy(self.b)
            self.b = None

    def __del__(self):
        self.close()

    def set_kv(self, seq, layer, start, k_f16, v_f16):
        k = np.ascontiguousarray(k_f16, np.float16)
        v = np.ascontiguousarray(v_f16, np.float16)
        check(capi().matmul_decoder_batch_set_kv(self.b, seq, layer, start, k.shape[0], k.ctypes.data,
                                                 v.ctypes.data), "batch_set_kv")

    def set_seq_len(self, seq, n):
        check(capi().matmul_decoder_batch_set_seq_len(self.b, seq, n), "batch_set_seq_len")

    def step(self, tokens, want_logits=False):
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.n, np.int32)
        logits = np.empty((self.n, self.cfg.vocab_size), np.float32) if want_logits else None
        check(capi().matmul_decoder_batch_step(self.b, t.ctypes.data, out.ctypes.data, _ptr(logits)),
              "batch_step")
        return (out, logits) if want_logits else out

    def shard_vocab(self, rank: int, world: int, nccl_id: bytes, rows_per_rank: int):
        """matmul_decoder_batch_shard_vocab (collective over the ranks)."""
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        check(capi().matmul_decoder_batch_shard_vocab(self.b, rank, world, buf, rows_per_rank), "batch_shard_vocab")

    def stats(self):
        s = MatmulDecoderStats()
        capi().matmul_decoder_batch_get_stats(self.b, ctypes.byref(s))
        return {f: getattr(s, f) for f, _ in MatmulDecoderStats._fields_}
