"""CPU ORACLE (test infrastructure, never the product).

Python driver over liboracle.so (ref_ops.c, the scalar C restatement of the
reference's CPU arithmetic).  `RefDecoder` restates the reference decoder's
host flow on a model directory in the reference's on-disk format:

* loading (src/matmul_decoder.c:698-826, :862-926, :1155-1168 of
  suharvest/rknn-matmul-parallel): FP32 embeddings, tied or separate lm_head,
  FP16 or pre-quantized projections, FP32 norms;
* the INT8 lm_head built at init from the FP16 copy of the table
  (:917-926, :1170-1275), or the FP16 CPU lm_head when disable_npu_lm_head
  (:1606-1610);
* `step` = matmul_decoder_step (:1430-1634): per-layer body, prefill mode when
  no logits are wanted, final norm, lm_head, seq_len++, argmax;
* `step_head` = matmul_decoder_step_head (:1636-1742), FP32 per-head tables;
* `prefill_batch` = matmul_decoder_prefill_batch (:1901-2065) including its
  chunking at max_batch_prefill (default 64).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
F32P = ctypes.POINTER(ctypes.c_float)
W_F16, W_I8, W_I4 = 0, 1, 2
PROJS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def build() -> str:
    """Compile liboracle.so with the committed Makefile if it is missing or stale."""
    src = os.path.join(HERE, "ref_ops.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
    return LIB_PATH


class RefDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("nq", ctypes.c_int), ("nkv", ctypes.c_int),
                ("hd", ctypes.c_int), ("ffn", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("rope_style", ctypes.c_int), ("has_qk_norm", ctypes.c_int),
                ("wtype", ctypes.c_int), ("eps", ctypes.c_float)]


class RefLayer(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p * 7), ("s", ctypes.c_void_p * 7),
                ("in_norm", ctypes.c_void_p), ("post_norm", ctypes.c_void_p),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sig = {
            "ref_rms_norm": [vp, vp, vp, i, f],
            "ref_rope_tables": [vp, vp, i, i, f],
            "ref_apply_rope": [vp, vp, vp, i, i, i],
            "ref_attention": [vp, vp, vp, vp, i, i, i, i],
            "ref_attention_batch_causal": [vp, vp, vp, vp, vp, vp, i, i, i, i, i],
            "ref_silu_mul": [vp, vp, vp, i],
            "ref_vec_add": [vp, vp, i],
            "ref_argmax": [vp, i],
            "ref_gemm": [vp, vp, i, vp, vp, i, i, i, i],
            "ref_quantize_cols": [vp, i, i, i, vp, vp],
            "ref_quantize_lm_head": [vp, i, i, i, vp, vp],
            "ref_lm_head_int8": [vp, vp, vp, vp, i, i, i, i],
            "ref_lm_head_f16": [vp, vp, vp, i, i, i],
            "ref_lm_head_f32": [vp, vp, vp, i, i],
            "ref_layer_decode": [vp, vp, vp, vp, vp, i, vp, vp, i],
            "ref_layer_prefill": [vp, i, vp, vp, vp, vp, i, f, i],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int if name == "ref_argmax" else None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data


# ─── op-level wrappers (used by the golden and kernel parity tests) ───

def rms_norm(x, w, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().ref_rms_norm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return out


def rope_tables(max_seq, head_dim, theta):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty_like(c)
    lib().ref_rope_tables(_p(c), _p(s), max_seq, head_dim, theta)
    return c, s


def apply_rope(x_heads, cos_row, sin_row, style):
    x = np.ascontiguousarray(x_heads, np.float32).copy()
    nh, hd = x.shape
    lib().ref_apply_rope(_p(x), _p(np.ascontiguousarray(cos_row, np.float32)),
                         _p(np.ascontiguousarray(sin_row, np.float32)), nh, hd, style)
    return x


def attention(q, k_cache, v_cache, nq, nkv, hd):
    """q [nq*hd]; caches [L][nkv][hd] FP32."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k_cache, np.float32)
    v = np.ascontiguousarray(v_cache, np.float32)
    out = np.empty(nq * hd, np.float32)
    lib().ref_attention(_p(out), _p(q), _p(k), _p(v), nq, nkv, hd, k.shape[0])
    return out


def silu_mul(g, u):
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(g)
    lib().ref_silu_mul(_p(out), _p(g), _p(np.ascontiguousarray(u, np.float32)), g.size)
    return out


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().ref_argmax(_p(x), x.size))


def gemm(x, w, scales=None, wtype=W_F16, n=None, nthreads=1):
    """x [M,K] FP32 -> [M,N] with the reference matmul semantics; w in the
    on-disk layout ([K,N] fp16/int8 or [K,N/2] packed int4)."""
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    M, K = x.shape
    w = np.ascontiguousarray(w)
    N = n if n is not None else (w.shape[1] * 2 if wtype == W_I4 else w.shape[1])
    y = np.empty((M, N), np.float32)
    sp = _p(np.ascontiguousarray(scales, np.float32)) if scales is not None else None
    lib().ref_gemm(_p(y), _p(x), M, _p(w), sp, K, N, wtype, nthreads)
    return y


def quantize_cols(w_f16, bits):
    w = np.ascontiguousarray(w_f16, np.float16)
    K, N = w.shape
    q = np.empty((K, N if bits == 8 else N // 2), np.uint8)
    s = np.empty(N, np.float32)
    lib().ref_quantize_cols(_p(w), K, N, bits, _p(q), _p(s))
    return (q.view(np.int8) if bits == 8 else q), s


def quantize_lm_head(table_f16, tile_n=4096):
    t = np.ascontiguousarray(table_f16, np.float16)
    V, K = t.shape
    n_tiles = (V + tile_n - 1) // tile_n
    q = np.empty((n_tiles, K, tile_n), np.int8)
    s = np.empty(n_tiles * tile_n, np.float32)
    lib().ref_quantize_lm_head(_p(t), V, K, tile_n, _p(q), _p(s))
    return q, s


# ─── model-level oracle ───

def _read(path, dtype, count):
    a = np.fromfile(path, dtype=dtype)
    if a.size != count:
        raise IOError(f"{path}: expected {count} elements, got {a.size}")
    return a


def _first(*paths):
    for p in paths:
        if os.path.exists(p):
            return p
    raise FileNotFoundError(paths[0])


class RefDecoder:
    """Whole-model oracle over a reference-format model directory."""

    def __init__(self, model_dir, quant="fp16", max_seq_len=4096, disable_npu_lm_head=False,
                 nthreads=1, max_batch_prefill=64):
        with open(os.path.join(model_dir, "config.json")) as f:
            cfg = json.load(f)
        self.cfg = cfg
        self.H, self.nq, self.nkv = cfg["hidden_dim"], cfg["num_q_heads"], cfg["num_kv_heads"]
        self.hd, self.F, self.nL = cfg["head_dim"], cfg["ffn_dim"], cfg["num_layers"]
        self.V = cfg["vocab_size"]
        self.eps = float(cfg.get("rms_eps", 1e-6))
        self.theta = float(cfg.get("rope_theta", 1e6))
        self.style = int(cfg.get("rope_style", 0))
        self.qk = int(cfg.get("has_qk_norm", 1))
        self.max_seq = max_seq_len
        self.nth = nthreads
        self.max_m = max_batch_prefill
        self.wtype = {"fp16": W_F16, "int8": W_I8, "int4": W_I4, "int4_g128": W_I4}[quant]
        H, qd, kvd = self.H, self.nq * self.hd, self.nkv * self.hd
        shapes = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
                  "gate_proj": (H, self.F), "up_proj": (H, self.F), "down_proj": (self.F, H)}

        self.emb = _read(os.path.join(model_dir, "embeddings.bin"), np.float32,
                         self.V * H).reshape(self.V, H)
        # multi-head mode (src/matmul_decoder.c:878-901): FP32 tables lm_head_NN.bin
        self.n_heads = int(cfg.get("num_lm_heads", 0))
        self.lm_vocab = int(cfg.get("lm_head_vocab_size", 0)) or self.V
        self.lm_heads = []
        if self.n_heads > 1:
            for i in range(self.n_heads):
                self.lm_heads.append(_read(os.path.join(model_dir, f"lm_head_{i:02d}.bin"), np.float32,
                                           self.lm_vocab * H).reshape(self.lm_vocab, H))
            disable_npu_lm_head = True  # no single table to quantize
            lm = self.emb
        else:
            lm_path = os.path.join(model_dir, "lm_head.bin")
            lm = (_read(lm_path, np.float32, self.V * H).reshape(self.V, H)
                  if os.path.exists(lm_path) else self.emb)
        self.lm_f16 = lm.astype(np.float16)
        self.disable_npu_lm_head = disable_npu_lm_head
        if not disable_npu_lm_head:
            self.lm_q, self.lm_s = quantize_lm_head(self.lm_f16)
        self.final_norm = _read(_first(os.path.join(model_dir, "final_norm.bin"),
                                       os.path.join(model_dir, "model_norm.bin")), np.float32, H)
        self.layers = []
        self._keep = []
        for l in range(self.nL):
            d = os.path.join(model_dir, "layers", f"layer_{l:02d}")
            if not os.path.isdir(d):
                d = os.path.join(model_dir, f"layer_{l:02d}")
            ent = {
                "in_norm": _read(_first(f"{d}/input_norm.bin", f"{d}/input_norm_weight.bin"),
                                 np.float32, H),
                "post_norm": _read(_first(f"{d}/post_attn_norm.bin", f"{d}/post_norm.bin",
                                          f"{d}/post_attn_norm_weight.bin"), np.float32, H),
                "q_norm": _read(_first(f"{d}/q_norm.bin", f"{d}/q_norm_weight.bin"),
                                np.float32, self.hd),
                "k_norm": _read(_first(f"{d}/k_norm.bin", f"{d}/k_norm_weight.bin"),
                                np.float32, self.hd),
            }
            ws, ss = [], []
            for p in PROJS:
                K, N = shapes[p]
                if self.wtype == W_F16:
                    ws.append(_read(f"{d}/{p}.bin", np.float16, K * N))
                    ss.append(None)
                else:
                    nb = K * N if self.wtype == W_I8 else K * N // 2
                    ws.append(_read(f"{d}/{p}_weight.bin", np.uint8, nb))
                    ss.append(_read(f"{d}/{p}_scales.bin", np.float32, N))
            ent["w"], ent["s"] = ws, ss
            rl = RefLayer()
            for i in range(7):
                rl.w[i] = ws[i].ctypes.data
                rl.s[i] = ss[i].ctypes.data if ss[i] is not None else None
            rl.in_norm = ent["in_norm"].ctypes.data
            rl.post_norm = ent["post_norm"].ctypes.data
            rl.q_norm = ent["q_norm"].ctypes.data
            rl.k_norm = ent["k_norm"].ctypes.data
            self._keep.append(ent)
            self.layers.append(rl)
        self.dims = RefDims(H, self.nq, self.nkv, self.hd, self.F, self.max_seq, self.style,
                            self.qk, self.wtype, self.eps)
        self.cos, self.sin = rope_tables(self.max_seq, self.hd, self.theta)
        self.k_cache = np.zeros((self.nL, self.max_seq, self.nkv, self.hd), np.float32)
        self.v_cache = np.zeros_like(self.k_cache)
        self.seq_len = 0
        self.last_hidden = None

    def clear(self):
        self.seq_len = 0

    def set_kv(self, layer, start, k_f16, v_f16):
        n = k_f16.shape[0]
        self.k_cache[layer, start:start + n] = np.asarray(k_f16, np.float32).reshape(
            n, self.nkv, self.hd)
        self.v_cache[layer, start:start + n] = np.asarray(v_f16, np.float32).reshape(
            n, self.nkv, self.hd)

    def logits_from_hidden(self, hidden):
        normed = rms_norm(hidden, self.final_norm, self.eps)
        logits = np.empty(self.V, np.float32)
        if self.disable_npu_lm_head:
            lib().ref_lm_head_f16(_p(logits), _p(normed), _p(self.lm_f16), self.V, self.H,
                                  self.nth)
        else:
            lib().ref_lm_head_int8(_p(logits), _p(normed), _p(self.lm_q), _p(self.lm_s),
                                   self.H, self.V, 4096, self.nth)
        return logits

    def step(self, token_id=-1, embedding=None, want_logits=True, layers=None):
        """Returns (token, logits|None).  Raises on the reference's error cases."""
        if embedding is not None:
            h = np.array(embedding, np.float32).reshape(self.H).copy()
        else:
            if token_id < 0 or token_id >= self.V:
                raise ValueError("invalid token")
            h = self.emb[token_id].copy()
        if self.seq_len >= self.max_seq:
            raise ValueError("KV cache full")
        pos = self.seq_len
        n_layers = self.nL if layers is None else layers
        for l in range(n_layers):
            lib().ref_layer_decode(_p(h), ctypes.byref(self.layers[l]), ctypes.byref(self.dims),
                                   _p(self.k_cache[l]), _p(self.v_cache[l]), pos,
                                   _p(self.cos), _p(self.sin), self.nth)
        self.last_hidden = h
        self.seq_len += 1
        if not want_logits:
            return 0, None
        logits = self.logits_from_hidden(h)
        return argmax(logits), logits

    def step_head(self, token_id=-1, lm_head_idx=0, embedding=None):
        """matmul_decoder_step_head (src/matmul_decoder.c:1636-1742): the layer
        body of `step`, final norm, then the FP32 GEMV of head lm_head_idx
        (gemv_f32_neon, :511-566) and argmax over its vocabulary."""
        if self.n_heads <= 1:
            return self.step(token_id, embedding)
        if not 0 <= lm_head_idx < self.n_heads:
            raise ValueError("invalid lm_head_idx")
        self.step(token_id, embedding, want_logits=False)
        normed = rms_norm(self.last_hidden, self.final_norm, self.eps)
        logits = np.empty(self.lm_vocab, np.float32)
        lib().ref_lm_head_f32(_p(logits), _p(normed), _p(np.ascontiguousarray(self.lm_heads[lm_head_idx])),
                              self.lm_vocab, self.H)
        return argmax(logits), logits

    def prefill_batch(self, embeds):
        x = np.ascontiguousarray(embeds, np.float32).reshape(-1, self.H)
        M = x.shape[0]
        if self.seq_len + M > self.max_seq:
            raise ValueError("KV cache overflow")
        for off in range(0, M, self.max_m):
            chunk = np.ascontiguousarray(x[off:off + self.max_m]).copy()
            m = chunk.shape[0]
            for l in range(self.nL):
                lib().ref_layer_prefill(_p(chunk), m, ctypes.byref(self.layers[l]),
                                        ctypes.byref(self.dims), _p(self.k_cache[l]),
                                        _p(self.v_cache[l]), self.seq_len, self.theta, self.nth)
            self.seq_len += m
            self.last_hidden = chunk[-1].copy()
        return 0
