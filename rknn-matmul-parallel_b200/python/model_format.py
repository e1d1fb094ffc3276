"""Reference on-disk model format: writer, reader helpers and seeded synthetic models.

The layout is the one the reference loader reads (src/matmul_decoder.c:635-826,
:862-926, :1155-1168 of suharvest/rknn-matmul-parallel):

    model_dir/config.json                 keys parsed by matmul_decoder_load_config
    model_dir/embeddings.bin              FP32 [vocab, hidden]
    model_dir/lm_head.bin                 FP32 [vocab, hidden] (only when untied)
    model_dir/lm_head_NN.bin              FP32 [lm_head_vocab, hidden] per head (multi-head)
    model_dir/final_norm.bin              FP32 [hidden]
    model_dir/layers/layer_NN/input_norm.bin, post_attn_norm.bin   FP32 [hidden]
    model_dir/layers/layer_NN/q_norm.bin, k_norm.bin               FP32 [head_dim]
    model_dir/layers/layer_NN/{proj}.bin                           FP16 [K, N]
    model_dir/layers/layer_NN/{proj}_weight.bin                    int8 [K, N] | int4 [K, N/2]
    model_dir/layers/layer_NN/{proj}_scales.bin                    FP32 [N]

The reference ships no writer for the quantized files; `quantize_model_dir`
fills that gap using the runtime's own quantizer (bit-exact per-column rule).

Synthetic models follow the seeded recipe of the benchmark configs: numpy
PCG64 streams, one seed per tensor (1000 * layer + tensor id), FP16 weights
N(0, 0.02), norm weights 1 + N(0, 0.01), FP32 embedding table N(0, 0.02).
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, field

import numpy as np

PROJS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
TENSOR_ID = {"input_norm": 0, "post_attn_norm": 1, "q_norm": 2, "k_norm": 3,
             "q_proj": 4, "k_proj": 5, "v_proj": 6, "o_proj": 7,
             "gate_proj": 8, "up_proj": 9, "down_proj": 10}
GLOBAL_SEED = {"embeddings": 900_000, "final_norm": 900_001, "lm_head": 900_002}


@dataclass
class ModelShape:
    hidden_dim: int = 1024
    num_q_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    ffn_dim: int = 3072
    num_layers: int = 28
    vocab_size: int = 151936
    max_seq_len: int = 4096
    rms_eps: float = 1e-6
    rope_theta: float = 1000000.0
    rope_style: int = 1
    has_qk_norm: int = 1
    tie_word_embeddings: bool = True
    name: str = "qwen3-0.6b-synthetic"
    num_lm_heads: int = 0         # > 1: multi-head model (lm_head_NN.bin tables, step_head)
    lm_head_vocab_size: int = 0   # vocabulary of each head in multi-head mode
    extra: dict = field(default_factory=dict)

    def proj_shapes(self):
        h, q, kv, f = self.hidden_dim, self.num_q_heads * self.head_dim, \
            self.num_kv_heads * self.head_dim, self.ffn_dim
        return {"q_proj": (h, q), "k_proj": (h, kv), "v_proj": (h, kv), "o_proj": (q, h),
                "gate_proj": (h, f), "up_proj": (h, f), "down_proj": (f, h)}

    def config_json(self) -> dict:
        d = {"name": self.name, "hidden_dim": self.hidden_dim, "num_q_heads": self.num_q_heads,
             "num_kv_heads": self.num_kv_heads, "head_dim": self.head_dim,
             "ffn_dim": self.ffn_dim, "num_layers": self.num_layers,
             "vocab_size": self.vocab_size, "max_seq_len": self.max_seq_len,
             "rms_eps": self.rms_eps, "rope_theta": self.rope_theta,
             "rope_style": self.rope_style, "has_qk_norm": self.has_qk_norm,
             "tie_word_embeddings": bool(self.tie_word_embeddings)}
        if self.num_lm_heads > 1:
            d["num_lm_heads"] = self.num_lm_heads
            d["lm_head_vocab_size"] = self.lm_head_vocab_size or self.vocab_size
        d.update(self.extra)
        return d


def write_config_json(path: str, cfg: dict) -> None:
    """Write config.json with floats in positional notation.

    The reference's config scanner (src/matmul_decoder.c:2245-2256) reads
    digits, one '.', digits: an exponent such as 1e-06 would parse as 1.
    """
    def fmt(v):
        if isinstance(v, bool):
            return "true" if v else "false"
        if isinstance(v, float):
            return np.format_float_positional(v, trim="-")
        return json.dumps(v)
    body = ",\n".join(f'  "{k}": {fmt(v)}' for k, v in cfg.items())
    with open(path, "w") as f:
        f.write("{\n" + body + "\n}\n")


def _normal(seed: int, shape, std: float, mean: float = 0.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    if mean != 0.0:
        x += np.float32(mean)
    return x


def layer_dir(model_dir: str, layer: int) -> str:
    return os.path.join(model_dir, "layers", f"layer_{layer:02d}")


def synth_layer_tensors(shape: ModelShape, layer: int) -> dict:
    """Seeded tensors of one layer: FP16 [K,N] projections and FP32 norms."""
    base = 1000 * layer
    out = {
        "input_norm": _normal(base + TENSOR_ID["input_norm"], (shape.hidden_dim,), 0.01, 1.0),
        "post_attn_norm": _normal(base + TENSOR_ID["post_attn_norm"], (shape.hidden_dim,), 0.01, 1.0),
        "q_norm": _normal(base + TENSOR_ID["q_norm"], (shape.head_dim,), 0.01, 1.0),
        "k_norm": _normal(base + TENSOR_ID["k_norm"], (shape.head_dim,), 0.01, 1.0),
    }
    for p, (k, n) in shape.proj_shapes().items():
        out[p] = _normal(base + TENSOR_ID[p], (k, n), 0.02).astype(np.float16)
    return out


def synth_embeddings(shape: ModelShape) -> np.ndarray:
    return _normal(GLOBAL_SEED["embeddings"], (shape.vocab_size, shape.hidden_dim), 0.02)


def write_synthetic_model(model_dir: str, shape: ModelShape, quant: str | None = None,
                          lib_path: str | None = None) -> str:
    """Write a seeded synthetic model in the reference layout.

    quant: None/'fp16' writes FP16 projections only; 'int8' or 'int4' also
    writes {proj}_weight.bin / {proj}_scales.bin quantized from the FP16 copy.
    A marker file records the recipe so an identical directory is reused.
    """
    os.makedirs(model_dir, exist_ok=True)
    marker = os.path.join(model_dir, ".synthetic.json")
    recipe = {"shape": shape.config_json(), "quant": quant or "fp16", "version": 1}
    if os.path.exists(marker):
        with open(marker) as f:
            if json.load(f) == recipe:
                return model_dir
    write_config_json(os.path.join(model_dir, "config.json"), shape.config_json())
    synth_embeddings(shape).tofile(os.path.join(model_dir, "embeddings.bin"))
    _normal(GLOBAL_SEED["final_norm"], (shape.hidden_dim,), 0.01, 1.0).tofile(
        os.path.join(model_dir, "final_norm.bin"))
    if shape.num_lm_heads > 1:  # one FP32 table per head (src/matmul_decoder.c:883-901)
        lv = shape.lm_head_vocab_size or shape.vocab_size
        for i in range(shape.num_lm_heads):
            _normal(GLOBAL_SEED["lm_head"] + 1 + i, (lv, shape.hidden_dim), 0.02).tofile(
                os.path.join(model_dir, f"lm_head_{i:02d}.bin"))
    elif not shape.tie_word_embeddings:
        _normal(GLOBAL_SEED["lm_head"], (shape.vocab_size, shape.hidden_dim), 0.02).tofile(
            os.path.join(model_dir, "lm_head.bin"))
    for layer in range(shape.num_layers):
        d = layer_dir(model_dir, layer)
        os.makedirs(d, exist_ok=True)
        t = synth_layer_tensors(shape, layer)
        for name in ("input_norm", "post_attn_norm", "q_norm", "k_norm"):
            t[name].tofile(os.path.join(d, f"{name}.bin"))
        for p in PROJS:
            t[p].tofile(os.path.join(d, f"{p}.bin"))
    if quant in ("int8", "int4"):
        quantize_model_dir(model_dir, quant, lib_path=lib_path)
    with open(marker, "w") as f:
        json.dump(recipe, f)
    return model_dir


def _quant_lib(lib_path: str | None):
    if lib_path is None:
        here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        lib_path = os.path.join(here, "lib", "libmatmul_decoder.so")
    lib = ctypes.CDLL(lib_path)
    fn = lib.matmul_decoder_quantize_weight
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def quantize_weight(w_f16: np.ndarray, bits: int, lib_path: str | None = None):
    """Quantize an FP16 [K,N] weight with the runtime's per-column rule.

    Returns (q, scales): int8 [K,N] (bits=8) or packed uint8 [K,N/2] (bits=4),
    and FP32 scales [N].
    """
    w = np.ascontiguousarray(w_f16, dtype=np.float16)
    K, N = w.shape
    q = np.empty((K, N if bits == 8 else N // 2), dtype=np.uint8)
    s = np.empty(N, dtype=np.float32)
    rc = _quant_lib(lib_path)(w.ctypes.data, K, N, bits, q.ctypes.data, s.ctypes.data)
    if rc != 0:
        raise ValueError(f"quantize_weight failed ({rc}) for K={K} N={N} bits={bits}")
    return (q.view(np.int8) if bits == 8 else q), s


def quantize_model_dir(model_dir: str, quant: str, lib_path: str | None = None) -> None:
    """Write {proj}_weight.bin and {proj}_scales.bin for every layer from {proj}.bin."""
    bits = {"int8": 8, "int4": 4}[quant]
    with open(os.path.join(model_dir, "config.json")) as f:
        cfg = json.load(f)
    shape = ModelShape(**{k: cfg[k] for k in ("hidden_dim", "num_q_heads", "num_kv_heads",
                                              "head_dim", "ffn_dim", "num_layers")})
    for layer in range(shape.num_layers):
        d = layer_dir(model_dir, layer)
        if not os.path.isdir(d):
            d = os.path.join(model_dir, f"layer_{layer:02d}")
        for p, (k, n) in shape.proj_shapes().items():
            w = np.fromfile(os.path.join(d, f"{p}.bin"), dtype=np.float16).reshape(k, n)
            q, s = quantize_weight(w, bits, lib_path)
            q.tofile(os.path.join(d, f"{p}_weight.bin"))
            s.tofile(os.path.join(d, f"{p}_scales.bin"))


# ─── seeded inputs of the benchmark configs ───

def seeded_hidden(seed: int, n: int, dim: int) -> np.ndarray:
    """N(0,1) FP32 rows (stand-in for audio-encoder embeddings)."""
    return _normal(seed, (n, dim), 1.0)


def seeded_kv(seed: int, length: int, num_kv_heads: int, head_dim: int) -> np.ndarray:
    """N(0,1) values rounded to FP16, [length][num_kv_heads][head_dim]."""
    return _normal(seed, (length, num_kv_heads, head_dim), 1.0).astype(np.float16)


def kv_seed(layer: int, which: int, seq: int = 0) -> int:
    """Seed of the pre-filled K (which=0) or V (which=1) of one layer/sequence."""
    return 700_000 + 100_000 * seq + 2 * layer + which
