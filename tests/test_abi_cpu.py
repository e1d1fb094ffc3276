"""C-ABI checks that need no GPU.

* libmatmul_decoder.so loads and exports every function include/*.h declares;
* the quantisers are bit-exact against the oracle's restatement of the
  reference rule (src/matmul_decoder.c:1216-1244);
* config.json parsing, sampling and argument validation of the C API.
No kernel is launched here.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

import b200_decoder as bd
import model_format as mf
import ref_decoder as ref

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("matmul_decoder.h", "b2_kernels.h"):
        text = open(os.path.join(REPO, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"static inline[^{]*\{.*?\n\}", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z][a-z0-9_]*)\s*\(", text, flags=re.M):
            if m.group(1) not in ("if", "sizeof", "void"):
                names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(bd.LIB_PATH)
    names = declared_functions()
    assert "matmul_decoder_step" in names and "b2_gemv" in names
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes table covers them all
    assert names <= set(bd.SIGNATURES), names - set(bd.SIGNATURES)
    bd.capi()


def test_pybind_module_surface():
    import matmul_decoder as md
    assert md.__version__ == "1.0.0"
    for name in ("step", "prefill", "prefill_batch", "step_get_token", "clear_kv_cache", "generate",
                 "seq_len", "config", "stats"):
        assert hasattr(md.MatmulDecoder, name), name
    c = md.config_qwen3_0_6b()
    assert c["hidden_dim"] == 1024 and c["num_kv_heads"] == 8 and c["exec_mode"] == "dual_core"
    assert md.config_qwen3_0_6b_single_core()["exec_mode"] == "single_core"
    with pytest.raises(RuntimeError):
        md.MatmulDecoder("/nonexistent-model-dir")


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("shape", [(64, 32), (1024, 2048), (3072, 64)])
def test_quantize_weight_bit_exact(bits, shape):
    rng = np.random.default_rng(bits * 100 + shape[0])
    w = (rng.standard_normal(shape) * 0.02).astype(np.float16)
    w[:, 3] = 0  # an all-zero column: scale 0, inv 0
    w[5, 7] = np.float16(0.5)  # a column dominated by one value
    q, s = mf.quantize_weight(w, bits)
    q_ref, s_ref = ref.quantize_cols(w, bits)
    np.testing.assert_array_equal(q.view(np.uint8), q_ref.view(np.uint8))
    np.testing.assert_array_equal(s.view(np.uint32), s_ref.view(np.uint32))


def test_quantize_rounding_half_away_from_zero():
    # w * (127 / max) landing exactly on .5 must round away from zero (roundf).
    w = np.array([[127.0], [0.5], [-0.5], [1.5], [-2.5]], np.float16)
    q, s = mf.quantize_weight(w, 8)
    assert q[:, 0].tolist() == [127, 1, -1, 2, -3]


def test_quantize_lm_head_bit_exact():
    rng = np.random.default_rng(7)
    V, K = 4100, 256  # crosses one 4096-column tile boundary
    table = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    q = np.empty((V, K), np.int8)
    s = np.empty(V, np.float32)
    bd.check(bd.capi().matmul_decoder_quantize_lm_head(table.ctypes.data, V, K, q.ctypes.data,
                                                        s.ctypes.data))
    q_tiles, s_ref = ref.quantize_lm_head(table.astype(np.float16), tile_n=4096)
    # reference tiles are [tile][K][4096]; a vocab row v is column v % 4096 of tile v // 4096
    q_ref = np.concatenate([q_tiles[t].T for t in range(q_tiles.shape[0])])[:V]
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(s.view(np.uint32), s_ref[:V].view(np.uint32))
    assert np.all(s_ref[V:] == 0)


def test_load_config_parses_reference_keys_and_exponents(tmp_path):
    p = tmp_path / "config.json"
    p.write_text('{"name": "x: y", "hidden_dim": 512, "num_layers": 3, "rms_eps": 1e-05,\n'
                 ' "rope_theta": 10000.0, "rope_style": 1, "tie_word_embeddings": false,\n'
                 ' "has_qk_norm": true, "vocab_size": 4096}')
    cfg = bd.MatmulDecoderConfig()
    assert bd.capi().matmul_decoder_load_config(str(p).encode(), ctypes.byref(cfg)) == 0
    assert (cfg.hidden_dim, cfg.num_layers, cfg.vocab_size, cfg.rope_style) == (512, 3, 4096, 1)
    assert abs(cfg.rms_eps - 1e-5) < 1e-12 and cfg.rope_theta == 10000.0
    assert cfg.tie_word_embeddings == 0 and cfg.has_qk_norm == 1
    assert cfg.num_q_heads == 16 and cfg.head_dim == 128  # defaults from the Qwen3 preset
    assert bd.capi().matmul_decoder_load_config(b"/nonexistent.json", ctypes.byref(cfg)) == -3


def test_written_config_round_trips(tmp_path):
    shape = mf.ModelShape(num_layers=2, vocab_size=4096)
    mf.write_config_json(str(tmp_path / "config.json"), shape.config_json())
    cfg = bd.MatmulDecoderConfig()
    assert bd.capi().matmul_decoder_load_config(str(tmp_path / "config.json").encode(),
                                                ctypes.byref(cfg)) == 0
    assert abs(cfg.rms_eps - 1e-6) < 1e-13 and cfg.rope_style == 1 and cfg.num_layers == 2


class SamplingParams(ctypes.Structure):
    _fields_ = [("top_k", ctypes.c_int), ("top_p", ctypes.c_float), ("temperature", ctypes.c_float),
                ("repeat_penalty", ctypes.c_float), ("repeat_tokens", ctypes.c_void_p),
                ("n_repeat_tokens", ctypes.c_int)]


def test_sample_token_greedy_and_topk():
    L = bd.capi()
    x = np.array([0.1, 3.0, 3.0, -1.0, 2.9], np.float32)
    p = SamplingParams(1, 1.0, 1.0, 1.0, None, 0)
    assert L.matmul_sample_token(x.ctypes.data, 5, ctypes.byref(p)) == 1  # first max
    p = SamplingParams(2, 1.0, 1.0, 1.0, None, 0)
    got = {L.matmul_sample_token(x.ctypes.data, 5, ctypes.byref(p)) for _ in range(200)}
    assert got <= {1, 2} and len(got) == 2
    rep = np.array([1, 2], np.int32)
    p = SamplingParams(1, 1.0, 1.0, 10.0, rep.ctypes.data, 2)
    assert L.matmul_sample_token(x.ctypes.data, 5, ctypes.byref(p)) == 4


def test_c_api_rejects_bad_arguments():
    L = bd.capi()
    assert L.matmul_decoder_step(None, 0, None, None) == -1
    assert L.matmul_decoder_prefill_batch(None, None, 4) == -1
    assert L.matmul_decoder_get_seq_len(None) == 0
    assert L.matmul_decoder_create(b"/nonexistent", None, 0, 16) is None
    assert L.matmul_decoder_export_hf_model(b"a", b"b", 0) == -5
    kv = L.matmul_kv_cache_create(2, 8, 128, 16)
    assert kv and L.matmul_kv_cache_get_seq_len(kv) == 0
    L.matmul_kv_cache_clear(kv)
    L.matmul_kv_cache_destroy(kv)
    assert L.matmul_kv_cache_create(0, 8, 128, 16) is None
