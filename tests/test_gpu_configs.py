"""GPU parity at the benchmark shapes the other decoder tests reduce, and for
the API entry points beside the decode step.

* cfg5 at its benchmark shape: 64 sequences, 28-layer W4A16 model, vocab
  151936, contexts U[128, 4096] from the benchmark's seed; sampled sequences
  (the shortest, the longest and others) checked against the oracle over two
  teacher-forced batched steps.
* batched decode at 20 sequences (INT4 and INT8): the tensor-core GEMMs with
  cluster split-K and the lm_head GEMM with the argmax epilogue over ragged
  contexts longer than one 512-position attention block; every row checked.
* cfg3 W8A16 at L = 1024 (split attention units of the persistent kernel on
  the 28-layer model).
* cfg4 M = 512 on the 28-layer FP16 model.
* matmul_decoder_step_head with 15 FP32 heads (the code-predictor preset of
  ref include/matmul_decoder.h:159-184; ref src/matmul_decoder.c:1636-1742).
* matmul_decoder_create_from_weights against the directory-loaded decoder.
* run_embed of the RKLLM-style wrapper (ref python/matmul_decoder.py:164-241).

Criteria as in test_gpu_decoder.py: cosine >= 0.9995 and max-abs <= 2e-2 per
step on logits and hidden states, tokens identical unless the oracle's top-2
gap is below 1e-3 * |top-1| (then the oracle's token is fed to both sides).
"""
from __future__ import annotations

import os
import shutil

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402
import model_format as mf  # noqa: E402
import ref_decoder as ref  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

GAP_TOL = 1e-3
NTH = max(1, min(32, os.cpu_count() or 1))
FIRST_TOKEN = 151644


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def assert_parity(got, exp, what=""):
    c = cos(got, exp)
    d = float(np.abs(np.asarray(got, np.float64) - np.asarray(exp, np.float64)).max())
    assert c >= 0.9995 and d <= 2e-2, f"{what}: cos={c:.6f} max_abs={d:.3e}"
    return c, d


def tokens_agree(t_got, t_exp, logits_exp, what=""):
    if t_got == t_exp:
        return True
    top = np.sort(logits_exp)[-2:]
    gap = float(top[1] - top[0])
    assert gap <= GAP_TOL * abs(float(top[1])), f"{what}: token {t_got} != {t_exp}, gap {gap}"
    return False


def model(cache, dirname, quant="fp16", **shape):
    d = os.path.join(cache, dirname)
    return mf.write_synthetic_model(d, mf.ModelShape(**shape), quant=quant if quant != "fp16" else None)


# ── batched decode at the cfg5 benchmark shape ──

def test_cfg5_benchmark_shape(model_cache):
    mdir = model(model_cache, "full_int4", "int4")
    n, nl = 64, 28
    lens = np.random.default_rng(55).integers(128, 4097, size=n)  # bench.py's cfg5 contexts
    order = np.argsort(lens, kind="stable")
    sampled = sorted({int(order[0]), int(order[-1]), int(order[n // 2]), 5, 37})
    bat = bd.BatchDecoder(mdir, n, "int4", max_seq_len=4096 + 8)
    orcs = {}
    for s in range(n):
        bat.set_seq_len(s, int(lens[s]))
    for s in sampled:
        L = int(lens[s])
        d = ref.RefDecoder(mdir, "int4", max_seq_len=L + 4, nthreads=NTH)
        for layer in range(nl):
            k = mf.seeded_kv(mf.kv_seed(layer, 0, s), L, 8, 128)
            v = mf.seeded_kv(mf.kv_seed(layer, 1, s), L, 8, 128)
            bat.set_kv(s, layer, 0, k, v)
            d.set_kv(layer, 0, k, v)
        d.seq_len = L
        orcs[s] = d
    toks = (np.arange(n, dtype=np.int32) * 977 + FIRST_TOKEN) % 151936
    for step in range(2):
        out, logits = bat.step(toks, want_logits=True)
        nxt = out.copy()
        for s in sampled:
            t_o, lo = orcs[s].step(int(toks[s]))
            assert_parity(logits[s], lo, f"seq {s} (L={int(lens[s])}) step {step}")
            tokens_agree(int(out[s]), t_o, lo, f"seq {s} step {step}")
            nxt[s] = t_o
        # argmax epilogue == argmax of the returned logits on every row
        for s in range(n):
            assert out[s] == int(np.argmax(logits[s])) or np.isclose(logits[s].max(), logits[s][out[s]])
        toks = nxt
    for s in range(n):
        assert bd.capi().matmul_decoder_batch_get_seq_len(bat.b, s) == int(lens[s]) + 2
    bat.close()


@pytest.mark.parametrize("quant", ["int4", "int8"])
def test_batched_twenty_sequences_ragged(model_cache, quant):
    """n >= 16 rows: tcgen05 GEMMs (cluster split-K) and the lm_head GEMM with
    its argmax epilogue, contexts up to 1500 (several attention blocks)."""
    mdir = model(model_cache, f"small_{quant}", quant, num_layers=4, vocab_size=8192, name="small")
    n = 20
    lens = np.random.default_rng(21).integers(8, 1500, size=n)
    lens[0], lens[1] = 1, 1499  # a one-position and a three-block context
    bat = bd.BatchDecoder(mdir, n, quant, max_seq_len=1536)
    orcs = []
    for s in range(n):
        L = int(lens[s])
        d = ref.RefDecoder(mdir, quant, max_seq_len=1536, nthreads=NTH)
        for layer in range(4):
            k = mf.seeded_kv(mf.kv_seed(layer, 0, s), L, 8, 128)
            v = mf.seeded_kv(mf.kv_seed(layer, 1, s), L, 8, 128)
            bat.set_kv(s, layer, 0, k, v)
            d.set_kv(layer, 0, k, v)
        bat.set_seq_len(s, L)
        d.seq_len = L
        orcs.append(d)
    toks = (np.arange(n, dtype=np.int32) * 131 + 7) % 8192
    for step in range(4):
        out, logits = bat.step(toks, want_logits=True)
        nxt = []
        for s in range(n):
            t_o, lo = orcs[s].step(int(toks[s]))
            assert_parity(logits[s], lo, f"{quant} seq {s} step {step}")
            tokens_agree(int(out[s]), t_o, lo, f"{quant} seq {s} step {step}")
            nxt.append(t_o)
        toks = np.array(nxt, np.int32)
    bat.close()


# ── cfg3 at L = 1024 ──

def test_cfg3_w8a16_context_1024(model_cache):
    mdir = model(model_cache, "full_int8", "int8")
    L, steps = 1024, 3
    dec = bd.Decoder(mdir, "int8", max_seq_len=L + 16)
    assert dec.uses_persistent_kernel()
    orc = ref.RefDecoder(mdir, "int8", max_seq_len=L + 16, nthreads=NTH)
    for layer in range(28):
        k = mf.seeded_kv(mf.kv_seed(layer, 0), L, 8, 128)
        v = mf.seeded_kv(mf.kv_seed(layer, 1), L, 8, 128)
        dec.set_kv(layer, 0, k, v)
        orc.set_kv(layer, 0, k, v)
    dec.set_seq_len(L)
    orc.seq_len = L
    tok = FIRST_TOKEN
    for i in range(steps):
        t_g, lg = dec.step_logits(tok)
        t_o, lo = orc.step(tok)
        assert_parity(lg, lo, f"L=1024 step {i} logits")
        assert_parity(dec.hidden(), orc.last_hidden, f"L=1024 step {i} hidden")
        tokens_agree(t_g, t_o, lo, f"L=1024 step {i}")
        tok = t_o


# ── cfg4 M = 512 on the 28-layer model ──

def test_cfg4_prefill_512_full_model(model_cache):
    mdir = model(model_cache, "full_fp16", "fp16")
    M = 512
    dec = bd.Decoder(mdir, "fp16", max_seq_len=M + 8)
    orc = ref.RefDecoder(mdir, "fp16", max_seq_len=M + 8, nthreads=NTH)
    emb = mf.seeded_hidden(830_000 + M, M, 1024)
    dec.prefill_batch(emb)
    orc.prefill_batch(emb)
    assert dec.seq_len == orc.seq_len == M
    assert_parity(dec.hidden(), orc.last_hidden, "M=512 last hidden")
    for layer in (0, 27):
        k, v = dec.get_kv(layer, 0, M)
        assert_parity(k.astype(np.float32), orc.k_cache[layer, :M], f"K layer {layer}")
        assert_parity(v.astype(np.float32), orc.v_cache[layer, :M], f"V layer {layer}")


# ── matmul_decoder_step_head: 15 FP32 heads ──

def test_step_head_fifteen_heads(model_cache):
    shape = dict(num_layers=5, vocab_size=2048, tie_word_embeddings=False, num_lm_heads=15,
                 lm_head_vocab_size=2048, name="tts_cp")
    mdir = model(model_cache, "tts_cp", "fp16", **shape)
    dec = bd.Decoder(mdir, "fp16", max_seq_len=20)
    assert not dec.uses_persistent_kernel()
    orc = ref.RefDecoder(mdir, "fp16", max_seq_len=20, nthreads=NTH)
    emb = mf.seeded_hidden(880_000, 2, 1024)
    tok = None
    for i in range(2):  # embedding inputs, as the code predictor is fed
        t_g, lg = dec.step_head(embedding=emb[i], lm_head_idx=0)
        t_o, lo = orc.step_head(embedding=emb[i], lm_head_idx=0)
        assert_parity(lg, lo, f"embedding step {i}")
        tokens_agree(t_g, t_o, lo, f"embedding step {i}")
        tok = t_o
    for idx in (1, 7, 14):  # one token per head
        t_g, lg = dec.step_head(tok, lm_head_idx=idx)
        t_o, lo = orc.step_head(tok, lm_head_idx=idx)
        assert lg.shape == (2048,)
        assert_parity(lg, lo, f"head {idx}")
        tokens_agree(t_g, t_o, lo, f"head {idx}")
        tok = t_o
    assert dec.seq_len == orc.seq_len == 5
    # error cases of the reference: head index out of range, bad token
    assert dec.step_head(tok, lm_head_idx=15)[0] == -1
    assert dec.step_head(tok, lm_head_idx=-1)[0] == -1
    assert dec.step_head(5000, lm_head_idx=0)[0] == -1
    assert dec.seq_len == 5


# ── matmul_decoder_create_from_weights ──

def _host_layers(mdir, quant, nl, shape):
    out = []
    for layer in range(nl):
        d = mf.layer_dir(mdir, layer)
        L = {}
        for p, (k, n) in shape.proj_shapes().items():
            if quant == "fp16":
                L[p] = (np.fromfile(os.path.join(d, f"{p}.bin"), np.float16).reshape(k, n), None)
            else:
                nb = k * n if quant == "int8" else k * n // 2
                L[p] = (np.fromfile(os.path.join(d, f"{p}_weight.bin"), np.uint8, nb),
                        np.fromfile(os.path.join(d, f"{p}_scales.bin"), np.float32, n))
        for f, name in (("input_norm_weight", "input_norm"), ("post_attn_norm_weight", "post_attn_norm"),
                        ("q_norm_weight", "q_norm"), ("k_norm_weight", "k_norm")):
            L[f] = np.fromfile(os.path.join(d, f"{name}.bin"), np.float32)
        out.append(L)
    return out


@pytest.mark.parametrize("quant", ["fp16", "int8"])
def test_create_from_weights_matches_directory(model_cache, quant):
    """The LayerWeights struct carries no final norm, so (as the reference
    loader does without final_norm.bin, src/matmul_decoder.c:1162-1165) the
    last layer's post-attention norm serves as the final norm.  The directory
    model here is written with that same final norm so both paths agree."""
    shape = mf.ModelShape(num_layers=3, vocab_size=4096, name=f"cfw_{quant}")
    src = model(model_cache, f"cfw_src_{quant}", quant, num_layers=3, vocab_size=4096, name=f"cfw_{quant}")
    mdir = os.path.join(model_cache, f"cfw_{quant}")
    if not os.path.exists(mdir):
        shutil.copytree(src, mdir)
        shutil.copyfile(os.path.join(mf.layer_dir(mdir, 2), "post_attn_norm.bin"),
                        os.path.join(mdir, "final_norm.bin"))
    a = bd.Decoder(mdir, quant, max_seq_len=64)
    cfg = bd.MatmulDecoderConfig()
    bd.check(bd.capi().matmul_decoder_load_config(os.path.join(mdir, "config.json").encode(),
                                                  bd.ctypes.byref(cfg)), "load_config")
    emb = np.fromfile(os.path.join(mdir, "embeddings.bin"), np.float32).reshape(4096, 1024)
    b = bd.Decoder.from_weights(cfg, emb, _host_layers(mdir, quant, 3, shape), None, quant, max_seq_len=64)
    orc = ref.RefDecoder(mdir, quant, max_seq_len=64, nthreads=NTH)
    pre = mf.seeded_hidden(890_000, 6, 1024)
    a.prefill_batch(pre)
    b.prefill_batch(pre)
    orc.prefill_batch(pre)
    tok = 11
    for i in range(5):
        ta, la = a.step_logits(tok)
        tb, lb = b.step_logits(tok)
        to, lo = orc.step(tok)
        # same weights and kernels; the decode kernel's cross-CTA float
        # additions land in a run-dependent order, so equal up to FP32 rounding
        np.testing.assert_allclose(la, lb, rtol=0, atol=1e-4)
        assert ta == tb or tokens_agree(tb, ta, la, "from_weights vs directory")
        assert_parity(lb, lo, f"from_weights step {i}")
        tokens_agree(tb, to, lo, f"from_weights step {i}")
        tok = to
    # reference error behaviour: NULL arguments give NULL
    assert not bd.capi().matmul_decoder_create_from_weights(None, None, None, None, 0, 64)


# ── RKLLM-style wrapper: run_embed ──

def test_wrapper_run_embed_matches_oracle(model_cache):
    import matmul_decoder_wrapper as w
    mdir = model(model_cache, "small_fp16", "fp16", num_layers=4, vocab_size=8192, name="small")
    dec = w.create_decoder(mdir, quant_type="fp16", max_context_len=96, max_new_tokens=10)
    emb = mf.seeded_hidden(895_000, 12, 1024)
    out = dec.run_embed(emb, 12)
    orc = ref.RefDecoder(mdir, "fp16", max_seq_len=96, nthreads=NTH)
    orc.prefill_batch(emb[:-1])
    assert out["n_tokens_generated"] == 10 and out["ret_code"] == 0
    assert dec.seq_len == 12 + 10 - 1
    got = out["token_ids"]
    t, lo = orc.step(embedding=emb[-1])
    for i, g in enumerate(got):  # identical up to the first near-tie, if any
        if not tokens_agree(g, t, lo, f"run_embed token {i}"):
            break
        if i + 1 < len(got):
            t, lo = orc.step(t)
    # keep_history=0 clears the cache: a second call reproduces the first
    out2 = dec.run_embed(emb, 12)
    assert out2["text"] == out["text"] and out2["n_tokens_generated"] == 10
    dec.release()
