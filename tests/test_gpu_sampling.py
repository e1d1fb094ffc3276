"""On-device sampling (b2_sample_token) against the sampling oracle
(oracle/ref_sample.py, pinned to the host sampler matmul_sample_token by
tests/test_sampling_cpu.py).

* greedy and repeat-penalty paths: the exact token;
* the kept set (top-k, ties at the threshold by lowest index, top-p cut):
  the kernel's count of kept entries equals the oracle's, every draw is in
  the oracle's set;
* the distribution: chi-square of many draws (one per counter) against the
  oracle's probabilities;
* determinism in (seed, counter); the decoder-level step_sample and
  matmul_decoder_generate.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402
import model_format as mf  # noqa: E402
import ref_sample as rs  # noqa: E402

scipy_stats = pytest.importorskip("scipy.stats")

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = torch.device("cuda:0")


def _sample(logits_d, V, top_k, top_p, temp, seed=1, counter=0, penalty=1.0, rep=None):
    """(token, info[4]) of one b2_sample_token call."""
    L = bd.capi()
    out = torch.full((8,), -7, dtype=torch.int32, device=DEV)
    rep_d = None if rep is None else torch.tensor(rep, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bd.check(L.b2_sample_token(logits_d.data_ptr(), V, None if rep_d is None else rep_d.data_ptr(),
                               0 if rep is None else len(rep), penalty, top_k, top_p, temp, seed, counter,
                               out.data_ptr(), out[1:].data_ptr(), stream), "b2_sample_token")
    o = out.cpu().tolist()
    return o[0], o[1:5]


def _draws(logits_d, V, top_k, top_p, temp, n, seed=3, penalty=1.0, rep=None):
    """n draws (counters 0 .. n-1), all kept on the device until the end."""
    L = bd.capi()
    toks = torch.full((n,), -7, dtype=torch.int32, device=DEV)
    rep_d = None if rep is None else torch.tensor(rep, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    base = toks.data_ptr()
    for i in range(n):
        bd.check(L.b2_sample_token(logits_d.data_ptr(), V, None if rep_d is None else rep_d.data_ptr(),
                                   0 if rep is None else len(rep), penalty, top_k, top_p, temp, seed, i,
                                   base + 4 * i, None, stream), "b2_sample_token")
    return toks.cpu().numpy()


def _chi2(draws, idx, prob):
    counts = np.array([(draws == i).sum() for i in idx], np.float64)
    exp = prob * draws.size
    big = exp >= 5
    obs = np.append(counts[big], counts[~big].sum())
    ex = np.append(exp[big], exp[~big].sum())
    if ex[-1] == 0:
        obs, ex = obs[:-1], ex[:-1]
    return scipy_stats.chisquare(obs, ex).pvalue


def test_greedy_first_maximum_and_penalty():
    V = 151936
    rng = np.random.default_rng(1)
    x = rng.standard_normal(V).astype(np.float32)
    x[5000] = x[140000] = x.max() + 2.0  # tie: the first index wins
    d = torch.from_numpy(x).to(DEV)
    tok, info = _sample(d, V, 1, 1.0, 0.5)
    assert tok == 5000 and info[0] == 1
    rep = [5000, 5000, 140000, 7]  # 5000 penalized twice
    tok, _ = _sample(d, V, 1, 1.0, 1.0, penalty=1.7, rep=rep)
    assert tok == int(rs.kept_distribution(x, 1, repeat_penalty=1.7, repeat_tokens=rep)[0][0])
    # negative logits are multiplied by the penalty
    y = -np.abs(x)
    y[123] = -1e-3
    dy = torch.from_numpy(y).to(DEV)
    tok, _ = _sample(dy, V, 1, 1.0, 1.0, penalty=3.0, rep=[123])
    assert tok == int(rs.kept_distribution(y, 1, repeat_penalty=3.0, repeat_tokens=[123])[0][0])


@pytest.mark.parametrize("top_k,top_p,temp", [(50, 1.0, 0.8), (50, 0.9, 0.8), (1000, 0.5, 1.0), (0, 0.7, 1.2),
                                              (0, 1.0, 1.0), (40000, 0.95, 2.0)])
def test_kept_set_matches_oracle(top_k, top_p, temp):
    V = 151936
    rng = np.random.default_rng(7 + top_k)
    x = (rng.standard_normal(V) * 3.0).astype(np.float32)
    rep = [int(i) for i in np.argsort(-x)[:5]] + [int(np.argmax(x))]
    d = torch.from_numpy(x).to(DEV)
    idx, prob = rs.kept_distribution(x, top_k, top_p, temp, 1.2, rep)
    kept = set(idx.tolist())
    for counter in range(8):
        tok, info = _sample(d, V, top_k, top_p, temp, seed=99, counter=counter, penalty=1.2, rep=rep)
        assert info[0] == idx.size, (info, idx.size)
        assert info[1] == (V if top_k <= 0 or top_k > V else top_k)
        assert tok in kept


def test_ties_at_the_top_k_threshold_go_to_lowest_indices():
    V = 4096
    x = np.full(V, -4.0, np.float32)
    x[[900, 30, 3000]] = 3.0
    fives = np.array([2500, 11, 4000, 700, 55, 1200, 3333, 18, 2048, 999, 1500, 600])
    x[fives] = 1.0
    d = torch.from_numpy(x).to(DEV)
    idx, prob = rs.kept_distribution(x, 10, 1.0, 1.0)
    assert set(idx.tolist()) == {30, 900, 3000} | set(np.sort(fives)[:7].tolist())
    draws = _draws(d, V, 10, 1.0, 1.0, 6000)
    assert set(draws.tolist()) <= set(idx.tolist())
    assert _chi2(draws, idx, prob) > 1e-4


@pytest.mark.parametrize("top_k,top_p,temp", [(12, 1.0, 1.0), (20, 0.9, 1.3), (0, 0.85, 0.9)])
def test_distribution_matches_oracle(top_k, top_p, temp):
    V = 3000
    rng = np.random.default_rng(21 + top_k)
    x = (rng.standard_normal(V) * 2.0).astype(np.float32)
    x[np.argsort(-x)[:30]] += 2.0  # a head of candidates that carries most mass
    rep = [int(np.argmax(x))] * 2
    d = torch.from_numpy(x).to(DEV)
    idx, prob = rs.kept_distribution(x, top_k, top_p, temp, 1.5, rep)
    draws = _draws(d, V, top_k, top_p, temp, 8000, penalty=1.5, rep=rep)
    assert set(draws.tolist()) <= set(idx.tolist())
    assert _chi2(draws, idx, prob) > 1e-4


def test_draw_is_a_function_of_seed_and_counter():
    V = 151936
    x = (np.random.default_rng(3).standard_normal(V) * 2).astype(np.float32)
    d = torch.from_numpy(x).to(DEV)
    a = [_sample(d, V, 0, 1.0, 1.0, seed=5, counter=c)[0] for c in range(6)]
    b = [_sample(d, V, 0, 1.0, 1.0, seed=5, counter=c)[0] for c in range(6)]
    assert a == b and len(set(a)) > 1
    assert _sample(d, V, 0, 1.0, 1.0, seed=6, counter=0)[0] != a[0] or \
        _sample(d, V, 0, 1.0, 1.0, seed=7, counter=0)[0] != a[0]


def test_rejects_bad_arguments():
    L = bd.capi()
    big = int(L.b2_sample_max_vocab()) + 1
    out = torch.zeros(8, dtype=torch.int32, device=DEV)
    assert L.b2_sample_token(out.data_ptr(), big, None, 0, 1.0, 0, 1.0, 1.0, 0, 0, out.data_ptr(), None, None) == -1
    assert L.b2_sample_token(out.data_ptr(), 16, None, 3, 1.0, 0, 1.0, 1.0, 0, 0, out.data_ptr(), None, None) == -1


@pytest.fixture(scope="module")
def small_model(model_cache):
    d = os.path.join(model_cache, "sample_l2_int8")
    mf.write_synthetic_model(d, mf.ModelShape(num_layers=2), quant="int8")
    return d


def test_decoder_step_sample_and_generate(small_model):
    dec = bd.Decoder(small_model, "int8", max_seq_len=64)
    greedy_ref = bd.Decoder(small_model, "int8", max_seq_len=64)
    # a near-zero temperature is the greedy choice
    p = bd.SamplingParams(0, 1.0, 1e-6, 1.0, None, 0)
    toks_a = []
    tok = 151644
    for _ in range(4):
        tok = dec.step_sample(tok, p)
        toks_a.append(tok)
    tok = 151644
    toks_b = []
    for _ in range(4):
        tok = greedy_ref.step_token(tok)
        toks_b.append(tok)
    assert toks_a == toks_b
    # seeded draws repeat after set_seed and a cleared cache
    p = bd.SamplingParams(40, 0.95, 1.5, 1.1, None, 0)
    runs = []
    for _ in range(2):
        bd.capi().matmul_decoder_clear_kv_cache(dec.ctx)
        dec.set_seed(1234)
        tok, seq = 151644, []
        for _ in range(6):
            tok = dec.step_sample(tok, p)
            seq.append(tok)
        runs.append(seq)
    assert runs[0] == runs[1] and all(0 <= t < dec.V for t in runs[0])
    # generate: the same draws through the reference entry point
    bd.capi().matmul_decoder_clear_kv_cache(dec.ctx)
    dec.set_seed(1234)
    prompt = np.array([151644], np.int32)
    out = []
    cb = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p)(lambda t, s, u: out.append(t))
    n = bd.capi().matmul_decoder_generate(dec.ctx, prompt.ctypes.data, 1, 6, ctypes.byref(p), cb, None)
    assert n == 6 and out == runs[0]
