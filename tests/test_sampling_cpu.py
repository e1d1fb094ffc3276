"""The sampling oracle (oracle/ref_sample.py) against the host sampler
matmul_sample_token, on CPU: same kept set (every draw lands in it) and the
same distribution (chi-square over repeated draws of the C library's
generator)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import b200_decoder as bd
import ref_sample as rs

scipy_stats = pytest.importorskip("scipy.stats")


def _params(top_k, top_p, temp, penalty=1.0, rep=None):
    return bd.SamplingParams(top_k, top_p, temp, penalty, None if rep is None else rep.ctypes.data,
                             0 if rep is None else rep.size)


def test_oracle_greedy_and_penalty_match_host_sampler():
    L = bd.capi()
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    x[100] = x[200] = x.max() + 1.0  # tie: first index wins
    p = _params(1, 1.0, 1.0)
    assert L.matmul_sample_token(x.ctypes.data, x.size, ctypes.byref(p)) == 100
    assert rs.kept_distribution(x, top_k=1)[0].tolist() == [100]
    rep = np.array([100, 100, 200], np.int32)  # 100 penalized twice
    p = _params(1, 1.0, 1.0, 1.5, rep)
    got = L.matmul_sample_token(x.ctypes.data, x.size, ctypes.byref(p))
    assert rs.kept_distribution(x, top_k=1, repeat_penalty=1.5, repeat_tokens=rep.tolist())[0].tolist() == [got]


@pytest.mark.parametrize("top_k,top_p,temp", [(8, 1.0, 1.0), (20, 0.9, 0.7), (0, 0.8, 1.3)])
def test_oracle_distribution_matches_host_sampler(top_k, top_p, temp):
    L = bd.capi()
    rng = np.random.default_rng(11 + top_k)
    x = (rng.standard_normal(48) * 1.5).astype(np.float32)
    x[7] = x[9]  # a tie inside the candidates
    rep = np.array([3, 3, 17], np.int32)
    idx, prob = rs.kept_distribution(x, top_k, top_p, temp, 1.3, rep.tolist())
    p = _params(top_k, top_p, temp, 1.3, rep)
    n = 6000
    draws = np.array([L.matmul_sample_token(x.ctypes.data, x.size, ctypes.byref(p)) for _ in range(n)])
    assert set(draws.tolist()) <= set(idx.tolist())
    counts = np.array([(draws == i).sum() for i in idx], np.float64)
    exp = prob * n
    big = exp >= 5  # pool the rare cells so the chi-square approximation holds
    obs = np.append(counts[big], counts[~big].sum())
    ex = np.append(exp[big], exp[~big].sum())
    if ex[-1] == 0:
        obs, ex = obs[:-1], ex[:-1]
    assert scipy_stats.chisquare(obs, ex).pvalue > 1e-4
