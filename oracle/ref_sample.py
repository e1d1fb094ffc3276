"""CPU ORACLE for token sampling (test infrastructure, never the product).

Restates, in numpy, the distribution a sampler draws from:

* temperature, then the top_k largest values, a softmax over them and one
  draw: top_k_sample_f32 (src/cpu_ops.c:593-647 of
  suharvest/rknn-matmul-parallel).  Its insertion scan keeps the earlier index
  on equal values, so ties order by index.
* top_k == 1 is greedy argmax, first index of the maximum
  (src/matmul_decoder.c:2316-2320, argmax_f32 src/cpu_ops.c:575-586); as there,
  no temperature is applied on that path.
* the extensions of this runtime's matmul_sample_token
  (csrc/host/md_generate.c): a repeat penalty applied once per listed
  occurrence before everything else (x > 0 ? x / p : x * p), and a top-p cut
  that keeps the shortest prefix of the sorted top-k whose probability reaches
  top_p (the reference's top_p_sample_f32, src/cpu_ops.c:649-672, returns the
  argmax instead: its "simplified" stub).

Weights are exp(v - v_max) in float64, as the host sampler computes them.
Only tests/ use it.
"""
from __future__ import annotations

import numpy as np


def penalized(logits, repeat_penalty=1.0, repeat_tokens=()):
    x = np.asarray(logits, np.float32).copy()
    if repeat_penalty != 1.0:
        p = np.float32(repeat_penalty)
        for t in repeat_tokens:  # once per occurrence, in list order
            if 0 <= t < x.size:
                x[t] = x[t] / p if x[t] > 0 else x[t] * p
    return x


def sorted_candidates(logits, top_k=0, temperature=1.0, repeat_penalty=1.0, repeat_tokens=()):
    """(indices, values v) of the top_k entries by v descending, index ascending."""
    x = penalized(logits, repeat_penalty, repeat_tokens)
    temp = np.float32(temperature if temperature > 0 else 1.0)
    v = (x / temp).astype(np.float32)
    order = np.lexsort((np.arange(v.size), -v.astype(np.float64)))
    k = v.size if top_k <= 0 or top_k > v.size else top_k
    idx = order[:k]
    return idx, v[idx]


def kept_distribution(logits, top_k=0, top_p=1.0, temperature=1.0, repeat_penalty=1.0, repeat_tokens=()):
    """(indices, probabilities) a draw picks from; greedy returns one index."""
    if top_k == 1:
        x = penalized(logits, repeat_penalty, repeat_tokens)
        return np.array([int(np.argmax(x))]), np.array([1.0])
    idx, v = sorted_candidates(logits, top_k, temperature, repeat_penalty, repeat_tokens)
    w = np.exp(v.astype(np.float64) - float(v[0]))
    keep = idx.size
    if 0.0 < top_p < 1.0:
        cum = np.cumsum(w / w.sum())
        hit = np.nonzero(cum >= np.float32(top_p))[0]
        if hit.size:
            keep = int(hit[0]) + 1
    w = w[:keep]
    return idx[:keep], w / w.sum()
