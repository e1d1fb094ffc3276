"""Vocab-sharded lm_head of the batched decoder (NCCL all-gather of the final
hidden rows, each rank's vocab slice, all-reduce MAX of packed argmax keys).

* One GPU: a one-rank shard must give exactly the tokens of the unsharded
  decoder (same GEMM over the whole vocabulary, plus the key merge and the
  NCCL collectives on one rank).
* Two GPUs (skipped with fewer): two ranks, each decoding half of the
  sequences with a vocabulary half, against an unsharded decoder of the same
  sequences on the same rank.  The global argmax is the reference's first
  maximum (src/cpu_ops.c:575-586), so tokens must agree exactly.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402
import model_format as mf  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

HERE = os.path.dirname(os.path.abspath(__file__))


def setup_batch(mdir, seqs, lens, quant="int8", layers=4):
    bat = bd.BatchDecoder(mdir, len(seqs), quant, max_seq_len=256)
    for i, s in enumerate(seqs):
        L = int(lens[s])
        for layer in range(layers):
            bat.set_kv(i, layer, 0, mf.seeded_kv(mf.kv_seed(layer, 0, s), L, 8, 128),
                       mf.seeded_kv(mf.kv_seed(layer, 1, s), L, 8, 128))
        bat.set_seq_len(i, L)
    return bat


def test_one_rank_shard_equals_unsharded(model_cache):
    mdir = mf.write_synthetic_model(os.path.join(model_cache, "small_int8"),
                                    mf.ModelShape(num_layers=4, vocab_size=8192, name="small"), quant="int8")
    n = 20
    lens = np.random.default_rng(3).integers(4, 200, size=n)
    a = setup_batch(mdir, list(range(n)), lens)
    b = setup_batch(mdir, list(range(n)), lens)
    b.shard_vocab(0, 1, bd.nccl_unique_id(), n + 3)
    toks = (np.arange(n, dtype=np.int32) * 37 + 5) % 8192
    for step in range(4):
        ta = a.step(toks)
        tb = b.step(toks)
        np.testing.assert_array_equal(ta, tb)
        toks = ta
    # a rank holds one vocab slice: full logits are not available
    logits = np.empty((n, 8192), np.float32)
    assert bd.capi().matmul_decoder_batch_step(b.b, toks.ctypes.data, np.empty(n, np.int32).ctypes.data,
                                               logits.ctypes.data) == -5
    a.close()
    b.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_shard_matches_unsharded(model_cache):
    mdir = mf.write_synthetic_model(os.path.join(model_cache, "small_int8"),
                                    mf.ModelShape(num_layers=4, vocab_size=8192, name="small"), quant="int8")
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "mp_vocab_shard.py"), mdir]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("rank ok") == 2, r.stdout[-3000:]
