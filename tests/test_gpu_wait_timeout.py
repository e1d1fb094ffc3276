"""Timed-out waits of the persistent decode kernel, made to happen on purpose.

Every spin-wait of the kernel is bounded; when one runs out, the kernel sets
the error word of its state block, stops, lets its in-flight copies land and
returns, and the host resets the kernel's scratch and state and returns
MATMUL_DECODER_ERR_RKNN.  Here a short poll limit (B2_MK_POLL_LIMIT, read at
create) and a wait that can never complete (B2_MK_STALL_TEST: the lm_head
phase waits for a flag value no CTA writes) exercise that path without any
fault: the GPU keeps running and the next step must succeed and still match
the oracle.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402
import model_format as mf  # noqa: E402
import ref_decoder as ref  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

ERR_RKNN = -4


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


@pytest.fixture
def stall_model(model_cache):
    d = os.path.join(model_cache, "stall2")
    return mf.write_synthetic_model(d, mf.ModelShape(num_layers=2, vocab_size=4096, name="stall2"))


def test_timed_out_wait_reports_and_recovers(stall_model, monkeypatch):
    monkeypatch.setenv("B2_MK_POLL_LIMIT", "20000")
    monkeypatch.setenv("B2_DECODE_KERNEL", "persistent")
    dec = bd.Decoder(stall_model, "fp16", max_seq_len=64)
    monkeypatch.delenv("B2_MK_POLL_LIMIT")
    monkeypatch.delenv("B2_DECODE_KERNEL")
    assert dec.uses_persistent_kernel()
    orc = ref.RefDecoder(stall_model, "fp16", max_seq_len=64)
    emb = mf.seeded_hidden(897_000, 5, 1024)
    dec.prefill_batch(emb)
    orc.prefill_batch(emb)
    # a normal step first
    t, lg = dec.step_logits(7)
    to, lo = orc.step(7)
    assert cos(lg, lo) >= 0.9995 and t == to
    # the lm_head phase can never start: every CTA's wait runs out
    monkeypatch.setenv("B2_MK_STALL_TEST", "1")
    logits = np.empty(4096, np.float32)
    assert dec.step(token_id=t, logits=logits) == ERR_RKNN
    assert dec.seq_len == 6  # the failed step did not advance the sequence
    toks = np.empty(3, np.int32)
    assert bd.capi().matmul_decoder_decode_greedy(dec.ctx, t, 3, toks.ctypes.data, None) == ERR_RKNN
    assert dec.seq_len == 6
    monkeypatch.delenv("B2_MK_STALL_TEST")
    # the state was reset: the same step now succeeds and matches the oracle
    for i in range(3):
        tg, lg = dec.step_logits(t)
        to, lo = orc.step(t)
        assert cos(lg, lo) >= 0.9995 and float(np.abs(lg - lo).max()) <= 2e-2, f"step {i} after recovery"
        assert tg == to
        t = to
    assert dec.seq_len == orc.seq_len == 9
