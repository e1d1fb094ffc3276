"""ASR front end on the GPU (b2_log_mel, b2_build_embed) against the oracle
(oracle/ref_mel.py, pinned to the reference's MelExtractor by
tests/test_asr_glue_cpu.py) and the reference's own golden output."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import asr_glue  # noqa: E402
import b200_decoder as bd  # noqa: E402
import model_format as mf  # noqa: E402
import ref_mel  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = torch.device("cuda:0")
TOL = 2e-4  # log10 units / 4: FP32 DFT against the float64 oracle


def test_mel_matches_reference_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "golden_mel.npz"))
    ext = asr_glue.MelExtractor(filters=ref_mel.mel_filters())
    for k in "ab":
        got = ext(g["audio_" + k])
        assert got.shape == g["mel_" + k].shape
        np.testing.assert_allclose(got, g["mel_" + k], atol=TOL, rtol=0)


@pytest.mark.parametrize("n", [201, 12345, 16000 * 30])
def test_mel_matches_oracle(n):
    rng = np.random.default_rng(n)
    t = np.arange(n) / 16000.0
    audio = (0.2 * np.sin(2 * np.pi * 440 * t) * (1 + np.sin(2 * np.pi * 0.7 * t))
             + 0.02 * rng.standard_normal(n)).astype(np.float32)
    audio[: n // 7] *= 1e-4  # a quiet stretch: the max - 8 clamp engages
    fb = ref_mel.mel_filters()
    want = ref_mel.log_mel(audio, fb)
    got = asr_glue.MelExtractor(filters=fb)(audio)
    assert got.shape == want.shape == (128, n // 160)
    np.testing.assert_allclose(got, want, atol=TOL, rtol=0)


def test_mel_device_entry_point_twice():
    L = bd.capi()
    n = 48000
    rng = np.random.default_rng(9)
    fb = ref_mel.mel_filters()
    a = torch.from_numpy((0.1 * rng.standard_normal(n)).astype(np.float32)).to(DEV)
    f = torch.from_numpy(fb).to(DEV)
    out = torch.empty((128, n // 160), dtype=torch.float32, device=DEV)
    work = torch.empty(L.b2_log_mel_workspace(n), dtype=torch.uint8, device=DEV)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    want = ref_mel.log_mel(a.cpu().numpy(), fb)
    for _ in range(2):  # the maximum slot is reset per call
        bd.check(L.b2_log_mel(a.data_ptr(), n, f.data_ptr(), out.data_ptr(), work.data_ptr(), s), "b2_log_mel")
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want, atol=TOL, rtol=0)
    assert L.b2_log_mel(a.data_ptr(), 200, f.data_ptr(), out.data_ptr(), work.data_ptr(), s) == -1


@pytest.fixture(scope="module")
def small_model(model_cache):
    d = os.path.join(model_cache, "asr_l1_fp16")
    mf.write_synthetic_model(d, mf.ModelShape(num_layers=1), quant=None)
    return d


def test_build_embed_matches_oracle(small_model):
    dec = bd.Decoder(small_model, "fp16", max_seq_len=64)
    V, H = dec.V, dec.cfg.hidden_dim
    table = np.fromfile(os.path.join(small_model, "embeddings.bin"), np.float32).reshape(V, H)
    rng = np.random.default_rng(3)
    pre = [151644, 8948, 198, 151645, 0]
    suf = [V - 1, 5, 151644]
    audio = rng.standard_normal((37, H)).astype(np.float32)
    rows, n = asr_glue.build_embed(dec, audio, pre, suf)
    assert n == len(pre) + 37 + len(suf)
    np.testing.assert_array_equal(rows, ref_mel.build_embed(table, pre, audio, suf))
    # audio only, and out-of-range ids refused
    rows2, n2 = asr_glue.build_embed(dec, audio[:3], [], [])
    assert n2 == 3
    np.testing.assert_array_equal(rows2, audio[:3])
    with pytest.raises(RuntimeError):
        asr_glue.build_embed(dec, audio, [V], [])
    dec.close()
