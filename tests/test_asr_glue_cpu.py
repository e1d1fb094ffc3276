"""The ASR front-end oracle (oracle/ref_mel.py) against golden vectors made by
the reference's own MelExtractor (tests/golden/make_golden_mel.py), and the
prompt assembly of python/asr_glue.py against the reference's layout
(examples/qwen3_asr/engine.py:243-306), on CPU."""
from __future__ import annotations

import os

import numpy as np

import asr_glue
import ref_mel


def test_oracle_matches_reference_mel(golden_dir):
    g = np.load(os.path.join(golden_dir, "golden_mel.npz"))
    fb = ref_mel.mel_filters()
    for k in "ab":
        got = ref_mel.log_mel(g["audio_" + k], fb)
        want = g["mel_" + k]
        assert got.shape == want.shape == (128, g["audio_" + k].size // 160)
        np.testing.assert_allclose(got, want, atol=2e-6, rtol=0)


def test_oracle_build_embed_rows():
    table = np.arange(40, dtype=np.float32).reshape(10, 4)
    audio = -np.ones((2, 4), np.float32)
    out = ref_mel.build_embed(table, [3, 1], audio, [9])
    assert out.shape == (5, 4)
    np.testing.assert_array_equal(out[0], table[3])
    np.testing.assert_array_equal(out[2:4], audio)
    np.testing.assert_array_equal(out[4], table[9])


def test_prompt_ids_follow_the_reference_layout():
    vocab = {}

    def encode(text):  # a stand-in tokenizer: one id per distinct character
        return [vocab.setdefault(c, 1000 + len(vocab)) for c in text]

    ids = {"im_start": 1, "im_end": 2, "audio_start": 3, "audio_end": 4, "asr_text": 5}
    pre, suf = asr_glue.asr_prompt_ids(encode, ids, language="Chinese", prefix_text="ab")
    assert pre == [1] + encode("system\nYou are a helpful assistant. ") + [2, 1] + encode("user\n") + [3]
    assert suf == ([4] + encode("转录：") + [2, 1] + encode("assistant\nlanguage Chinese") + [5]
                   + encode("ab"))
    pre2, _ = asr_glue.asr_prompt_ids(encode, ids, skip_prefix=True)
    assert pre2 == []
    _, suf3 = asr_glue.asr_prompt_ids(encode, ids, compact_suffix=False)
    long_instr = encode("数字用0123456789，语音转录：")
    assert suf3[1:1 + len(long_instr)] == long_instr
