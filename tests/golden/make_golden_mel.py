"""Golden vectors for the log-mel front end, made by the reference's own
MelExtractor (examples/qwen3_asr/mel.py, imported from a checkout of
suharvest/rknn-matmul-parallel; numpy only).  Run from the repository root:

    python tests/golden/make_golden_mel.py <reference checkout>

writes tests/golden/golden_mel.npz: seeded waveforms (0.5 s chirp + noise,
and 2001 samples of quiet noise) and the reference's (128, T) output for the
filter bank oracle.ref_mel.mel_filters() builds."""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import ref_mel  # noqa: E402


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "examples", "qwen3_asr"))
    import mel as ref  # noqa: E402  (the reference's module)

    fb = ref_mel.mel_filters()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "mel_filters.npy")
        np.save(path, fb)
        ext = ref.MelExtractor(path)
    rng = np.random.default_rng(4242)
    t = np.arange(8000) / 16000.0
    a = (0.3 * np.sin(2 * np.pi * (200 + 3000 * t) * t) + 0.01 * rng.standard_normal(8000)).astype(np.float32)
    b = (1e-3 * rng.standard_normal(2001)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "golden_mel.npz"), audio_a=a, mel_a=ext(a), audio_b=b, mel_b=ext(b))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_mel.py <reference checkout>")
    main(sys.argv[1])
