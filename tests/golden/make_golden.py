"""Generate golden vectors from the reference's own numpy oracle.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference /path/to/rknn-matmul-parallel

It imports tests/generate_reference.py of suharvest/rknn-matmul-parallel (pure
numpy) and evaluates its functions on seeded synthetic inputs:

* golden_ops.npz     rms_norm, silu, rope_interleaved at several positions;
* golden_layer.npz   forward_layer on one seeded Qwen3-0.6B-shaped layer at
                     pos 0 with all of the reference's saved intermediates;
* golden_model/      the reference's main() (its whole fixture pipeline) on a
                     2-layer, 4096-vocab seeded model: input_embedding,
                     layer intermediates, final_normed, top-100 logits + idx.

Weights are not stored: the tests regenerate them from the same seeds with
model_format.write_synthetic_model.  Only the small output vectors are
committed.  Nothing here runs at test time.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "rknn-matmul-parallel_b200", "python"))
import model_format as mf  # noqa: E402

LAYER_SHAPE = dict(num_layers=1, vocab_size=4096, rope_style=0, name="golden-layer")
MODEL_SHAPE = dict(num_layers=2, vocab_size=4096, rope_style=0, name="golden-model")
OPS_SEED = 123_000
LAYER_INPUT_SEED = 124_000
MODEL_TOKEN = 1234


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "tests", "generate_reference.py")
    spec = importlib.util.spec_from_file_location("generate_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def golden_ops(gr, out):
    rng = np.random.default_rng(OPS_SEED)
    x = rng.standard_normal(1024, dtype=np.float32)
    w = (1.0 + 0.01 * rng.standard_normal(1024, dtype=np.float32)).astype(np.float32)
    xs = (rng.standard_normal(3072, dtype=np.float32) * 4).astype(np.float32)
    xs[:4] = np.array([-100.0, 100.0, 0.0, -0.5], np.float32)
    heads = rng.standard_normal((16, 128), dtype=np.float32)
    positions = np.array([0, 1, 7, 127, 1000, 4095])
    rope = np.stack([gr.rope_interleaved(heads, int(p), 128, 1000000.0) for p in positions])
    np.savez(out, rms_x=x, rms_w=w, rms_out=gr.rms_norm(x, w, 1e-6).astype(np.float32),
             silu_x=xs, silu_out=gr.silu(xs).astype(np.float32),
             rope_x=heads, rope_pos=positions, rope_out=rope.astype(np.float32))


def golden_layer(gr, out):
    shape = mf.ModelShape(**LAYER_SHAPE)
    with tempfile.TemporaryDirectory() as d:
        mf.write_synthetic_model(d, shape)
        cfg = json.load(open(os.path.join(d, "config.json")))
        x = mf.seeded_hidden(LAYER_INPUT_SEED, 1, shape.hidden_dim)[0]
        inter = os.path.join(d, "inter")
        os.makedirs(inter)
        hid = gr.forward_layer(x.copy(), mf.layer_dir(d, 0), pos=0, config=cfg,
                               save_prefix="layer_00", out_dir=inter)
        arrays = {f[len("layer_00_"):-4]: np.load(os.path.join(inter, f))
                  for f in os.listdir(inter)}
        np.savez(out, x=x, out=hid.astype(np.float32), **arrays)


def golden_model(gr, out_dir):
    shape = mf.ModelShape(**MODEL_SHAPE)
    os.makedirs(out_dir, exist_ok=True)
    with tempfile.TemporaryDirectory() as d:
        mf.write_synthetic_model(d, shape)
        argv = sys.argv
        sys.argv = ["generate_reference.py", "--model-dir", d, "--output-dir", out_dir,
                    "--token-id", str(MODEL_TOKEN), "--save-all-layers"]
        try:
            gr.main()
        finally:
            sys.argv = argv
    cfgp = os.path.join(out_dir, "config.json")
    cfg = json.load(open(cfgp))
    cfg["model_dir"] = "<regenerated from seeds: model_format.ModelShape(**MODEL_SHAPE)>"
    cfg["shape"] = MODEL_SHAPE
    json.dump(cfg, open(cfgp, "w"), indent=2)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    gr = load_reference(a.reference)
    golden_ops(gr, os.path.join(HERE, "golden_ops.npz"))
    golden_layer(gr, os.path.join(HERE, "golden_layer.npz"))
    golden_model(gr, os.path.join(HERE, "golden_model"))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
