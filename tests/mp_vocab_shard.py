"""Rank program of test_gpu_vocab_shard.py (launched by torch.distributed.run):
rank r decodes sequences r, r + 2, ... of a 4-layer INT8 model with half of
the vocabulary and compares its tokens with an unsharded decoder of the same
sequences on its own GPU."""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "rknn-matmul-parallel_b200", "python"))
sys.path.insert(0, os.path.join(REPO, "rknn-matmul-parallel_b200"))
sys.path.insert(0, HERE)

import b200_decoder as bd  # noqa: E402
from test_gpu_vocab_shard import setup_batch  # noqa: E402


def main():
    mdir = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    bd.check(bd.capi().b2_set_device(rank), "set_device")
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    n_total = 24
    lens = np.random.default_rng(4).integers(4, 200, size=n_total)
    mine = list(range(rank, n_total, world))
    ref = setup_batch(mdir, mine, lens)
    sh = setup_batch(mdir, mine, lens)
    obj = [bd.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    sh.shard_vocab(rank, world, obj[0], (n_total + world - 1) // world)
    toks = (np.array(mine, np.int32) * 37 + 5) % 8192
    for step in range(4):
        t_ref = ref.step(toks)
        t_sh = sh.step(toks)
        if not np.array_equal(t_ref, t_sh):
            print(f"rank {rank} step {step}: {t_ref} != {t_sh}", flush=True)
            sys.exit(1)
        toks = t_ref
    sh.close()
    ref.close()
    print(f"rank ok {rank}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
