"""Multi-rank host logic of bench.py on CPU: two gloo ranks on 127.0.0.1.

The batched-decode workload shards its sequences over ranks with no
collective in the data path; the only collectives are the barrier around the
timed region and the max-over-ranks reduction of the time.  These tests run
exactly those bench.py functions in two processes, plus the sequence
bin-packing every rank computes on its own."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port), B2_DIST_BACKEND="gloo", B2_DIST_TIMEOUT="60")
        sys.path.insert(0, REPO)
        import torch.distributed as dist

        import bench
        w, r, _ = bench.dist_setup()
        lens = np.random.default_rng(55).integers(128, 4097, size=64)
        mine = bench.shard_sequences(lens, w)[r]
        bench.barrier(w)
        slowest = bench.max_over_ranks(w, float(r + 1) * 0.25)
        parts = [None] * w
        dist.all_gather_object(parts, mine)
        dist.destroy_process_group()
        q.put((r, w, slowest, parts, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, world, None, None, repr(e)))


def test_two_gloo_ranks_shard_and_time_like_bench():
    pytest.importorskip("torch")
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    for r, w, slowest, parts, err in results:
        assert err is None, err
        assert w == world
        assert slowest == pytest.approx(0.5)  # max over ranks of (rank + 1) / 4
        assert sorted(i for part in parts for i in part) == list(range(64))  # every sequence exactly once
    assert results[0][3] == results[1][3]  # every rank computed the same assignment


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_sequences_balances_context(world):
    import bench
    lens = np.random.default_rng(55).integers(128, 4097, size=64)
    parts = bench.shard_sequences(lens, world)
    assert sorted(i for p in parts for i in p) == list(range(64))
    load = [int(sum(lens[i] for i in p)) for p in parts]
    assert max(load) - min(load) <= int(lens.max())  # greedy longest-first bound
    assert all(len(p) > 0 for p in parts)


# ── vocab-sharded lm_head: the argmax-key protocol of
# matmul_decoder_batch_shard_vocab (csrc/host/md_batch.c), on gloo ranks ──
# Each rank holds a contiguous slice of the vocabulary.  Its best key per row
# is (orderable(logit) << 32) | (0xFFFFFFFF - global index); an all-reduce MAX
# of the keys over the ranks picks the largest logit and, on ties, the lowest
# global index: the first maximum of the reference argmax
# (src/cpu_ops.c:575-586).  NaN is ordered below every number.

def _order(v: np.ndarray) -> np.ndarray:
    u = v.astype(np.float32).view(np.uint32).astype(np.uint64)
    out = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return np.where(np.isnan(v), 0, out).astype(np.uint64)


def _keys(logits: np.ndarray, offset: int) -> np.ndarray:
    idx = np.arange(logits.shape[1], dtype=np.uint64) + np.uint64(offset)
    k = (_order(logits) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idx)
    return k.max(axis=1)


def _vocab_rank(rank: int, world: int, port: int, logits: np.ndarray, q) -> None:
    try:
        import torch
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        V = logits.shape[1]
        lo, hi = rank * V // world, (rank + 1) * V // world
        k = torch.from_numpy(_keys(logits[:, lo:hi], lo).view(np.int64))  # same bits, signed view
        # MAX over unsigned keys via the signed view: flip the top bit first
        k ^= torch.tensor(np.int64(-0x8000000000000000))
        dist.all_reduce(k, op=dist.ReduceOp.MAX)
        k ^= torch.tensor(np.int64(-0x8000000000000000))
        toks = (np.uint64(0xFFFFFFFF) - (k.numpy().view(np.uint64) & np.uint64(0xFFFFFFFF))).astype(np.int64)
        dist.destroy_process_group()
        q.put((rank, toks.tolist(), None))
    except Exception as e:
        q.put((rank, None, repr(e)))


def test_vocab_shard_argmax_keys_over_gloo_ranks():
    pytest.importorskip("torch")
    rng = np.random.default_rng(8)
    logits = rng.standard_normal((6, 1000)).astype(np.float32)
    logits[1, [10, 600]] = 9.0        # tie across the two slices: the lower index wins
    logits[2, [700, 900]] = 9.0       # tie inside one slice
    logits[3, 0] = np.nan             # NaN never wins
    logits[4, :] = -3.0               # all equal: index 0
    logits[5, 999] = 50.0
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_vocab_rank, args=(r, world, port, logits, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r, toks, err in res:
        assert err is None, err
        want = [int(np.nanargmax(np.where(np.isnan(row), -np.inf, row))) for row in logits]
        assert toks == want, (r, toks, want)
