#!/usr/bin/env python3
"""Decode benchmark of the B200 decoder runtime (one JSON line on rank 0).

Workloads (the default is the one its metric is quoted on):
  cfg2  28-layer Qwen3-0.6B-shaped decoder, FP16 layers + INT8 lm_head,
        60-token batch prefill of N(0,1) embeddings, then greedy decode at B=1
        from token 151644.  A step is one decode token.          (default)
  cfg3  same model quantized W8A16, KV cache pre-filled to --context L.
  cfg4  batch prefill of --rows (60 or 512) N(0,1) embeddings through the
        28-layer FP16 model; a step is one prefill.  The four projections run on
        the tcgen05 tensor cores; `roofline` is the gate|up GEMM timed alone.
  cfg5  batched W4A16 decode of 64 sequences with contexts U[128, 4096],
        sharded over ranks; a step advances every sequence by one token.

Arms:
  --impl b200       (default) this runtime.  `value` is device-timed (CUDA
                    events on the decoder's stream) greedy decode with the token
                    feedback on the device (matmul_decoder_decode_greedy), inputs
                    resident in HBM; `e2e` is the same metric through the C API
                    call a user makes (matmul_decoder_step_token: host->device
                    parameter block, device->host token id, both inside the
                    timed region), host-timed.
  --impl reference  the reference's CPU path (the oracle's scalar C port of
                    src/cpu_ops.c + the matmul semantics, since the reference
                    itself needs an ARM NPU) on the host cores with all threads,
                    rank 0 only.

Multi-GPU (torchrun, one rank per GPU): cfg2/cfg3 run one independent sequence
per rank (weak scaling, no collective in the data path); cfg5 shards the 64
sequences over the ranks.  Times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "rknn-matmul-parallel_b200")
sys.path.insert(0, os.path.join(PKG, "python"))
sys.path.insert(0, PKG)

import model_format as mf  # noqa: E402

METRIC = "decode ms/token (B=1) & tok/s (B=64, 1–8 GPU); % of HBM roofline"
FIRST_TOKEN = 151644
PREFILL = 60


# ─── algorithmic bytes per decode token ───

def layer_weight_bytes(shape: mf.ModelShape, quant: str) -> int:
    elems = sum(k * n for k, n in shape.proj_shapes().values()) * shape.num_layers
    n_cols = sum(n for _, n in shape.proj_shapes().values()) * shape.num_layers
    if quant == "fp16":
        return elems * 2
    return (elems if quant == "int8" else elems // 2) + n_cols * 4


def token_bytes(shape: mf.ModelShape, quant: str, attended: float) -> float:
    """Bytes one decode token must move: all layer weights (+scales), the INT8
    lm_head and its scales, norm weights, the embedding row, the K/V read over
    `attended` positions and the K/V write of the new position."""
    H, nl, kvd = shape.hidden_dim, shape.num_layers, shape.num_kv_heads * shape.head_dim
    lm = shape.vocab_size * H + shape.vocab_size * 4
    norms = nl * (2 * H + 2 * shape.head_dim) * 4 + H * 4
    kv = nl * 2 * kvd * 2 * attended + nl * 2 * kvd * 2
    return layer_weight_bytes(shape, quant) + lm + norms + H * 4 + kv


def cpu_model() -> str:
    """The host CPU's model name (lscpu's "Model name"), for the CPU baselines."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def load_peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    return json.load(open(path)) if os.path.exists(path) else {}


def single_stream_config(workload: str, context: int, quant: str, world: int) -> dict:
    """`config` of a B=1 decode line; both arms build it here so they match key for key."""
    shape = mf.ModelShape()
    w = layer_weight_bytes(shape, quant) + shape.vocab_size * (shape.hidden_dim + 4)
    return {"workload": workload, "model": "qwen3-0.6b-shaped (28 layers, vocab 151936)",
            "batch_per_gpu": 1, "context_start": context, "quant": quant, "lm_head": "int8",
            "parallelism": f"replicas x{world} (independent sequences)",
            "l2": "inputs larger than L2: %.2f GB of weights streamed per token" % (w / 1e9)}


def prefill_config(rows: int, world: int) -> dict:
    return {"workload": "cfg4", "model": "qwen3-0.6b-shaped (28 layers), FP16 layers", "rows": rows,
            "parallelism": f"replicas x{world}"}


# ─── clocks during the timed region ───

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int):
        self.samples = []
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "20", "-i", str(device)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi needs a moment to start: have it sampling before the timed region does
            t_end = time.perf_counter() + 3.0
            while not self.samples and time.perf_counter() < t_end:
                time.sleep(0.01)
        except OSError:
            self.p = None

    def _read(self):
        for line in self.p.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.perf_counter(), parts))

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self, t0: float, t1: float) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        win = [s for t, s in self.samples if t0 - 0.03 <= t <= t1 + 0.03]
        note = "timed region"
        if not win:  # a region shorter than the sampling period: the samples nearest to it
            near = sorted(self.samples, key=lambda ts: min(abs(ts[0] - t0), abs(ts[0] - t1)))[:3]
            win = [s for _, s in near]
            note = "samples nearest to the timed region"

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(s[1]) for s in win if num(s[1]) is not None]
        reasons = set()
        for s in win:
            for name, flag in zip(self.NAMES, s[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(win[0][2]),
                "reasons": sorted(reasons), "samples": len(win), "window": note}


# ─── distributed plumbing ───

def dist_setup():
    """One process per GPU under torchrun (RANK / WORLD_SIZE / LOCAL_RANK /
    MASTER_* from the environment): NCCL on GPUs, gloo on a host without one
    (or when B2_DIST_BACKEND=gloo), with a short timeout so that ranks which
    wait for a missing peer end with an error."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        backend = os.environ.get("B2_DIST_BACKEND") or ("nccl" if torch.cuda.is_available() else "gloo")
        timeout = datetime.timedelta(seconds=int(os.environ.get("B2_DIST_TIMEOUT", "120")))
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=timeout)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, x: float) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def model_dir(cache: str, quant: str, rank: int, world: int) -> str:
    shape = mf.ModelShape()
    d = os.path.join(cache, f"qwen3_0p6b_{quant}")
    if rank == 0:
        mf.write_synthetic_model(d, shape, quant=None if quant == "fp16" else quant)
    barrier(world)
    return d


# ─── CPU baseline (oracle port) ───

def cpu_decode_rate(mdir: str, quant: str, context: int, tokens: int, nthreads: int):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import ref_decoder as ref
    dec = ref.RefDecoder(mdir, quant, max_seq_len=context + tokens + 4, nthreads=nthreads)
    for layer in range(dec.nL):  # seeded context instead of a (slow) CPU prefill
        k = mf.seeded_kv(mf.kv_seed(layer, 0), context, dec.nkv, dec.hd)
        v = mf.seeded_kv(mf.kv_seed(layer, 1), context, dec.nkv, dec.hd)
        dec.set_kv(layer, 0, k, v)
    dec.seq_len = context
    tok = FIRST_TOKEN
    t0 = time.perf_counter()
    for _ in range(tokens):
        tok, _ = dec.step(tok)
    return tokens / (time.perf_counter() - t0)


def cpu_prefill_rate(mdir: str, rows: int, nthreads: int):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import ref_decoder as ref
    dec = ref.RefDecoder(mdir, "fp16", max_seq_len=rows + 4, nthreads=nthreads)
    emb = mf.seeded_hidden(830_000, rows, mf.ModelShape().hidden_dim)
    t0 = time.perf_counter()
    dec.prefill_batch(emb)
    return rows / (time.perf_counter() - t0)


# ─── arms ───

def run_reference(args, world, rank):
    if rank != 0:
        return None
    import torch  # noqa: F401  (only so the arm's environment matches the b200 arm)
    nth = os.cpu_count() or 1
    quant = {"cfg2": "fp16", "cfg3": "int8", "cfg4": "fp16", "cfg5": "int4"}[args.workload]
    mdir = model_dir(args.model_cache, quant, 0, 1)
    context = PREFILL if args.workload == "cfg2" else args.context
    tokens = args.warmup + args.steps
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import ref_decoder as ref
    common = {"metric": METRIC, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "vs_baseline": None, "dtype": "f32", "impl": "reference"}
    if args.workload == "cfg4":  # bounded sample: cpu_rows prefill rows per step
        rows = max(1, args.cpu_rows)
        emb = mf.seeded_hidden(830_000, rows, mf.ModelShape().hidden_dim)
        d = ref.RefDecoder(mdir, quant, max_seq_len=rows + 4, nthreads=nth)
        for _ in range(args.warmup):
            d.seq_len = 0
            d.prefill_batch(emb)
        t = 0.0
        for _ in range(args.steps):
            d.seq_len = 0
            t0 = time.perf_counter()
            d.prefill_batch(emb)
            t += time.perf_counter() - t0
        rate = args.steps * rows / t
        sample = f"{args.steps} prefills of {rows} rows of the 28-layer FP16 model, oracle C port, {nth} threads"
        return dict(common, value=round(rate, 3), ms_per_step=round(t * 1e3 / args.steps, 3), scaling="weak",
                    data="synthetic (seeded N(0,0.02) weights, N(0,1) embeddings)",
                    config=prefill_config(args.rows, world),
                    cpu_baseline={"value": round(rate, 3), "unit": "tok/s", "cores": nth, "kind": "port",
                                  "cpu": cpu_model(), "sample": sample},
                    e2e={"value": round(rate, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
    dec = ref.RefDecoder(mdir, quant, max_seq_len=context + tokens + 4, nthreads=nth)
    for layer in range(dec.nL):
        dec.set_kv(layer, 0, mf.seeded_kv(mf.kv_seed(layer, 0), context, dec.nkv, dec.hd),
                   mf.seeded_kv(mf.kv_seed(layer, 1), context, dec.nkv, dec.hd))
    dec.seq_len = context
    tok = FIRST_TOKEN
    for _ in range(args.warmup):
        tok, _ = dec.step(tok)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok, _ = dec.step(tok)
    dt = time.perf_counter() - t0
    rate = args.steps / dt
    sample = (f"{args.steps} full decode tokens of the 28-layer {quant} model at context {context}"
              f" (KV seeded), oracle C port, {nth} threads")
    return dict(common, value=round(rate, 3), ms_per_step=round(dt * 1e3 / args.steps, 3), scaling="weak",
                data="synthetic (seeded N(0,0.02) weights, seeded N(0,1) FP16 KV)",
                config=single_stream_config(args.workload, context, quant, world),
                cpu_baseline={"value": round(rate, 3), "unit": "tok/s", "cores": nth, "kind": "port",
                              "cpu": cpu_model(), "sample": sample},
                e2e={"value": round(rate, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})


def measure_single_stream(args, world, rank, local, workload, context, steps, warmup):
    """B=1 greedy decode of `steps` tokens on this rank's GPU.  Returns the
    device time (CUDA events on the decoder's stream, max over ranks), the host
    time of the same tokens through matmul_decoder_step_token, and the clocks
    sampled during the device-timed region."""
    import b200_decoder as bd
    quant = "fp16" if workload == "cfg2" else "int8"
    mdir = model_dir(args.model_cache, quant, rank, world)
    bd.check(bd.capi().b2_set_device(local), "set_device")
    shape = mf.ModelShape()
    max_seq = (PREFILL if workload == "cfg2" else context) + max(steps, warmup) + 8
    dec = bd.Decoder(mdir, quant, max_seq_len=max_seq)

    def reset():
        bd.capi().matmul_decoder_clear_kv_cache(dec.ctx)
        if workload == "cfg2":
            dec.prefill_batch(mf.seeded_hidden(820_000, PREFILL, shape.hidden_dim))
            return PREFILL
        dec.set_seq_len(context)
        return context

    if workload == "cfg3":
        for layer in range(shape.num_layers):
            dec.set_kv(layer, 0, mf.seeded_kv(mf.kv_seed(layer, 0), context, 8, 128),
                       mf.seeded_kv(mf.kv_seed(layer, 1), context, 8, 128))
    reset()
    dec.decode_greedy(FIRST_TOKEN, warmup)  # warm-up: first launches, clocks, caches
    ctx0 = reset()

    clocks = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    t0 = time.perf_counter()
    toks, dev_ms = dec.decode_greedy(FIRST_TOKEN, steps)
    t1 = time.perf_counter()
    barrier(world)
    clk = clocks.summary(t0, t1)
    clocks.stop()
    ms = max_over_ranks(world, dev_ms)

    # e2e through the C API with host buffers, same context and token count
    assert reset() == ctx0
    barrier(world)
    tok = FIRST_TOKEN
    e0 = time.perf_counter()
    for _ in range(steps):
        tok = dec.step_token(tok)
        if tok < 0:
            raise RuntimeError(f"step_token failed ({tok})")
    e_s = max_over_ranks(world, time.perf_counter() - e0)
    kinds = {dec.step_kernel(ctx0), dec.step_kernel(ctx0 + steps - 1)}
    persistent = kinds.pop() if len(kinds) == 1 else -1  # -1: the run crossed a routing boundary
    dec.close()
    attended = ctx0 + (steps + 1) / 2.0
    return {"quant": quant, "mdir": mdir, "ctx0": ctx0, "ms": ms, "e2e_s": e_s, "clocks": clk,
            "toks": toks, "bytes": token_bytes(shape, quant, attended), "persistent": persistent}


KERNEL_NAMES = {2: "tile-stream persistent kernel b2_mk2_decode (mk2_kernel), one launch per token",
                1: "persistent kernel b2_mk_decode, one launch per token",
                0: "CUDA graph of per-op kernels"}


def decode_roofline(m: dict, steps: int, peaks: dict, traffic=None) -> dict:
    peak = float(peaks.get("hbm_gbs", 6650.0))
    ms_tok = m["ms"] / steps
    achieved = m["bytes"] / (ms_tok * 1e-3) / 1e9
    r = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
         "frac": round(achieved / peak, 4), "traffic": traffic,
         "kernel": "whole decode step (" + KERNEL_NAMES.get(m["persistent"], "mixed routing") + ")",
         "bytes_per_token": int(m["bytes"]),
         "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured, of measured)" if peaks else "fallback 6.65 TB/s"}
    return r


def run_single_stream(args, world, rank, local):
    K, W = args.steps, args.warmup
    shape = mf.ModelShape()
    ctx_arg = PREFILL if args.workload == "cfg2" else args.context
    m = measure_single_stream(args, world, rank, local, args.workload, ctx_arg, K, W)
    peaks = load_peaks()
    traffic, traffic_note = None, None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        t = json.load(open(tp))
        traffic = t.get(f"{args.workload}_bytes_per_token")
        traffic_note = t.get("source")
    roof = decode_roofline(m, K, peaks, traffic)
    if traffic is not None:
        roof["traffic_source"] = ("copied from an ncu capture of the same command, not measured in this run: "
                                  + (traffic_note or "profiles/traffic.json"))
    quant = m["quant"]
    launches_per_token = 1 if m["persistent"] else 1 + shape.num_layers * 7 + 2 + 1
    line = {
        "metric": METRIC, "value": round(world * K / (m["ms"] * 1e-3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(m["ms"] / K, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16" if quant == "fp16" else "int8 weights / fp16 act",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) prefill embeddings)",
        "config": single_stream_config(args.workload, m["ctx0"], quant, world),
        "roofline": roof,
        "clocks": m["clocks"],
        # bytes a step_token call moves: the persistent kernels take 4 ints of
        # step state and return the error flag and the token; the graph path
        # uploads its parameter block (8 ints + an embedding row) and reads
        # the token
        "e2e": {"value": round(world * K / m["e2e_s"], 2), "unit": "tok/s",
                "h2d_bytes_per_step": 16 if m["persistent"] else 4 * (8 + shape.hidden_dim),
                "d2h_bytes_per_step": 8 if m["persistent"] else 4,
                "api": "matmul_decoder_step_token (C ABI)"},
        "gpu_launches": launches_per_token * K,
        "tokens_check": [int(t) for t in m["toks"][:4]],
    }
    if args.workload == "cfg2" and not args.no_extras:
        # the north star's target config next to the headline: W8A16, L = 128
        m3 = measure_single_stream(args, world, rank, local, "cfg3", 128, K, W)
        line["cfg3"] = {"workload": "cfg3", "quant": "int8", "context_start": 128,
                        "ms_per_token": round(m3["ms"] / K, 4),
                        "value": round(world * K / (m3["ms"] * 1e-3), 2), "unit": "tok/s",
                        "e2e": round(world * K / m3["e2e_s"], 2),
                        "roofline": decode_roofline(m3, K, peaks), "clocks": m3["clocks"]}
        line["gpu_launches"] += (1 if m3["persistent"] else 1 + shape.num_layers * 7 + 3) * K
        # the batched workload at this N: 64 sequences sharded over the ranks
        b = run_batched(args, world, rank, local, sub=True)
        if b is not None:
            line["batched"] = b
            line["gpu_launches"] += b.pop("_launches")
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        rate = cpu_decode_rate(m["mdir"], quant, m["ctx0"], args.cpu_tokens, 1)
        line["cpu_baseline"] = {
            "value": round(rate, 4), "unit": "tok/s", "cores": 1, "kind": "port", "cpu": cpu_model(),
            "sample": f"{args.cpu_tokens} decode tokens of the same 28-layer model at context {m['ctx0']} "
                      f"(KV seeded), oracle scalar C port, 1 thread",
            "role": "the stated CPU baseline: one thread, as the reference decoder runs its CPU ops; the "
                    "--impl reference arm times the same port with every host thread"}
    return line if rank == 0 else None


def prefill_flops(shape: mf.ModelShape, rows: int) -> tuple[float, float]:
    """(projection FLOPs, causal attention FLOPs) of one prefill of `rows` rows."""
    proj = 2.0 * rows * sum(k * n for k, n in shape.proj_shapes().values()) * shape.num_layers
    attn = 4.0 * shape.head_dim * shape.num_q_heads * shape.num_layers * rows * (rows + 1) / 2
    return proj, attn


def time_gemm_alone(rows: int, iters: int = 20):
    """CUDA-event time of the gate|up b2_gemm launch (K=1024, 2x3072 rows) on
    torch's current stream, L2 flushed (256 MB write) before every launch."""
    import ctypes
    import torch
    import b200_decoder as bd
    K, F = 1024, 3072
    g = torch.Generator(device="cuda").manual_seed(7)
    x16 = torch.randn((rows, K), device="cuda", generator=g).half()
    w = (torch.randn((2 * F, K), device="cuda", generator=g) * 0.02).half()
    y = torch.empty((rows, F), device="cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    a = bd.B2GemmArgs(y.data_ptr(), F, x16.data_ptr(), K, rows, K, F, w.data_ptr(), None, bd.W_F16,
                      bd.EPI_SILU_PAIR)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    times = []
    for i in range(iters + 3):
        flush.fill_(float(i))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        bd.check(bd.capi().b2_gemm(ctypes.byref(a), st), "b2_gemm")
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    ms = statistics.mean(times)
    flops = 2.0 * rows * K * 2 * F
    return ms, flops, w.numel() * 2 + x16.numel() * 2 + y.numel() * 4


def run_prefill(args, world, rank, local):
    import b200_decoder as bd
    mdir = model_dir(args.model_cache, "fp16", rank, world)
    bd.check(bd.capi().b2_set_device(local), "set_device")
    import torch
    torch.cuda.set_device(local)
    shape = mf.ModelShape()
    M, K, W = args.rows, args.steps, args.warmup
    dec = bd.Decoder(mdir, "fp16", max_seq_len=M + 8)
    emb = mf.seeded_hidden(830_000 + M, M, shape.hidden_dim)
    for _ in range(W):
        bd.capi().matmul_decoder_clear_kv_cache(dec.ctx)
        dec.prefill_batch(emb)
    clocks = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    dev_ms, host_s = [], []
    t0 = time.perf_counter()
    for _ in range(K):
        bd.capi().matmul_decoder_clear_kv_cache(dec.ctx)
        h0 = time.perf_counter()
        dec.prefill_batch(emb)        # host embeddings -> device, all layers, synchronous
        last = dec.hidden()           # device -> host read of the step's result
        host_s.append(time.perf_counter() - h0)
        dev_ms.append(dec.stats()["matmul_ms"])
    t1 = time.perf_counter()
    barrier(world)
    clk = clocks.summary(t0, t1)
    clocks.stop()
    assert np.isfinite(last).all()
    ms = max_over_ranks(world, statistics.mean(dev_ms))
    e2e = max_over_ranks(world, statistics.mean(host_s))
    g_ms, g_flops, g_bytes = time_gemm_alone(M)
    g_ms = max_over_ranks(world, g_ms)
    proj, attn = prefill_flops(shape, M)
    peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    ach = g_flops / (g_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(world * M / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) embeddings)",
        "config": dict(prefill_config(M, world),
                       l2="weights 0.88 GB per prefill (> L2); gate|up GEMM timing flushes L2 (256 MB write) "
                          "per launch"),
        "prefill": {"tflops_projections": round(proj / (ms * 1e-3) / 1e12, 2),
                    "tflops_with_attention": round((proj + attn) / (ms * 1e-3) / 1e12, 2),
                    "projection_gflop": round(proj / 1e9, 2), "attention_gflop": round(attn / 1e9, 2)},
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(ach / peak, 4), "traffic": None,
                     "kernel": f"b2_gemm gate|up + SiLU (M={M}, K=1024, N=2x3072), {round(g_ms * 1e3, 2)} us/launch",
                     "peak_source": "MEASURED_PEAKS.json bf16_tflops (measured, burst)" if peaks else "fallback"},
        "clocks": clk,
        "e2e": {"value": round(world * M / e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": M * shape.hidden_dim * 4,
                "d2h_bytes_per_step": shape.hidden_dim * 4, "api": "matmul_decoder_prefill_batch (C ABI)"},
        "gpu_launches": K * shape.num_layers * 11,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        rows = max(1, args.cpu_rows)
        rate = cpu_prefill_rate(mdir, rows, os.cpu_count() or 1)
        line["cpu_baseline"] = {"value": round(rate, 4), "unit": "tok/s", "cores": os.cpu_count() or 1,
                                "cpu": cpu_model(),
                                "kind": "port", "sample": f"one {rows}-row prefill of the same 28-layer FP16 model, "
                                                          f"oracle C port, all threads"}
    dec.close()
    return line if rank == 0 else None


def shard_sequences(lens, world):
    """Greedy bin-packing of sequences on context length (KV bytes dominate a
    batched step): longest first, each to the rank with the least work so far.
    Every rank computes the same assignment."""
    load = [0] * world
    parts = [[] for _ in range(world)]
    for s in sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i)):
        r = min(range(world), key=lambda i: (load[i], i))
        parts[r].append(s)
        load[r] += int(lens[s])
    return [sorted(p) for p in parts]


def run_batched(args, world, rank, local, sub=False):
    """cfg5: 64 W4A16 sequences with contexts U[128, 4096], bin-packed over the
    ranks.  sub=True returns the `batched` sub-object of the default line."""
    import b200_decoder as bd
    mdir = model_dir(args.model_cache, "int4", rank, world)
    bd.check(bd.capi().b2_set_device(local), "set_device")
    shape = mf.ModelShape()
    n_total = args.seqs
    lens = np.random.default_rng(55).integers(128, 4097, size=n_total)
    if n_total < world:
        raise SystemExit(f"cfg5 needs at least one sequence per GPU ({n_total} sequences, {world} GPUs)")
    mine = shard_sequences(lens, world)[rank]
    K, W = args.steps, args.warmup
    bat = bd.BatchDecoder(mdir, len(mine), "int4", max_seq_len=4096 + K + W + 8)
    sharded = world > 1 and os.environ.get("B2_SHARD_VOCAB", "1") != "0"
    if sharded:  # each rank keeps 1/world of the lm_head; NCCL all-gather + all-reduce MAX per step
        import torch.distributed as dist
        obj = [bd.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        bat.shard_vocab(rank, world, obj[0], max(len(p) for p in shard_sequences(lens, world)))

    def reset():
        for i, s in enumerate(mine):
            bat.set_seq_len(i, int(lens[s]))
    reset()
    toks = np.full(len(mine), FIRST_TOKEN, np.int32)
    for _ in range(W):
        toks = bat.step(toks)
    reset()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    t0 = time.perf_counter()
    dev_ms = 0.0
    for _ in range(K):  # each step: tokens in from host memory, next tokens back (C ABI)
        toks = bat.step(toks)
        st = bat.stats()  # device time of the step's layers and lm_head (CUDA events on its stream)
        dev_ms += st["matmul_ms"] + st["lm_head_ms"]
    t1 = time.perf_counter()
    barrier(world)
    clk = clocks.summary(t0, t1)
    clocks.stop()
    bat.close()
    dt = max_over_ranks(world, t1 - t0)
    dev_s = max_over_ranks(world, dev_ms * 1e-3)
    my_lens = [int(lens[s]) for s in mine]
    attended = float(np.mean(my_lens)) + (K + 1) / 2.0
    kv_bytes = len(mine) * shape.num_layers * 2 * shape.num_kv_heads * shape.head_dim * 2 * attended
    kv_max = max_over_ranks(world, kv_bytes)  # the rank with the most KV bytes sets the step time
    lm_bytes = shape.vocab_size * (shape.hidden_dim + 4) / (world if sharded else 1)
    bytes_step = layer_weight_bytes(shape, "int4") + lm_bytes + kv_bytes
    bytes_step_max = layer_weight_bytes(shape, "int4") + lm_bytes + kv_max
    peaks = load_peaks()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = bytes_step_max / (dev_s / K) / 1e9
    # per step: embed, 9 per layer (2 row norms, 4 GEMMs, rope+KV store, attention, combine),
    # final norm, lm_head GEMM, argmax reduce
    launches_per_step = 1 + 9 * shape.num_layers + 3
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": None,
            "kernel": "whole batched step on the busiest rank (CUDA graph; weights + lm_head + its KV)",
            "bytes_per_step": int(bytes_step_max),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured, of measured)" if peaks else "fallback"}
    if sub:
        if rank != 0:
            return None
        return {"workload": "cfg5", "sequences": n_total, "per_gpu_max": max(len(p) for p in
                                                                             shard_sequences(lens, world)),
                "n_gpus": world, "value": round(n_total * K / dev_s, 2), "unit": "tok/s",
                "ms_per_step": round(dev_s * 1e3 / K, 3), "scaling": "strong",
                "e2e": round(n_total * K / dt, 2), "roofline": roof, "clocks": clk,
                "lm_head": f"vocab-sharded over {world} ranks (NCCL all-gather + all-reduce MAX)" if sharded
                           else "replicated",
                "note": "all 64 sequences advance one greedy token per step; device time is the max over ranks",
                "_launches": launches_per_step * K}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        ctx = int(round(float(np.mean(lens))))
        threads = os.cpu_count() or 1
        rate = cpu_decode_rate(mdir, "int4", ctx, 1, threads)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
               "sample": f"1 decode token of one sequence at the mean context {ctx} of the same W4A16 model, "
                         f"oracle C port, {threads} threads"}
    line = {"metric": METRIC, "value": round(n_total * K / dev_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(dev_s * 1e3 / K, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights / fp16 act",
            "data": "synthetic; KV contents zero (attention cost is value-independent)",
            "config": {"workload": "cfg5", "sequences": n_total, "per_gpu": len(mine), "context": "U[128,4096]",
                       "parallelism": f"sequences sharded over {world} GPUs"
                                      + (", lm_head vocab-sharded (NCCL)" if sharded else ""),
                       "l2": "inputs larger than L2: %.2f GB of weights and KV per step per GPU" % (bytes_step / 1e9)},
            "roofline": roof,
            "clocks": clk,
            "e2e": {"value": round(n_total * K / dt, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": 12 * len(mine), "d2h_bytes_per_step": 4 * (len(mine) + 1),
                    "api": "matmul_decoder_batch_step (C ABI)"},
            "gpu_launches": launches_per_step * K}
    if cpu:
        line["cpu_baseline"] = cpu
    return line if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("cfg2", "cfg3", "cfg4", "cfg5"), default="cfg2")
    ap.add_argument("--rows", type=int, default=512, help="cfg4 prefill rows (60 or 512)")
    ap.add_argument("--cpu-rows", type=int, default=4, help="cfg4 CPU baseline sample rows")
    ap.add_argument("--context", type=int, default=128, help="cfg3 pre-filled context")
    ap.add_argument("--seqs", type=int, default=64, help="cfg5 total sequences")
    ap.add_argument("--model-cache", default=os.environ.get("B2_MODEL_CACHE", "/tmp/b2_bench_models"))
    ap.add_argument("--cpu-tokens", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="cfg2: omit the cfg3 and batched sub-objects of the default line")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "cfg5":
            line = run_batched(args, world, rank, local)
        elif args.workload == "cfg4":
            line = run_prefill(args, world, rank, local)
        else:
            line = run_single_stream(args, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
