"""Time one kernel of the decoder alone, at the shapes of the benchmark
workloads (Qwen3-0.6B: hidden 1024, 16 q / 8 kv heads of 128, ffn 3072).

    python rknn-matmul-parallel_b200/python/kernel_bench.py attn-blocks [--rows 64] [--block 512]
    python rknn-matmul-parallel_b200/python/kernel_bench.py attn-split  [--rows 64]
    python rknn-matmul-parallel_b200/python/kernel_bench.py gemm-gu     [--rows 64] [--wtype i4] [--split 0]
    (gemm-qkv, gemm-o, gemm-down likewise)
    python rknn-matmul-parallel_b200/python/kernel_bench.py log-mel     [--seconds 30]
    python rknn-matmul-parallel_b200/python/kernel_bench.py sample      [--top-k 50] [--top-p 0.9]

Attention rows are independent sequences whose cache lengths are drawn
uniformly from [128, 4096) (the batched-decode workload, seeded); GEMM
weights are random bytes of the given type.  Each timed iteration follows
a 256 MB write that flushes L2; the line printed per case gives the median
and minimum device time (CUDA events around the C-ABI call) and the
algorithmic bytes (weights, or the K and V rows attended) per microsecond;
for log-mel (the ASR front end) the FLOPs of the direct 400-point DFT and
the mel product per second; for sample (on-device sampling over the 151936
logits of one token) the logit bytes read per second.
Every kernel runs through the library's C-ABI (libmatmul_decoder.so)."""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import b200_decoder as bd  # noqa: E402

H, NQ, NKV, HD, FFN = 1024, 16, 8, 128, 3072
GEMMS = {  # name: (epilogue, K, N)
    "gemm-qkv": (bd.EPI_STORE, H, (NQ + 2 * NKV) * HD),
    "gemm-o": (bd.EPI_ADD, NQ * HD, H),
    "gemm-gu": (bd.EPI_SILU_PAIR, H, FFN),
    "gemm-down": (bd.EPI_ADD, FFN, H),
}
WTYPES = {"f16": (bd.W_F16, 2.0), "i8": (bd.W_I8, 1.0), "i4": (bd.W_I4, 0.5)}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=["attn-blocks", "attn-split", "log-mel", "sample"] + sorted(GEMMS))
    ap.add_argument("--top-k", type=int, default=50, help="sample: top_k (0: all)")
    ap.add_argument("--top-p", type=float, default=0.9, help="sample: top_p")
    ap.add_argument("--seconds", type=float, default=30.0, help="log-mel: audio length at 16 kHz")
    ap.add_argument("--rows", type=int, default=64, help="token rows (sequences for attention)")
    ap.add_argument("--wtype", choices=sorted(WTYPES), default="i4")
    ap.add_argument("--split", type=int, default=0, help="GEMM split-K cluster size (0: automatic)")
    ap.add_argument("--block", type=int, default=512, help="attention positions per work unit")
    ap.add_argument("--max-seq", type=int, default=4108)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--seed", type=int, default=5)
    a = ap.parse_args()
    if not torch.cuda.is_available():
        print("kernel_bench needs a CUDA device", file=sys.stderr)
        return 2
    dev = torch.device("cuda:0")
    lib = bd.capi()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(a.seed)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    M = a.rows
    keep = []

    if a.kernel == "sample":
        V = 151936
        logits = torch.randn(V, device=dev) * 3.0
        rep = torch.from_numpy(rng.integers(0, V, 64).astype(np.int32)).to(dev)
        tok = torch.zeros(8, dtype=torch.int32, device=dev)
        keep += [logits, rep, tok]
        nbytes = V * 4.0
        label = f"sample V={V} top_k={a.top_k} top_p={a.top_p} temperature=0.8 penalty=1.1 (64 repeat tokens)"
        counter = [0]

        def run():
            counter[0] += 1
            bd.check(lib.b2_sample_token(logits.data_ptr(), V, rep.data_ptr(), 64, 1.1, a.top_k, a.top_p, 0.8, 7,
                                         counter[0], tok.data_ptr(), None, stream), a.kernel)
    elif a.kernel == "log-mel":
        n = int(a.seconds * 16000)
        audio = torch.from_numpy((0.1 * rng.standard_normal(n)).astype(np.float32)).to(dev)
        filt = torch.from_numpy(rng.random((201, 128), dtype=np.float32) * 0.01).to(dev)
        out = torch.empty((128, n // 160), dtype=torch.float32, device=dev)
        work = torch.empty(lib.b2_log_mel_workspace(n), dtype=torch.uint8, device=dev)
        keep += [audio, filt, out, work]
        frames = n // 160 + 1
        nbytes = frames * 201 * 400 * 4.0 + frames * 128 * 201 * 2.0  # FLOPs here
        label = f"log-mel {a.seconds:g} s audio ({frames} frames)"

        def run():
            bd.check(lib.b2_log_mel(audio.data_ptr(), n, filt.data_ptr(), out.data_ptr(), work.data_ptr(), stream),
                     a.kernel)
    elif a.kernel in GEMMS:
        epi, K, N = GEMMS[a.kernel]
        wt, bpw = WTYPES[a.wtype]
        rows = 2 * N if epi == bd.EPI_SILU_PAIR else N
        if wt == bd.W_F16:
            w = (torch.randn((rows, K), device=dev) * 0.02).half()
        else:
            w = torch.from_numpy(rng.integers(0, 256, (rows, int(K * bpw)), dtype=np.uint8)).to(dev)
        sc = torch.full((rows,), 0.01, dtype=torch.float32, device=dev)
        x16 = torch.randn((M, K), device=dev).half()
        y = torch.zeros((M, N), dtype=torch.float32, device=dev)
        args = bd.B2GemmArgs(y.data_ptr(), N, x16.data_ptr(), K, M, K, N, w.data_ptr(),
                             sc.data_ptr() if wt != bd.W_F16 else None, wt, epi, None, None, None, a.split)
        keep += [w, sc, x16, y]
        nbytes = rows * K * bpw
        label = f"{a.kernel} {a.wtype} M={M} K={K} N={N} split={a.split or 'auto'}"

        def run():
            bd.check(lib.b2_gemm(ctypes.byref(args), stream), a.kernel)
    else:
        max_seq = a.max_seq
        pos = rng.integers(128, min(4096, max_seq), M).astype(np.int32)
        seq_stride = NKV * max_seq * HD
        k = (torch.randn((M * seq_stride,), device=dev) * 0.1).half()
        v = torch.randn((M * seq_stride,), device=dev).half()
        pos_d = torch.from_numpy(pos).to(dev)
        rows_seq = torch.arange(M, dtype=torch.int32, device=dev)
        kv = bd.B2KVRef(k.data_ptr(), v.data_ptr(), seq_stride, seq_stride, 0, max_seq, rows_seq.data_ptr(),
                        pos_d.data_ptr(), M)
        q = torch.randn((M, (NQ + 2 * NKV) * HD), device=dev)
        out16 = torch.empty((M, NQ * HD), dtype=torch.float16, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        if a.kernel == "attn-blocks":
            ns = lib.b2_attention_blocks_split(max_seq, a.block)
        else:
            ns = (8 * 148 + M * NKV - 1) // (M * NKV)
        work = torch.empty(lib.b2_attention_workspace(M, NQ, HD, ns), dtype=torch.uint8, device=dev)
        keep += [k, v, pos_d, rows_seq, q, out16, err, work]
        nbytes = float((pos.astype(np.int64) + 1).sum()) * NKV * HD * 2 * 2
        label = f"{a.kernel} rows={M} ctx=U[128,4096) " + (f"block={a.block}" if a.kernel == "attn-blocks" else f"split={ns}")

        def run():
            if a.kernel == "attn-blocks":
                bd.check(lib.b2_attention_blocks(None, out16.data_ptr(), q.data_ptr(), q.shape[1], M, NQ, NKV, HD,
                                                 ctypes.byref(kv), work.data_ptr(), a.block, err.data_ptr(), stream),
                         a.kernel)
            else:
                bd.check(lib.b2_attention_f16(out16.data_ptr(), q.data_ptr(), q.shape[1], M, NQ, NKV, HD,
                                              ctypes.byref(kv), work.data_ptr(), ns, stream), a.kernel)

    run()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.iters):
        flush.zero_()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        run()
        t1.record()
        torch.cuda.synchronize()
        times.append(t0.elapsed_time(t1) * 1e3)
    med = sorted(times)[len(times) // 2]
    unit = "GFLOP/s" if a.kernel == "log-mel" else "GB/s"
    print(f"{label}: median {med:.1f} us, min {min(times):.1f} us, {nbytes / med / 1e3:.1f} {unit} algorithmic")
    return 0


if __name__ == "__main__":
    sys.exit(main())
