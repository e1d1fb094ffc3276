"""Argument validation of the kernel entry points (include/b2_kernels.h) on a
host without a GPU: every call below must be refused before any CUDA call.

The pointers passed are placeholders that are never dereferenced.  So that a
validation bug can never launch a kernel on them, the module runs only where
no CUDA device is present; on GPU hosts the same refusals are exercised by
test_gpu_kernels.py."""
from __future__ import annotations

import ctypes

import pytest

import b200_decoder as bd

try:  # a CUDA device makes a wrongly accepted call dangerous: skip there
    import torch

    _HAS_GPU = torch.cuda.is_available()
except ImportError:  # pragma: no cover
    _HAS_GPU = False

pytestmark = pytest.mark.skipif(_HAS_GPU, reason="placeholder pointers; GPU hosts run test_gpu_kernels.py")

P = 4096  # placeholder address, 16-byte aligned, never dereferenced


def gemm(**kw):
    a = dict(y=P, ldy=4096, x16=P, ldx=1024, M=64, K=1024, N=4096, w=P, scales=P, wtype=bd.W_F16,
             epilogue=bd.EPI_STORE, keys=None, tokens=None, y16=None, split_k=0)
    a.update(kw)
    args = bd.B2GemmArgs(*[a[f] for f, _ in bd.B2GemmArgs._fields_])
    return bd.capi().b2_gemm(ctypes.byref(args), None)


@pytest.mark.parametrize("bad", [
    dict(K=1000, ldx=1000),                      # K not a multiple of 64
    dict(wtype=bd.W_I8, scales=None),            # INT8 without scales
    dict(wtype=bd.W_I4, scales=None),            # INT4 without scales
    dict(N=4000, ldy=4000),                      # N not a multiple of 128
    dict(ldx=1020),                              # ldx not a multiple of 8
    dict(x16=P + 8),                             # activation rows not 16-byte aligned
    dict(w=P + 4),                               # weights not 16-byte aligned
    dict(y=None),                                # no output
    dict(y=None, y16=P, epilogue=bd.EPI_ADD),    # FP16 output only for STORE / SILU_PAIR
    dict(epilogue=bd.EPI_ARGMAX),                # argmax without keys / tokens
    dict(epilogue=7),                            # unknown epilogue
    dict(split_k=3),                             # cluster size not a power of two
    dict(split_k=16),                            # larger than a portable cluster
    dict(K=128, ldx=128, split_k=4),             # more CTAs than k stages
    dict(wtype=9),                               # unknown weight type
])
def test_gemm_refuses(bad):
    assert gemm(**bad) == -1
    assert b"b2_gemm" in bd.capi().b2_last_error()


def test_gemm_argmax_keys_size():
    assert bd.capi().b2_gemm_argmax_keys(64, 151936) == 64 * 1187 * 8
    assert bd.capi().b2_gemm_argmax_keys(3, 128) == 3 * 1 * 8


def test_rows_to_f16_refuses():
    L = bd.capi()
    assert L.b2_rows_to_f16(P, 1000, P, 1024, 4, 1024, None, 1e-6, None) == -1  # ldy < K
    assert L.b2_rows_to_f16(P, 1028, P, 1024, 4, 1024, None, 1e-6, None) == -1  # ldy % 8
    assert L.b2_rows_to_f16(None, 1024, P, 1024, 4, 1024, None, 1e-6, None) == -1


def test_attention_blocks_split():
    L = bd.capi()
    assert L.b2_attention_blocks_split(4108, 512) == 9
    assert L.b2_attention_blocks_split(4096, 1024) == 4
    assert L.b2_attention_blocks_split(4096, 96) == -1  # not a multiple of 64
    assert L.b2_attention_blocks_split(4096, 0) == -1


def test_attention_blocks_refuses():
    L = bd.capi()
    kv = bd.B2KVRef(P, P, 8 * 64 * 128, 8 * 64 * 128, 0, 64, None, P, 1)

    def call(kvr, M=16, nq=16, nkv=8, hd=128, block=64, err=P, out=P):
        return L.b2_attention_blocks(out, None, P, 2048, M, nq, nkv, hd, ctypes.byref(kvr), P, block, err, None)

    assert call(kv, block=100) == -1           # block not a multiple of 64
    assert call(kv, err=None) == -1            # no error flag
    assert call(kv, out=None) == -1            # no output
    assert call(kv, hd=64) == -1               # head_dim 128 only
    assert call(kv, nq=12) == -1               # nq not a multiple of nkv
    assert call(kv, M=513) == -1               # more rows than one launch takes
    bad = bd.B2KVRef(P + 8, P, 8 * 64 * 128, 8 * 64 * 128, 0, 64, None, P, 1)
    assert call(bad) == -1                     # K cache not 16-byte aligned
    odd = bd.B2KVRef(P, P, 8 * 64 * 128 + 64, 8 * 64 * 128, 0, 64, None, P, 1)
    assert call(odd) == -1                     # sequence stride not a whole number of rows


def test_attention_prefill_refuses():
    L = bd.capi()
    kv = bd.B2KVRef(P, P, 0, 0, 0, 64, None, P, 1)
    assert L.b2_attention_prefill(P, None, P, 2048, 8, 24, 8, 128, ctypes.byref(kv), 0, None) == -1  # G = 3
    assert L.b2_attention_prefill(P, None, P, 2048, 8, 16, 8, 128, ctypes.byref(kv), 60, None) == -1  # past max_seq
    assert L.b2_attention_prefill(None, None, P, 2048, 8, 16, 8, 128, ctypes.byref(kv), 0, None) == -1  # no output
    rows = bd.B2KVRef(P, P, 0, 0, 0, 64, P, P, 1)
    assert L.b2_attention_prefill(P, None, P, 2048, 8, 16, 8, 128, ctypes.byref(rows), 0, None) == -1  # several seqs
