"""The allocation-free lm_head + argmax entry point (b2_lm_head_argmax_noalloc).

Some callers cannot call cudaMalloc for a workspace: a host that owns all
device memory in its own pool, or code enqueued while another framework is
capturing the stream into a CUDA graph.  For them the library keeps the
argmax scratch in a fixed device array.  This test calls that entry point
through the C-ABI and checks it against the workspace entry point
(b2_lm_head_argmax) on the same inputs, twice in a row, and checks that an
oversized request is refused.  It lives in its own file, collected last, so a
failure here never hides the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = torch.device("cuda:0")


def _lm_head(L, wtype, V, K, rng):
    """Seeded lm_head weights in the given storage type, on the device."""
    emb = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    if wtype == bd.W_I8:
        table = np.empty((V, K), np.int8)
        scales = np.empty(V, np.float32)
        bd.check(L.matmul_decoder_quantize_lm_head(emb.ctypes.data, V, K, table.ctypes.data, scales.ctypes.data))
        return torch.from_numpy(table).to(DEV), torch.from_numpy(scales).to(DEV)
    table = emb.astype(np.float16) if wtype == bd.W_F16 else emb
    return torch.from_numpy(table).to(DEV), None


def _pair(L, wtype, M, V, K, t_d, s_d, nw_d, x_d, work, stream):
    """(logits, tokens) of the workspace and the no-alloc entry points."""
    la = torch.empty((M, V), dtype=torch.float32, device=DEV)
    lb = torch.empty((M, V), dtype=torch.float32, device=DEV)
    ta = torch.full((M,), -1, dtype=torch.int32, device=DEV)
    tb = torch.full((M,), -1, dtype=torch.int32, device=DEV)
    sp = s_d.data_ptr() if s_d is not None else None
    bd.check(L.b2_lm_head_argmax(x_d.data_ptr(), K, M, K, V, t_d.data_ptr(), sp, wtype, nw_d.data_ptr(), 1e-6,
                                 la.data_ptr(), V, ta.data_ptr(), work.data_ptr(), stream), "workspace entry point")
    bd.check(L.b2_lm_head_argmax_noalloc(x_d.data_ptr(), K, M, K, V, t_d.data_ptr(), sp, wtype, nw_d.data_ptr(),
                                         1e-6, lb.data_ptr(), V, tb.data_ptr(), stream), "no-alloc entry point")
    return la, ta, lb, tb


# (weight type, vocab): the F32 / F16 vocabularies stay inside the 1 MiB key
# array at M = 9 (8 and 16 vocab rows per CTA)
CASES = [(bd.W_I8, 151936), (bd.W_F16, 60000), (bd.W_F32, 50000)]


@pytest.mark.parametrize("wtype,V", CASES, ids=["int8", "f16", "f32"])
@pytest.mark.parametrize("M", [1, 2, 5, 9])
def test_noalloc_lm_head_matches_workspace_entry_point_twice(wtype, V, M):
    L = bd.capi()
    K = 1024
    rng = np.random.default_rng(2024 + 7 * wtype + M)
    t_d, s_d = _lm_head(L, wtype, V, K, rng)
    nw_d = torch.from_numpy((1 + 0.01 * rng.standard_normal(K)).astype(np.float32)).to(DEV)
    work = torch.empty(L.b2_lm_head_workspace(M, V), dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # two calls in a row: the shared scratch keeps no stale state
        x_d = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to(DEV)
        la, ta, lb, tb = _pair(L, wtype, M, V, K, t_d, s_d, nw_d, x_d, work, stream)
        torch.cuda.synchronize()
        a, b = la.cpu().numpy(), lb.cpu().numpy()
        # same kernel and inputs: equal within the tolerance the other tests use
        np.testing.assert_allclose(b, a, rtol=1e-6, atol=1e-6)
        assert tb.cpu().tolist() == ta.cpu().tolist(), f"call {call}"
        assert tb.cpu().tolist() == [int(np.argmax(b[m])) for m in range(M)]


def test_noalloc_lm_head_inside_cuda_graph_capture():
    """First call outside capture (it looks up the key array's address), then
    the same call enqueued while torch captures the stream into a CUDA graph;
    the replayed graph matches the workspace entry point."""
    L = bd.capi()
    V, K, M = 151936, 1024, 5
    rng = np.random.default_rng(77)
    t_d, s_d = _lm_head(L, bd.W_I8, V, K, rng)
    nw_d = torch.from_numpy((1 + 0.01 * rng.standard_normal(K)).astype(np.float32)).to(DEV)
    x_d = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to(DEV)
    work = torch.empty(L.b2_lm_head_workspace(M, V), dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    la, ta, _, _ = _pair(L, bd.W_I8, M, V, K, t_d, s_d, nw_d, x_d, work, stream)
    torch.cuda.synchronize()
    lg = torch.zeros((M, V), dtype=torch.float32, device=DEV)
    tg = torch.full((M,), -1, dtype=torch.int32, device=DEV)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cs = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        bd.check(L.b2_lm_head_argmax_noalloc(x_d.data_ptr(), K, M, K, V, t_d.data_ptr(), s_d.data_ptr(), bd.W_I8,
                                             nw_d.data_ptr(), 1e-6, lg.data_ptr(), V, tg.data_ptr(), cs),
                 "no-alloc entry point under capture")
    torch.cuda.synchronize()
    assert tg.cpu().tolist() == [-1] * M  # capture recorded the work without running it
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    np.testing.assert_allclose(lg.cpu().numpy(), la.cpu().numpy(), rtol=1e-6, atol=1e-6)
    assert tg.cpu().tolist() == ta.cpu().tolist()
    del g


def test_noalloc_lm_head_rejects_oversized_request():
    L = bd.capi()
    V, K = 151936, 1024
    per_row = (V + 31) // 32  # int8: 32 vocab rows per CTA
    M = L.b2_lm_head_noalloc_max_keys() // per_row + 1
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    rc = L.b2_lm_head_argmax_noalloc(dummy.data_ptr(), K, M, K, V, dummy.data_ptr(), dummy.data_ptr(), bd.W_I8,
                                     None, 1e-6, None, V, dummy.data_ptr(), None)
    assert rc == -1
    assert b"exceeds the fixed scratch" in L.b2_last_error()
