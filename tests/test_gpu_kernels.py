"""Kernel-level parity: each b2_* kernel (called through the C-ABI) against the
CPU oracle on the same seeded inputs.

Tolerances: floating-point outputs must reach cosine >= 0.9995 and
max-abs <= 2e-2 (the north-star criterion), and additionally stay within
rtol/atol 2e-3 of the oracle where only summation order differs.  Integer
results (argmax token ids, KV bytes of exactly representable values) are
compared exactly.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import b200_decoder as bd  # noqa: E402
import ref_decoder as ref  # noqa: E402

if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

DEV = torch.device("cuda:0")


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def assert_close(got, exp, rtol=2e-3, atol=2e-3):
    assert cos(got, exp) >= 0.9995, cos(got, exp)
    assert np.abs(np.asarray(got) - np.asarray(exp)).max() <= 2e-2
    np.testing.assert_allclose(got, exp, rtol=rtol, atol=atol)


_LIVE = []


def dev(a):
    """Device copy of a numpy array, kept alive until the end of the test: a
    temporary whose data_ptr() is passed to the C-ABI would otherwise be freed
    (and its block reused) before the asynchronous kernel reads it."""
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _LIVE.append(t)
    return t


@pytest.fixture(autouse=True)
def _keep_device_buffers_alive():
    yield
    torch.cuda.synchronize()
    _LIVE.clear()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def device_rows(w_file, wtype, N):
    """File layout ([K,N] fp16/int8, [K,N/2] int4) -> device rows [N, K(/2)]."""
    if wtype == bd.W_I4:
        lo = (w_file & 15).astype(np.uint8)
        hi = (w_file >> 4).astype(np.uint8)
        nib = np.empty((w_file.shape[0], N), np.uint8)
        nib[:, 0::2], nib[:, 1::2] = lo, hi
        t = nib.T  # [N, K]
        return np.ascontiguousarray((t[:, 0::2] | (t[:, 1::2] << 4)).astype(np.uint8))
    return np.ascontiguousarray(w_file.T)


def make_weight(rng, K, N, wtype):
    w16 = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    if wtype == bd.W_F16:
        return w16, None, ref.W_F16
    bits = 8 if wtype == bd.W_I8 else 4
    q, s = ref.quantize_cols(w16, bits)
    return q, s, (ref.W_I8 if bits == 8 else ref.W_I4)


@pytest.mark.parametrize("wtype", [bd.W_F16, bd.W_I8, bd.W_I4])
@pytest.mark.parametrize("M", [1, 3, 8, 13])
@pytest.mark.parametrize("KN", [(1024, 4096), (3072, 1024), (2048, 96)])
def test_gemv_store_and_add(wtype, M, KN):
    K, N = KN
    rng = np.random.default_rng(1000 * wtype + 10 * M + K // 1024)
    wf, s, rwt = make_weight(rng, K, N, wtype)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    y0 = rng.standard_normal((M, N), dtype=np.float32)
    for norm, epi in ((False, bd.EPI_STORE), (True, bd.EPI_STORE), (False, bd.EPI_ADD)):
        xn = np.stack([ref.rms_norm(r, norm_w) for r in x]) if norm else x
        exp = ref.gemm(xn, wf, s, wtype=rwt, n=N)
        if epi == bd.EPI_ADD:
            exp = exp + y0
        w_d, x_d = dev(device_rows(wf, wtype, N)), dev(x)
        s_d = dev(s) if s is not None else None
        nw_d = dev(norm_w)
        y_d = dev(y0.copy())
        a = bd.B2GemvArgs(y_d.data_ptr(), N, x_d.data_ptr(), K, M, K, N, w_d.data_ptr(),
                          s_d.data_ptr() if s_d is not None else None, wtype,
                          nw_d.data_ptr() if norm else None, 1e-6, epi)
        bd.check(bd.capi().b2_gemv(ctypes.byref(a), stream()), "b2_gemv")
        torch.cuda.synchronize()
        assert_close(y_d.cpu().numpy(), exp)


@pytest.mark.parametrize("wtype", [bd.W_F16, bd.W_I8, bd.W_I4])
@pytest.mark.parametrize("M", [1, 5])
def test_gemv_silu_pair(wtype, M):
    K, F = 1024, 3072
    rng = np.random.default_rng(77 + wtype + M)
    wg, sg, rwt = make_weight(rng, K, F, wtype)
    wu, su, _ = make_weight(rng, K, F, wtype)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    xn = np.stack([ref.rms_norm(r, norm_w) for r in x])
    g = ref.gemm(xn, wg, sg, wtype=rwt, n=F)
    u = ref.gemm(xn, wu, su, wtype=rwt, n=F)
    exp = np.stack([ref.silu_mul(g[i], u[i]) for i in range(M)])
    rows = np.concatenate([device_rows(wg, wtype, F), device_rows(wu, wtype, F)])
    scales = np.concatenate([sg, su]) if sg is not None else None
    w_d, x_d, nw_d = dev(rows), dev(x), dev(norm_w)
    s_d = dev(scales) if scales is not None else None
    y_d = torch.zeros((M, F), dtype=torch.float32, device=DEV)
    a = bd.B2GemvArgs(y_d.data_ptr(), F, x_d.data_ptr(), K, M, K, F, w_d.data_ptr(),
                      s_d.data_ptr() if s_d is not None else None, wtype, nw_d.data_ptr(), 1e-6,
                      bd.EPI_SILU_PAIR)
    bd.check(bd.capi().b2_gemv(ctypes.byref(a), stream()), "b2_gemv pair")
    torch.cuda.synchronize()
    assert_close(y_d.cpu().numpy(), exp)


# ── tensor-core GEMM (batch prefill) ──

def rows_f16(x_d, M, K, norm_w=None):
    """b2_rows_to_f16 of device rows x_d [M, K] -> device FP16 [M, K]."""
    y16 = torch.empty((M, K), dtype=torch.float16, device=DEV)
    _LIVE.append(y16)
    nw = dev(norm_w) if norm_w is not None else None
    bd.check(bd.capi().b2_rows_to_f16(y16.data_ptr(), K, x_d.data_ptr(), K, M, K,
                                      nw.data_ptr() if nw is not None else None, 1e-6, stream()),
             "b2_rows_to_f16")
    return y16


def test_rows_to_f16_matches_oracle_rounding():
    rng = np.random.default_rng(4242)
    M, K = 37, 3072
    x = rng.standard_normal((M, K), dtype=np.float32) * 3
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    got = rows_f16(dev(x), M, K, norm_w).cpu().numpy().astype(np.float32)
    exp = np.stack([ref.rms_norm(r, norm_w) for r in x]).astype(np.float16).astype(np.float32)
    # the device RMS sum runs in another order: an element may land on the
    # neighbouring FP16 value, never further
    ulp = np.abs(np.spacing(exp.astype(np.float16)).astype(np.float32))
    assert np.all(np.abs(got - exp) <= ulp)
    assert np.mean(got == exp) > 0.99
    plain = rows_f16(dev(x), M, K).cpu().numpy()
    np.testing.assert_array_equal(plain, x.astype(np.float16))


def gemm_ref(x, w16, norm_w=None):
    """FP32 reference of the GEMM numerics: FP16-rounded activations times FP16
    weights, summed in FP32 (numpy BLAS)."""
    xn = np.stack([ref.rms_norm(r, norm_w) for r in x]) if norm_w is not None else x
    return xn.astype(np.float16).astype(np.float32) @ w16.astype(np.float32)


@pytest.mark.parametrize("M", [16, 60, 130, 512])
@pytest.mark.parametrize("KN", [(1024, 4096), (2048, 1024), (3072, 1024)])
def test_gemm_tensor_cores_store_and_add(M, KN):
    K, N = KN
    rng = np.random.default_rng(5000 + M + K // 1024)
    w16 = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    y0 = rng.standard_normal((M, N), dtype=np.float32)
    w_d, x_d = dev(np.ascontiguousarray(w16.T)), dev(x)
    for norm, epi in ((True, bd.EPI_STORE), (False, bd.EPI_ADD)):
        exp = gemm_ref(x, w16, norm_w if norm else None) + (y0 if epi == bd.EPI_ADD else 0)
        x16 = rows_f16(x_d, M, K, norm_w if norm else None)
        y_d = dev(y0.copy())
        a = bd.B2GemmArgs(y_d.data_ptr(), N, x16.data_ptr(), K, M, K, N, w_d.data_ptr(), None, bd.W_F16, epi)
        bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm")
        torch.cuda.synchronize()
        assert_close(y_d.cpu().numpy(), exp)


def test_gemm_tensor_cores_matches_oracle():
    """One prefill-shaped case against the C oracle's reference matmul."""
    M, K, N = 60, 1024, 1024
    rng = np.random.default_rng(777)
    w16 = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K), dtype=np.float32)
    exp = ref.gemm(x, w16, None, wtype=ref.W_F16, n=N)
    x16 = rows_f16(dev(x), M, K)
    y_d = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    w_d = dev(np.ascontiguousarray(w16.T))
    a = bd.B2GemmArgs(y_d.data_ptr(), N, x16.data_ptr(), K, M, K, N, w_d.data_ptr(), None, bd.W_F16,
                      bd.EPI_STORE)
    bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm")
    torch.cuda.synchronize()
    assert_close(y_d.cpu().numpy(), exp)


@pytest.mark.parametrize("M", [16, 60, 512])
def test_gemm_tensor_cores_silu_pair(M):
    K, F = 1024, 3072
    rng = np.random.default_rng(900 + M)
    wg = (rng.standard_normal((K, F)) * 0.02).astype(np.float16)
    wu = (rng.standard_normal((K, F)) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    g, u = gemm_ref(x, wg, norm_w), gemm_ref(x, wu, norm_w)
    exp = g / (1 + np.exp(-g)) * u
    rows = np.concatenate([np.ascontiguousarray(wg.T), np.ascontiguousarray(wu.T)])
    x16 = rows_f16(dev(x), M, K, norm_w)
    y_d = torch.zeros((M, F), dtype=torch.float32, device=DEV)
    a = bd.B2GemmArgs(y_d.data_ptr(), F, x16.data_ptr(), K, M, K, F, dev(rows).data_ptr(), None, bd.W_F16,
                      bd.EPI_SILU_PAIR)
    bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm pair")
    torch.cuda.synchronize()
    assert_close(y_d.cpu().numpy(), exp)


@pytest.mark.parametrize("wtype", [bd.W_I8, bd.W_I4])
@pytest.mark.parametrize("M", [16, 64, 130])
def test_gemm_tensor_cores_quantized_weights(wtype, M):
    """INT8 / INT4 rows widened on chip to FP16 for tcgen05, against the C oracle."""
    rng = np.random.default_rng(6100 + 10 * wtype + M)
    for (K, N), epi in (((1024, 4096), bd.EPI_STORE), ((2048, 1024), bd.EPI_ADD)):
        wf, s, rwt = make_weight(rng, K, N, wtype)
        x = rng.standard_normal((M, K), dtype=np.float32)
        y0 = rng.standard_normal((M, N), dtype=np.float32)
        exp = ref.gemm(x, wf, s, wtype=rwt, n=N) + (y0 if epi == bd.EPI_ADD else 0)
        x16 = rows_f16(dev(x), M, K)
        y_d = dev(y0.copy())
        a = bd.B2GemmArgs(y_d.data_ptr(), N, x16.data_ptr(), K, M, K, N, dev(device_rows(wf, wtype, N)).data_ptr(),
                          dev(s).data_ptr(), wtype, epi, None, None)
        bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm quantized")
        torch.cuda.synchronize()
        assert_close(y_d.cpu().numpy(), exp)


@pytest.mark.parametrize("wtype", [bd.W_I8, bd.W_I4])
def test_gemm_tensor_cores_quantized_silu_pair(wtype):
    K, F, M = 1024, 3072, 64
    rng = np.random.default_rng(6200 + wtype)
    wg, sg, rwt = make_weight(rng, K, F, wtype)
    wu, su, _ = make_weight(rng, K, F, wtype)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    xn = np.stack([ref.rms_norm(r, norm_w) for r in x])
    g, u = ref.gemm(xn, wg, sg, wtype=rwt, n=F), ref.gemm(xn, wu, su, wtype=rwt, n=F)
    exp = np.stack([ref.silu_mul(g[i], u[i]) for i in range(M)])
    rows = np.concatenate([device_rows(wg, wtype, F), device_rows(wu, wtype, F)])
    x16 = rows_f16(dev(x), M, K, norm_w)
    y_d = torch.zeros((M, F), dtype=torch.float32, device=DEV)
    a = bd.B2GemmArgs(y_d.data_ptr(), F, x16.data_ptr(), K, M, K, F, dev(rows).data_ptr(),
                      dev(np.concatenate([sg, su])).data_ptr(), wtype, bd.EPI_SILU_PAIR, None, None)
    bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm quantized pair")
    torch.cuda.synchronize()
    assert_close(y_d.cpu().numpy(), exp)


@pytest.mark.parametrize("V", [8192, 151936, 70001])
def test_gemm_tensor_cores_lm_head_argmax(V):
    """Batched INT8 lm_head on the tensor cores: logits vs the oracle and
    argmax of the kernel's own logits (first index on ties)."""
    K, M = 1024, 64
    rng = np.random.default_rng(6300 + V)
    emb = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    table = np.empty((V, K), np.int8)
    scales = np.empty(V, np.float32)
    bd.check(bd.capi().matmul_decoder_quantize_lm_head(emb.ctypes.data, V, K, table.ctypes.data, scales.ctypes.data))
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    x16 = rows_f16(dev(x), M, K, norm_w)
    logits_d = torch.empty((M, V), dtype=torch.float32, device=DEV)
    tok_d = torch.empty(M, dtype=torch.int32, device=DEV)
    keys = torch.empty(bd.capi().b2_gemm_argmax_keys(M, V), dtype=torch.uint8, device=DEV)
    a = bd.B2GemmArgs(logits_d.data_ptr(), V, x16.data_ptr(), K, M, K, V, dev(table).data_ptr(),
                      dev(scales).data_ptr(), bd.W_I8, bd.EPI_ARGMAX, keys.data_ptr(), tok_d.data_ptr())
    bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), "b2_gemm argmax")
    torch.cuda.synchronize()
    logits, toks = logits_d.cpu().numpy(), tok_d.cpu().numpy()
    for m in range(0, M, 9):
        exp = lm_reference(x[m], norm_w, table, scales, bd.W_I8)
        assert_close(logits[m], exp, rtol=1e-3, atol=1e-3)
    for m in range(M):
        assert toks[m] == int(np.argmax(logits[m]))


@pytest.mark.parametrize("wtype", [bd.W_F16, bd.W_I8, bd.W_I4])
@pytest.mark.parametrize("split", [1, 2, 4, 8])
@pytest.mark.parametrize("M", [40, 130])
def test_gemm_split_k_cluster_all_epilogues(wtype, split, M):
    """Split-K over a thread-block cluster (each CTA sums K / split, the
    partial sums are reduced through distributed shared memory and each CTA
    finishes 1/split of the token columns) against the oracle for every
    epilogue: STORE (FP32 and FP16 rows), ADD, SILU_PAIR (FP16 rows) and
    ARGMAX.  M = 40 leaves whole token slices empty at split 8."""
    K, N = 1024, 1024
    rng = np.random.default_rng(7000 + 100 * wtype + 10 * split + M)
    wf, s, rwt = make_weight(rng, K, N, wtype)
    wu, su, _ = make_weight(rng, K, N, wtype)
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    xn = np.stack([ref.rms_norm(r, norm_w) for r in x])
    exp = ref.gemm(xn, wf, s, wtype=rwt, n=N)
    x16 = rows_f16(dev(x), M, K, norm_w)
    w_d = dev(device_rows(wf, wtype, N))
    s_d = dev(s).data_ptr() if s is not None else None

    def run(y, epi, w=w_d.data_ptr(), sc=s_d, y16=None, keys=None, toks=None):
        a = bd.B2GemmArgs(y, N, x16.data_ptr(), K, M, K, N, w, sc, wtype, epi, keys, toks, y16, split)
        bd.check(bd.capi().b2_gemm(ctypes.byref(a), stream()), f"b2_gemm split {split}")
        torch.cuda.synchronize()

    y_d = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    run(y_d.data_ptr(), bd.EPI_STORE)
    assert_close(y_d.cpu().numpy(), exp)
    h_d = torch.zeros((M, N), dtype=torch.float16, device=DEV)
    run(None, bd.EPI_STORE, y16=h_d.data_ptr())
    np.testing.assert_array_equal(h_d.cpu().numpy(), y_d.cpu().numpy().astype(np.float16))
    y0 = rng.standard_normal((M, N), dtype=np.float32)
    y_d = dev(y0.copy())
    run(y_d.data_ptr(), bd.EPI_ADD)
    assert_close(y_d.cpu().numpy(), y0 + exp)
    # gate|up pair: gate rows then up rows, SiLU(gate) * up as FP16 rows
    up = ref.gemm(xn, wu, su, wtype=rwt, n=N)
    pair_exp = np.stack([ref.silu_mul(exp[i], up[i]) for i in range(M)])
    rows = dev(np.concatenate([device_rows(wf, wtype, N), device_rows(wu, wtype, N)]))
    sc2 = dev(np.concatenate([s, su])).data_ptr() if s is not None else None
    h_d = torch.zeros((M, N), dtype=torch.float16, device=DEV)
    run(None, bd.EPI_SILU_PAIR, w=rows.data_ptr(), sc=sc2, y16=h_d.data_ptr())
    assert_close(h_d.float().cpu().numpy(), pair_exp, rtol=4e-3, atol=4e-3)
    # argmax of the kernel's own logits, first index on ties
    logits_d = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    tok_d = torch.full((M,), -1, dtype=torch.int32, device=DEV)
    keys = torch.empty(bd.capi().b2_gemm_argmax_keys(M, N), dtype=torch.uint8, device=DEV)
    run(logits_d.data_ptr(), bd.EPI_ARGMAX, keys=keys.data_ptr(), toks=tok_d.data_ptr())
    logits = logits_d.cpu().numpy()
    assert_close(logits, exp)
    np.testing.assert_array_equal(tok_d.cpu().numpy(), logits.argmax(axis=1))


def test_gemm_rejects_unsupported_shapes():
    a = bd.B2GemmArgs(16, 128, 16, 100, 32, 100, 128, 16, None, bd.W_F16, 0, None, None)  # K % 64
    assert bd.capi().b2_gemm(ctypes.byref(a), None) == -1
    a = bd.B2GemmArgs(16, 128, 16, 128, 32, 128, 128, 16, None, bd.W_I8, 0, None, None)  # INT8 without scales
    assert bd.capi().b2_gemm(ctypes.byref(a), None) == -1
    a = bd.B2GemmArgs(16, 96, 16, 128, 32, 128, 96, 16, None, bd.W_F16, 0, None, None)   # N % 128
    assert bd.capi().b2_gemm(ctypes.byref(a), None) == -1
    a = bd.B2GemmArgs(None, 0, 16, 128, 32, 128, 1000, 16, None, bd.W_F16, bd.EPI_ARGMAX, None, None)  # no keys
    assert bd.capi().b2_gemm(ctypes.byref(a), None) == -1
    for split in (3, 16, 4):  # not a power of two <= 8; more CTAs than k stages (K = 128: 2 stages)
        a = bd.B2GemmArgs(16, 128, 16, 128, 32, 128, 128, 16, None, bd.W_F16, 0, None, None, None, split)
        assert bd.capi().b2_gemm(ctypes.byref(a), None) == -1


def test_gemv_rejects_bad_shapes():
    a = bd.B2GemvArgs(1, 8, 1, 8, 1, 1000, 8, 16, None, bd.W_I4, None, 0.0, 0)
    assert bd.capi().b2_gemv(ctypes.byref(a), None) == -1
    a = bd.B2GemvArgs(1, 8, 1, 8, 1, 1024, 8, 16, None, bd.W_I8, None, 0.0, 0)  # no scales
    assert bd.capi().b2_gemv(ctypes.byref(a), None) == -1


def kv_ref(k, v, layer_stride, max_seq, pos_d, rows_seq_d=None, seq_stride=0, layer=0, n_seqs=1):
    return bd.B2KVRef(k.data_ptr(), v.data_ptr(), seq_stride, layer_stride, layer, max_seq,
                      rows_seq_d.data_ptr() if rows_seq_d is not None else None, pos_d.data_ptr(), n_seqs)


@pytest.mark.parametrize("style", [0, 1])
def test_qk_rope_kv(style):
    nq, nkv, hd, max_seq, L = 16, 8, 128, 256, 2
    rng = np.random.default_rng(5 + style)
    M = 4
    qkv = rng.standard_normal((M, (nq + 2 * nkv) * hd), dtype=np.float32) * 2
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    pos = np.array([0, 1, 100, 255], np.int32)
    cos_t, sin_t = ref.rope_tables(max_seq, hd, 1e6)
    kc = torch.zeros((L, nkv, max_seq, hd), dtype=torch.float16, device=DEV)
    vc = torch.zeros_like(kc)
    qkv_d, pos_d = dev(qkv), dev(pos)
    kv = kv_ref(kc, vc, nkv * max_seq * hd, max_seq, pos_d, layer=1)
    bd.check(bd.capi().b2_qk_rope_kv(qkv_d.data_ptr(), qkv.shape[1], M, nq, nkv, hd, dev(qn).data_ptr(),
                                     dev(kn).data_ptr(), 1e-6, dev(cos_t).data_ptr(), dev(sin_t).data_ptr(),
                                     style, ctypes.byref(kv), stream()), "qk_rope_kv")
    torch.cuda.synchronize()
    got_q = qkv_d.cpu().numpy()[:, :nq * hd]
    kc_h, vc_h = kc.cpu().numpy(), vc.cpu().numpy()
    for m in range(M):
        q = qkv[m, :nq * hd].reshape(nq, hd)
        k = qkv[m, nq * hd:(nq + nkv) * hd].reshape(nkv, hd)
        v = qkv[m, (nq + nkv) * hd:].reshape(nkv, hd)
        qe = ref.apply_rope(np.stack([ref.rms_norm(r, qn) for r in q]), cos_t[pos[m]], sin_t[pos[m]], style)
        ke = ref.apply_rope(np.stack([ref.rms_norm(r, kn) for r in k]), cos_t[pos[m]], sin_t[pos[m]], style)
        np.testing.assert_allclose(got_q[m].reshape(nq, hd), qe, rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(kc_h[1, :, pos[m]].astype(np.float32), ke.astype(np.float16).astype(np.float32),
                                   rtol=1e-3, atol=1e-3)
        np.testing.assert_array_equal(vc_h[1, :, pos[m]], v.astype(np.float16))
    assert not kc_h[0].any()  # layer 0 untouched


@pytest.mark.parametrize("G", [2, 1])
def test_attention_rows_and_sequences(G):
    nkv, hd, max_seq = 8, 128, 4100
    nq = nkv * G
    rng = np.random.default_rng(9 + G)
    n_seq = 3
    kc = rng.standard_normal((n_seq, nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((n_seq, nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    rows_seq = np.array([0, 2, 1, 2, 0], np.int32)
    pos = np.array([0, 1, 127, 1023, 4095], np.int32)
    M = len(pos)
    q = rng.standard_normal((M, nq * hd), dtype=np.float32)
    kc_d, vc_d = dev(kc), dev(vc)
    for nsplit in (0, 1, 7):
        work = torch.empty(bd.capi().b2_attention_workspace(M, nq, hd, nsplit), dtype=torch.uint8, device=DEV)
        out_d = torch.empty((M, nq * hd), dtype=torch.float32, device=DEV)
        kv = kv_ref(kc_d, vc_d, 0, max_seq, dev(pos), dev(rows_seq), seq_stride=nkv * max_seq * hd, n_seqs=n_seq)
        bd.check(bd.capi().b2_attention(out_d.data_ptr(), dev(q).data_ptr(), nq * hd, M, nq, nkv, hd,
                                        ctypes.byref(kv), work.data_ptr(), nsplit, stream()), "attention")
        torch.cuda.synchronize()
        out = out_d.cpu().numpy()
        for m in range(M):
            s, L = rows_seq[m], pos[m] + 1
            kk = kc[s, :, :L].transpose(1, 0, 2).astype(np.float32)  # [L][nkv][hd]
            vv = vc[s, :, :L].transpose(1, 0, 2).astype(np.float32)
            exp = ref.attention(q[m], kk, vv, nq, nkv, hd)
            assert_close(out[m], exp, rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("G", [1, 2, 4])
@pytest.mark.parametrize("block", [64, 256])
def test_attention_blocks_rows_and_sequences(G, block):
    """Batched-decode attention in fixed position blocks (TMA into a
    shared-memory ring, scores and P.V on the tensor cores with FP16 Q and P)
    against the oracle: rows of different sequences and lengths, including
    partial last stages and blocks past a row's end, in FP32 and FP16 output."""
    nkv, hd, max_seq = 8, 128, 4100
    nq = nkv * G
    rng = np.random.default_rng(90 + G + block)
    n_seq = 3
    kc = rng.standard_normal((n_seq, nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((n_seq, nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    rows_seq = np.array([0, 2, 1, 2, 0, 1], np.int32)
    pos = np.array([0, 1, 31, 127, 1000, 4095], np.int32)
    M = len(pos)
    q = rng.standard_normal((M, nq * hd), dtype=np.float32)
    kc_d, vc_d, q_d = dev(kc), dev(vc), dev(q)
    nsplit = bd.capi().b2_attention_blocks_split(max_seq, block)
    assert nsplit == -(-max_seq // block)
    work = torch.empty(bd.capi().b2_attention_workspace(M, nq, hd, nsplit), dtype=torch.uint8, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kv = kv_ref(kc_d, vc_d, 0, max_seq, dev(pos), dev(rows_seq), seq_stride=nkv * max_seq * hd, n_seqs=n_seq)
    out_d = torch.empty((M, nq * hd), dtype=torch.float32, device=DEV)
    bd.check(bd.capi().b2_attention_blocks(out_d.data_ptr(), None, q_d.data_ptr(), nq * hd, M, nq, nkv, hd,
                                           ctypes.byref(kv), work.data_ptr(), block, err.data_ptr(), stream()),
             "attention_blocks")
    out_h = torch.empty((M, nq * hd), dtype=torch.float16, device=DEV)
    bd.check(bd.capi().b2_attention_blocks(None, out_h.data_ptr(), q_d.data_ptr(), nq * hd, M, nq, nkv, hd,
                                           ctypes.byref(kv), work.data_ptr(), block, err.data_ptr(), stream()),
             "attention_blocks f16")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    out = out_d.cpu().numpy()
    np.testing.assert_array_equal(out_h.cpu().numpy(), out.astype(np.float16))
    for m in range(M):
        sq, L = rows_seq[m], pos[m] + 1
        kk = kc[sq, :, :L].transpose(1, 0, 2).astype(np.float32)
        vv = vc[sq, :, :L].transpose(1, 0, 2).astype(np.float32)
        assert_close(out[m], ref.attention(q[m], kk, vv, nq, nkv, hd), rtol=2e-2, atol=5e-3)


def test_attention_blocks_rejects_bad_arguments():
    kv = bd.B2KVRef(16, 16, 0, 0, 0, 64, None, 16, 1)
    assert bd.capi().b2_attention_blocks_split(4096, 96) == -1  # not a multiple of 64
    assert bd.capi().b2_attention_blocks(16, None, 16, 2048, 8, 16, 8, 128, ctypes.byref(kv), 16, 100, 16, None) == -1
    assert bd.capi().b2_attention_blocks(16, None, 16, 2048, 8, 16, 8, 128, ctypes.byref(kv), 16, 64, None, None) == -1
    kv = bd.B2KVRef(24, 16, 0, 0, 0, 64, None, 16, 1)  # K cache not 16-byte aligned
    assert bd.capi().b2_attention_blocks(16, None, 16, 2048, 8, 16, 8, 128, ctypes.byref(kv), 16, 64, 16, None) == -1


@pytest.mark.parametrize("M, base", [(16, 0), (60, 0), (77, 100), (512, 0), (200, 3000)])
def test_attention_prefill_flash_matches_oracle(M, base):
    """Causal flash attention of a prefill chunk (tensor cores, FP16 Q and P)
    against the oracle's FP32 attention on sampled rows, and against the
    per-row split kernel on every row."""
    nkv, hd, G = 8, 128, 2
    nq, max_seq = nkv * G, base + M + 4
    rng = np.random.default_rng(7000 + M + base)
    kc = rng.standard_normal((nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((nkv, max_seq, hd), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((M, nq * hd), dtype=np.float32)
    pos = (base + np.arange(M)).astype(np.int32)
    kc_d, vc_d, q_d = dev(kc), dev(vc), dev(q)
    kv = kv_ref(kc_d, vc_d, 0, max_seq, dev(pos))
    out_f = torch.empty((M, nq * hd), dtype=torch.float32, device=DEV)
    bd.check(bd.capi().b2_attention_prefill(out_f.data_ptr(), None, q_d.data_ptr(), nq * hd, M, nq, nkv, hd,
                                            ctypes.byref(kv), base, stream()), "attention_prefill")
    out_h = torch.empty((M, nq * hd), dtype=torch.float16, device=DEV)
    bd.check(bd.capi().b2_attention_prefill(None, out_h.data_ptr(), q_d.data_ptr(), nq * hd, M, nq, nkv, hd,
                                            ctypes.byref(kv), base, stream()), "attention_prefill f16")
    work = torch.empty(bd.capi().b2_attention_workspace(M, nq, hd, 0), dtype=torch.uint8, device=DEV)
    out_s = torch.empty((M, nq * hd), dtype=torch.float32, device=DEV)
    bd.check(bd.capi().b2_attention(out_s.data_ptr(), q_d.data_ptr(), nq * hd, M, nq, nkv, hd, ctypes.byref(kv),
                                    work.data_ptr(), 0, stream()), "attention")
    torch.cuda.synchronize()
    flash, split = out_f.cpu().numpy(), out_s.cpu().numpy()
    assert_close(flash, split, rtol=2e-2, atol=5e-3)
    np.testing.assert_array_equal(out_h.cpu().numpy(), flash.astype(np.float16))  # same values, rounded
    for m in sorted({0, M // 3, M - 1}):
        L = base + m + 1
        exp = ref.attention(q[m], kc[:, :L].transpose(1, 0, 2).astype(np.float32),
                            vc[:, :L].transpose(1, 0, 2).astype(np.float32), nq, nkv, hd)
        assert_close(flash[m], exp, rtol=2e-2, atol=5e-3)


def test_attention_prefill_rejects_unsupported():
    kv = bd.B2KVRef(16, 16, 0, 0, 0, 64, None, 16, 1)
    assert bd.capi().b2_attention_prefill(16, None, 16, 2048, 8, 24, 8, 128, ctypes.byref(kv), 0, None) == -1  # G = 3
    assert bd.capi().b2_attention_prefill(16, None, 16, 2048, 8, 16, 8, 128, ctypes.byref(kv), 60, None) == -1  # past max_seq


def lm_reference(x, norm_w, table, scales, wtype):
    xn = ref.rms_norm(x, norm_w)
    if wtype == bd.W_I8:
        x16 = xn.astype(np.float16).astype(np.float64)
        return (table.astype(np.float64) @ x16) * scales
    return table.astype(np.float64) @ xn.astype(np.float64)


@pytest.mark.parametrize("wtype", [bd.W_I8, bd.W_F16, bd.W_F32])
@pytest.mark.parametrize("M", [1, 3])
def test_lm_head_argmax(wtype, M):
    V, K = 151936, 1024
    rng = np.random.default_rng(31 + wtype + M)
    emb = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    if wtype == bd.W_I8:
        table = np.empty((V, K), np.int8)
        scales = np.empty(V, np.float32)
        bd.check(bd.capi().matmul_decoder_quantize_lm_head(emb.ctypes.data, V, K, table.ctypes.data,
                                                            scales.ctypes.data))
    elif wtype == bd.W_F16:
        table, scales = emb.astype(np.float16), None
    else:
        table, scales = emb, None
    x = rng.standard_normal((M, K), dtype=np.float32)
    norm_w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    t_d = dev(table)
    s_d = dev(scales) if scales is not None else None
    logits_d = torch.empty((M, V), dtype=torch.float32, device=DEV)
    tok_d = torch.empty(M, dtype=torch.int32, device=DEV)
    work = torch.empty(bd.capi().b2_lm_head_workspace(M, V), dtype=torch.uint8, device=DEV)
    bd.check(bd.capi().b2_lm_head_argmax(dev(x).data_ptr(), K, M, K, V, t_d.data_ptr(),
                                         s_d.data_ptr() if s_d is not None else None, wtype,
                                         dev(norm_w).data_ptr(), 1e-6, logits_d.data_ptr(), V,
                                         tok_d.data_ptr(), work.data_ptr(), stream()), "lm_head")
    torch.cuda.synchronize()
    logits, toks = logits_d.cpu().numpy(), tok_d.cpu().numpy()
    for m in range(M):
        exp = lm_reference(x[m], norm_w, table, scales, wtype)
        assert_close(logits[m], exp, rtol=1e-3, atol=1e-3)
        assert toks[m] == int(np.argmax(logits[m]))  # first max of the kernel's own logits
        top2 = np.sort(exp)[-2:]
        if top2[1] - top2[0] > 1e-3:
            assert toks[m] == int(np.argmax(exp))


def test_lm_head_ties_pick_lowest_index():
    V, K = 70000, 1024
    table = np.zeros((V, K), np.float16)
    table[:, 0] = np.float16(0.001)
    for v in (123, 40000, 69999):  # equal maxima far apart (different CTAs)
        table[v, 0] = np.float16(0.5)
    x = np.zeros((1, K), np.float32)
    x[0, 0] = 1.0
    logits_d = torch.empty((1, V), dtype=torch.float32, device=DEV)
    tok_d = torch.empty(1, dtype=torch.int32, device=DEV)
    work = torch.empty(bd.capi().b2_lm_head_workspace(1, V), dtype=torch.uint8, device=DEV)
    bd.check(bd.capi().b2_lm_head_argmax(dev(x).data_ptr(), K, 1, K, V, dev(table).data_ptr(), None,
                                         bd.W_F16, None, 0.0, logits_d.data_ptr(), V, tok_d.data_ptr(),
                                         work.data_ptr(), stream()), "lm_head ties")
    torch.cuda.synchronize()
    assert int(tok_d.cpu()[0]) == 123
    assert ref.argmax(logits_d.cpu().numpy()[0]) == 123


def test_embed_token_and_staged():
    V, H = 64, 1024
    rng = np.random.default_rng(2)
    table = rng.standard_normal((V, H), dtype=np.float32)
    staged = rng.standard_normal((1, H), dtype=np.float32)
    out = torch.empty((2, H), dtype=torch.float32, device=DEV)
    toks = dev(np.array([5, 63], np.int32))
    bd.check(bd.capi().b2_embed(out.data_ptr(), dev(table).data_ptr(), toks.data_ptr(), None, None, 2, H,
                                stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), table[[5, 63]])
    flag = dev(np.array([1], np.int32))
    bd.check(bd.capi().b2_embed(out.data_ptr(), dev(table).data_ptr(), toks.data_ptr(), flag.data_ptr(),
                                dev(staged).data_ptr(), 1, H, stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy()[0], staged[0])
