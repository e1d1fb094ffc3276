// Embedding gather and the q/k post-processing of the decode/prefill step.
//
// b2_qk_rope_kv fuses what the reference does on the CPU between the q/k/v
// matmuls and attention (src/matmul_decoder.c:1495-1516): per-head RMSNorm of
// q and k with the shared q_norm/k_norm weights, RoPE (apply_rope_f32,
// src/cpu_ops.c:109-155, both pairings) with the host-computed cos/sin tables
// (precompute_rope_tables, src/matmul_decoder.c:620-631), and the store of k
// and v into the KV cache.  One warp owns one head of one row.
#include "b2_common.cuh"

namespace {

__global__ void embed_kernel(float* hidden, const float* table, const int* tokens,
                             const int* use_staged, const float* staged, int dim) {
    b2::pdl_trigger();
    b2::pdl_wait();
    const int m = blockIdx.x;
    const bool st = use_staged && *use_staged;
    const float* src = st ? staged + (size_t)m * dim : table + (size_t)tokens[m] * dim;
    float* dst = hidden + (size_t)m * dim;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) dst[k] = src[k];
}

template <int EPL>  // elements per lane = head_dim / 32
__global__ void __launch_bounds__(128) qk_rope_kv_kernel(
    float* qkv, int ldqkv, int nq, int nkv, const float* q_norm_w, const float* k_norm_w,
    float eps, const float* cos_tab, const float* sin_tab, int rope_style, B2KVRef kv) {
    constexpr int HD = EPL * 32;
    constexpr int HALF = HD / 2;
    b2::pdl_trigger();
    b2::pdl_wait();
    const int m = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
    if (h >= nq + 2 * nkv) return;
    const int pos = kv.pos[m];
    const int seq = kv.rows_seq ? kv.rows_seq[m] : 0;
    if (pos < 0 || pos >= kv.max_seq || seq < 0 || seq >= kv.n_seqs) return;  // invalid row: no access
    float* xp = qkv + (size_t)m * ldqkv + (size_t)h * HD + lane * EPL;
    float x[EPL];
#pragma unroll
    for (int j = 0; j < EPL; j++) x[j] = xp[j];

    const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
    if (is_q || is_k) {
        const float* nw = is_q ? q_norm_w : k_norm_w;
        if (nw) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < EPL; j++) ss = fmaf(x[j], x[j], ss);
            ss = b2::warp_sum(ss);
            const float rms = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
            for (int j = 0; j < EPL; j++) x[j] = (x[j] * rms) * nw[lane * EPL + j];
        }
        const float* c = cos_tab + (size_t)pos * HALF;
        const float* sn = sin_tab + (size_t)pos * HALF;
        if (rope_style == 0) {
#pragma unroll
            for (int j = 0; j < EPL; j += 2) {
                const int i = (lane * EPL + j) >> 1;
                const float x0 = x[j], x1 = x[j + 1];
                x[j] = x0 * c[i] - x1 * sn[i];
                x[j + 1] = x1 * c[i] + x0 * sn[i];
            }
        } else {
#pragma unroll
            for (int j = 0; j < EPL; j++) {
                const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
                const int e = lane * EPL + j;
                if (lane < 16) {
                    x[j] = x[j] * c[e] - other * sn[e];
                } else {
                    const int i = e - HALF;
                    x[j] = x[j] * c[i] + other * sn[i];
                }
            }
        }
    }
    if (is_q) {
#pragma unroll
        for (int j = 0; j < EPL; j++) xp[j] = x[j];
        return;
    }
    const int g = is_k ? h - nq : h - nq - nkv;
    uint16_t* base = is_k ? kv.k_base : kv.v_base;
    __half* dst = reinterpret_cast<__half*>(base + seq * kv.seq_stride + kv.layer * kv.layer_stride +
                                            ((size_t)g * kv.max_seq + pos) * HD) + lane * EPL;
#pragma unroll
    for (int j = 0; j < EPL; j++) dst[j] = __float2half_rn(x[j]);
}

__global__ void loop_advance_kernel(int* loop, int* hist, int hist_len) {
    b2::pdl_wait();
    const int step = loop[2];
    if (step < hist_len) hist[step] = loop[0];
    loop[1] += 1;
    loop[2] = step + 1;
}

}  // namespace

extern "C" int b2_loop_advance(int* loop, int* hist, int hist_len, b2_stream_t s) {
    if (!loop || !hist) return b2_set_error(B2_ERR_INVALID_ARG, "b2_loop_advance: null pointer");
    cudaError_t e = b2::launch_pdl(loop_advance_kernel, dim3(1), dim3(1), 0, (cudaStream_t)s, loop, hist, hist_len);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_loop_advance: %s", cudaGetErrorString(e));
    return 0;
}

extern "C" int b2_embed(float* hidden, const float* table, const int* tokens, const int* use_staged,
                        const float* staged, int M, int dim, b2_stream_t s) {
    if (M <= 0) return 0;
    if (!hidden || (!table && !staged)) return b2_set_error(B2_ERR_INVALID_ARG, "b2_embed: null pointer");
    cudaError_t e = b2::launch_pdl(embed_kernel, dim3(M), dim3(256), 0, (cudaStream_t)s, hidden, table, tokens,
                                   use_staged, staged, dim);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_embed: %s", cudaGetErrorString(e));
    return 0;
}

extern "C" int b2_qk_rope_kv(float* qkv, int ldqkv, int M, int nq, int nkv, int hd,
                             const float* q_norm_w, const float* k_norm_w, float eps,
                             const float* cos_tab, const float* sin_tab, int rope_style,
                             const B2KVRef* kv, b2_stream_t s) {
    if (M <= 0) return 0;
    if (!qkv || !kv || !kv->pos || !cos_tab || !sin_tab)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_qk_rope_kv: null pointer");
    dim3 grid(M, (nq + 2 * nkv + 3) / 4);
    cudaStream_t st = (cudaStream_t)s;
    cudaError_t e = cudaSuccess;
    switch (hd) {
        case 64:
            e = b2::launch_pdl(qk_rope_kv_kernel<2>, grid, dim3(128), 0, st, qkv, ldqkv, nq, nkv, q_norm_w,
                               k_norm_w, eps, cos_tab, sin_tab, rope_style, *kv);
            break;
        case 128:
            e = b2::launch_pdl(qk_rope_kv_kernel<4>, grid, dim3(128), 0, st, qkv, ldqkv, nq, nkv, q_norm_w,
                               k_norm_w, eps, cos_tab, sin_tab, rope_style, *kv);
            break;
        case 256:
            e = b2::launch_pdl(qk_rope_kv_kernel<8>, grid, dim3(128), 0, st, qkv, ldqkv, nq, nkv, q_norm_w,
                               k_norm_w, eps, cos_tab, sin_tab, rope_style, *kv);
            break;
        default:
            return b2_set_error(B2_ERR_INVALID_ARG, "b2_qk_rope_kv: head_dim %d not in {64,128,256}", hd);
    }
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_qk_rope_kv: %s", cudaGetErrorString(e));
    return 0;
}
