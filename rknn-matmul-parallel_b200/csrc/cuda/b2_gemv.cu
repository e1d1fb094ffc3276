// Weight-only GEMV / skinny GEMM for the decode path (b2_gemv).
//
// Semantics follow the reference matmul (run_persistent_matmul,
// src/matmul_decoder.c:382-445): the FP32 activation row is rounded to FP16,
// products with FP16 / int8 / int4 weights accumulate in FP32, and the FP32
// per-column scale multiplies the sum.  The RMSNorm that precedes q/k/v and
// gate/up in the reference (src/cpu_ops.c:18-55) is recomputed in each CTA's
// prologue, and the residual add (vec_add_f32) or SiLU*mul (silu_mul_f32)
// that follows is the epilogue, so each reference matmul + CPU op pair is one
// kernel.
//
// Layout: weights are stored one row per output column with K contiguous,
// so a warp streams a row with coalesced 16-byte loads that bypass L1.  Each
// warp owns R rows (R = 1, 2, 4 by weight width so that every warp keeps
// 32-64 bytes per lane in flight); the CTA's 8 warps share the FP16
// activation rows staged in shared memory.
#include "b2_common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <int WT>
struct WTraits;
template <>
struct WTraits<B2_W_F16> {
    static constexpr int kElems = 8;   // elements per 16-byte chunk
    static constexpr int kRows = 1;    // weight rows per warp
};
template <>
struct WTraits<B2_W_I8> {
    static constexpr int kElems = 16;
    static constexpr int kRows = 2;
};
template <>
struct WTraits<B2_W_I4> {
    static constexpr int kElems = 32;
    static constexpr int kRows = 4;
};

// acc += sum over 8 staged activations x[0..8) times w[8].
__device__ __forceinline__ float dot8(const float4 x0, const float4 x1, const float (&w)[8], float acc) {
    acc = fmaf(x0.x, w[0], acc);
    acc = fmaf(x0.y, w[1], acc);
    acc = fmaf(x0.z, w[2], acc);
    acc = fmaf(x0.w, w[3], acc);
    acc = fmaf(x1.x, w[4], acc);
    acc = fmaf(x1.y, w[5], acc);
    acc = fmaf(x1.z, w[6], acc);
    acc = fmaf(x1.w, w[7], acc);
    return acc;
}

template <int WT, int MR, bool PAIR>
__global__ void __launch_bounds__(kThreads) gemv_kernel(B2GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    // [MR][K] activations, FP16-rounded, held as FP32 times x_scale<WT>()
    float* xs = reinterpret_cast<float*>(smem);
    __shared__ float red[kWarps][MR];
    const int K = a.K;
    const int m0 = blockIdx.y * MR;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int R = WTraits<WT>::kRows;
    const size_t row_bytes = WT == B2_W_F16 ? (size_t)K * 2 : WT == B2_W_I8 ? (size_t)K : (size_t)K / 2;

    // The weight rows of this CTA do not depend on the previous kernel: start
    // pulling them into L2 before waiting for it.
    if (tid == 0 && blockIdx.y == 0) {
        const int n0 = blockIdx.x * kWarps * R;
        const int n1 = min(a.N, n0 + kWarps * R);
        if (n0 < n1) {
            const unsigned char* wb = reinterpret_cast<const unsigned char*>(a.w);
            b2::prefetch_l2(wb + (size_t)n0 * row_bytes, (uint32_t)((n1 - n0) * row_bytes));
            if (PAIR) b2::prefetch_l2(wb + (size_t)(n0 + a.N) * row_bytes, (uint32_t)((n1 - n0) * row_bytes));
        }
    }
    b2::pdl_trigger();
    b2::pdl_wait();

    // ── prologue: activation rows -> (optional RMSNorm) -> FP16 rounding -> smem ──
    float rms[MR];
    if (a.norm_w) {
        float ss[MR];
#pragma unroll
        for (int r = 0; r < MR; r++) {
            ss[r] = 0.f;
            if (m0 + r < a.M) {
                const float* xr = a.x + (size_t)(m0 + r) * a.ldx;
                for (int k = tid; k < K; k += kThreads) ss[r] = fmaf(xr[k], xr[k], ss[r]);
            }
            ss[r] = b2::warp_sum(ss[r]);
            if (lane == 0) red[warp][r] = ss[r];
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < MR; r++) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; w++) t += red[w][r];
            rms[r] = 1.0f / sqrtf(t / (float)K + a.eps);
        }
    }
#pragma unroll
    for (int r = 0; r < MR; r++) {
        const bool live = m0 + r < a.M;
        const float* xr = a.x + (size_t)(m0 + r) * a.ldx;
        for (int k = tid; k < K; k += kThreads) {
            float v = live ? xr[k] : 0.f;
            if (a.norm_w) v = (v * rms[r]) * a.norm_w[k];
            xs[r * K + k] = __half2float(__float2half_rn(v)) * b2::x_scale<WT>();
        }
    }
    __syncthreads();

    // ── main loop: each warp streams R weight rows (2R for the gate/up pair) ──
    constexpr int RR = PAIR ? 2 * R : R;
    constexpr int E = WTraits<WT>::kElems;
    constexpr int U = RR >= 8 ? 1 : 8 / RR;  // chunks per lane in flight per row
    const int n_base = (blockIdx.x * kWarps + warp) * R;
    if (n_base >= a.N) return;
    const int nchunks = (int)(row_bytes / 16);
    const unsigned char* wrow[RR];
    bool rlive[RR];
#pragma unroll
    for (int j = 0; j < RR; j++) {
        int n = n_base + (j % R);
        rlive[j] = n < a.N;
        int row = (PAIR && j >= R) ? n + a.N : n;
        wrow[j] = reinterpret_cast<const unsigned char*>(a.w) + (size_t)(rlive[j] ? row : 0) * row_bytes;
    }
    float acc[RR][MR];
#pragma unroll
    for (int j = 0; j < RR; j++)
#pragma unroll
        for (int r = 0; r < MR; r++) acc[j][r] = 0.f;

    for (int c0 = lane; c0 < nchunks; c0 += 32 * U) {
        uint4 wv[RR][U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            int c = c0 + 32 * u;
#pragma unroll
            for (int j = 0; j < RR; j++)
                if (c < nchunks && rlive[j]) wv[j][u] = b2::ld_stream16(wrow[j] + (size_t)c * 16);
                else wv[j][u] = make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            int c = c0 + 32 * u;
            if (c >= nchunks) break;
#pragma unroll
            for (int g = 0; g < E / 8; g++) {
                float w[RR][8];
#pragma unroll
                for (int j = 0; j < RR; j++) b2::expand8_exact<WT>(wv[j][u], g, w[j]);
#pragma unroll
                for (int r = 0; r < MR; r++) {
                    const float4* xp = reinterpret_cast<const float4*>(xs + r * K + c * E + g * 8);
                    const float4 x0 = xp[0], x1 = xp[1];
#pragma unroll
                    for (int j = 0; j < RR; j++) acc[j][r] = dot8(x0, x1, w[j], acc[j][r]);
                }
            }
        }
    }

    // ── epilogue ──
#pragma unroll
    for (int j = 0; j < RR; j++)
#pragma unroll
        for (int r = 0; r < MR; r++) acc[j][r] = b2::warp_sum(acc[j][r]);

#pragma unroll
    for (int j = 0; j < R; j++) {
        const int n = n_base + j;
        if (n >= a.N) break;
#pragma unroll
        for (int r = 0; r < MR; r++) {
            if (lane != r || m0 + r >= a.M) continue;
            float* yp = a.y + (size_t)(m0 + r) * a.ldy + n;
            float v = acc[j][r];
            if (a.scales) v = v * a.scales[n];
            if constexpr (PAIR) {
                float u = acc[R + j][r];
                if (a.scales) u = u * a.scales[a.N + n];
                float sig = 1.0f / (1.0f + expf(-v));
                *yp = (v * sig) * u;
            } else {
                if (a.epilogue == B2_EPI_ADD) *yp = *yp + v;
                else *yp = v;
            }
        }
    }
}

template <int WT, int MR, bool PAIR>
int launch(const B2GemvArgs* a, cudaStream_t s) {
    constexpr int R = WTraits<WT>::kRows;
    dim3 grid((a->N + kWarps * R - 1) / (kWarps * R), (a->M + MR - 1) / MR);
    size_t smem = (size_t)MR * a->K * sizeof(float);
    auto fn = gemv_kernel<WT, MR, PAIR>;
    if (smem + 2048 > 48 * 1024) {  // static shared memory counts against the same limit
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "gemv smem attr: %s", cudaGetErrorString(e));
    }
    cudaError_t e = b2::launch_pdl(fn, grid, dim3(kThreads), smem, s, *a);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_gemv launch: %s", cudaGetErrorString(e));
    return 0;
}

template <int WT, bool PAIR>
int dispatch_mr(const B2GemvArgs* a, cudaStream_t s) {
    if (a->M <= 1) return launch<WT, 1, PAIR>(a, s);
    if (a->M <= 2) return launch<WT, 2, PAIR>(a, s);
    if (a->M <= 4) return launch<WT, 4, PAIR>(a, s);
    return launch<WT, 8, PAIR>(a, s);
}

template <int WT>
int dispatch_pair(const B2GemvArgs* a, cudaStream_t s) {
    if (a->epilogue == B2_EPI_SILU_PAIR) return dispatch_mr<WT, true>(a, s);
    return dispatch_mr<WT, false>(a, s);
}

}  // namespace

extern "C" int b2_gemv(const B2GemvArgs* a, b2_stream_t stream) {
    if (!a || !a->y || !a->x || !a->w || a->M < 0 || a->K <= 0 || a->N <= 0)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemv: bad arguments");
    if (a->M == 0) return 0;
    const int need = a->wtype == B2_W_F16 ? 8 : a->wtype == B2_W_I8 ? 16 : 32;
    if (a->K % need != 0 || a->K > 6144)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemv: K=%d must be a multiple of %d and <= 6144",
                            a->K, need);
    if ((reinterpret_cast<uintptr_t>(a->w) & 15) != 0)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemv: weight pointer not 16-byte aligned");
    if (a->wtype != B2_W_F16 && !a->scales)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemv: quantized weights need scales");
    cudaStream_t s = (cudaStream_t)stream;
    switch (a->wtype) {
        case B2_W_F16: return dispatch_pair<B2_W_F16>(a, s);
        case B2_W_I8: return dispatch_pair<B2_W_I8>(a, s);
        case B2_W_I4: return dispatch_pair<B2_W_I4>(a, s);
        default: return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemv: unsupported wtype %d", a->wtype);
    }
}
