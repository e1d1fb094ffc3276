// Final RMSNorm + lm_head GEMV + greedy argmax (b2_lm_head_argmax).
//
// Replaces the tail of matmul_decoder_step (src/matmul_decoder.c:1563-1633):
// final rms_norm_f32, then either the tiled INT8 NPU lm_head (FP16-rounded
// input, FP32 accumulation, per-vocab-column FP32 scale; :1569-1605), the FP16
// CPU GEMV with FP32 input (gemv_f16_neon, :572-616, disable_npu_lm_head) or the
// FP32 GEMV of step_head (gemv_f32_neon, :511-566), and argmax_f32
// (src/cpu_ops.c:575-586).  The argmax is fused: every CTA reduces its rows to
// one packed (value, index) key, a second tiny kernel reduces the keys per
// row, and only the token id has to leave the device.  Logits are stored only
// when the caller asks for them.
//
// Table layout: one row per vocab entry, K contiguous (int8 rows are 1 KB at
// K = 1024), streamed with 16-byte no-L1-allocate loads.
#include "b2_common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <int WT>
struct LmTraits;
template <>
struct LmTraits<B2_W_I8> {
    static constexpr int kElems = 16;
    static constexpr int kRows = 4;
};
template <>
struct LmTraits<B2_W_F16> {
    static constexpr int kElems = 8;
    static constexpr int kRows = 2;
};
template <>
struct LmTraits<B2_W_F32> {
    static constexpr int kElems = 4;
    static constexpr int kRows = 1;
};

template <int WT, int MR>
__global__ void __launch_bounds__(kThreads) lm_head_kernel(const float* __restrict__ x, int ldx, int M,
                                                           int K, int V, const void* __restrict__ table,
                                                           const float* __restrict__ scales,
                                                           const float* __restrict__ norm_w, float eps,
                                                           float* __restrict__ logits, int ldl,
                                                           unsigned long long* __restrict__ part) {
    extern __shared__ __align__(16) float xs[];  // [MR][K] FP32 (FP16-rounded values for int8)
    __shared__ float red[kWarps][MR];
    __shared__ unsigned long long best_sm[kWarps][MR];
    const int m0 = blockIdx.y * MR;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        constexpr int RPC = kWarps * LmTraits<WT>::kRows;
        const size_t rb = (size_t)K * (WT == B2_W_I8 ? 1 : WT == B2_W_F16 ? 2 : 4);
        const int v0 = blockIdx.x * RPC, v1 = min(V, v0 + RPC);
        if (tid == 0 && blockIdx.y == 0 && v0 < v1)
            b2::prefetch_l2(reinterpret_cast<const unsigned char*>(table) + (size_t)v0 * rb, (uint32_t)((v1 - v0) * rb));
    }
    b2::pdl_trigger();
    b2::pdl_wait();

    float rms[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) rms[r] = 1.f;
    if (norm_w) {
#pragma unroll
        for (int r = 0; r < MR; r++) {
            float ss = 0.f;
            if (m0 + r < M)
                for (int k = tid; k < K; k += kThreads) {
                    float v = x[(size_t)(m0 + r) * ldx + k];
                    ss = fmaf(v, v, ss);
                }
            ss = b2::warp_sum(ss);
            if (lane == 0) red[warp][r] = ss;
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < MR; r++) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; w++) t += red[w][r];
            rms[r] = 1.0f / sqrtf(t / (float)K + eps);
        }
    }
#pragma unroll
    for (int r = 0; r < MR; r++)
        for (int k = tid; k < K; k += kThreads) {
            float v = m0 + r < M ? x[(size_t)(m0 + r) * ldx + k] : 0.f;
            if (norm_w) v = (v * rms[r]) * norm_w[k];
            if (WT == B2_W_I8) v = __half2float(__float2half_rn(v));
            xs[r * K + k] = v;
        }
    __syncthreads();

    constexpr int R = LmTraits<WT>::kRows;
    constexpr int E = LmTraits<WT>::kElems;
    constexpr int U = 8 / R;
    const int esz = WT == B2_W_I8 ? 1 : WT == B2_W_F16 ? 2 : 4;
    const size_t row_bytes = (size_t)K * esz;
    const int nchunks = (int)(row_bytes / 16);
    const int v_base = (blockIdx.x * kWarps + warp) * R;

    unsigned long long best[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) best[r] = 0ull;

    float acc[R][MR];
#pragma unroll
    for (int j = 0; j < R; j++)
#pragma unroll
        for (int r = 0; r < MR; r++) acc[j][r] = 0.f;
    for (int c0 = lane; c0 < nchunks; c0 += 32 * U) {
        uint4 wv[R][U];
#pragma unroll
        for (int u = 0; u < U; u++)
#pragma unroll
            for (int j = 0; j < R; j++) {
                const int c = c0 + 32 * u, v = v_base + j;
                wv[j][u] = (c < nchunks && v < V)
                               ? b2::ld_stream16(reinterpret_cast<const unsigned char*>(table) +
                                                 (size_t)v * row_bytes + (size_t)c * 16)
                               : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = c0 + 32 * u;
            if (c >= nchunks) break;
#pragma unroll
            for (int j = 0; j < R; j++) {
                float w[E];
                const uint32_t* wu = &wv[j][u].x;
                if constexpr (WT == B2_W_I8) {
                    b2::expand8_exact<B2_W_I8>(wv[j][u], 0, *reinterpret_cast<float(*)[8]>(w));
                    b2::expand8_exact<B2_W_I8>(wv[j][u], 1, *reinterpret_cast<float(*)[8]>(w + 8));
                } else if constexpr (WT == B2_W_F16) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        float2 f = b2::h2_to_f2(wu[i]);
                        w[2 * i] = f.x;
                        w[2 * i + 1] = f.y;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) w[i] = __uint_as_float(wu[i]);
                }
#pragma unroll
                for (int r = 0; r < MR; r++) {
                    const float4* xp = reinterpret_cast<const float4*>(xs + r * K + c * E);
                    float a = acc[j][r];
#pragma unroll
                    for (int i = 0; i < E / 4; i++) {
                        float4 xv = xp[i];
                        a = fmaf(xv.x, w[4 * i], a);
                        a = fmaf(xv.y, w[4 * i + 1], a);
                        a = fmaf(xv.z, w[4 * i + 2], a);
                        a = fmaf(xv.w, w[4 * i + 3], a);
                    }
                    acc[j][r] = a;
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < R; j++) {
        const int v = v_base + j;
#pragma unroll
        for (int r = 0; r < MR; r++) {
            float t = b2::warp_sum(acc[j][r]);
            if (v < V && m0 + r < M) {
                if (WT == B2_W_I8) t = t * scales[v];
                if (logits && lane == r) logits[(size_t)(m0 + r) * ldl + v] = t;
                unsigned long long k = b2::argmax_key(t, (uint32_t)v);
                best[r] = k > best[r] ? k : best[r];
            }
        }
    }
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < MR; r++) best_sm[warp][r] = best[r];
    __syncthreads();
    if (tid < MR && m0 + tid < M) {
        unsigned long long b = 0ull;
#pragma unroll
        for (int w = 0; w < kWarps; w++) b = best_sm[w][tid] > b ? best_sm[w][tid] : b;
        part[(size_t)(m0 + tid) * gridDim.x + blockIdx.x] = b;
    }
}

__global__ void argmax_final_kernel(const unsigned long long* __restrict__ part, int nblocks,
                                    int* __restrict__ tokens) {
    __shared__ unsigned long long sm[32];
    b2::pdl_trigger();
    b2::pdl_wait();
    const int m = blockIdx.x;
    unsigned long long b = 0ull;
    for (int i = threadIdx.x; i < nblocks; i += blockDim.x) {
        unsigned long long k = part[(size_t)m * nblocks + i];
        b = k > b ? k : b;
    }
    b = b2::warp_max_u64(b);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = b;
    __syncthreads();
    if (threadIdx.x < 32) {
        b = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0ull;
        b = b2::warp_max_u64(b);
        if (threadIdx.x == 0) tokens[m] = (int)b2::key_index(b);
    }
}

int rows_per_cta(int wtype) {
    return kWarps * (wtype == B2_W_I8 ? 4 : wtype == B2_W_F16 ? 2 : 1);
}

template <int WT, int MR>
int launch(const float* x, int ldx, int M, int K, int V, const void* table, const float* scales,
           const float* norm_w, float eps, float* logits, int ldl, unsigned long long* part,
           cudaStream_t s) {
    const int nb = (V + rows_per_cta(WT) - 1) / rows_per_cta(WT);
    size_t smem = (size_t)MR * K * sizeof(float);
    auto fn = lm_head_kernel<WT, MR>;
    if (smem + 2048 > 48 * 1024) {  // static shared memory counts against the same limit
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "lm_head smem attr: %s", cudaGetErrorString(e));
    }
    cudaError_t e = b2::launch_pdl(fn, dim3(nb, (M + MR - 1) / MR), dim3(kThreads), smem, s, x, ldx, M, K, V, table,
                                   scales, norm_w, eps, logits, ldl, part);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_lm_head: %s", cudaGetErrorString(e));
    return 0;
}

template <int WT>
int dispatch(const float* x, int ldx, int M, int K, int V, const void* table, const float* scales,
             const float* norm_w, float eps, float* logits, int ldl, unsigned long long* part,
             cudaStream_t s) {
    if (M <= 1) return launch<WT, 1>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s);
    if (M <= 2) return launch<WT, 2>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s);
    if (M <= 4) return launch<WT, 4>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s);
    return launch<WT, 8>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s);
}

}  // namespace

extern "C" size_t b2_lm_head_workspace(int M, int V) {
    const int nb = (V + rows_per_cta(B2_W_F32) - 1) / rows_per_cta(B2_W_F32);  // largest grid
    return (size_t)M * nb * sizeof(unsigned long long) + 256;
}

extern "C" int b2_lm_head_argmax(const float* x, int ldx, int M, int K, int V, const void* table,
                                 const float* scales, int wtype, const float* norm_w, float eps,
                                 float* logits, int ldl, int* tokens, void* work, b2_stream_t stream) {
    if (M <= 0) return 0;
    if (!x || !table || !tokens || !work || K <= 0 || V <= 0 || K % 16 != 0 || K > 8192)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax: bad arguments (K=%d V=%d)", K, V);
    if (wtype == B2_W_I8 && !scales) return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax: int8 needs scales");
    cudaStream_t s = (cudaStream_t)stream;
    auto* part = reinterpret_cast<unsigned long long*>(work);
    int rc;
    switch (wtype) {
        case B2_W_I8: rc = dispatch<B2_W_I8>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
        case B2_W_F16: rc = dispatch<B2_W_F16>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
        case B2_W_F32: rc = dispatch<B2_W_F32>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
        default: return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax: wtype %d", wtype);
    }
    if (rc) return rc;
    const int nb = (V + rows_per_cta(wtype) - 1) / rows_per_cta(wtype);
    cudaError_t e = b2::launch_pdl(argmax_final_kernel, dim3(M), dim3(256), 0, s, (const unsigned long long*)part, nb,
                                   tokens);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_argmax_final: %s", cudaGetErrorString(e));
    return 0;
}

// ─── the same lm_head + argmax for callers that cannot allocate ───
//
// Callers embedded in a host that owns all device memory (a serving runtime
// that pre-reserves HBM in its own pool) or that enqueue work while another
// framework is capturing the stream into a CUDA graph cannot call cudaMalloc
// for a workspace: cudaMalloc is not capturable, it can synchronize the
// device, and the pool may leave nothing outside its arena.  This entry point
// keeps the per-CTA argmax keys in a file-scope device array instead.
#include <mutex>

namespace {

constexpr size_t kNoAllocKeys = (size_t)1 << 17;  // 131072 keys = 1 MiB per device
static __device__ __align__(256) unsigned long long g_lm_noalloc_keys[kNoAllocKeys];

constexpr int kMaxDevices = 64;
unsigned long long* g_noalloc_addr[kMaxDevices];
std::mutex g_noalloc_mu;

// Device address of g_lm_noalloc_keys on the current device.  In host code the
// symbol name is only a host-side handle: the address must come from
// cudaGetSymbolAddress, once per device, with that device current.
int noalloc_keys(unsigned long long** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return b2_set_error(B2_ERR_INVALID_ARG, "noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_lm_noalloc_keys);
        if (e != cudaSuccess)
            return b2_set_error(B2_ERR_CUDA, "noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_noalloc_addr[dev] = static_cast<unsigned long long*>(p);
    }
    *out = g_noalloc_addr[dev];
    return 0;
}

}  // namespace

extern "C" size_t b2_lm_head_noalloc_max_keys(void) { return kNoAllocKeys; }

extern "C" int b2_lm_head_argmax_noalloc(const float* x, int ldx, int M, int K, int V, const void* table,
                                         const float* scales, int wtype, const float* norm_w, float eps,
                                         float* logits, int ldl, int* tokens, b2_stream_t stream) {
    if (M <= 0) return 0;
    if (!x || !table || !tokens || K <= 0 || V <= 0 || K % 16 != 0 || K > 8192)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax_noalloc: bad arguments (K=%d V=%d)", K, V);
    if (wtype != B2_W_I8 && wtype != B2_W_F16 && wtype != B2_W_F32)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax_noalloc: wtype %d", wtype);
    if (wtype == B2_W_I8 && !scales)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_lm_head_argmax_noalloc: int8 needs scales");
    const int nb = (V + rows_per_cta(wtype) - 1) / rows_per_cta(wtype);
    if ((size_t)M * (size_t)nb > kNoAllocKeys)
        return b2_set_error(B2_ERR_INVALID_ARG,
                            "b2_lm_head_argmax_noalloc: M=%d x %d CTA keys exceeds the fixed scratch of %zu keys "
                            "(1 MiB); use b2_lm_head_argmax with a workspace",
                            M, nb, kNoAllocKeys);
    unsigned long long* part = nullptr;
    int rc = noalloc_keys(&part);
    if (rc) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    switch (wtype) {
        case B2_W_I8: rc = dispatch<B2_W_I8>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
        case B2_W_F16: rc = dispatch<B2_W_F16>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
        default: rc = dispatch<B2_W_F32>(x, ldx, M, K, V, table, scales, norm_w, eps, logits, ldl, part, s); break;
    }
    if (rc) return rc;
    cudaError_t e = b2::launch_pdl(argmax_final_kernel, dim3(M), dim3(256), 0, s, (const unsigned long long*)part, nb,
                                   tokens);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_argmax_final: %s", cudaGetErrorString(e));
    return 0;
}

// ─── vocab-sharded lm_head: keys across ranks ───
//
// With the vocabulary split over ranks, each rank's lm_head GEMM leaves per
// CTA keys (orderable value << 32 | ~local index) for every row.  The merge
// keeps each row's largest key and rewrites its index as a global vocab index
// (local + offset), so an all-reduce MAX over the ranks picks the largest
// logit and, among equal logits, the lowest global index: the first maximum
// of the reference argmax (src/cpu_ops.c:575-586).
namespace {

__global__ void __launch_bounds__(128) keys_merge_kernel(const unsigned long long* __restrict__ keys, int parts,
                                                         unsigned offset, unsigned long long* __restrict__ out) {
    unsigned long long k = 0ull;
    for (int i = threadIdx.x; i < parts; i += blockDim.x) {
        const unsigned long long v = keys[(size_t)blockIdx.x * parts + i];
        k = v > k ? v : k;
    }
    k = b2::warp_max_u64(k);
    __shared__ unsigned long long w[4];
    if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < 4; i++) k = w[i] > k ? w[i] : k;
        k = w[0] > k ? w[0] : k;
        const uint32_t idx = b2::key_index(k) + offset;
        out[blockIdx.x] = (k & 0xFFFFFFFF00000000ull) | (0xFFFFFFFFull - idx);
    }
}

__global__ void keys_tokens_kernel(const unsigned long long* __restrict__ keys, int n, int* __restrict__ tokens) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) tokens[i] = (int)b2::key_index(keys[i]);
}

}  // namespace

extern "C" int b2_argmax_keys_merge(const unsigned long long* keys, int M, int parts, unsigned index_offset,
                                    unsigned long long* out, b2_stream_t s) {
    if (!keys || !out || M <= 0 || parts <= 0)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_argmax_keys_merge: bad arguments");
    keys_merge_kernel<<<M, 128, 0, (cudaStream_t)s>>>(keys, parts, index_offset, out);
    return b2_check_launch("b2_argmax_keys_merge");
}

extern "C" int b2_keys_tokens(const unsigned long long* keys, int n, int* tokens, b2_stream_t s) {
    if (!keys || !tokens || n <= 0) return b2_set_error(B2_ERR_INVALID_ARG, "b2_keys_tokens: bad arguments");
    keys_tokens_kernel<<<(n + 127) / 128, 128, 0, (cudaStream_t)s>>>(keys, n, tokens);
    return b2_check_launch("b2_keys_tokens");
}
