// Shared device helpers for the sm_100a kernels of the decoder runtime.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "b2_kernels.h"

#define B2_ERR_INVALID_ARG (-1)
#define B2_ERR_CUDA (-4)

// Records an error message for b2_last_error(); defined in b2_runtime.cu.
int b2_set_error(int code, const char* fmt, ...);
int b2_check_launch(const char* what);
// 2-D FP16 tensor map (CUtensorMap, 64 bytes) over [outer][inner] rows
// row_bytes apart, boxes of box_outer x box_inner elements with the 128-byte
// swizzle; defined in b2_gemm.cu.
int b2_tensor_map_f16(void* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                      uint32_t box_inner, uint32_t box_outer);

#define B2_TRY(expr)                                                                   \
    do {                                                                               \
        cudaError_t e__ = (expr);                                                      \
        if (e__ != cudaSuccess)                                                        \
            return b2_set_error(B2_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e__)); \
    } while (0)

namespace b2 {

// Launch with programmatic dependent launch (PDL) enabled: the kernel may
// start while the previous kernel on the stream is still running.  Every
// kernel launched this way calls pdl_wait() before it reads anything an
// earlier kernel of the same step writes, and before its first global store;
// only reads of data written by earlier steps (weights, older KV positions)
// and L2 prefetches may come before it.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Wait until the preceding kernel of the stream has completed and its
// writes are visible (no-op when launched without a programmatic edge).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next kernel of the stream to be scheduled.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk prefetch of [p, p + bytes) into L2; p and bytes multiples of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 16-byte global load that does not allocate in L1 (weights are
// read exactly once per step).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
}

// ── Exact weight expansion with integer/logic instructions only ──
// The GEMV inner loops are issue-bound on type conversions, so weights are
// widened to FP32 by bit manipulation instead.  All three forms are exact.
//
// F16 (exponent rebias by multiplication, F. Giesen, "Half to float done
// quic", 2012): moving a half's exponent+mantissa up 13 bits and keeping its
// sign gives an FP32 whose value is the half's times 2^-112 (subnormal halves
// become FP32 denormals, also exact).  The 2^112 is folded into the staged
// activation instead (kF16XScale), so a dot product needs no multiply here.
// Finite halves only (weights are finite).
constexpr float kF16XScale = 0x1p112f;
__device__ __forceinline__ float f16lo_scaled(uint32_t u) {
    return __uint_as_float(((u << 13) & 0x0FFFE000u) | ((u << 16) & 0x80000000u));
}
__device__ __forceinline__ float f16hi_scaled(uint32_t u) {
    return __uint_as_float(((u >> 3) & 0x0FFFE000u) | (u & 0x80000000u));
}

// INT8 / INT4 (the "magic number" method): an unsigned integer n < 2^23
// placed in the mantissa of 2^23 (bits 0x4B000000 | n) reads as 2^23 + n,
// and one FP32 subtraction removes the bias exactly.  Signed values are made
// unsigned by flipping the top bit of each field (s + 128, s + 8).
__device__ __forceinline__ uint32_t i8x4_bias(uint32_t w) { return w ^ 0x80808080u; }
template <int I>
__device__ __forceinline__ float i8_from_biased(uint32_t u) {
    return __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u | I)) - 8388736.0f;  // 2^23 + 128
}
__device__ __forceinline__ uint32_t i4x8_bias(uint32_t w) { return w ^ 0x88888888u; }
template <int I>
__device__ __forceinline__ float i4_from_biased(uint32_t u) {
    return __uint_as_float(((u >> (4 * I)) & 0xFu) | 0x4B000000u) - 8388616.0f;  // 2^23 + 8
}

// Eight consecutive weights of one 16-byte chunk (group g of 8) as FP32.
// F16 values come out scaled by 2^-112 (pair them with kF16XScale).
template <int WT>
__device__ __forceinline__ void expand8_exact(const uint4 wv, int g, float (&w)[8]) {
    const uint32_t* u = &wv.x;
    if constexpr (WT == B2_W_F16) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = f16lo_scaled(u[i]);
            w[2 * i + 1] = f16hi_scaled(u[i]);
        }
    } else if constexpr (WT == B2_W_I8) {
        const uint32_t a = i8x4_bias(u[2 * g]), b = i8x4_bias(u[2 * g + 1]);
        w[0] = i8_from_biased<0>(a);
        w[1] = i8_from_biased<1>(a);
        w[2] = i8_from_biased<2>(a);
        w[3] = i8_from_biased<3>(a);
        w[4] = i8_from_biased<0>(b);
        w[5] = i8_from_biased<1>(b);
        w[6] = i8_from_biased<2>(b);
        w[7] = i8_from_biased<3>(b);
    } else {  // int4: word g holds 8 nibbles, element i at bits [4i, 4i+4)
        const uint32_t a = i4x8_bias(u[g]);
        w[0] = i4_from_biased<0>(a);
        w[1] = i4_from_biased<1>(a);
        w[2] = i4_from_biased<2>(a);
        w[3] = i4_from_biased<3>(a);
        w[4] = i4_from_biased<4>(a);
        w[5] = i4_from_biased<5>(a);
        w[6] = i4_from_biased<6>(a);
        w[7] = i4_from_biased<7>(a);
    }
}

// Activation scale that pairs with expand8_exact<WT>.
template <int WT>
__host__ __device__ constexpr float x_scale() {
    return WT == B2_W_F16 ? kF16XScale : 1.0f;
}

// Orderable encoding of a float: a larger float maps to a larger unsigned.
// NaN maps to 0, below every number: the reference argmax's strict '>' scan
// never moves to a NaN after its first element (src/cpu_ops.c:575-586).
// (It differs only when element 0 itself is NaN: the scan then returns 0.)
__device__ __forceinline__ uint32_t float_order(float f) {
    uint32_t u = __float_as_uint(f);
    if (f != f) return 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (value, index) packed so that max() picks the largest value and, among
// equal values, the smallest index — the reference argmax's strict '>'
// scan keeps the first maximum (src/cpu_ops.c:575-586).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)float_order(v) << 32) | (0xFFFFFFFFu - idx);
}

__device__ __forceinline__ uint32_t key_index(unsigned long long k) {
    return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

}  // namespace b2
