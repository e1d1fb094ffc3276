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

// Orderable encoding of a float: a larger float maps to a larger unsigned.
__device__ __forceinline__ uint32_t float_order(float f) {
    uint32_t u = __float_as_uint(f);
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
