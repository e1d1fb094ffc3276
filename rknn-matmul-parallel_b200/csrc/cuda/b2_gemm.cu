// Tensor-core GEMM for M > 1 rows (batch prefill, batched decode, batched
// lm_head): b2_gemm, b2_rows_to_f16.
//
// Same contract as b2_gemv (the reference's run_batch_matmul,
// src/matmul_decoder.c:1841-1899: FP16-rounded activations, FP16 / INT8 / INT4
// weights, FP32 accumulation, per-column scale, then the residual add or
// SiLU*mul of src/cpu_ops.c:296-319, :350-359, or the lm_head argmax of
// src/cpu_ops.c:575-586), but the sums run on the sm_100 tensor cores:
//
//   warp 0       one thread issues TMA tile loads (cp.async.bulk.tensor) of a
//                128-row weight tile and a BN-row activation tile (128-byte
//                swizzle) per 64-wide k step into a shared-memory ring;
//   warp 1       allocates the tensor-memory accumulator and one thread issues
//                tcgen05.mma (M=128, N=BN, K=16, FP16 x FP16 -> FP32),
//                committing each stage back to the loader;
//   warps 2-5    for INT8 / INT4 weights, widen each stage's raw weight tile
//                exactly to FP16 in the swizzled layout the MMA reads (the
//                integer in the mantissa of 1024 and one half2 subtraction);
//                at the end, read the accumulator with tcgen05.ld (warp w owns
//                TMEM lanes 32*(w%4)..+31) and apply the epilogue.
//
// The weight tile is the MMA's A operand (output columns are TMEM lanes) and
// the activation tile its B operand (token rows are TMEM columns), so one
// CTA computes a 128-column x BN-row block of y.  For SILU_PAIR the stage
// holds 128 gate rows and the 128 matching up rows; two MMAs per k step sum
// them into TMEM columns [0, BN) and [BN, 2 BN), so each epilogue thread
// finds the gate and up sums of its channel side by side.  For ARGMAX each
// CTA reduces its 128 vocab rows to one packed (logit, index) key per token
// and a second kernel reduces the CTAs' keys.
#include <cuda.h>  // CUtensorMap and its enums; the encoder is looked up at run time

#include <mutex>

#include "b2_common.cuh"

namespace {

constexpr int kBM = 128;     // weight rows per tile (MMA M)
constexpr int kBK = 64;      // k per stage: 64 FP16 = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr long long kWaitLimit = 1ll << 22;

enum { MODE_ROWS = 0, MODE_PAIR = 1, MODE_ARGMAX = 2 };

// bytes of one weight row's 64-wide k step as stored (FP16 128, INT8 64, INT4 32)
template <int WT>
__host__ __device__ constexpr int raw_row_bytes() {
    return WT == B2_W_F16 ? 128 : WT == B2_W_I8 ? 64 : 32;
}

// Stage layout: [FP16 A tile(s), 16 KB each][B tile, BN x 128 B][raw A tile(s)]
template <int BN, int MODE, int WT>
struct Layout {
    static constexpr int kATiles = MODE == MODE_PAIR ? 2 : 1;
    static constexpr int kA = kATiles * kBM * 128;
    static constexpr int kB = BN * 128;
    static constexpr int kRaw = WT == B2_W_F16 ? 0 : kATiles * kBM * raw_row_bytes<WT>();
    static constexpr int kStage = kA + kB + kRaw;
    static constexpr int kStages = (192 * 1024) / kStage > kMaxStages ? kMaxStages : (192 * 1024) / kStage;
    static constexpr int kCols = MODE == MODE_PAIR ? 2 * BN : BN;  // TMEM columns (a power of two >= 32)
};

struct GemmParams {
    float* y;
    int ldy;
    int M, K, N;
    const float* scales;
    int epilogue;
    unsigned long long* keys;  // ARGMAX: [M][gridDim.x] per-CTA keys
    __half* y16;               // STORE / SILU_PAIR: FP16 output (row stride ldy) instead of y
};

struct Bars {
    uint64_t full[kMaxStages];
    uint64_t conv[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t done;
    uint32_t tmem;
    int failed;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false (and the CTA's failure flag) after kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, Bars* b) {
    for (long long it = 0; !mbar_try_wait(bar, parity); it++) {
        if (it > kWaitLimit || *(volatile int*)&b->failed) {
            b->failed = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile stored as 128-byte rows
// with the 128-byte swizzle (8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4)  // start address
           | ((uint64_t)1 << 16)                // leading byte offset (fixed for swizzled K-major)
           | ((uint64_t)(1024 >> 4) << 32)      // stride byte offset: one 8-row group
           | ((uint64_t)1 << 46)                // descriptor version
           | ((uint64_t)2 << 61);               // 128-byte swizzle
}

// Instruction descriptor of kind::f16: FP16 A and B (both K-major), FP32 D.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Eight consecutive weights (k = 8c .. 8c+7 of a row) widened exactly to FP16.
template <int WT>
__device__ __forceinline__ uint4 widen8(const unsigned char* raw) {
    uint4 h;
    if constexpr (WT == B2_W_I8) {
        const uint2 w = *reinterpret_cast<const uint2*>(raw);
        const uint32_t bias = 0x64806480u;  // half2(1152): 1024 + 128
        const uint32_t a = w.x ^ 0x80808080u, b = w.y ^ 0x80808080u;
        h.x = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4140), bias);
        h.y = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4342), bias);
        h.z = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4140), bias);
        h.w = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4342), bias);
    } else {  // INT4: nibble i of the word is k = 8c + i (even k in the low nibble of its byte)
        const uint32_t u = *reinterpret_cast<const uint32_t*>(raw) ^ 0x88888888u;
        const uint32_t bias = 0x64086408u;  // half2(1032): 1024 + 8
        h.x = hsub2_u32((u & 0x0000000Fu) | ((u << 12) & 0x000F0000u) | 0x64006400u, bias);
        h.y = hsub2_u32(((u >> 8) & 0x0000000Fu) | ((u << 4) & 0x000F0000u) | 0x64006400u, bias);
        h.z = hsub2_u32(((u >> 16) & 0x0000000Fu) | ((u >> 4) & 0x000F0000u) | 0x64006400u, bias);
        h.w = hsub2_u32(((u >> 24) & 0x0000000Fu) | ((u >> 12) & 0x000F0000u) | 0x64006400u, bias);
    }
    return h;
}

template <int BN, int MODE, int WT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const GemmParams g) {
    using Lay = Layout<BN, MODE, WT>;
    constexpr bool kConvert = WT != B2_W_F16;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    Bars* b = reinterpret_cast<Bars*>(smem + Lay::kStages * Lay::kStage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BN;
    // split-K (ADD epilogue only): this CTA sums k stages [kt0, kt0 + KT)
    const int KT_all = g.K / kBK;
    const int kt0 = (int)((long long)KT_all * blockIdx.z / gridDim.z);
    const int KT = (int)((long long)KT_all * (blockIdx.z + 1) / gridDim.z) - kt0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Lay::kStages; s++) {
            mbar_init(&b->full[s], 1);
            mbar_init(&b->conv[s], 4);
            mbar_init(&b->empty[s], 1);
        }
        mbar_init(&b->done, 1);
        b->failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tw) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tx) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&b->tmem)),
                     "r"(Lay::kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = b->tmem;
    // The activation rows come from the previous kernel of the stream.
    b2::pdl_wait();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            constexpr uint32_t kTx = Lay::kB + (kConvert ? Lay::kRaw : Lay::kA);
            constexpr int kWTile = kConvert ? kBM * raw_row_bytes<WT>() : kBM * 128;
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % Lay::kStages;
                if (kt >= Lay::kStages && !mbar_wait(&b->empty[s], (uint32_t)((kt / Lay::kStages - 1) & 1), b)) break;
                unsigned char* st = smem + s * Lay::kStage;
                unsigned char* wdst = kConvert ? st + Lay::kA + Lay::kB : st;
                // x coordinate of the weight map: elements for FP16, bytes for INT8/INT4
                const int wx = (kt0 + kt) * (WT == B2_W_F16 ? kBK : raw_row_bytes<WT>());
                mbar_expect_tx(&b->full[s], kTx);
                tma_load_2d(wdst, &tw, wx, kBM * blockIdx.x, &b->full[s]);
                if (MODE == MODE_PAIR) tma_load_2d(wdst + kWTile, &tw, wx, g.N + kBM * blockIdx.x, &b->full[s]);
                tma_load_2d(st + Lay::kA, &tx, (kt0 + kt) * kBK, m0, &b->full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_f16(kBM, BN);
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % Lay::kStages;
                const uint32_t par = (uint32_t)((kt / Lay::kStages) & 1);
                if (!mbar_wait(kConvert ? &b->conv[s] : &b->full[s], par, b)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * Lay::kStage), sb = sa + Lay::kA;
#pragma unroll
                for (int k = 0; k < kBK / 16; k++) {  // K = 16 per MMA: 32 bytes along the swizzled row
                    umma_f16(tmem, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), idesc, (kt | k) != 0);
                    if (MODE == MODE_PAIR)  // up rows into the next BN columns
                        umma_f16(tmem + BN, sw128_desc(sa + kBM * 128 + 32 * k), sw128_desc(sb + 32 * k), idesc,
                                 (kt | k) != 0);
                }
                umma_commit(&b->empty[s]);
            }
            umma_commit(&b->done);
        }
    } else {  // warps 2..5
        const int et = threadIdx.x - 64;  // 0..127
        if constexpr (kConvert) {
            // raw [rows][raw_row_bytes] -> FP16 [rows][128 B] with chunk c of row r at (c ^ (r % 8)) * 16
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % Lay::kStages;
                if (!mbar_wait(&b->full[s], (uint32_t)((kt / Lay::kStages) & 1), b)) break;
                unsigned char* st = smem + s * Lay::kStage;
                const unsigned char* raw = st + Lay::kA + Lay::kB;
#pragma unroll 4
                for (int job = et; job < Lay::kATiles * kBM * 8; job += 128) {
                    const int tile = job / (kBM * 8), r = (job >> 3) % kBM, c = job & 7;
                    const uint4 h = widen8<WT>(raw + (size_t)(tile * kBM + r) * raw_row_bytes<WT>() +
                                               c * (raw_row_bytes<WT>() / 8));
                    *reinterpret_cast<uint4*>(st + tile * kBM * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                                              ((c ^ (r & 7)) << 4)) = h;
                }
                // the tensor cores read shared memory through the async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&b->conv[s]);
            }
        }
        const int quad = warp & 3;  // TMEM lanes this warp may read
        const bool ok = mbar_wait(&b->done, 0, b);
        tc_fence_after();
        const int n = kBM * blockIdx.x + 32 * quad + lane;
        if (MODE == MODE_ROWS) {
            const float sc = g.scales ? g.scales[n] : 1.f;
            const bool split = gridDim.z > 1;  // partial sums: add atomically into y
#pragma unroll 1
            for (int c0 = 0; c0 < BN && ok; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + c0, v);
                const int jn = min(16, g.M - (m0 + c0));
                if (jn <= 0) break;
                float* yp = g.y + (size_t)(m0 + c0) * g.ldy + n;
                if (split) {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < jn) atomicAdd(yp + (size_t)j * g.ldy, __uint_as_float(v[j]) * sc);
                } else if (g.epilogue == B2_EPI_ADD) {
                    float old[16];  // all loads first, then the stores
#pragma unroll
                    for (int j = 0; j < 16; j++) old[j] = j < jn ? yp[(size_t)j * g.ldy] : 0.f;
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < jn) yp[(size_t)j * g.ldy] = old[j] + __uint_as_float(v[j]) * sc;
                } else if (g.y16) {
                    __half* hp = g.y16 + (size_t)(m0 + c0) * g.ldy + n;
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < jn) hp[(size_t)j * g.ldy] = __float2half_rn(__uint_as_float(v[j]) * sc);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        if (j < jn) yp[(size_t)j * g.ldy] = __uint_as_float(v[j]) * sc;
                }
            }
        } else if (MODE == MODE_PAIR) {
            // lane = channel n: gate sum in columns [0, BN), up sum in [BN, 2 BN)
            const float sg = g.scales ? g.scales[n] : 1.f, su = g.scales ? g.scales[g.N + n] : 1.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN && ok; c0 += 16) {
                uint32_t vg[16], vu[16];
                tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + c0, vg);
                tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + BN + c0, vu);
                const int jn = min(16, g.M - (m0 + c0));
                if (jn <= 0) break;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (j >= jn) break;
                    const float gv = __uint_as_float(vg[j]) * sg, uv = __uint_as_float(vu[j]) * su;
                    const float sig = 1.0f / (1.0f + expf(-gv));
                    const size_t o = (size_t)(m0 + c0 + j) * g.ldy + n;
                    if (g.y16) g.y16[o] = __float2half_rn((gv * sig) * uv);  // the down GEMM's FP16 input
                    else g.y[o] = (gv * sig) * uv;
                }
            }
        } else {  // ARGMAX over this CTA's 128 vocab rows, per token
            unsigned long long* kq = reinterpret_cast<unsigned long long*>(smem);  // [4][BN]; the ring is idle
            const bool live = n < g.N;
            const float sc = live ? (g.scales ? g.scales[n] : 1.f) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                if (ok) tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + c0, v);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int m = m0 + c0 + j;
                    const float logit = ok ? __uint_as_float(v[j]) * sc : 0.f;
                    if (g.y && live && m < g.M) g.y[(size_t)m * g.ldy + n] = logit;
                    unsigned long long key = live ? b2::argmax_key(logit, (uint32_t)n) : 0ull;
                    key = b2::warp_max_u64(key);
                    if (lane == 0) kq[quad * BN + c0 + j] = key;
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            for (int j = et; j < BN; j += 128) {
                unsigned long long key = kq[j];
#pragma unroll
                for (int q = 1; q < 4; q++) key = kq[q * BN + j] > key ? kq[q * BN + j] : key;
                if (m0 + j < g.M) g.keys[(size_t)(m0 + j) * gridDim.x + blockIdx.x] = key;
            }
        }
    }
    b2::pdl_trigger();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Lay::kCols)
                     : "memory");
    }
}

// tokens[m] = index of the largest key of row m over its nparts CTA keys
__global__ void __launch_bounds__(256) argmax_parts_kernel(const unsigned long long* __restrict__ keys, int nparts,
                                                           int* __restrict__ tokens) {
    __shared__ unsigned long long sm[8];
    b2::pdl_wait();
    unsigned long long k = 0ull;
    for (int i = threadIdx.x; i < nparts; i += 256) {
        const unsigned long long v = keys[(size_t)blockIdx.x * nparts + i];
        k = v > k ? v : k;
    }
    k = b2::warp_max_u64(k);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 0; w < 8; w++) k = sm[w] > k ? sm[w] : k;
        tokens[blockIdx.x] = (int)b2::key_index(k);
    }
    b2::pdl_trigger();
}

// ── b2_rows_to_f16: one CTA per row ──
__global__ void __launch_bounds__(256) rows_to_f16_kernel(uint16_t* __restrict__ y16, int ldy,
                                                         const float* __restrict__ x, int ldx, int K,
                                                         const float* __restrict__ norm_w, float eps) {
    __shared__ float red[8];
    b2::pdl_wait();
    const float* xr = x + (size_t)blockIdx.x * ldx;
    __half* yr = reinterpret_cast<__half*>(y16) + (size_t)blockIdx.x * ldy;
    const int tid = threadIdx.x;
    float rms = 1.f;
    if (norm_w) {
        float ss = 0.f;
        for (int k = tid; k < K; k += 256) ss = fmaf(xr[k], xr[k], ss);
        ss = b2::warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) t += red[w];
        rms = 1.0f / sqrtf(t / (float)K + eps);
    }
    for (int k = tid; k < K; k += 256) {
        float v = xr[k];
        if (norm_w) v = (v * rms) * norm_w[k];
        yr[k] = __float2half_rn(v);
    }
    b2::pdl_trigger();
}

// ── host side ──

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// 2-D tensor [outer][inner] with rows row_bytes apart, loaded in boxes of
// box_outer rows x box_inner elements.  FP16 boxes use the 128-byte swizzle
// (the MMA operand layout); UINT8 boxes (raw quantized rows) land unswizzled.
int make_map(CUtensorMap* m, const void* base, bool f16, uint64_t inner, uint64_t outer, uint64_t row_bytes,
             uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn enc = encoder();
    if (!enc) return b2_set_error(B2_ERR_CUDA, "b2_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                           const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           f16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return b2_set_error(B2_ERR_CUDA, "b2_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 0;
}

template <int BN, int MODE, int WT>
int launch(const B2GemmArgs* a, cudaStream_t s, int sms) {
    using Lay = Layout<BN, MODE, WT>;
    CUtensorMap tw, tx;
    const uint64_t wrows = (uint64_t)(MODE == MODE_PAIR ? 2 * a->N : a->N);
    const uint64_t wrow_bytes = (uint64_t)a->K / kBK * raw_row_bytes<WT>();
    int rc = WT == B2_W_F16 ? make_map(&tw, a->w, true, (uint64_t)a->K, wrows, wrow_bytes, kBK, kBM)
                            : make_map(&tw, a->w, false, wrow_bytes, wrows, wrow_bytes, raw_row_bytes<WT>(), kBM);
    if (!rc) rc = make_map(&tx, a->x16, true, (uint64_t)a->K, (uint64_t)a->M, (uint64_t)a->ldx * 2, kBK, BN);
    if (rc) return rc;
    constexpr size_t smem = (size_t)Lay::kStages * Lay::kStage + sizeof(Bars) + 1024;
    auto fn = gemm_kernel<BN, MODE, WT>;
    static std::once_flag once[8];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = cudaSuccess;
    std::call_once(once[dev & 7], [&] { e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_gemm smem attr: %s", cudaGetErrorString(e));
    GemmParams g{a->y, a->ldy, a->M, a->K, a->N, a->scales, a->epilogue, a->keys,
                 reinterpret_cast<__half*>(a->y16)};
    const int gx = (a->N + kBM - 1) / kBM, gy = (a->M + BN - 1) / BN;
    // A residual-add GEMM whose grid leaves SMs idle splits K over more CTAs
    // (each adds its partial sum into y; at least 4 k stages per split).
    int split = 1;
    if (MODE == MODE_ROWS && a->epilogue == B2_EPI_ADD)
        while (gx * gy * split * 2 <= sms && (a->K / kBK) / (split * 2) >= 4) split *= 2;
    e = b2::launch_pdl(fn, dim3(gx, gy, split), dim3(kThreads), smem, s, tw, tx, g);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_gemm launch: %s", cudaGetErrorString(e));
    if (MODE == MODE_ARGMAX) {
        e = b2::launch_pdl(argmax_parts_kernel, dim3(a->M), dim3(256), 0, s, (const unsigned long long*)a->keys, gx,
                           a->tokens);
        if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_gemm argmax: %s", cudaGetErrorString(e));
    }
    return 0;
}

template <int MODE, int WT>
int by_bn(const B2GemmArgs* a, cudaStream_t s, int sms) {
    return a->M <= 64 ? launch<64, MODE, WT>(a, s, sms) : launch<128, MODE, WT>(a, s, sms);
}

template <int MODE>
int by_wtype(const B2GemmArgs* a, cudaStream_t s, int sms) {
    switch (a->wtype) {
        case B2_W_F16: return by_bn<MODE, B2_W_F16>(a, s, sms);
        case B2_W_I8: return by_bn<MODE, B2_W_I8>(a, s, sms);
        default: return by_bn<MODE, B2_W_I4>(a, s, sms);
    }
}

}  // namespace

extern "C" size_t b2_gemm_argmax_keys(int M, int N) { return (size_t)M * ((N + kBM - 1) / kBM) * 8; }

extern "C" int b2_gemm(const B2GemmArgs* a, b2_stream_t stream) {
    if (!a || !a->x16 || !a->w || a->M < 0 || a->K <= 0 || a->N <= 0)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemm: bad arguments");
    if (a->M == 0) return 0;
    const int epi = a->epilogue;
    const bool argmax = epi == B2_EPI_ARGMAX;
    if (epi < B2_EPI_STORE || epi > B2_EPI_ARGMAX || (!argmax && !a->y && !a->y16) ||
        (a->y16 && epi != B2_EPI_STORE && epi != B2_EPI_SILU_PAIR) || (argmax && (!a->keys || !a->tokens)))
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_gemm: missing output for epilogue %d", epi);
    if ((a->wtype != B2_W_F16 && a->wtype != B2_W_I8 && a->wtype != B2_W_I4) ||
        (a->wtype != B2_W_F16 && !a->scales) || a->K % kBK || (!argmax && a->N % kBM) || a->ldx % 8 ||
        a->ldx < a->K || ((a->y || a->y16) && a->ldy < a->N) || (reinterpret_cast<uintptr_t>(a->x16) & 15) ||
        (reinterpret_cast<uintptr_t>(a->w) & 15))
        return b2_set_error(B2_ERR_INVALID_ARG,
                            "b2_gemm: needs F16/I8/I4 weights (scales for I8/I4), K %% 64 == 0, N %% 128 == 0, "
                            "ldx %% 8 == 0, aligned operands");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (epi == B2_EPI_SILU_PAIR) return by_wtype<MODE_PAIR>(a, s, sms);
    if (argmax) return by_wtype<MODE_ARGMAX>(a, s, sms);
    return by_wtype<MODE_ROWS>(a, s, sms);
}

extern "C" int b2_rows_to_f16(uint16_t* y16, int ldy, const float* x, int ldx, int M, int K, const float* norm_w,
                              float eps, b2_stream_t stream) {
    if (!y16 || !x || M < 0 || K <= 0 || ldy < K || ldx < K || ldy % 8)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_rows_to_f16: bad arguments");
    if (M == 0) return 0;
    cudaError_t e = b2::launch_pdl(rows_to_f16_kernel, dim3(M), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                                   y16, ldy, x, ldx, K, norm_w, eps);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_rows_to_f16 launch: %s", cudaGetErrorString(e));
    return 0;
}
