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
//   warps 2-9    for INT8 / INT4 weights, widen each stage's raw weight tile
//                exactly to FP16 in the swizzled layout the MMA reads (the
//                integer in the mantissa of 1024 and one half2 subtraction);
//                at the end, read the accumulator with tcgen05.ld (warp w owns
//                TMEM lanes 32*(w%4)..+31; warps 2-5 and 6-9 take alternate
//                16-column chunks) and apply the epilogue.
//
// The weight tile is the MMA's A operand (output columns are TMEM lanes) and
// the activation tile its B operand (token rows are TMEM columns), so one
// CTA computes a 128-column x BN-row block of y.  For SILU_PAIR the stage
// holds 128 gate rows and the 128 matching up rows; two MMAs per k step sum
// them into TMEM columns [0, BN) and [BN, 2 BN), so each epilogue thread
// finds the gate and up sums of its channel side by side.  For ARGMAX each
// CTA reduces its 128 vocab rows to one packed (logit, index) key per token
// and a second kernel reduces the CTAs' keys.
//
// When the tiles alone would leave SMs idle (few token rows), the K range of
// a tile is split over a thread-block cluster of 2, 4 or 8 CTAs.  Each CTA
// pushes its partial accumulator columns into the shared memory of the CTA
// that finishes that slice of the token columns (st.shared::cluster between
// two cluster barriers), so every epilogue sees whole sums without atomics.
#include <cuda.h>  // CUtensorMap and its enums; the encoder is looked up at run time

#include <mutex>
#include <stdlib.h>

#include "b2_common.cuh"

namespace {

constexpr int kBM = 128;     // weight rows per tile (MMA M)
constexpr int kBK = 64;      // k per stage: 64 FP16 = one 128-byte swizzle row
constexpr int kThreads = 320;  // producer warp, MMA warp, 8 converter / epilogue warps
constexpr int kWork = kThreads - 64;
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
    // The lm_head (ARGMAX) grid runs many waves of short CTAs: half the ring
    // lets two CTAs share an SM, so one's prologue and epilogue overlap the
    // other's weight stream.  The other modes keep one deep ring per SM.
    static constexpr int kBudget = (MODE == MODE_ARGMAX ? 96 : 192) * 1024;
    static constexpr int kStages = kBudget / kStage > kMaxStages ? kMaxStages : kBudget / kStage;
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
    int peer_failed[8];  // split-K: failure flag of each cluster rank, pushed by that rank
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

// Eight consecutive weights widened exactly to FP16 (the integer in the
// mantissa of 1024 and one half2 subtraction of 1024 + bias).
// INT8: two words, byte i of the pair is k = i.
__device__ __forceinline__ uint4 widen8_i8(uint32_t w0, uint32_t w1) {
    const uint32_t bias = 0x64806480u;  // half2(1152): 1024 + 128
    const uint32_t a = w0 ^ 0x80808080u, b = w1 ^ 0x80808080u;
    uint4 h;
    h.x = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4140), bias);
    h.y = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4342), bias);
    h.z = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4140), bias);
    h.w = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4342), bias);
    return h;
}
// INT4: one word, nibble i is k = i (even k in the low nibble of its byte).
__device__ __forceinline__ uint4 widen8_i4(uint32_t w) {
    const uint32_t u = w ^ 0x88888888u;
    const uint32_t bias = 0x64086408u;  // half2(1032): 1024 + 8
    uint4 h;
    h.x = hsub2_u32((u & 0x0000000Fu) | ((u << 12) & 0x000F0000u) | 0x64006400u, bias);
    h.y = hsub2_u32(((u >> 8) & 0x0000000Fu) | ((u << 4) & 0x000F0000u) | 0x64006400u, bias);
    h.z = hsub2_u32(((u >> 16) & 0x0000000Fu) | ((u >> 4) & 0x000F0000u) | 0x64006400u, bias);
    h.w = hsub2_u32(((u >> 24) & 0x0000000Fu) | ((u >> 12) & 0x000F0000u) | 0x64006400u, bias);
    return h;
}

// ── thread-block cluster helpers (split-K partial sums through distributed shared memory) ──
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// Stores into another CTA's shared memory do not stall the issuing thread;
// the cluster barrier's release / acquire makes them visible.
__device__ __forceinline__ void st_dsmem4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared::cluster.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ void st_dsmem_s32(uint32_t addr, int v) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Split-K receive buffer of the CTA that finishes a slice of W accumulator
// columns: slot r (the sending rank) holds its partial sums of the slice as
// groups of 4 columns, [r][lc / 4][128 rows][4] FP32, so one warp's 16-byte
// accesses to a column group are 512 contiguous bytes.  lc is the column
// within the slice (a multiple of 4 here).
__device__ __forceinline__ uint32_t part_off(int r, int W, int lc, int li) {
    return (uint32_t)((((r * W + lc) >> 2) * kBM + li) * 16);
}

// silu(g) * u with the sigmoid as 1 / (1 + e^-g) from the fast exponential
// and divide (relative error ~1e-6, inside the FP32 parity tolerance); the
// exponent is capped where e^-g would leave the divide's range.
__device__ __forceinline__ float silu_mul(float gv, float uv) {
    return gv * __fdividef(1.0f, 1.0f + __expf(fminf(-gv, 80.0f))) * uv;
}

template <int BN, int MODE, int WT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const GemmParams g) {
    using Lay = Layout<BN, MODE, WT>;
    constexpr bool kConvert = WT != B2_W_F16;
    static_assert(kBM * Lay::kCols * 4 + 4 * BN * 8 <= Lay::kStages * Lay::kStage, "epilogue scratch exceeds the ring");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    Bars* b = reinterpret_cast<Bars*>(smem + Lay::kStages * Lay::kStage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BN;
    // split-K: the gridDim.z CTAs of a tile form one cluster; this CTA sums k
    // stages [kt0, kt0 + KT) and the cluster reduces the partial sums.
    const int S = (int)gridDim.z;
    const int KT_all = g.K / kBK;
    const int kt0 = (int)((long long)KT_all * blockIdx.z / S);
    const int KT = (int)((long long)KT_all * (blockIdx.z + 1) / S) - kt0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Lay::kStages; s++) {
            mbar_init(&b->full[s], 1);
            mbar_init(&b->conv[s], kWork / 32);
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
    bool ok = true;
    // Let the next kernel of the stream start its own prologue on the SMs
    // this grid leaves free; it waits for this grid's completion before it
    // reads anything this grid writes.
    b2::pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            constexpr uint32_t kTx = Lay::kB + (kConvert ? Lay::kRaw : Lay::kA);
            constexpr int kWTile = kConvert ? kBM * raw_row_bytes<WT>() : kBM * 128;
            auto load_w = [&](int kt) {
                const int s = kt % Lay::kStages;
                unsigned char* st = smem + s * Lay::kStage;
                unsigned char* wdst = kConvert ? st + Lay::kA + Lay::kB : st;
                // x coordinate of the weight map: elements for FP16, bytes for INT8/INT4
                const int wx = (kt0 + kt) * (WT == B2_W_F16 ? kBK : raw_row_bytes<WT>());
                mbar_expect_tx(&b->full[s], kTx);
                tma_load_2d(wdst, &tw, wx, kBM * blockIdx.x, &b->full[s]);
                if (MODE == MODE_PAIR) tma_load_2d(wdst + kWTile, &tw, wx, g.N + kBM * blockIdx.x, &b->full[s]);
            };
            auto load_x = [&](int kt) {
                const int s = kt % Lay::kStages;
                tma_load_2d(smem + s * Lay::kStage + Lay::kA, &tx, (kt0 + kt) * kBK, m0, &b->full[s]);
            };
            // The weights do not depend on earlier kernels of the stream: the
            // first ring's worth is requested before waiting for them.
            const int pre = KT < Lay::kStages ? KT : Lay::kStages;
            for (int kt = 0; kt < pre; kt++) load_w(kt);
            // The activation rows come from the previous kernel of the stream.
            b2::pdl_wait();
            for (int kt = 0; kt < pre; kt++) load_x(kt);
            for (int kt = pre; kt < KT; kt++) {
                const int s = kt % Lay::kStages;
                if (!mbar_wait(&b->empty[s], (uint32_t)((kt / Lay::kStages - 1) & 1), b)) break;
                load_w(kt);
                load_x(kt);
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
    } else {  // warps 2..9
        const int et = threadIdx.x - 64;  // 0..kWork-1
        if constexpr (kConvert) {
            // raw [rows][raw_row_bytes] -> FP16 [rows][128 B] with 16-byte chunk c of row r at (c ^ (r % 8)) * 16.
            // Each thread widens whole 16-byte raw chunks (16 INT8 or 32 INT4 weights); all of a stage's
            // loads are issued before its stores.
            constexpr int kRowChunks = raw_row_bytes<WT>() / 16;               // raw chunks per row
            constexpr int kOut = 8 / kRowChunks;                               // FP16 chunks per raw chunk
            constexpr int kPer = Lay::kATiles * kBM * kRowChunks / kWork;      // raw chunks per thread
            static_assert(kPer * kWork == Lay::kATiles * kBM * kRowChunks, "converter jobs must divide evenly");
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % Lay::kStages;
                if (!mbar_wait(&b->full[s], (uint32_t)((kt / Lay::kStages) & 1), b)) break;
                unsigned char* st = smem + s * Lay::kStage;
                const uint4* raw = reinterpret_cast<const uint4*>(st + Lay::kA + Lay::kB);
                uint4 rv[kPer];
#pragma unroll
                for (int i = 0; i < kPer; i++) rv[i] = raw[et + kWork * i];
#pragma unroll
                for (int i = 0; i < kPer; i++) {
                    const int job = et + kWork * i;
                    const int R = job / kRowChunks, h = job % kRowChunks;  // row of the stage, raw chunk
                    const int tile = R / kBM, r = R % kBM;
                    unsigned char* row = st + tile * kBM * 128 + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                    for (int o = 0; o < kOut; o++) {
                        const int c = h * kOut + o;
                        const uint32_t* w = &rv[i].x;
                        const uint4 hv = WT == B2_W_I8 ? widen8_i8(w[2 * o], w[2 * o + 1]) : widen8_i4(w[o]);
                        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = hv;
                    }
                }
                // the tensor cores read shared memory through the async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&b->conv[s]);
            }
        }
        ok = mbar_wait(&b->done, 0, b);
        tc_fence_after();
    }
    // Split-K reduction.  The token columns [0, BN) are cut into S slices;
    // rank j finishes slice j (for SILU_PAIR the gate and the up columns of
    // those tokens).  Once every CTA of the cluster has finished its k loop
    // (its ring is idle), each pushes the partial sums of slice j into rank
    // j's ring, then the owners add the S partials from their own memory.
    constexpr int kSliceCols = MODE == MODE_PAIR ? 2 : 1;  // accumulator columns per token
    const int W = kSliceCols * BN / S;                      // accumulator columns per slice
    if (S > 1) {
        cluster_sync();
        if (warp >= 2) {
            const int quad = warp & 3, li = 32 * quad + lane, half = (warp - 2) >> 2;
            const int me = (int)cluster_rank();
            const bool bad = !ok || *(volatile int*)&b->failed;
            if (threadIdx.x == 64)
                for (int j = 0; j < S; j++) st_dsmem_s32(dsmem_addr(smem_u32(&b->peer_failed[me]), j), bad ? 1 : 0);
            if (!bad) {
                // chunks in an order rotated by rank, so the ranks start on different owners
                constexpr int kChunks = Lay::kCols / 16;
#pragma unroll 1
                for (int i = half; i < kChunks; i += 2) {
                    const int c0 = 16 * ((i + me * kChunks / S) % kChunks);
                    uint32_t v[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + c0, v);
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int col = c0 + 4 * q, tok = col % BN, j = tok / (BN / S);
                        const int lc = (col >= BN ? W / 2 : 0) + tok - j * (BN / S);
                        st_dsmem4(dsmem_addr(smem_u32(smem + part_off(me, W, lc, li)), j), v[4 * q], v[4 * q + 1],
                                  v[4 * q + 2], v[4 * q + 3]);
                    }
                }
            }
        }
        cluster_sync();
    }
    if (warp >= 2) {
        const int et = threadIdx.x - 64;
        const int quad = warp & 3, li = 32 * quad + lane, half = (warp - 2) >> 2;
        const int n = kBM * blockIdx.x + li;
        // This CTA's token columns: all of them, or with split-K its slice.
        const int rank = S > 1 ? (int)cluster_rank() : 0;
        const int cb = rank * BN / S, ce = (rank + 1) * BN / S;
        if (S > 1)
            for (int r = 0; r < S; r++) ok = ok && *(volatile int*)&b->peer_failed[r] == 0;
        // v[j] = accumulator column col + j (j < cnt) of row li; with split-K
        // col is relative to the slice (lc) and the S partials are summed.
        auto acc16 = [&](int col, int cnt, uint32_t (&v)[16]) {
            if (S == 1) {
                tmem_ld16(tmem + ((uint32_t)(32 * quad) << 16) + col, v);
                return;
            }
            float f[16];
#pragma unroll
            for (int j = 0; j < 16; j++) f[j] = 0.f;
            for (int r = 0; r < S; r++) {
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    if (4 * q >= cnt) break;
                    const float4 p = *reinterpret_cast<const float4*>(smem + part_off(r, W, col + 4 * q, li));
                    f[4 * q] += p.x;
                    f[4 * q + 1] += p.y;
                    f[4 * q + 2] += p.z;
                    f[4 * q + 3] += p.w;
                }
            }
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = __float_as_uint(f[j]);
        };
        b2::pdl_wait();  // y may be read (residual) and is written below
        if (MODE == MODE_ROWS) {
            const float sc = g.scales ? g.scales[n] : 1.f;
#pragma unroll 1
            for (int c0 = cb + 16 * half; c0 < ce && ok; c0 += 32) {
                uint32_t v[16];
                acc16(S > 1 ? c0 - cb : c0, min(16, ce - c0), v);
                const int jn = min(min(16, ce - c0), g.M - (m0 + c0));
                if (jn <= 0) break;
                float* yp = g.y + (size_t)(m0 + c0) * g.ldy + n;
                if (g.epilogue == B2_EPI_ADD) {
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
            for (int c0 = cb + 16 * half; c0 < ce && ok; c0 += 32) {
                uint32_t vg[16], vu[16];
                acc16(S > 1 ? c0 - cb : c0, min(16, ce - c0), vg);
                acc16(S > 1 ? W / 2 + c0 - cb : BN + c0, min(16, ce - c0), vu);
                const int jn = min(min(16, ce - c0), g.M - (m0 + c0));
                if (jn <= 0) break;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (j >= jn) break;
                    const float h = silu_mul(__uint_as_float(vg[j]) * sg, __uint_as_float(vu[j]) * su);
                    const size_t o = (size_t)(m0 + c0 + j) * g.ldy + n;
                    if (g.y16) g.y16[o] = __float2half_rn(h);  // the down GEMM's FP16 input
                    else g.y[o] = h;
                }
            }
        } else {  // ARGMAX over this CTA's 128 vocab rows, per token
            // [4][BN] keys after the partial-sum area; the ring is idle
            unsigned long long* kq = reinterpret_cast<unsigned long long*>(smem + kBM * Lay::kCols * 4);
            const bool live = n < g.N;
            const float sc = live ? (g.scales ? g.scales[n] : 1.f) : 0.f;
#pragma unroll 1
            for (int c0 = cb + 16 * half; c0 < ce; c0 += 32) {
                uint32_t v[16];
                if (ok) acc16(S > 1 ? c0 - cb : c0, min(16, ce - c0), v);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (c0 + j >= ce) break;  // uniform across the warp
                    const int m = m0 + c0 + j;
                    const float logit = ok ? __uint_as_float(v[j]) * sc : 0.f;
                    if (g.y && live && m < g.M) g.y[(size_t)m * g.ldy + n] = logit;
                    unsigned long long key = live ? b2::argmax_key(logit, (uint32_t)n) : 0ull;
                    key = b2::warp_max_u64(key);
                    if (lane == 0) kq[quad * BN + c0 + j] = key;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kWork) : "memory");
            for (int j = cb + et; j < ce; j += kWork) {
                unsigned long long key = kq[j];
#pragma unroll
                for (int q = 1; q < 4; q++) key = kq[q * BN + j] > key ? kq[q * BN + j] : key;
                if (m0 + j < g.M) g.keys[(size_t)(m0 + j) * gridDim.x + blockIdx.x] = key;
            }
        }
    }
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
    b2::pdl_trigger();
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
}

// ── b2_rows_to_f16: one CTA per row ──
__global__ void __launch_bounds__(256) rows_to_f16_kernel(uint16_t* __restrict__ y16, int ldy,
                                                         const float* __restrict__ x, int ldx, int K,
                                                         const float* __restrict__ norm_w, float eps) {
    __shared__ float red[8];
    b2::pdl_trigger();
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

// B2_GEMM_SPLIT=1|2|4|8 fixes the split-K cluster size of every call that
// leaves it to the library (split_k == 0); unset or 0 keeps the automatic choice.
int split_override() {
    static const int v = [] {
        const char* e = getenv("B2_GEMM_SPLIT");
        const int x = e ? atoi(e) : 0;
        return (x == 1 || x == 2 || x == 4 || x == 8) ? x : 0;
    }();
    return v;
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
    const int gx = (a->N + kBM - 1) / kBM, gy = (a->M + BN - 1) / BN, KT = a->K / kBK;
    // Split-K over a cluster of S CTAs per tile when the tiles alone leave
    // SMs idle (each CTA keeps at least two k stages); the cluster reduces
    // the partial sums, so every epilogue sees whole sums.
    int S = a->split_k;
    if (S <= 0) S = split_override();
    if (S <= 0) {
        S = 1;
        while (S < 8 && gx * gy * S * 2 <= sms && KT / (S * 2) >= 2) S *= 2;
    }
    while (S > KT) S /= 2;
    if (S > 1) {  // a cluster of S full-shared-memory CTAs must fit the GPU
        static int fits[4] = {-1, -1, -1, -1};  // S = 2, 4, 8 (index log2 S)
        int& f = fits[S == 2 ? 1 : S == 4 ? 2 : 3];
        if (f < 0) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(gx, gy, S);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 1;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = S;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            f = cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n > 0;
            cudaGetLastError();
        }
        if (!f) S = 1;
    }
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(gx, gy, S);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = 1;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = S;
        cfg.attrs = at;
        cfg.numAttrs = S > 1 ? 2 : 1;
        e = cudaLaunchKernelEx(&cfg, fn, tw, tx, g);
    }
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

// FP16 2-D tensor map with the 128-byte swizzle for other kernels of the library.
int b2_tensor_map_f16(void* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                      uint32_t box_inner, uint32_t box_outer) {
    return make_map(reinterpret_cast<CUtensorMap*>(map), base, true, inner, outer, row_bytes, box_inner, box_outer);
}

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
        a->ldx < a->K || ((a->y || a->y16) && a->ldy < a->N) ||
        (a->split_k != 0 && a->split_k != 1 && a->split_k != 2 && a->split_k != 4 && a->split_k != 8) ||
        a->split_k > a->K / kBK || (reinterpret_cast<uintptr_t>(a->x16) & 15) ||
        (reinterpret_cast<uintptr_t>(a->w) & 15))
        return b2_set_error(B2_ERR_INVALID_ARG,
                            "b2_gemm: needs F16/I8/I4 weights (scales for I8/I4), K %% 64 == 0, N %% 128 == 0, "
                            "ldx %% 8 == 0, aligned operands, split_k in {0, 1, 2, 4, 8} and <= K / 64");
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
