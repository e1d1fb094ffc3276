// GQA attention over the FP16 KV cache, three entry points:
//   b2_attention / b2_attention_f16  rows of any lengths, split-KV on CUDA cores
//                                    (decode graph path; this header);
//   b2_attention_blocks              many sequences of different lengths:
//                                    persistent CTAs over fixed position blocks,
//                                    TMA ring, tensor cores (batched decode);
//   b2_attention_prefill             causal flash attention of consecutive rows
//                                    of one sequence (batch prefill).
//
// Computes what attention_f32 (src/cpu_ops.c:202-264) and, per row,
// attention_batch_causal_f32 (:459-571) compute: for q head h the kv head is
// h / (nq / nkv), scores are dot(q, k) * (1 / sqrtf(hd)), softmax subtracts the
// maximum and uses expf, and the output is the probability-weighted sum of v.
//
// B200 shape: the cache of one (sequence, layer, kv head) is one contiguous
// [max_seq][hd] FP16 block, so a K or V row is 256 contiguous bytes.  The
// positions [0, pos] of a row are cut into nsplit ranges; one CTA per (range,
// kv head, row) streams its K and V rows once and serves all q heads of the
// GQA group from registers, keeping an online (running max / running sum)
// softmax.  Eight lanes cover one 128-wide row (16 dims each), so a 128-thread
// CTA walks 16 positions per iteration.  A second kernel merges the ranges.
#include <cuda.h>  // CUtensorMap
#include <math.h>

#include "b2_common.cuh"

namespace {

constexpr int kHD = 128;
constexpr int kThreads = 128;
constexpr int kGroups = kThreads / 8;  // positions in flight per CTA

template <int G>
__global__ void __launch_bounds__(kThreads) attn_split_kernel(const float* __restrict__ q, int ldq,
                                                              int nq, int nkv, B2KVRef kv,
                                                              float* __restrict__ part_ml,
                                                              float* __restrict__ part_o, int nsplit) {
    __shared__ float sm_m[kGroups][G], sm_l[kGroups][G];
    __shared__ float sm_o[kGroups][G][kHD];
    const int split = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane & 7, grp = warp * 4 + (lane >> 3);
    int seq = kv.rows_seq ? kv.rows_seq[m] : 0;
    int L = kv.pos[m] + 1;
    if (L < 1 || L > kv.max_seq || seq < 0 || seq >= kv.n_seqs) {  // invalid row: attend to nothing
        L = 0;
        seq = 0;
    }
    const int chunk = (L + nsplit - 1) / nsplit;
    const int p0 = split * chunk;
    const int p1 = min(L, p0 + chunk);
    const float scale = 1.0f / sqrtf((float)kHD);
    const size_t head_off = seq * kv.seq_stride + kv.layer * kv.layer_stride + (size_t)g * kv.max_seq * kHD;
    // Start pulling this range of K and V into L2 while the previous kernel
    // finishes.  pos[] and rows_seq[] are written before the step's first
    // kernel, so reading them here is safe; lines the previous kernel is still
    // storing are harmless to prefetch because stores land in L2 and every
    // read below follows pdl_wait().
    // Only the head of the range: with many sequences a whole-range prefetch
    // would exceed L2 and evict itself before the loop gets there.
    if (threadIdx.x == 0 && p1 - 1 > p0) {
        const uint32_t bytes = (uint32_t)min(p1 - 1 - p0, 4 * kGroups) * kHD * 2;
        b2::prefetch_l2(kv.k_base + head_off + (size_t)p0 * kHD, bytes);
        b2::prefetch_l2(kv.v_base + head_off + (size_t)p0 * kHD, bytes);
    }
    b2::pdl_trigger();
    b2::pdl_wait();

    float qv[G][16];
#pragma unroll
    for (int h = 0; h < G; h++) {
        const float* qp = q + (size_t)m * ldq + (size_t)(g * G + h) * kHD + sub * 16;
#pragma unroll
        for (int j = 0; j < 16; j++) qv[h][j] = qp[j];
    }
    float mx[G], ls[G], o[G][16];
#pragma unroll
    for (int h = 0; h < G; h++) {
        mx[h] = -INFINITY;
        ls[h] = 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) o[h][j] = 0.f;
    }
    const __half* kb = reinterpret_cast<const __half*>(kv.k_base + head_off) + sub * 16;
    const __half* vb = reinterpret_cast<const __half*>(kv.v_base + head_off) + sub * 16;

    // The loop bound is uniform across the warp (its four lane groups take
    // positions pb + {0,1,2,3} + 16 u) so every lane reaches the shuffles
    // below; a group past the end of the range computes on zeros and keeps
    // its state.  The K and V rows of kU positions per group are requested
    // before any is used, so each lane keeps 4 x 64 bytes in flight.
    constexpr int kU = 4;
    for (int pb = p0 + warp * 4; pb < p1; pb += kGroups * kU) {
        uint4 kr[kU][2], vr[kU][2];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int p = pb + u * kGroups + (lane >> 3);
            if (p < p1) {
                const uint4* kp = reinterpret_cast<const uint4*>(kb + (size_t)p * kHD);
                const uint4* vp = reinterpret_cast<const uint4*>(vb + (size_t)p * kHD);
                kr[u][0] = kp[0];
                kr[u][1] = kp[1];
                vr[u][0] = vp[0];
                vr[u][1] = vp[1];
            } else {
                kr[u][0] = kr[u][1] = vr[u][0] = vr[u][1] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; u++) {
            if (pb + u * kGroups >= p1) break;  // uniform across the warp
            const bool live = pb + u * kGroups + (lane >> 3) < p1;
            float kf[16], vf[16];
            const uint32_t* ku0 = &kr[u][0].x;
            const uint32_t* ku1 = &kr[u][1].x;
            const uint32_t* vu0 = &vr[u][0].x;
            const uint32_t* vu1 = &vr[u][1].x;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float2 a = b2::h2_to_f2(ku0[i]), b = b2::h2_to_f2(ku1[i]);
                kf[2 * i] = a.x; kf[2 * i + 1] = a.y; kf[8 + 2 * i] = b.x; kf[8 + 2 * i + 1] = b.y;
                float2 c = b2::h2_to_f2(vu0[i]), d = b2::h2_to_f2(vu1[i]);
                vf[2 * i] = c.x; vf[2 * i + 1] = c.y; vf[8 + 2 * i] = d.x; vf[8 + 2 * i + 1] = d.y;
            }
#pragma unroll
            for (int h = 0; h < G; h++) {
                float d = 0.f;
#pragma unroll
                for (int j = 0; j < 16; j++) d = fmaf(qv[h][j], kf[j], d);
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                d += __shfl_xor_sync(0xffffffffu, d, 4);
                if (!live) continue;
                const float sc = d * scale;
                const float mn = fmaxf(mx[h], sc);
                const float corr = expf(mx[h] - mn);
                const float pr = expf(sc - mn);
                ls[h] = ls[h] * corr + pr;
#pragma unroll
                for (int j = 0; j < 16; j++) o[h][j] = fmaf(pr, vf[j], o[h][j] * corr);
                mx[h] = mn;
            }
        }
    }
#pragma unroll
    for (int h = 0; h < G; h++) {
        if (sub == 0) {
            sm_m[grp][h] = mx[h];
            sm_l[grp][h] = ls[h];
        }
#pragma unroll
        for (int j = 0; j < 16; j++) sm_o[grp][h][sub * 16 + j] = o[h][j];
    }
    __syncthreads();
    const int d = threadIdx.x;  // one thread per head dimension
#pragma unroll
    for (int h = 0; h < G; h++) {
        float M = -INFINITY;
        for (int r = 0; r < kGroups; r++) M = fmaxf(M, sm_m[r][h]);
        float lsum = 0.f, acc = 0.f;
        if (M != -INFINITY) {
            for (int r = 0; r < kGroups; r++) {
                if (sm_m[r][h] == -INFINITY) continue;
                const float w = expf(sm_m[r][h] - M);
                lsum = fmaf(sm_l[r][h], w, lsum);
                acc = fmaf(sm_o[r][h][d], w, acc);
            }
        }
        const size_t slot = ((size_t)m * nq + g * G + h) * nsplit + split;
        part_o[slot * kHD + d] = acc;
        if (d == 0) {
            part_ml[slot * 2] = M;
            part_ml[slot * 2 + 1] = lsum;
        }
    }
}

// Merges the nsplit partial (max, sum, output) slots of each (row, q head).
// With block > 0 (b2_attention_blocks) only the slots of the row's blocks,
// ceil((pos[m] + 1) / block), were written.
__global__ void __launch_bounds__(kHD) attn_combine_kernel(float* __restrict__ out, __half* __restrict__ out16,
                                                           int nq, const float* __restrict__ part_ml,
                                                           const float* __restrict__ part_o, int nsplit,
                                                           const int* __restrict__ pos, int block, int max_seq) {
    b2::pdl_trigger();
    b2::pdl_wait();
    const int h = blockIdx.x, m = blockIdx.y, d = threadIdx.x;
    const size_t base = ((size_t)m * nq + h) * nsplit;
    int ns = nsplit;
    if (block > 0) {
        const int L = pos[m] + 1;
        ns = (L < 1 || L > max_seq) ? 0 : min(nsplit, (L + block - 1) / block);
    }
    float M = -INFINITY;
    for (int s = 0; s < ns; s++) M = fmaxf(M, part_ml[(base + s) * 2]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < ns; s++) {
        const float ms = part_ml[(base + s) * 2];
        if (ms == -INFINITY) continue;
        const float w = expf(ms - M);
        den = fmaf(part_ml[(base + s) * 2 + 1], w, den);
        num = fmaf(part_o[(base + s) * kHD + d], w, num);
    }
    const float r = den > 0.f ? num / den : 0.f;  // a row that attends to nothing gives zeros
    if (out16) out16[((size_t)m * nq + h) * kHD + d] = __float2half_rn(r);
    else out[((size_t)m * nq + h) * kHD + d] = r;
}

int pick_split(int M, int nkv, int nsplit) {
    if (nsplit > 0) return nsplit > 256 ? 256 : nsplit;
    int want = (2 * 148 + M * nkv - 1) / (M * nkv);
    return want < 1 ? 1 : (want > 64 ? 64 : want);
}

}  // namespace

extern "C" size_t b2_attention_workspace(int M, int nq, int hd, int nsplit) {
    (void)hd;
    nsplit = pick_split(M, 1, nsplit);  // worst case over nkv when nsplit <= 0
    return (size_t)M * nq * nsplit * (2 + kHD) * sizeof(float) + 256;
}

static int attention_impl(float* out, __half* out16, const float* q, int ldq, int M, int nq, int nkv, int hd,
                          const B2KVRef* kv, void* work, int nsplit, b2_stream_t s) {
    if (M <= 0) return 0;
    if (hd != kHD) return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention: head_dim %d != 128", hd);
    if ((!out && !out16) || !q || !kv || !kv->pos || !work || nkv <= 0 || nq % nkv != 0)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention: bad arguments");
    nsplit = pick_split(M, nkv, nsplit);
    float* part_ml = reinterpret_cast<float*>(work);
    float* part_o = part_ml + (size_t)M * nq * nsplit * 2;
    dim3 grid(nsplit, nkv, M);
    cudaStream_t st = (cudaStream_t)s;
    cudaError_t e = cudaSuccess;
    switch (nq / nkv) {
        case 1: e = b2::launch_pdl(attn_split_kernel<1>, grid, dim3(kThreads), 0, st, q, ldq, nq, nkv, *kv, part_ml, part_o, nsplit); break;
        case 2: e = b2::launch_pdl(attn_split_kernel<2>, grid, dim3(kThreads), 0, st, q, ldq, nq, nkv, *kv, part_ml, part_o, nsplit); break;
        case 4: e = b2::launch_pdl(attn_split_kernel<4>, grid, dim3(kThreads), 0, st, q, ldq, nq, nkv, *kv, part_ml, part_o, nsplit); break;
        default: return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention: GQA group %d not in {1,2,4}", nq / nkv);
    }
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention split: %s", cudaGetErrorString(e));
    e = b2::launch_pdl(attn_combine_kernel, dim3(nq, M), dim3(kHD), 0, st, out, out16, nq, (const float*)part_ml,
                       (const float*)part_o, nsplit, (const int*)nullptr, 0, 0);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention combine: %s", cudaGetErrorString(e));
    return 0;
}

extern "C" int b2_attention(float* out, const float* q, int ldq, int M, int nq, int nkv, int hd,
                            const B2KVRef* kv, void* work, int nsplit, b2_stream_t s) {
    return attention_impl(out, nullptr, q, ldq, M, nq, nkv, hd, kv, work, nsplit, s);
}

extern "C" int b2_attention_f16(uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv, int hd,
                                const B2KVRef* kv, void* work, int nsplit, b2_stream_t s) {
    return attention_impl(nullptr, reinterpret_cast<__half*>(out16), q, ldq, M, nq, nkv, hd, kv, work, nsplit, s);
}

// ─── many sequences: fixed-size position blocks on the tensor cores (b2_attention_blocks) ───
//
// attention_f32 (src/cpu_ops.c:202-264) per row for batched decode, where the
// rows have very different lengths.  Each CTA takes one block of `block`
// consecutive cache positions of one (row, kv head), so the work per CTA does
// not depend on the row's length and the grid's tail is short.  The block's
// K and V rows stream through a ring of shared-memory stages by TMA (128-byte
// swizzled boxes of 64 positions x 64 dims), and the four warps compute on
// the stage before, each on 16 positions of a stage:
//
//   S^T = K Q^T    mma.sync m16n8k16: the warp's 16 positions are the M
//                  rows, the GQA group's q heads the N columns (G <= 8, the
//                  rest zero), head dims the K dimension;
//   online softmax per q head over the 16 positions (8-lane shuffles);
//   O^T += V^T P^T  the 128 head dims are M (8 tiles), the positions K; P^T
//                  moves from the accumulator layout to the B-operand layout
//                  with movmatrix.trans (FP16 P).
//
// Q and P are FP16, sums and the softmax FP32 (as in the prefill kernel).
// Rows of a partial last stage are masked (V rows past the end are zeroed).
namespace {

constexpr int kBlkChunk = 64;                            // positions per stage (16 per warp)
constexpr int kBlkStages = 3;
constexpr int kBlkBox = 64 * 128;                        // one 64 x 64 FP16 box, bytes
constexpr int kBlkStageBytes = 4 * kBlkBox;              // K dims 0-63, K 64-127, V 0-63, V 64-127
constexpr long long kBlkWaitLimit = 1ll << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of (row r, 8-dim chunk c) in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

constexpr int kBlkMaxRows = 512;  // rows one launch takes (the per-row unit prefix lives in shared memory)

// One unit of work: block b of row m, kv head g (positions [p0, p1)).
struct BlkUnit {
    int m, g, b, p0, p1, nch, row0;
};

// Unit u of the launch: units are ordered by row, then kv head, then block;
// pre[m] is the number of units of rows < m.
__device__ __forceinline__ BlkUnit blk_unit(int u, const int* pre, int M, int nkv, int block, const B2KVRef& kv) {
    int lo = 0, hi = M;  // largest m with pre[m] <= u
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] <= u) lo = mid;
        else hi = mid;
    }
    BlkUnit x;
    x.m = lo;
    const int nb = (pre[lo + 1] - pre[lo]) / nkv, r = u - pre[lo];
    x.g = r / nb;
    x.b = r % nb;
    const int L = kv.pos[lo] + 1;
    const int seq = kv.rows_seq ? kv.rows_seq[lo] : 0;
    x.p0 = x.b * block;
    x.p1 = min(L, x.p0 + block);
    x.nch = (x.p1 - x.p0 + kBlkChunk - 1) / kBlkChunk;
    x.row0 = (int)((seq * kv.seq_stride + kv.layer * kv.layer_stride + (long long)x.g * kv.max_seq * kHD) / kHD);
    return x;
}

// Persistent: CTA i takes units i, i + gridDim.x, ...  Thread 0 keeps the
// ring kBlkStages chunks ahead of the warps, across unit boundaries, so the
// memory pipe does not drain between units.
template <int G>
__global__ void __launch_bounds__(kThreads) attn_block_kernel(const __grid_constant__ CUtensorMap tk,
                                                              const __grid_constant__ CUtensorMap tv,
                                                              const float* __restrict__ q, int ldq, int M, int nq,
                                                              int nkv, B2KVRef kv, int block,
                                                              float* __restrict__ part_ml, float* __restrict__ part_o,
                                                              int nsplit, int* __restrict__ err) {
    static_assert(G >= 1 && G <= 8, "GQA group must fit the 8 MMA columns");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* ring =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full[kBlkStages];
    __shared__ int pre[kBlkMaxRows + 1];
    __shared__ float mg_m[4][8], mg_l[4][8];
    __shared__ float mg_o[4][G][kHD];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    b2::pdl_trigger();
    // units per row: ceil(L / block) blocks per kv head (none for an invalid
    // row); positions and rows are written before the step's first kernel
    if (warp == 0) {
        int carry = 0;
        for (int base = 0; base < M; base += 32) {
            const int m = base + lane;
            int n = 0;
            if (m < M) {
                const int L = kv.pos[m] + 1, seq = kv.rows_seq ? kv.rows_seq[m] : 0;
                if (L >= 1 && L <= kv.max_seq && seq >= 0 && seq < kv.n_seqs) n = (L + block - 1) / block * nkv;
            }
            int incl = n;  // inclusive warp scan
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            if (m < M) pre[m + 1] = carry + incl;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) pre[0] = 0;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kBlkStages; s++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tk) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tv) : "memory");
    }
    __syncthreads();
    const int U = pre[M];
    // The newest position's K and V come from the previous kernel (every CTA
    // waits, so this grid never completes before its predecessor).
    b2::pdl_wait();
    if ((int)blockIdx.x >= U) return;

    // producer cursor (thread 0 only): next chunk to request
    int iu = blockIdx.x, ic = 0, kin = 0;
    BlkUnit iun = blk_unit(iu, pre, M, nkv, block, kv);
    auto issue_next = [&]() {
        if (iu >= U) return;
        const int s = kin % kBlkStages, y = iun.row0 + iun.p0 + ic * kBlkChunk;
        unsigned char* st = ring + s * kBlkStageBytes;
        const uint32_t bar = smem_addr(&full[s]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBlkStageBytes)
                     : "memory");
#pragma unroll
        for (int i = 0; i < 4; i++)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
                "[%4];" ::"r"(smem_addr(st + i * kBlkBox)),
                "l"(i < 2 ? &tk : &tv), "r"((i & 1) * 64), "r"(y), "r"(bar)
                : "memory");
        kin++;
        if (++ic == iun.nch) {
            ic = 0;
            iu += gridDim.x;
            if (iu < U) iun = blk_unit(iu, pre, M, nkv, block, kv);
        }
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < kBlkStages; i++) issue_next();

    const float scale = 1.0f / sqrtf((float)kHD);
    const int pw = warp * 16;  // this warp's positions within a stage
    uint32_t qb[8][2];
    float o[8][4], mx[2], ls[2];
    bool ok = true;
    int kout = 0;  // chunks consumed
    for (int cu = blockIdx.x; cu < U && ok; cu += gridDim.x) {
        const BlkUnit un = blk_unit(cu, pre, M, nkv, block, kv);
        // Q^T as the B operand of S^T = K Q^T: column n = lane / 4 is q head
        // g*G + n (zero for n >= G); k step t covers dims 16t .. 16t+15.
        {
            const int n = lane >> 2, d0 = 2 * (lane & 3);
            const float* qp = q + (size_t)un.m * ldq + (size_t)(un.g * G + n) * kHD;
#pragma unroll
            for (int t = 0; t < 8; t++) {
                if (n < G) {
                    qb[t][0] = pack_h2(qp[16 * t + d0], qp[16 * t + d0 + 1]);
                    qb[t][1] = pack_h2(qp[16 * t + d0 + 8], qp[16 * t + d0 + 9]);
                } else {
                    qb[t][0] = qb[t][1] = 0u;
                }
            }
        }
        // O^T accumulator (8 tiles of 16 dims x 8 q columns), running max /
        // sum of this lane's two columns j0 = 2 (lane % 4) and j0 + 1.
#pragma unroll
        for (int t = 0; t < 8; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
        mx[0] = mx[1] = -INFINITY;
        ls[0] = ls[1] = 0.f;
        for (int c = 0; c < un.nch; c++, kout++) {
            const int s = kout % kBlkStages, np = min(kBlkChunk, un.p1 - (un.p0 + c * kBlkChunk));
            const uint32_t bar = smem_addr(&full[s]), par = (uint32_t)((kout / kBlkStages) & 1);
            uint32_t done = 0;
            for (long long it = 0; ok && !done; it++) {
                asm volatile(
                    "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, "
                    "0, p;\n}\n"
                    : "=r"(done)
                    : "r"(bar), "r"(par)
                    : "memory");
                if (!done && it > kBlkWaitLimit) ok = false;
            }
            // one decision for the whole CTA, so every thread meets the same barriers
            if (__syncthreads_or(!ok)) {
                ok = false;
                break;
            }
            unsigned char* st = ring + s * kBlkStageBytes;
            const uint32_t sk = smem_addr(st), sv = smem_addr(st + 2 * kBlkBox);
            const bool zero_tail = np < kBlkChunk && pw + 16 > np;
            if (zero_tail) {
                // V rows past the block's end may hold anything: zero this
                // warp's (P is zero there, and 0 x inf would not be)
                for (int r = max(pw, np) + (lane >> 4); r < pw + 16; r += 2) {
                    uint4* z = reinterpret_cast<uint4*>(st + 2 * kBlkBox + ((lane >> 3) & 1) * kBlkBox + r * 128) +
                               (lane & 7);
                    *z = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
            }
            if (pw < np) {
                float sc[4] = {0.f, 0.f, 0.f, 0.f};  // S^T [16 positions x 8 columns]
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    // A = K rows pw.., dims 16t..: sub-matrix j = lane / 8 -> (+8 rows if j odd, +8 dims if j >= 2)
                    const int r = pw + (lane & 7) + ((lane >> 3) & 1) * 8, d = 16 * t + (lane >> 4) * 8;
                    uint32_t a[4];
                    ldsm_x4(sk + (d >> 6) * kBlkBox + sw128(r, (d & 63) >> 3), a);
                    mma16816(sc, a, qb[t][0], qb[t][1]);
                }
                const int pa = pw + (lane >> 2), pb = pa + 8;
#pragma unroll
                for (int i = 0; i < 4; i++) sc[i] = (i < 2 ? pa : pb) < np ? sc[i] * scale : -INFINITY;
                float corr[2], pr[4];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float cm = fmaxf(sc[j], sc[j + 2]);
                    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
                    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 8));
                    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 16));
                    const float mn = fmaxf(mx[j], cm);
                    const bool none = mn == -INFINITY;
                    corr[j] = none ? 1.f : expf(mx[j] - mn);
                    pr[j] = none ? 0.f : expf(sc[j] - mn);
                    pr[j + 2] = none ? 0.f : expf(sc[j + 2] - mn);
                    float rs = pr[j] + pr[j + 2];
                    rs += __shfl_xor_sync(0xffffffffu, rs, 4);
                    rs += __shfl_xor_sync(0xffffffffu, rs, 8);
                    rs += __shfl_xor_sync(0xffffffffu, rs, 16);
                    ls[j] = ls[j] * corr[j] + rs;
                    mx[j] = mn;
                }
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    o[t][0] *= corr[0];
                    o[t][1] *= corr[1];
                    o[t][2] *= corr[0];
                    o[t][3] *= corr[1];
                }
                // P^T as the B operand: rows (positions) 0-7 and 8-15 transposed
                const uint32_t pb0 = movm_t(pack_h2(pr[0], pr[1])), pb1 = movm_t(pack_h2(pr[2], pr[3]));
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    // A = V^T dims 16t.., positions pw..: sub-matrix j -> (+8 dims if j odd, +8 rows if j >= 2)
                    const int r = pw + (lane & 7) + (lane >> 4) * 8, d = 16 * t + ((lane >> 3) & 1) * 8;
                    uint32_t a[4];
                    ldsm_x4_t(sv + (d >> 6) * kBlkBox + sw128(r, (d & 63) >> 3), a);
                    mma16816(o[t], a, pb0, pb1);
                }
            }
            // every warp is done with stage s (and, after a zeroing, the
            // generic-proxy writes are ordered before the next TMA into it)
            if (zero_tail) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            if (threadIdx.x == 0) issue_next();
        }
        if (!ok) break;
        // merge the four warps' states of this unit and write its partial slot
        {
            const int j0 = 2 * (lane & 3);
            if (lane < 4) {
                mg_m[warp][j0] = mx[0];
                mg_m[warp][j0 + 1] = mx[1];
                mg_l[warp][j0] = ls[0];
                mg_l[warp][j0 + 1] = ls[1];
            }
#pragma unroll
            for (int t = 0; t < 8; t++) {
                const int d = 16 * t + (lane >> 2);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int j = j0 + (i & 1), dd = d + (i >> 1) * 8;
                    if (j < G) mg_o[warp][j][dd] = o[t][i];
                }
            }
        }
        __syncthreads();
        {
            const int d = threadIdx.x;  // one thread per head dimension
#pragma unroll
            for (int h = 0; h < G; h++) {
                float Mx = -INFINITY;
#pragma unroll
                for (int w = 0; w < 4; w++) Mx = fmaxf(Mx, mg_m[w][h]);
                float lsum = 0.f, acc = 0.f;
                if (Mx != -INFINITY) {
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        if (mg_m[w][h] == -INFINITY) continue;
                        const float wt = expf(mg_m[w][h] - Mx);
                        lsum = fmaf(mg_l[w][h], wt, lsum);
                        acc = fmaf(mg_o[w][h][d], wt, acc);
                    }
                }
                const size_t slot = ((size_t)un.m * nq + un.g * G + h) * nsplit + un.b;
                part_o[slot * kHD + d] = acc;
                if (d == 0) {
                    part_ml[slot * 2] = Mx;
                    part_ml[slot * 2 + 1] = lsum;
                }
            }
        }
        __syncthreads();  // the merge area is free for the next unit
    }
    if (!ok) {
        if ((threadIdx.x & 31) == 0) atomicExch(err, 1);
        // requested chunks [kout, kin) may still be landing in the ring: wait
        // for them (again bounded) before the CTA exits
        if (threadIdx.x == 0) {
            for (int kk = kout; kk < kin; kk++) {
                const uint32_t bar = smem_addr(&full[kk % kBlkStages]), par = (uint32_t)((kk / kBlkStages) & 1);
                uint32_t done = 0;
                for (long long it = 0; !done && it <= kBlkWaitLimit; it++)
                    asm volatile(
                        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, "
                        "1, 0, p;\n}\n"
                        : "=r"(done)
                        : "r"(bar), "r"(par)
                        : "memory");
            }
        }
    }
}

}  // namespace

extern "C" int b2_attention_blocks_split(int max_seq, int block) {
    return block > 0 && block % kBlkChunk == 0 ? (max_seq + block - 1) / block : -1;
}

extern "C" int b2_attention_blocks(float* out, uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv,
                                   int hd, const B2KVRef* kv, void* work, int block, int* err, b2_stream_t s) {
    if (M <= 0) return 0;
    if (hd != kHD) return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention_blocks: head_dim %d != 128", hd);
    if ((!out && !out16) || !q || !kv || !kv->pos || !work || !err || nkv <= 0 || nq % nkv != 0 ||
        block <= 0 || block % kBlkChunk != 0 || kv->max_seq <= 0 || kv->n_seqs <= 0 || M > kBlkMaxRows ||
        (reinterpret_cast<uintptr_t>(kv->k_base) & 15) || (reinterpret_cast<uintptr_t>(kv->v_base) & 15) ||
        kv->seq_stride % kHD || kv->layer_stride % kHD)
        return b2_set_error(B2_ERR_INVALID_ARG,
                            "b2_attention_blocks: bad arguments (block %% %d, M <= %d, 16-byte caches, strides %% 128)",
                            kBlkChunk, kBlkMaxRows);
    const int nsplit = (kv->max_seq + block - 1) / block;
    // rows of 128 dims the caches span for these rows (reads past it are zero-filled)
    const long long rows = ((long long)(kv->n_seqs - 1) * kv->seq_stride + (long long)kv->layer * kv->layer_stride +
                            (long long)nkv * kv->max_seq * kHD) / kHD;
    if (rows >= (1ll << 31)) return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention_blocks: cache too large");
    CUtensorMap tk, tv;
    int rc = b2_tensor_map_f16(&tk, kv->k_base, kHD, (uint64_t)rows, kHD * 2, 64, 64);
    if (!rc) rc = b2_tensor_map_f16(&tv, kv->v_base, kHD, (uint64_t)rows, kHD * 2, 64, 64);
    if (rc) return rc;
    float* part_ml = reinterpret_cast<float*>(work);
    float* part_o = part_ml + (size_t)M * nq * nsplit * 2;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    dim3 grid(2 * sms);  // two CTAs per SM; each walks its share of the units
    cudaStream_t st = (cudaStream_t)s;
    constexpr size_t smem = (size_t)kBlkStages * kBlkStageBytes + 1024;
    cudaError_t e = cudaSuccess;
    {  // more than the default 48 KB of dynamic shared memory: opt in once per device
        static bool set[8] = {};
        if (!set[dev & 7]) {
            e = cudaFuncSetAttribute(attn_block_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(attn_block_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(attn_block_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess)
                return b2_set_error(B2_ERR_CUDA, "b2_attention_blocks smem attr: %s", cudaGetErrorString(e));
            set[dev & 7] = true;
        }
    }
    switch (nq / nkv) {
        case 1: e = b2::launch_pdl(attn_block_kernel<1>, grid, dim3(kThreads), smem, st, tk, tv, q, ldq, M, nq, nkv, *kv, block, part_ml, part_o, nsplit, err); break;
        case 2: e = b2::launch_pdl(attn_block_kernel<2>, grid, dim3(kThreads), smem, st, tk, tv, q, ldq, M, nq, nkv, *kv, block, part_ml, part_o, nsplit, err); break;
        case 4: e = b2::launch_pdl(attn_block_kernel<4>, grid, dim3(kThreads), smem, st, tk, tv, q, ldq, M, nq, nkv, *kv, block, part_ml, part_o, nsplit, err); break;
        default: return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention_blocks: GQA group %d not in {1,2,4}", nq / nkv);
    }
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention_blocks: %s", cudaGetErrorString(e));
    e = b2::launch_pdl(attn_combine_kernel, dim3(nq, M), dim3(kHD), 0, st, out, reinterpret_cast<__half*>(out16), nq,
                       (const float*)part_ml, (const float*)part_o, nsplit, (const int*)kv->pos, block, kv->max_seq);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention_blocks combine: %s", cudaGetErrorString(e));
    return 0;
}

// ─── causal flash attention for batch prefill (b2_attention_prefill) ───
//
// attention_batch_causal_f32 (src/cpu_ops.c:459-571) for M consecutive rows
// of one sequence at positions base .. base + M - 1, whose K and V are
// already in the cache: row m attends positions [0, base + m].  One CTA takes
// 32 rows and the Gq q heads of one kv head (64 query rows for Gq = 2), four
// warps of 16 query rows.  Scores and P.V run on the tensor cores
// (mma.sync m16n8k16, FP16 operands, FP32 accumulation) in the register
// layout of FlashAttention-2 (Dao, 2023): each warp owns whole query rows, so
// the online softmax needs only quad shuffles, and the score accumulators
// become the A operand of P.V without leaving registers.  Two groups of four
// warps own the same query rows and take alternate K/V blocks of 64 positions
// (even / odd), each double-buffering its blocks in shared memory with
// cp.async; at the end group 1 leaves its softmax state in shared memory and
// group 0 merges it.  The causal triangle gives the last rows 8 blocks at
// M = 512, so splitting them over two groups halves the longest CTA.  Rows
// are padded by 16 bytes so ldmatrix reads are conflict-free.  Q and P are
// rounded to FP16 (the reference keeps them FP32; the difference is far
// inside the parity tolerance, see the prefill tests).

namespace {

constexpr int kFaRows = 32;            // tokens per CTA
constexpr int kFaKv = 64;              // positions per K/V block
constexpr int kFaPad = kHD + 8;        // padded row (halves)
constexpr int kFaGroups = 2;           // warp groups splitting the K/V blocks
constexpr int kFaThreads = 128 * kFaGroups;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

template <int G>
__global__ void __launch_bounds__(kFaThreads) flash_prefill_kernel(float* __restrict__ out, __half* __restrict__ out16,
                                                                   const float* __restrict__ q, int ldq, int M, int nq,
                                                                   B2KVRef kv, int base) {
    static_assert(G * kFaRows == 64, "four warps of 16 query rows per group");
    extern __shared__ __align__(16) unsigned char fsm[];
    __half* sq = reinterpret_cast<__half*>(fsm);                 // [64][kFaPad]
    const int tid = threadIdx.x, lane = tid & 31, grp = tid >> 7, gtid = tid & 127, warp = (tid >> 5) & 3;
    // this group's [2 buffers][K, V][kFaKv][kFaPad]
    __half* skv = sq + 64 * kFaPad + (size_t)grp * 4 * kFaKv * kFaPad;
    const int m0 = blockIdx.x * kFaRows, g = blockIdx.y;
    const int last = base + M - 1;                                // last filled cache position
    const int pmax = min(last, base + m0 + kFaRows - 1);          // last position any row of the CTA attends
    const size_t head_off = kv.layer * kv.layer_stride + (size_t)g * kv.max_seq * kHD;
    const __half* kg = reinterpret_cast<const __half*>(kv.k_base + head_off);
    const __half* vg = reinterpret_cast<const __half*>(kv.v_base + head_off);
    b2::pdl_trigger();
    b2::pdl_wait();

    // Q rows: r = h * 32 + t (q head g*G + h, token m0 + t), FP16
    for (int i = tid; i < 64 * (kHD / 4); i += kFaThreads) {
        const int r = i / (kHD / 4), c = (i % (kHD / 4)) * 4;
        const int h = r / kFaRows, t = r % kFaRows, m = min(m0 + t, M - 1);
        const float4 x = *reinterpret_cast<const float4*>(q + (size_t)m * ldq + (size_t)(g * G + h) * kHD + c);
        uint2 hv;
        hv.x = pack_h2(x.x, x.y);
        hv.y = pack_h2(x.z, x.w);
        *reinterpret_cast<uint2*>(sq + r * kFaPad + c) = hv;
    }
    const int nblk = pmax / kFaKv + 1;
    auto load_block = [&](int blk, int buf) {
        __half* dk = skv + (size_t)buf * 2 * kFaKv * kFaPad;
        __half* dv = dk + kFaKv * kFaPad;
        for (int i = gtid; i < kFaKv * (kHD / 8); i += 128) {
            const int r = i / (kHD / 8), c = (i % (kHD / 8)) * 8;
            const int p = min(blk * kFaKv + r, pmax);  // rows past pmax repeat it (masked below)
            cp_async16(dk + r * kFaPad + c, kg + (size_t)p * kHD + c);
            cp_async16(dv + r * kFaPad + c, vg + (size_t)p * kHD + c);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto group_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory"); };
    if (grp < nblk) load_block(grp, 0);
    __syncthreads();  // Q rows staged for both groups

    const int g8 = lane >> 2, q4 = lane & 3;
    // the two query rows of this lane: warp rows 16 warp + g8 and + 8
    const int rA = warp * 16 + g8, rB = rA + 8;
    const int posA = base + m0 + (rA % kFaRows), posB = base + m0 + (rB % kFaRows);
    const float scale = 1.0f / sqrtf((float)kHD);
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    float o[kHD / 8][4];
#pragma unroll
    for (int j = 0; j < kHD / 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int blk = grp, it = 0; blk < nblk; blk += kFaGroups, it++) {
        if (blk + kFaGroups < nblk) {
            load_block(blk + kFaGroups, (it + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        group_sync();
        const __half* sk = skv + (size_t)(it & 1) * 2 * kFaKv * kFaPad;
        const __half* sv = sk + kFaKv * kFaPad;
        // S = Q K^T for this warp's 16 rows x 64 positions
        float s[kFaKv / 8][4];
#pragma unroll
        for (int j = 0; j < kFaKv / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kHD / 16; kk++) {
            uint32_t a[4];
            {
                const int mi = lane >> 3, rr = warp * 16 + (mi & 1) * 8 + (lane & 7), cc = kk * 16 + (mi >> 1) * 8;
                ldsm_x4(a, sq + rr * kFaPad + cc);
            }
#pragma unroll
            for (int j = 0; j < kFaKv / 8; j += 2) {
                // B fragments of position tiles j and j + 1: K rows, columns kk*16 .. +15
                uint32_t b[4];
                const int mi = lane >> 3, pr = (j + (mi >> 1)) * 8 + (lane & 7), cc = kk * 16 + (mi & 1) * 8;
                ldsm_x4(b, sk + pr * kFaPad + cc);
                mma_f16(s[j], a, b[0], b[1]);
                mma_f16(s[j + 1], a, b[2], b[3]);
            }
        }
        // online softmax (rows rA: c0, c1; rB: c2, c3)
        float mxA = mA, mxB = mB;
#pragma unroll
        for (int j = 0; j < kFaKv / 8; j++) {
            const int p = blk * kFaKv + j * 8 + 2 * q4;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                s[j][e] = p + e <= posA ? s[j][e] * scale : -INFINITY;
                s[j][2 + e] = p + e <= posB ? s[j][2 + e] * scale : -INFINITY;
                mxA = fmaxf(mxA, s[j][e]);
                mxB = fmaxf(mxB, s[j][2 + e]);
            }
        }
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
        const float cA = mA == -INFINITY ? 0.f : expf(mA - mxA), cB = mB == -INFINITY ? 0.f : expf(mB - mxB);
        mA = mxA;
        mB = mxB;
        float sumA = 0.f, sumB = 0.f;
        uint32_t pa[kFaKv / 8][2];  // P as FP16 pairs: [tile][row A / row B]
#pragma unroll
        for (int j = 0; j < kFaKv / 8; j++) {
            const float p0 = mxA == -INFINITY ? 0.f : expf(s[j][0] - mxA);
            const float p1 = mxA == -INFINITY ? 0.f : expf(s[j][1] - mxA);
            const float p2 = mxB == -INFINITY ? 0.f : expf(s[j][2] - mxB);
            const float p3 = mxB == -INFINITY ? 0.f : expf(s[j][3] - mxB);
            sumA += p0 + p1;
            sumB += p2 + p3;
            pa[j][0] = pack_h2(p0, p1);
            pa[j][1] = pack_h2(p2, p3);
        }
        sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
        sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
        sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
        sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
        lA = lA * cA + sumA;
        lB = lB * cB + sumB;
#pragma unroll
        for (int j = 0; j < kHD / 8; j++) {
            o[j][0] *= cA;
            o[j][1] *= cA;
            o[j][2] *= cB;
            o[j][3] *= cB;
        }
        // O += P V: k = positions (16 per step), n = head dims
#pragma unroll
        for (int kk = 0; kk < kFaKv / 16; kk++) {
            const uint32_t a[4] = {pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1]};
#pragma unroll
            for (int j = 0; j < kHD / 8; j += 2) {
                // V rows kk*16 .. +15 (positions), columns of dim tiles j and j + 1, transposed
                uint32_t b[4];
                const int mi = lane >> 3, pr = kk * 16 + (mi & 1) * 8 + (lane & 7), cc = (j + (mi >> 1)) * 8;
                ldsm_x4_t(b, sv + pr * kFaPad + cc);
                mma_f16(o[j], a, b[0], b[1]);
                mma_f16(o[j + 1], a, b[2], b[3]);
            }
        }
        group_sync();  // the buffer is refilled two blocks later
    }
    // group 1 hands its state to group 0 through its (now idle) K/V buffers:
    // [warp][lane][mA, mB, lA, lB, o[16][4]]
    constexpr int kSt = 4 + 4 * (kHD / 8);
    float* st = reinterpret_cast<float*>(sq + 64 * kFaPad + 4 * kFaKv * kFaPad) + (size_t)(warp * 32 + lane) * kSt;
    if (grp == 1) {
        st[0] = mA, st[1] = mB, st[2] = lA, st[3] = lB;
#pragma unroll
        for (int j = 0; j < kHD / 8; j++)
            *reinterpret_cast<float4*>(st + 4 + 4 * j) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
    }
    __syncthreads();
    if (grp == 1) return;
    {
        const float m1A = st[0], m1B = st[1], l1A = st[2], l1B = st[3];
        const float nA = fmaxf(mA, m1A), nB = fmaxf(mB, m1B);
        const float a0 = mA == -INFINITY ? 0.f : expf(mA - nA), a1 = m1A == -INFINITY ? 0.f : expf(m1A - nA);
        const float b0 = mB == -INFINITY ? 0.f : expf(mB - nB), b1 = m1B == -INFINITY ? 0.f : expf(m1B - nB);
        lA = lA * a0 + l1A * a1;
        lB = lB * b0 + l1B * b1;
#pragma unroll
        for (int j = 0; j < kHD / 8; j++) {
            const float4 u = *reinterpret_cast<const float4*>(st + 4 + 4 * j);
            o[j][0] = o[j][0] * a0 + u.x * a1;
            o[j][1] = o[j][1] * a0 + u.y * a1;
            o[j][2] = o[j][2] * b0 + u.z * b1;
            o[j][3] = o[j][3] * b0 + u.w * b1;
        }
    }
    // out[m][(g*G + h) * 128 + d] = O / l
    const int tA = rA % kFaRows, tB = rB % kFaRows;
    const int hA = rA / kFaRows, hB = rB / kFaRows;
    const float iA = 1.0f / lA, iB = 1.0f / lB;
#pragma unroll
    for (int j = 0; j < kHD / 8; j++) {
        const int d = j * 8 + 2 * q4;
        const size_t oA = (size_t)(m0 + tA) * nq * kHD + (size_t)(g * G + hA) * kHD + d;
        const size_t oB = (size_t)(m0 + tB) * nq * kHD + (size_t)(g * G + hB) * kHD + d;
        if (out16) {  // FP16 rows for the o_proj GEMM
            if (m0 + tA < M) *reinterpret_cast<__half2*>(out16 + oA) = __floats2half2_rn(o[j][0] * iA, o[j][1] * iA);
            if (m0 + tB < M) *reinterpret_cast<__half2*>(out16 + oB) = __floats2half2_rn(o[j][2] * iB, o[j][3] * iB);
        } else {
            if (m0 + tA < M) *reinterpret_cast<float2*>(out + oA) = make_float2(o[j][0] * iA, o[j][1] * iA);
            if (m0 + tB < M) *reinterpret_cast<float2*>(out + oB) = make_float2(o[j][2] * iB, o[j][3] * iB);
        }
    }
}

}  // namespace

extern "C" int b2_attention_prefill(float* out, uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv,
                                    int hd, const B2KVRef* kv, int base, b2_stream_t s) {
    if (M <= 0) return 0;
    if (hd != kHD || (!out && !out16) || !q || !kv || nkv <= 0 || nq != 2 * nkv || base < 0 || base + M > kv->max_seq ||
        ldq % 4 || kv->rows_seq)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention_prefill: needs hd 128, GQA group 2, one sequence");
    const size_t smem = (size_t)(64 + 4 * kFaGroups * kFaKv) * kFaPad * sizeof(__half);
    static int configured = 0;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(flash_prefill_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "flash prefill smem: %s", cudaGetErrorString(e));
        configured = 1;
    }
    const dim3 grid((M + kFaRows - 1) / kFaRows, nkv);
    cudaError_t e = b2::launch_pdl(flash_prefill_kernel<2>, grid, dim3(kFaThreads), smem, (cudaStream_t)s, out,
                                   reinterpret_cast<__half*>(out16), q, ldq, M, nq, *kv, base);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention_prefill: %s", cudaGetErrorString(e));
    return 0;
}
