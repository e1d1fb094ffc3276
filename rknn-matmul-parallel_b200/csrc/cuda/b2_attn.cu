// GQA attention over the FP16 KV cache (b2_attention).
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

__global__ void __launch_bounds__(kHD) attn_combine_kernel(float* __restrict__ out, __half* __restrict__ out16,
                                                           int nq, const float* __restrict__ part_ml,
                                                           const float* __restrict__ part_o, int nsplit) {
    b2::pdl_trigger();
    b2::pdl_wait();
    const int h = blockIdx.x, m = blockIdx.y, d = threadIdx.x;
    const size_t base = ((size_t)m * nq + h) * nsplit;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, part_ml[(base + s) * 2]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; s++) {
        const float ms = part_ml[(base + s) * 2];
        if (ms == -INFINITY) continue;
        const float w = expf(ms - M);
        den = fmaf(part_ml[(base + s) * 2 + 1], w, den);
        num = fmaf(part_o[(base + s) * kHD + d], w, num);
    }
    if (out16) out16[((size_t)m * nq + h) * kHD + d] = __float2half_rn(num / den);
    else out[((size_t)m * nq + h) * kHD + d] = num / den;
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
                       (const float*)part_o, nsplit);
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
// become the A operand of P.V without leaving registers.  K and V blocks of 64
// positions are double-buffered in shared memory with cp.async; rows are
// padded by 16 bytes so ldmatrix reads are conflict-free.  Q and P are
// rounded to FP16 (the reference keeps them FP32; the difference is far
// inside the parity tolerance, see the prefill tests).

namespace {

constexpr int kFaRows = 32;            // tokens per CTA
constexpr int kFaKv = 64;              // positions per K/V block
constexpr int kFaPad = kHD + 8;        // padded row (halves)
constexpr int kFaThreads = 128;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int G>
__global__ void __launch_bounds__(kFaThreads) flash_prefill_kernel(float* __restrict__ out, __half* __restrict__ out16,
                                                                   const float* __restrict__ q, int ldq, int M, int nq,
                                                                   B2KVRef kv, int base) {
    static_assert(G * kFaRows == 64, "four warps of 16 query rows");
    extern __shared__ __align__(16) unsigned char fsm[];
    __half* sq = reinterpret_cast<__half*>(fsm);                 // [64][kFaPad]
    __half* skv = sq + 64 * kFaPad;                               // [2 buffers][K, V][kFaKv][kFaPad]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
        for (int i = tid; i < kFaKv * (kHD / 8); i += kFaThreads) {
            const int r = i / (kHD / 8), c = (i % (kHD / 8)) * 8;
            const int p = min(blk * kFaKv + r, pmax);  // rows past pmax repeat it (masked below)
            cp_async16(dk + r * kFaPad + c, kg + (size_t)p * kHD + c);
            cp_async16(dv + r * kFaPad + c, vg + (size_t)p * kHD + c);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_block(0, 0);

    const int g8 = lane >> 2, q4 = lane & 3;
    // the two query rows of this lane: warp rows 16 warp + g8 and + 8
    const int rA = warp * 16 + g8, rB = rA + 8;
    const int posA = base + m0 + (rA % kFaRows), posB = base + m0 + (rB % kFaRows);
    const float scale = 1.0f / sqrtf((float)kHD);
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    float o[kHD / 8][4];
#pragma unroll
    for (int j = 0; j < kHD / 8; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int blk = 0; blk < nblk; blk++) {
        if (blk + 1 < nblk) {
            load_block(blk + 1, (blk + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const __half* sk = skv + (size_t)(blk & 1) * 2 * kFaKv * kFaPad;
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
        __syncthreads();  // the buffer is refilled two blocks later
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
    const size_t smem = (size_t)(64 + 4 * kFaKv) * kFaPad * sizeof(__half);
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
