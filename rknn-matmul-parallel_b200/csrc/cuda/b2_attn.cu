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

__global__ void __launch_bounds__(kHD) attn_combine_kernel(float* __restrict__ out, int nq,
                                                           const float* __restrict__ part_ml,
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
    out[((size_t)m * nq + h) * kHD + d] = num / den;
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

extern "C" int b2_attention(float* out, const float* q, int ldq, int M, int nq, int nkv, int hd,
                            const B2KVRef* kv, void* work, int nsplit, b2_stream_t s) {
    if (M <= 0) return 0;
    if (hd != kHD) return b2_set_error(B2_ERR_INVALID_ARG, "b2_attention: head_dim %d != 128", hd);
    if (!out || !q || !kv || !kv->pos || !work || nkv <= 0 || nq % nkv != 0)
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
    e = b2::launch_pdl(attn_combine_kernel, dim3(nq, M), dim3(kHD), 0, st, out, nq, (const float*)part_ml,
                       (const float*)part_o, nsplit);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_attention combine: %s", cudaGetErrorString(e));
    return 0;
}
