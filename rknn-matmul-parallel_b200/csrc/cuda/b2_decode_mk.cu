// Persistent single-token decode kernel (b2_mk_decode).
//
// One cooperative launch runs a whole matmul_decoder_step
// (src/matmul_decoder.c:1430-1634 of suharvest/rknn-matmul-parallel): the
// embedding row, every layer's RMSNorm / q|k|v / per-head q,k norm / RoPE /
// KV append / GQA attention / o_proj + residual / RMSNorm / gate|up SiLU /
// down + residual, then optionally the final RMSNorm, the INT8 lm_head and
// the argmax.  Numerics are those of the multi-kernel path (b2_gemv,
// b2_qk_rope_kv, b2_attention, b2_lm_head_argmax).
//
// Why one kernel: a decode token is ~0.6-1.05 GB of weights spread over 28
// short dependent phases; with one launch per phase the boundaries, not HBM,
// set the time.  Here every CTA (one per SM) owns a fixed slice of every
// phase: a row range of each projection, a (kv head, position range) unit of
// attention and a row range of the lm_head.  Warp 8 of each CTA is a producer
// that streams the CTA's weight rows for the whole token — and the K/V rows
// written by earlier steps — through a ring of shared-memory stages with
// cp.async.bulk + mbarrier transaction counts.  It never waits for another
// CTA, so HBM streaming continues while the consumer warps 0-7 wait on the
// dependency chain.  The consumers order the phases with device-scope
// acquire/release counters in global memory:
//
//   QKV(l)   waits DOWN(l-1) of every CTA      signals QKV(l)[kv group] += rows
//   ATTN(l)  waits QKV(l)[its group]           last unit of a group combines the
//                                              split partials, signals ATTN_DONE(l)
//   O(l)     waits ATTN_DONE(l) == nkv         signals O(l)
//   GU(l)    waits O(l) of every CTA           signals GU(l)
//   DOWN(l)  waits GU(l) of every CTA          signals DOWN(l)
//   LM       waits DOWN(L-1) of every CTA      atomicMax of (value, ~index) keys
//   FIN      last CTA to arrive publishes the token and advances the state
//
// Counters grow monotonically by a fixed amount per step; a wait's target is
// (amount) x (generation + 1), where the generation (state[B2_MK_GEN]) counts
// completed launches.  Every wait is bounded: on timeout the CTA sets
// state[B2_MK_ERR], stops, lets its in-flight copies land and returns.
#include "b2_common.cuh"

namespace {

constexpr int kCWarps = 8;
constexpr int kConsumers = kCWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kStages = 3;
constexpr int kStageBytes = 64 * 1024;
constexpr int kHD = 128;
constexpr int kMaxK = 3072;        // longest staged activation (hidden, q_dim, ffn)
constexpr int kV = kMaxK / (4 * kConsumers);  // float4 groups of a staged vector per consumer thread
// Copies of each layer-output accumulator: CTA c adds its down partial into
// copy c % kOutCopies and readers sum the copies, so each address takes
// G / kOutCopies atomic adds instead of G (the adds of all CTAs land on the
// same H addresses; fewer per address finish sooner).
constexpr int kOutCopies = 4;
constexpr int kMaxSplit = 32;      // attention position ranges per kv head
constexpr int kMaxGq = 2;          // q heads per kv head handled by one attention unit
constexpr int kScCap = 1040;       // per-item scales prefetched into shared memory
constexpr int kResCap = 64;        // per-item residual rows prefetched into shared memory
constexpr long long kPollLimit = 1ll << 22;
constexpr long long kBarLimit = 1ll << 22;

enum { IT_QKV, IT_ATTN, IT_O, IT_GU, IT_DN, IT_LM, IT_DNT, IT_AO, IT_OSEG };
constexpr int kFuseL = 256;   // contexts up to which attention and o_proj run as one phase
constexpr int kActCap = 64;   // gate|up channels per CTA (the down partial's inputs)

// Vectors passed between CTAs are "LL" words (the low-latency protocol of
// NCCL's LL transport): one 64-bit store holds an FP32 value in the low half
// and the step's generation tag in the high half.  A reader polls the words
// it needs until every tag is this step's, so producers need no fence and no
// flag, and a consumer starts as soon as its own inputs have landed.
struct Scratch {
    unsigned long long* cnt;   // [8 + 2L]: [0] CTAs finished, [1] best argmax key, [8 + l] down partials of
                               // layer l, [8 + L + l] attention + o_proj units of layer l
    float* hacc;               // [L][2][kOutCopies][H] layer outputs, summed from down partials (two token
                               // parities; a layer output is the sum of its copies)
    float* macc;               // [L][2][H] hidden after attention, summed from o_proj partials (fused phase)
    unsigned long long* hbuf;  // LL [L+1][H] layer inputs (row 0 unused: layer 0 reads the embedding)
    unsigned long long* hmid;  // LL [L][H] hidden after attention + residual
    unsigned long long* qkv;   // LL [L][qd + 2 kvd]
    unsigned long long* part;  // LL [L][nkv][kMaxSplit][Gq][2 + hd] attention partials (m, l, o[hd])
    unsigned long long* act;   // LL [L][F] SiLU(gate) * up
    float* hfinal;             // [H] final hidden state (plain FP32, read by the host)
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline Scratch scratch_layout(void* base, int L, int H, int F, int nq, int nkv, int hd,
                                                  size_t* total) {
    unsigned char* p = static_cast<unsigned char*>(base);
    size_t off = 0;
    Scratch s;
    const size_t qd = (size_t)nq * hd, kvd = (size_t)nkv * hd;
    auto take = [&](size_t bytes) {
        unsigned char* r = p + off;
        off += align256(bytes);
        return r;
    };
    s.cnt = reinterpret_cast<unsigned long long*>(take((size_t)(8 + 2 * L) * 8));
    s.hacc = reinterpret_cast<float*>(take((size_t)L * 2 * kOutCopies * H * 4));
    s.macc = reinterpret_cast<float*>(take((size_t)L * 2 * H * 4));
    s.hbuf = reinterpret_cast<unsigned long long*>(take((size_t)(L + 1) * H * 8));
    s.hmid = reinterpret_cast<unsigned long long*>(take((size_t)L * H * 8));
    s.qkv = reinterpret_cast<unsigned long long*>(take((size_t)L * (qd + 2 * kvd) * 8));
    s.part = reinterpret_cast<unsigned long long*>(take((size_t)L * nkv * kMaxSplit * (nq / nkv) * (2 + hd) * 8));
    s.act = reinterpret_cast<unsigned long long*>(take((size_t)L * F * 8));
    s.hfinal = reinterpret_cast<float*>(take((size_t)H * 4));
    if (total) *total = off;
    return s;
}

// ─── small PTX helpers ───

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
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

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory; completion is counted
// on `bar` in bytes.  Addresses and size are multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ unsigned long long atom_add_acqrel(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Four FP32 additions into global memory in one request.
__device__ __forceinline__ void red_add_v4(float* p, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Barrier over the 256 consumer threads that also returns the AND of `pred`
// across them, so every consumer takes the same branch afterwards.
__device__ __forceinline__ bool consumer_all(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.and.pred po, 1, 256, pi;\n"
        " selp.u32 %0, 1, 0, po;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

// ── LL words ──
__device__ __forceinline__ void ll_put(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_get(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Two adjacent words (16-byte aligned); each word is read atomically.
__device__ __forceinline__ ulonglong2 ll_get2(const unsigned long long* p) {
    ulonglong2 r;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ bool ll_ok(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// ─── dot products from shared memory ───

// ─── tensor-core row dots ───
//
// mma.m16n8k16 (FP16 operands, FP32 accumulation: every product is exact and
// the sum is FP32, the reference's matmul numerics) takes 16 weight rows at
// once: the rows are the A operand and the staged FP16 activation, repeated
// in all 8 columns, the B operand.  Each row is cut into 64-byte
// super-blocks; lane (g = lane / 4, q = lane % 4) feeds rows g and g + 8
// with the 16 bytes at offset 16 q of every super-block and takes the
// activation elements of the same k positions.  Inside a super-block the
// k order is permuted identically for A and B, which a dot product does
// not see.  Int8 and int4 weights widen to FP16 exactly with byte permutes
// (the value plus 1024 sits in the mantissa of 1024, one half2 subtraction
// removes the bias).

template <int WT>
__host__ __device__ constexpr int sb_k() {  // k positions per 64-byte super-block
    return WT == B2_W_F16 ? 32 : WT == B2_W_I8 ? 64 : 128;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// One super-block of rows g and g + 8 (wg, wh: this lane's 16 bytes of each)
// against this lane's activation words xw; consecutive steps alternate
// between two accumulators so neighbouring MMAs do not wait on each other.
template <int WT>
__device__ __forceinline__ void sb_mma(float (&d0)[4], float (&d1)[4], const uint4 wg, const uint4 wh,
                                       const uint32_t* xw) {
    const uint32_t* g = &wg.x;
    const uint32_t* h = &wh.x;
    if constexpr (WT == B2_W_F16) {
        mma16816(d0, g[0], h[0], g[1], h[1], xw[0], xw[1]);
        mma16816(d1, g[2], h[2], g[3], h[3], xw[2], xw[3]);
    } else if constexpr (WT == B2_W_I8) {
        const uint32_t bias = 0x64806480u;  // half2(1152, 1152) = 1024 + 128
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t ug = g[t] ^ 0x80808080u, uh = h[t] ^ 0x80808080u;
            const uint32_t glo = hsub2_u32(__byte_perm(ug, 0x64646464u, 0x4140), bias);
            const uint32_t ghi = hsub2_u32(__byte_perm(ug, 0x64646464u, 0x4342), bias);
            const uint32_t hlo = hsub2_u32(__byte_perm(uh, 0x64646464u, 0x4140), bias);
            const uint32_t hhi = hsub2_u32(__byte_perm(uh, 0x64646464u, 0x4342), bias);
            mma16816(t & 1 ? d1 : d0, glo, hlo, ghi, hhi, xw[2 * t], xw[2 * t + 1]);
        }
    } else {
        const uint32_t bias = 0x64086408u;  // half2(1032, 1032) = 1024 + 8
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t ug = g[t] ^ 0x88888888u, uh = h[t] ^ 0x88888888u;
            // word t holds k = 8t + i at nibble i; half2 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7)
            mma16816(d0, hsub2_u32((ug & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32((uh & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32(((ug >> 4) & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32(((uh >> 4) & 0x000F000Fu) | 0x64006400u, bias), xw[4 * t], xw[4 * t + 1]);
            mma16816(d1, hsub2_u32(((ug >> 8) & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32(((uh >> 8) & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32(((ug >> 12) & 0x000F000Fu) | 0x64006400u, bias),
                     hsub2_u32(((uh >> 12) & 0x000F000Fu) | 0x64006400u, bias), xw[4 * t + 2], xw[4 * t + 3]);
        }
    }
}

// Dots of rows rg (row g) and rh (row g + 8) over super-blocks [s0, s1)
// with the staged activation xs (FP16, in the k order sb_mma expects).
// Returns this lane's row-g sum in out[0] and row-(g+8) sum in out[1].
template <int WT>
__device__ __forceinline__ void tile_dot(const unsigned char* rg, const unsigned char* rh, const __half* xs,
                                         int s0, int s1, int lane, float (&out)[2]) {
    constexpr int XW = sb_k<WT>() / 8;  // activation words (half2) per lane per super-block
    const int q = lane & 3;
    // four accumulators (FP16 / INT8): consecutive super-blocks use different
    // pairs, so a warp's dependent MMA chains are a quarter of its MMAs long
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    float d2[4] = {0.f, 0.f, 0.f, 0.f}, d3[4] = {0.f, 0.f, 0.f, 0.f};
    auto step = [&](int sb, float (&da)[4], float (&db)[4]) {
        const uint4 wg = *reinterpret_cast<const uint4*>(rg + sb * 64 + q * 16);
        const uint4 wh = *reinterpret_cast<const uint4*>(rh + sb * 64 + q * 16);
        uint32_t xw[XW];
        const uint4* xp = reinterpret_cast<const uint4*>(xs + sb * sb_k<WT>() + q * (sb_k<WT>() / 4));
#pragma unroll
        for (int i = 0; i < XW / 4; i++) *reinterpret_cast<uint4*>(xw + 4 * i) = xp[i];
        sb_mma<WT>(da, db, wg, wh, xw);
    };
    int sb = s0;
    if constexpr (WT == B2_W_I4) {  // eight MMAs per super-block already; two accumulators keep registers
        for (; sb < s1; sb++) step(sb, d0, d1);
    } else {
        for (; sb + 1 < s1; sb += 2) {
            step(sb, d0, d1);
            step(sb + 1, d2, d3);
        }
        if (sb < s1) step(sb, d0, d1);
    }
    // all 8 columns hold the same sums: column 2q of rows g and g + 8
    out[0] = (d0[0] + d1[0]) + (d2[0] + d3[0]);
    out[1] = (d0[2] + d1[2]) + (d2[2] + d3[2]);
}

__host__ __device__ inline size_t row_bytes(int wtype, int K) {
    return wtype == B2_W_F16 ? (size_t)K * 2 : wtype == B2_W_I8 ? (size_t)K : (size_t)K / 2;
}

__device__ __forceinline__ int split_lo(int n, int parts, int i) { return (int)(((long long)n * i) / parts); }

// ─── the per-CTA schedule, shared by producer and consumers ───

struct Geo {
    int L, pos, S, G, cta, qd, kvd, nqkv, Gq;
    int R;  // fused attention + o_proj: o_proj row slices per kv head (0: split attention and o_proj)
};

struct Chunk {
    int type, l, a, b, g, s;
    const void* src0;
    uint32_t bytes0;
    const void* src1;
    uint32_t bytes1;
    uint32_t off1;
    int nseg = 0;            // > 0: nseg copies of bytes0 from src0 + i * seg_stride, packed
    uint32_t seg_stride = 0;
};

struct Item {
    int type, l, r0, r1, g, s, p0, p1;
};

// Visits, in order, every item of this CTA and the shared-memory chunks its
// weights arrive in.  Producer and consumers run the same walk, so the k-th
// chunk the producer fills is the k-th chunk the consumers read.
template <int WT, class V>
__device__ void walk(const B2MkPlan& p, const Geo& geo, V& v) {
    const int H = p.hidden, F = p.ffn;
    const size_t rb_h = row_bytes(WT, H), rb_q = row_bytes(WT, geo.qd), rb_f = row_bytes(WT, F);
    // rows per stage, at most 64 (four 16-row tensor-core tiles)
    const int cap_h = min(64, kStageBytes / (int)rb_h), cap_q = min(64, kStageBytes / (int)rb_q);
    const int cap_pair = min(32, kStageBytes / (2 * (int)rb_h));
    const int cap_t = min(64, kStageBytes / (int)rb_h);  // input-major down rows: H values each
    (void)rb_f;
    for (int l = 0; l < p.n_layers; l++) {
        const B2MkLayer& Lw = p.layers[l];
        if (v.stop()) return;
        {  // q|k|v rows
            Item it{IT_QKV, l, split_lo(geo.nqkv, geo.G, geo.cta), split_lo(geo.nqkv, geo.G, geo.cta + 1), 0, 0, 0, 0};
            v.begin(it);
            for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_h) {
                const int b = min(it.r1, a + cap_h);
                Chunk c{IT_QKV, l, a, b, 0, 0, (const unsigned char*)Lw.qkv + a * rb_h, (uint32_t)((b - a) * rb_h),
                        nullptr, 0, 0};
                v.chunk(c);
            }
            v.end(it);
        }
        if (geo.R > 0) {  // fused: unit (kv head g, o_proj rows [n0, n1)) = attention of g + its o_proj columns
            if (geo.cta < p.nkv * geo.R) {
                const int g = geo.cta / geo.R, r = geo.cta % geo.R;
                Item it{IT_AO, l, split_lo(H, geo.R, r), split_lo(H, geo.R, r + 1), g, r, 0, geo.L};
                v.begin(it);
                const size_t head = (size_t)l * p.layer_stride + (size_t)g * p.max_seq * kHD;
                for (int a = 0; a < geo.L - 1 && !v.stop(); a += kStageBytes / (4 * kHD)) {
                    const int b = min(geo.L - 1, a + kStageBytes / (4 * kHD));
                    const uint32_t bytes = (uint32_t)(b - a) * kHD * 2;
                    Chunk c{IT_ATTN, l, a, b, g, 0, p.k_cache + head + (size_t)a * kHD, bytes,
                            p.v_cache + head + (size_t)a * kHD, bytes, bytes};
                    v.chunk(c);
                }
                v.mid(it);
                // o_proj rows n0..n1, only the columns of kv head g's q heads
                const uint32_t seg = (uint32_t)row_bytes(WT, geo.Gq * kHD);
                const int cap = min(64, kStageBytes / (int)seg);
                for (int a = it.r0; a < it.r1 && !v.stop(); a += cap) {
                    const int b = min(it.r1, a + cap);
                    Chunk c{IT_OSEG, l, a, b, g, 0, (const unsigned char*)Lw.o + a * rb_q + (size_t)g * seg, seg,
                            nullptr, 0, 0, b - a, (uint32_t)rb_q};
                    v.chunk(c);
                }
                v.end(it);
            }
        } else {
            for (int u = geo.cta; u < p.nkv * geo.S && !v.stop(); u += geo.G) {  // attention units
                const int g = u / geo.S, s = u % geo.S;
                const int chunk = (geo.L + geo.S - 1) / geo.S;
                const int p0 = min(geo.L, s * chunk), p1 = min(geo.L, p0 + chunk);
                const int pc = min(p1, geo.L - 1);  // positions cached by earlier steps
                Item it{IT_ATTN, l, 0, 0, g, s, p0, p1};
                v.begin(it);
                const size_t head = (size_t)l * p.layer_stride + (size_t)g * p.max_seq * kHD;
                for (int a = p0; a < pc && !v.stop(); a += kStageBytes / (4 * kHD)) {
                    const int b = min(pc, a + kStageBytes / (4 * kHD));
                    const uint32_t bytes = (uint32_t)(b - a) * kHD * 2;
                    Chunk c{IT_ATTN, l, a, b, g, s, p.k_cache + head + (size_t)a * kHD, bytes,
                            p.v_cache + head + (size_t)a * kHD, bytes, bytes};
                    v.chunk(c);
                }
                v.end(it);
            }
            if (v.stop()) return;
            {  // o_proj rows
                Item it{IT_O, l, split_lo(H, geo.G, geo.cta), split_lo(H, geo.G, geo.cta + 1), 0, 0, 0, 0};
                v.begin(it);
                for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_q) {
                    const int b = min(it.r1, a + cap_q);
                    Chunk c{IT_O, l, a, b, 0, 0, (const unsigned char*)Lw.o + a * rb_q, (uint32_t)((b - a) * rb_q),
                            nullptr, 0, 0};
                    v.chunk(c);
                }
                v.end(it);
            }
            if (v.stop()) return;
        }
        if (v.stop()) return;
        {  // gate|up channel pairs, then the same channels' rows of the input-major down weight
            Item it{IT_GU, l, split_lo(F, geo.G, geo.cta), split_lo(F, geo.G, geo.cta + 1), 0, 0, 0, 0};
            v.begin(it);
            for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_pair) {
                const int b = min(it.r1, a + cap_pair);
                const uint32_t bytes = (uint32_t)((b - a) * rb_h);
                Chunk c{IT_GU, l, a, b, 0, 0, (const unsigned char*)Lw.gu + a * rb_h, bytes,
                        (const unsigned char*)Lw.gu + (size_t)(F + a) * rb_h, bytes, bytes};
                v.chunk(c);
            }
            for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_t) {
                const int b = min(it.r1, a + cap_t);
                Chunk c{IT_DNT, l, a, b, 0, 0, (const unsigned char*)Lw.dn_t + (size_t)a * rb_h,
                        (uint32_t)((b - a) * rb_h), nullptr, 0, 0};
                v.chunk(c);
            }
            v.end(it);
        }
    }
    if (p.do_lm && !v.stop()) {
        Item it{IT_LM, p.n_layers, split_lo(p.vocab, geo.G, geo.cta), split_lo(p.vocab, geo.G, geo.cta + 1), 0, 0,
                0, 0};
        v.begin(it);
        const int cap = min(64, kStageBytes / H);  // int8 rows
        for (int a = it.r0; a < it.r1 && !v.stop(); a += cap) {
            const int b = min(it.r1, a + cap);
            Chunk c{IT_LM, p.n_layers, a, b, 0, 0, (const unsigned char*)p.lm + (size_t)a * H,
                    (uint32_t)((b - a) * H), nullptr, 0, 0};
            v.chunk(c);
        }
        v.end(it);
    }
}

struct Shared {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    int abort;                  // set by the producer (or a consumer) to stop the CTA
    int cabort;                 // consumers gave up (read by the producer)
    int issued, consumed;
    float red[kCWarps];
    unsigned long long best[kCWarps];
    float q[kMaxGq][kHD];                  // normalized + rotated q heads of the group
    float k[kHD], v[kHD];                  // new k (rotated) and v of the kv head
    float gm[kCWarps][kMaxGq], gl[kCWarps][kMaxGq];  // per-warp softmax state
    float go[kCWarps][kMaxGq][kHD];                   // per-warp partial outputs
    float pr[kCWarps][16];      // per-warp partial row sums of a chunk
    float act[kActCap];         // FP16-rounded SiLU(gate) * up of this CTA's channels
    float sc[2][kScCap];        // prefetched scales of the current / next item
    float res[2][kResCap];      // prefetched residual rows of the current / next item
};

__device__ __forceinline__ void set_error(const B2MkPlan& p, Shared& sh, int code) {
    sh.abort = 1;
    atomicOr(p.state + B2_MK_ERR, code);
}

// ─── producer ───

template <int WT>
struct Producer {
    const B2MkPlan& p;
    Shared& sh;
    unsigned char* ring;
    int n = 0;
    bool dead = false;
    __device__ bool stop() const {
        return dead || *(volatile const int*)&sh.abort || *(volatile const int*)&sh.cabort;
    }
    __device__ void begin(const Item&) {}
    __device__ void mid(const Item&) {}
    __device__ void end(const Item&) {}
    __device__ void chunk(const Chunk& c) {
        const int stage = n % kStages;
        if (n >= kStages) {  // wait until the consumers released this stage's previous fill
            const uint32_t parity = (uint32_t)((n / kStages - 1) & 1);
            long long it = 0;
            while (!mbar_try_wait(&sh.empty[stage], parity)) {
                if (*(volatile int*)&sh.abort || *(volatile int*)&sh.cabort) {
                    dead = true;
                    return;
                }
                if (++it > kBarLimit) {
                    set_error(p, sh, 2);
                    dead = true;
                    return;
                }
            }
        }
        unsigned char* dst = ring + (size_t)stage * kStageBytes;
        if (c.nseg > 0) {  // row segments, packed back to back
            mbar_expect_tx(&sh.full[stage], (uint32_t)c.nseg * c.bytes0);
            for (int i = 0; i < c.nseg; i++)
                bulk_g2s(dst + (size_t)i * c.bytes0, (const unsigned char*)c.src0 + (size_t)i * c.seg_stride, c.bytes0,
                         &sh.full[stage]);
        } else {
            mbar_expect_tx(&sh.full[stage], c.bytes0 + c.bytes1);
            bulk_g2s(dst, c.src0, c.bytes0, &sh.full[stage]);
            if (c.bytes1) bulk_g2s(dst + c.off1, c.src1, c.bytes1, &sh.full[stage]);
        }
        n++;
        *(volatile int*)&sh.issued = n;
    }
};

// ─── consumers ───

template <int WT>
struct Consumer {
    const B2MkPlan& p;
    const Geo& geo;
    Shared& sh;
    unsigned char* ring;
    __half* xs;
    const Scratch& S;
    uint32_t tag;  // generation tag of this step's LL words
    const float* emb_row;
    int tid, lane, warp;
    int n = 0;       // chunks consumed
    int items = 0;   // items begun; its parity selects the prefetch buffers
    int buf = 0, r0 = 0, nrows = 0;  // current item: prefetch buffer, first row, row count
    const float* isc = nullptr;       // current item's scale array (null: FP16 weights)
    float dacc_[4];                   // down partial of outputs 4 tid .. 4 tid + 3 (gate|up item)
    float4 res4_;                     // CTA 0: hmid at those outputs (the residual it adds)
    // attention state of this thread's lane group (positions of group grp)
    float m_[kMaxGq], l_[kMaxGq], o_[kMaxGq][16], qv_[kMaxGq][16];
    unsigned long long best = 0ull;
    bool aborted = false;  // identical in every consumer thread (set only at barriers)

    __device__ bool stop() const { return aborted; }

    __device__ bool abort_seen() const {
        return *(volatile int*)&sh.abort || *(volatile const int*)(p.state + B2_MK_ERR);
    }

    // Every consumer votes; a failed wait anywhere stops the whole CTA.
    __device__ void settle(bool ok) {
        if (consumer_all(ok)) return;
        if (tid == 0) {
            sh.cabort = 1;
            atomicOr(p.state + B2_MK_ERR, 1);
        }
        aborted = true;
    }

    // Bounded poll of one LL word.
    __device__ bool ll_wait(const unsigned long long* w, float& out) const {
        for (long long it = 0;; it++) {
            const unsigned long long v = ll_get(w);
            if (ll_ok(v, tag)) {
                out = ll_val(v);
                return true;
            }
            if (it > kPollLimit || ((it & 63) == 63 && abort_seen())) return false;
            __nanosleep(64);
        }
    }

    // Lane 0 polls one word until it carries the tag; the lanes wait for it
    // with the warp.  Only one request per warp and round reaches the L2
    // (148 CTAs x 256 threads polling the same lines would congest it).
    __device__ bool warp_lead_wait(const unsigned long long* w, bool has_word) const {
        bool ok = true;
        if (lane == 0 && has_word) {
            for (long long it = 0;; it++) {
                if (ll_ok(ll_get(w), tag)) break;
                if (it > kPollLimit || ((it & 63) == 63 && abort_seen())) {
                    ok = false;
                    break;
                }
                __nanosleep(96);
            }
        }
        return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }

    // This thread's float4 groups q = tid + j * kConsumers (elements 4q..4q+3)
    // of the LL vector src[0..K), polled until every word carries the tag.
    // The warp's first word gates the first read; writers of neighbouring
    // rows finish together, so the rest is almost always already there.
    __device__ bool ll_gather(const unsigned long long* src, int K, float4 (&v)[kV]) const {
        if (!warp_lead_wait(src + (size_t)(warp * 32) * 4, warp * 32 * 4 < K)) return false;
        unsigned pending = 0;
#pragma unroll
        for (int j = 0; j < kV; j++)
            if ((tid + j * kConsumers) * 4 < K) pending |= 1u << j;
        for (long long it = 0; pending; it++) {
#pragma unroll
            for (int j = 0; j < kV; j++) {
                if (!((pending >> j) & 1)) continue;
                const unsigned long long* w = src + (size_t)(tid + j * kConsumers) * 4;
                const ulonglong2 a = ll_get2(w), b = ll_get2(w + 2);
                if (ll_ok(a.x, tag) && ll_ok(a.y, tag) && ll_ok(b.x, tag) && ll_ok(b.y, tag)) {
                    v[j] = make_float4(ll_val(a.x), ll_val(a.y), ll_val(b.x), ll_val(b.y));
                    pending &= ~(1u << j);
                }
            }
            if (!pending) break;
            if (it > kPollLimit || ((it & 63) == 63 && abort_seen())) return false;
            __nanosleep(128);
        }
        return true;
    }

    // Consumer 0 waits until *cnt >= want (bounded); the decision reaches every
    // consumer through the barrier, and the barrier orders their reads of the
    // data the counter publishes after consumer 0's acquire.
    __device__ void wait_counter(const unsigned long long* cnt, unsigned long long want) {
        if (tid == 0) {
            for (long long it = 0; ld_acquire(cnt) < want; it++) {
                if ((it & 63) == 63 && abort_seen()) {
                    sh.cabort = 1;
                    break;
                }
                if (it > kPollLimit) {
                    sh.cabort = 1;
                    atomicOr(p.state + B2_MK_ERR, 1);
                    break;
                }
                if (it > 32) __nanosleep(64);
            }
        }
        consumer_sync();
        aborted = *(volatile int*)&sh.cabort != 0;
    }
    __device__ unsigned long long* dn_count(int l) const { return S.cnt + 8 + l; }
    __device__ unsigned long long* ao_count(int l) const { return S.cnt + 8 + p.n_layers + l; }
    __device__ float* mid_acc(int l) const { return S.macc + ((size_t)l * 2 + (tag & 1)) * p.hidden; }
    __device__ int ao_units() const { return p.nkv * (geo.G / p.nkv); }
    // output of layer l (input of layer l + 1) for this step's parity
    __device__ float* layer_out(int l) const {
        return S.hacc + ((size_t)l * 2 + (tag & 1)) * kOutCopies * p.hidden;
    }
    // copies summed in a layer-output read (1 for the embedding row)
    __device__ int out_copies(int l) const { return l < 0 ? 1 : kOutCopies; }
    // groups of a vector summed by other CTAs in this launch: read through L2
    // (the sum of `copies` copies K values apart)
    __device__ void cg_gather(const float* src, int K, float4 (&v)[kV], int copies = 1) const {
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            if (q * 4 >= K) continue;
            float4 a = __ldcg(reinterpret_cast<const float4*>(src) + q);
            for (int c = 1; c < copies; c++) {
                const float4 b = __ldcg(reinterpret_cast<const float4*>(src + (size_t)c * K) + q);
                a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
            }
            v[j] = a;
        }
    }

    // Same groups of a plain FP32 vector that is constant during the launch.
    __device__ void plain_gather(const float* src, int K, float4 (&v)[kV]) const {
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            if (q * 4 < K) v[j] = __ldg(reinterpret_cast<const float4*>(src) + q);
        }
    }

    // The attention output of layer l (q_dim values) for this thread's groups:
    // the S position-range partials of each head merged with the online
    // softmax rule (the split-KV combine of flash decoding).  The poll only
    // checks tags; the merge re-reads the (now cached) words.
    __device__ const unsigned long long* part_rec(int l, int e, int s) const {
        const int Gq = geo.Gq, hq = e / kHD, g = hq / Gq, h = hq % Gq;
        return S.part + ((((size_t)l * p.nkv + g) * kMaxSplit + s) * Gq + h) * (2 + kHD);
    }
    __device__ bool attn_gather(int l, float4 (&v)[kV]) const {
        if (!warp_lead_wait(part_rec(l, warp * 32 * 4, geo.S - 1), warp * 32 * 4 < geo.qd)) return false;
        for (int j = 0; j < kV; j++) {
            const int e = (tid + j * kConsumers) * 4;
            if (e >= geo.qd) break;
            const int d = e % kHD;
            for (int s = 0; s < geo.S; s++) {
                const unsigned long long* rec = part_rec(l, e, s);
                for (long long it = 0;; it++) {
                    const ulonglong2 ml = ll_get2(rec), o01 = ll_get2(rec + 2 + d), o23 = ll_get2(rec + 4 + d);
                    if (ll_ok(ml.x, tag) && ll_ok(ml.y, tag) && ll_ok(o01.x, tag) && ll_ok(o01.y, tag) &&
                        ll_ok(o23.x, tag) && ll_ok(o23.y, tag))
                        break;
                    if (it > kPollLimit || ((it & 63) == 63 && abort_seen())) return false;
                    __nanosleep(128);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int e = (tid + j * kConsumers) * 4;
            if (e >= geo.qd) break;
            const int d = e % kHD;
            float M = -INFINITY, den = 0.f;
            float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s = 0; s < geo.S; s++) {
                const unsigned long long* rec = part_rec(l, e, s);
                const ulonglong2 ml = ll_get2(rec);
                const float m = ll_val(ml.x);
                if (m == -INFINITY) continue;
                const ulonglong2 o01 = ll_get2(rec + 2 + d), o23 = ll_get2(rec + 4 + d);
                const float Mn = fmaxf(M, m);
                const float a = M == -INFINITY ? 0.f : expf(M - Mn);
                const float b = expf(m - Mn);
                den = den * a + ll_val(ml.y) * b;
                num.x = num.x * a + ll_val(o01.x) * b;
                num.y = num.y * a + ll_val(o01.y) * b;
                num.z = num.z * a + ll_val(o23.x) * b;
                num.w = num.w * a + ll_val(o23.y) * b;
                M = Mn;
            }
            v[j] = make_float4(num.x / den, num.y / den, num.z / den, num.w / den);
        }
        return true;
    }

    // Static per-item inputs, requested before the item's wait so their
    // latency hides behind it.  Norm weights are only pulled into L1 (this
    // thread's 16-byte groups; registers are the scarce resource here) and
    // read again by stage().
    __device__ void load_norm(const float* nw, int K) {
        if (!nw) return;
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            if (q * 4 < K) asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const float4*>(nw) + q));
        }
    }
    // scales of rows [r0, r0 + nrows) (then of rows [r0 + off2, ...) when off2 > 0)
    __device__ void load_scales(const float* sc, int off2) {
        const int tot = off2 > 0 ? 2 * nrows : nrows;
        if (!sc || tot > kScCap) return;
        for (int i = tid; i < tot; i += kConsumers)
            sh.sc[buf][i] = __ldg(sc + (i < nrows ? r0 + i : r0 + off2 + (i - nrows)));
    }
    __device__ float scale(const float* sc, int i, int off2) const {  // i-th scale of the item
        if (!sc) return 1.f;
        const int tot = off2 > 0 ? 2 * nrows : nrows;
        if (tot <= kScCap) return sh.sc[buf][i];
        return __ldg(sc + (i < nrows ? r0 + i : r0 + off2 + (i - nrows)));
    }
    // residual rows of the item: LL words already validated by this CTA's
    // previous stage (so the poll ends at once), or the plain embedding row
    // plain[r0 + i] summed over `copies` copies p.hidden apart (layer outputs)
    __device__ float plain_sum(const float* plain, int i, int copies) const {
        float v = __ldcg(plain + r0 + i);
        for (int c = 1; c < copies; c++) v += __ldcg(plain + (size_t)c * p.hidden + r0 + i);
        return v;
    }
    __device__ bool load_res(const unsigned long long* ll, const float* plain, int copies = 1) {
        if (nrows > kResCap) return true;
        bool ok = true;
        for (int i = tid; i < nrows; i += kConsumers) {
            float v = 0.f;
            if (ll) ok = ll_wait(ll + r0 + i, v) && ok;
            else v = plain_sum(plain, i, copies);
            sh.res[buf][i] = v;
        }
        return ok;
    }
    __device__ float resid(const unsigned long long* ll, const float* plain, int i, int copies = 1) const {
        if (nrows <= kResCap) return sh.res[buf][i];
        float v = 0.f;
        if (!ll) return plain_sum(plain, i, copies);
        ll_wait(ll + r0 + i, v);  // validated by this CTA's previous stage
        return v;
    }

    // Optional RMSNorm (weights nw) and FP16 rounding into xs, in the k order
    // the tensor-core dot of the coming rows expects: natural, or for int4
    // rows each group of 8 as (0 4 1 5 2 6 3 7).  Runs after the vote, so
    // every consumer has finished with the old xs.
    __device__ void stage(const float4 (&v)[kV], int K, const float* nw, bool perm8) {
        float rms = 1.f;
        if (nw) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < kV; j++)
                if ((tid + j * kConsumers) * 4 < K)
                    ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
            ss = b2::warp_sum(ss);
            if (lane == 0) sh.red[warp] = ss;
            consumer_sync();
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kCWarps; w++) t += sh.red[w];
            rms = 1.0f / sqrtf(t / (float)K + p.eps);
        }
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            if (q * 4 >= K) break;
            float4 x = v[j];
            if (nw) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(nw) + q);
                x.x = (x.x * rms) * w.x;
                x.y = (x.y * rms) * w.y;
                x.z = (x.z * rms) * w.z;
                x.w = (x.w * rms) * w.w;
            }
            if (perm8) {  // elements 4q..4q+3 are i = 0..3 or 4..7 of their group of 8
                const int base = (q >> 1) * 8 + (q & 1);
                xs[base] = __float2half_rn(x.x);
                xs[base + 2] = __float2half_rn(x.y);
                xs[base + 4] = __float2half_rn(x.z);
                xs[base + 6] = __float2half_rn(x.w);
            } else {
                __half2* d = reinterpret_cast<__half2*>(xs + q * 4);
                d[0] = __floats2half2_rn(x.x, x.y);
                d[1] = __floats2half2_rn(x.z, x.w);
            }
        }
        consumer_sync();
    }

    __device__ void begin(const Item& it) {
        buf = items & 1;
        items++;
        r0 = it.r0;
        nrows = it.r1 - it.r0;
        const int H = p.hidden;
        const B2MkLayer& Lw = p.layers[it.type == IT_LM ? 0 : it.l];
        constexpr bool perm = WT == B2_W_I4;
        float4 v[kV];
        bool ok = true;
        switch (it.type) {
            case IT_QKV:
                isc = Lw.qkv_s;
                load_scales(Lw.qkv_s, 0);
                load_norm(Lw.in_norm, H);
                if (it.l == 0) {
                    plain_gather(emb_row, H, v);
                } else {
                    wait_counter(dn_count(it.l - 1), (unsigned long long)geo.G * tag);
                    if (stop()) return;
                    cg_gather(layer_out(it.l - 1), H, v, kOutCopies);
                }
                settle(ok);
                if (!stop()) stage(v, H, Lw.in_norm, perm);
                break;
            case IT_ATTN: attn_prologue(it); break;
            case IT_AO:
                isc = Lw.o_s;
                load_scales(Lw.o_s, 0);
                if (it.g == 0) load_res(nullptr, it.l == 0 ? emb_row : layer_out(it.l - 1), out_copies(it.l - 1));
                attn_prologue(it);
                break;
            case IT_O:
                isc = Lw.o_s;
                load_scales(Lw.o_s, 0);
                ok = load_res(nullptr, it.l == 0 ? emb_row : layer_out(it.l - 1), out_copies(it.l - 1));
                ok = attn_gather(it.l, v) && ok;
                settle(ok);
                if (!stop()) stage(v, geo.qd, nullptr, perm);
                break;
            case IT_GU:
                isc = Lw.gu_s;
                load_scales(Lw.gu_s, p.ffn);
                load_norm(Lw.post_norm, H);
                if (geo.R > 0) {
                    wait_counter(ao_count(it.l), (unsigned long long)ao_units() * tag);
                    if (stop()) return;
                    cg_gather(mid_acc(it.l), H, v);
                } else {
                    ok = ll_gather(S.hmid + (size_t)it.l * H, H, v);
                }
#pragma unroll
                for (int i = 0; i < 4; i++) dacc_[i] = 0.f;
                res4_ = v[0];  // CTA 0 adds hmid (outputs 4 tid ..) into the layer output
                settle(ok);
                if (!stop()) stage(v, H, Lw.post_norm, perm);
                break;
            case IT_LM:
                isc = p.lm_s;
                load_scales(p.lm_s, 0);
                load_norm(p.final_norm, H);
                wait_counter(dn_count(p.n_layers - 1), (unsigned long long)geo.G * tag);
                if (stop()) return;
                cg_gather(layer_out(p.n_layers - 1), H, v, kOutCopies);
                if (geo.cta == 0) write_final(v);
                settle(ok);
                if (!stop()) stage(v, H, p.final_norm, false);  // int8 table
                best = 0ull;
                break;
        }
    }

    __device__ void mid(const Item& it) {
        if (stop()) return;
        if (it.type == IT_AO) attn_to_xs(it);
    }

    // Every consumer waits for the stage itself (so the bulk-copied bytes are
    // visible to it); the vote makes the outcome uniform.
    __device__ bool wait_full(int stage, uint32_t parity) {
        long long it = 0;
        bool ok = true;
        while (!mbar_try_wait(&sh.full[stage], parity)) {
            if (*(volatile int*)&sh.abort || ++it > kBarLimit) {
                ok = false;
                break;
            }
        }
        if (consumer_all(ok)) return true;
        if (tid == 0) {
            sh.cabort = 1;
            atomicOr(p.state + B2_MK_ERR, 3);
        }
        aborted = true;
        return false;
    }

    __device__ void chunk(const Chunk& c) {
        const int stage = n % kStages;
        if (aborted || !wait_full(stage, (uint32_t)((n / kStages) & 1))) return;
        const unsigned char* buf_ = ring + (size_t)stage * kStageBytes;
        switch (c.type) {
            case IT_QKV: rows_qkv(c, buf_); break;
            case IT_ATTN: attn_chunk(c, buf_); break;
            case IT_O: rows_resid(c, buf_, geo.qd); break;
            case IT_GU: rows_gu(c, buf_); break;
            case IT_DNT: rows_dnt(c, buf_); break;
            case IT_OSEG: rows_oseg(c, buf_); break;
            case IT_LM: rows_lm(c, buf_); break;
        }
        __syncwarp();  // this warp is done reading the stage
        if (lane == 0) mbar_arrive(&sh.empty[stage]);
        if (tid == 0) *(volatile int*)&sh.consumed = n + 1;
        n++;
    }

    // Rows publish their LL words as they are computed; only attention (its
    // partial) and the lm_head (its argmax) have work at the end of an item.
    __device__ void end(const Item& it) {
        if (stop()) return;
        if (it.type == IT_ATTN) {
            attn_epilogue(it);
        } else if (it.type == IT_AO) {
            consumer_sync();  // every consumer's o_proj additions precede the release
            if (tid == 0) red_release(ao_count(it.l), 1ull);
        } else if (it.type == IT_O) {
            // split phase: keep the fused phase's counter in step (one unit count per step)
            if (geo.cta == 0 && tid == 0) red_release(ao_count(it.l), (unsigned long long)ao_units());
        } else if (it.type == IT_GU) {
            // this CTA's down partial (its gate|up channels) into the layer
            // output; CTA 0 also adds the residual hmid.  The barrier orders
            // every consumer's additions before consumer 0's release.
            const int n = 4 * tid;
            if (n < p.hidden) {
                const float* ds = p.layers[it.l].dn_s;
                float4 d = make_float4(dacc_[0], dacc_[1], dacc_[2], dacc_[3]);
                if (ds) {
                    const float4 sc = __ldg(reinterpret_cast<const float4*>(ds + n));
                    d.x *= sc.x, d.y *= sc.y, d.z *= sc.z, d.w *= sc.w;
                }
                if (geo.cta == 0) d.x += res4_.x, d.y += res4_.y, d.z += res4_.z, d.w += res4_.w;
                red_add_v4(layer_out(it.l) + (size_t)(geo.cta % kOutCopies) * p.hidden + n, d);
            }
            consumer_sync();
            if (tid == 0) red_release(dn_count(it.l), 1ull);
        } else if (it.type == IT_LM) {
            unsigned long long b = best;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long x = __shfl_xor_sync(0xffffffffu, b, o);
                b = x > b ? x : b;
            }
            if (lane == 0) sh.best[warp] = b;
            consumer_sync();
            if (tid == 0) {
                unsigned long long m = 0ull;
                for (int w = 0; w < kCWarps; w++) m = sh.best[w] > m ? sh.best[w] : m;
                atomicMax(S.cnt + 1, m);
            }
        }
    }

    // ── row kernels ──

    // Sums of the chunk's nr rows (row(r) points at row r in the stage),
    // split over the 8 warps by 16-row tile and super-block range; the
    // partials meet in shared memory and thread r (< nr) receives row r.
    template <int W, class RowPtr>
    __device__ float chunk_dot(int nr, int K, RowPtr row) {
        const int nt = (nr + 15) >> 4;  // <= 4 (a stage holds at most 64 rows)
        const int ks = kCWarps / (nt == 3 ? 4 : nt);
        const int tile = warp / ks, part = warp % ks;
        if (tile < nt) {
            const int nsb = K / sb_k<W>();
            const int g = lane >> 2;
            const int ra = min(tile * 16 + g, nr - 1), rb = min(tile * 16 + g + 8, nr - 1);
            float o[2];
            tile_dot<W>(row(ra), row(rb), xs, split_lo(nsb, ks, part), split_lo(nsb, ks, part + 1), lane, o);
            if ((lane & 3) == 0) {
                sh.pr[warp][g] = o[0];
                sh.pr[warp][g + 8] = o[1];
            }
        }
        consumer_sync();
        float sum = 0.f;
        if (tid < nr) {
            const int t = tid >> 4, r = tid & 15;
            for (int w = t * ks; w < t * ks + ks; w++) sum += sh.pr[w][r];
        }
        return sum;
    }

    __device__ void rows_qkv(const Chunk& c, const unsigned char* buf_) {
        const size_t rb = row_bytes(WT, p.hidden);
        const int n = c.b - c.a;
        const float v = chunk_dot<WT>(n, p.hidden, [&](int r) { return buf_ + (size_t)r * rb; });
        if (tid < n) {
            const int r = c.a + tid;
            ll_put(S.qkv + (size_t)c.l * geo.nqkv + r, v * scale(isc, r - r0, 0), tag);
        }
    }

    // out[r] = resid[r] + s[r] * dot(row r, xs): o_proj into hmid, down into hbuf[l+1]
    __device__ void rows_resid(const Chunk& c, const unsigned char* buf_, int K) {
        const size_t rb = row_bytes(WT, K);
        const int H = p.hidden, n = c.b - c.a;
        const float v = chunk_dot<WT>(n, K, [&](int r) { return buf_ + (size_t)r * rb; });
        if (tid < n) {
            const int r = c.a + tid;
            const float y = resid(nullptr, c.l == 0 ? emb_row : layer_out(c.l - 1), r - r0, out_copies(c.l - 1)) +
                            v * scale(isc, r - r0, 0);
            ll_put(S.hmid + (size_t)c.l * H + r, y, tag);
        }
    }

    // rows 2j / 2j+1 of the dot are gate / up of channel c.a + j
    __device__ void rows_gu(const Chunk& c, const unsigned char* buf_) {
        const size_t rb = row_bytes(WT, p.hidden);
        const int n = c.b - c.a;
        const float v = chunk_dot<WT>(2 * n, p.hidden, [&](int r) {
            return buf_ + (r & 1 ? c.off1 : 0) + (size_t)(r >> 1) * rb;
        });
        const float u = __shfl_down_sync(0xffffffffu, v, 1);
        if (tid < 2 * n && (tid & 1) == 0) {
            const int jj = tid >> 1, j = c.a + jj;
            const float g = v * scale(isc, j - r0, p.ffn);
            const float up = u * scale(isc, nrows + (j - r0), p.ffn);
            const float sig = 1.0f / (1.0f + expf(-g));
            sh.act[j - r0] = __half2float(__float2half_rn((g * sig) * up));  // the down matmul's FP16 input
        }
    }

    // Down partial: outputs 4 tid .. 4 tid + 3 of rows j in [c.a, c.b) of the
    // input-major down weight times the staged act[j] (exact FP16 x weight
    // products, FP32 sums; the per-output scale is applied at the end).
    __device__ void rows_dnt(const Chunk& c, const unsigned char* buf_) {
        const int n = 4 * tid;
        if (n >= p.hidden) return;
        const size_t rb = row_bytes(WT, p.hidden);
        for (int j = c.a; j < c.b; j++) {
            const float a = sh.act[j - r0];
            const unsigned char* row = buf_ + (size_t)(j - c.a) * rb;
            float w[4];
            if constexpr (WT == B2_W_F16) {
                const uint2 h = *reinterpret_cast<const uint2*>(row + n * 2);
                const float2 w01 = b2::h2_to_f2(h.x), w23 = b2::h2_to_f2(h.y);
                w[0] = w01.x, w[1] = w01.y, w[2] = w23.x, w[3] = w23.y;
            } else if constexpr (WT == B2_W_I8) {
                const uint32_t u = b2::i8x4_bias(*reinterpret_cast<const uint32_t*>(row + n));
                w[0] = b2::i8_from_biased<0>(u), w[1] = b2::i8_from_biased<1>(u);
                w[2] = b2::i8_from_biased<2>(u), w[3] = b2::i8_from_biased<3>(u);
            } else {
                const uint32_t u = b2::i4x8_bias(*reinterpret_cast<const uint16_t*>(row + n / 2));
                w[0] = b2::i4_from_biased<0>(u), w[1] = b2::i4_from_biased<1>(u);
                w[2] = b2::i4_from_biased<2>(u), w[3] = b2::i4_from_biased<3>(u);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) dacc_[i] = fmaf(a, w[i], dacc_[i]);
        }
    }

    // Fused phase: o_proj rows [c.a, c.b) restricted to kv head c.g's columns,
    // times the unit's attention output; the partial (plus the residual, from
    // kv head 0's units) is added into this step's hidden-after-attention.
    __device__ void rows_oseg(const Chunk& c, const unsigned char* buf_) {
        const int K = geo.Gq * kHD;
        const size_t rb = row_bytes(WT, K);
        const int n = c.b - c.a;
        const float v = chunk_dot<WT>(n, K, [&](int r) { return buf_ + (size_t)r * rb; });
        if (tid < n) {
            const int r = c.a + tid;
            float y = v * scale(isc, r - r0, 0);
            if (c.g == 0) y += resid(nullptr, c.l == 0 ? emb_row : layer_out(c.l - 1), r - r0, out_copies(c.l - 1));
            atomicAdd(mid_acc(c.l) + r, y);
        }
    }

    // CTA 0: the final residual stream (before the final norm) for the host.
    __device__ void write_final(const float4 (&v)[kV]) const {
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            if (q * 4 < p.hidden) reinterpret_cast<float4*>(S.hfinal)[q] = v[j];
        }
    }

    __device__ void rows_lm(const Chunk& c, const unsigned char* buf_) {
        const int n = c.b - c.a;
        const size_t rb = (size_t)p.hidden;
        const float v = chunk_dot<B2_W_I8>(n, p.hidden, [&](int r) { return buf_ + (size_t)r * rb; });
        if (tid < n) {
            const int r = c.a + tid;
            const float logit = v * scale(isc, r - r0, 0);
            if (p.logits) p.logits[r] = logit;
            const unsigned long long k = b2::argmax_key(logit, (uint32_t)r);
            best = k > best ? k : best;
        }
    }

    // ── attention: one (kv head g, position range) unit ──

    __device__ void attn_prologue(const Item& it) {
        // The unit's softmax state starts here on every path, so it is dead
        // (holds no registers) outside attention items.
#pragma unroll
        for (int h2 = 0; h2 < kMaxGq; h2++) {
            m_[h2] = -INFINITY;
            l_[h2] = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) o_[h2][j] = qv_[h2][j] = 0.f;
        }
        const int Gq = geo.Gq;
        const unsigned long long* qkv = S.qkv + (size_t)it.l * geo.nqkv;
        const B2MkLayer& Lw = p.layers[it.l];
        const int h = warp;  // warps 0..Gq-1: q heads, Gq: k head, Gq+1: v head
        const int e0 = lane * 4;
        bool ok = true;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        float nw[4] = {1.f, 1.f, 1.f, 1.f}, cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
        const float* nwp = h < Gq ? Lw.q_norm : h == Gq ? Lw.k_norm : nullptr;
        if (h <= Gq + 1) {
            // static inputs first: their latency overlaps the poll below
            if (nwp) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(nwp + e0));
                nw[0] = t.x, nw[1] = t.y, nw[2] = t.z, nw[3] = t.w;
            }
            if (h <= Gq) {
                const float* ct = p.cos_tab + (size_t)geo.pos * (kHD / 2);
                const float* st = p.sin_tab + (size_t)geo.pos * (kHD / 2);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    // interleaved pairs (2i, 2i+1) use angle i; split halves (e, e + hd/2) use angle e
                    const int i = p.rope_style == 0 ? (e0 + j) >> 1 : (lane < 16 ? e0 + j : e0 + j - kHD / 2);
                    cs[j] = __ldg(ct + i);
                    sn[j] = __ldg(st + i);
                }
            }
            const unsigned long long* src = h < Gq ? qkv + (size_t)(it.g * Gq + h) * kHD
                                            : h == Gq ? qkv + geo.qd + (size_t)it.g * kHD
                                                      : qkv + geo.qd + geo.kvd + (size_t)it.g * kHD;
            ok = warp_lead_wait(src, true);
            for (long long t = 0; ok; t++) {
                const ulonglong2 a = ll_get2(src + e0), b = ll_get2(src + e0 + 2);
                if (ll_ok(a.x, tag) && ll_ok(a.y, tag) && ll_ok(b.x, tag) && ll_ok(b.y, tag)) {
                    x[0] = ll_val(a.x), x[1] = ll_val(a.y), x[2] = ll_val(b.x), x[3] = ll_val(b.y);
                    break;
                }
                if (t > kPollLimit || ((t & 63) == 63 && abort_seen())) {
                    ok = false;
                    break;
                }
                __nanosleep(128);
            }
        }
        settle(ok);
        if (stop()) return;
        if (h <= Gq + 1) {
            if (h <= Gq) {
                if (nwp) {
                    float ss = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; j++) ss = fmaf(x[j], x[j], ss);
                    ss = b2::warp_sum(ss);
                    const float rms = 1.0f / sqrtf(ss / (float)kHD + p.eps);
#pragma unroll
                    for (int j = 0; j < 4; j++) x[j] = (x[j] * rms) * nw[j];
                }
                if (p.rope_style == 0) {
#pragma unroll
                    for (int j = 0; j < 4; j += 2) {
                        const float x0 = x[j], x1 = x[j + 1];
                        x[j] = x0 * cs[j] - x1 * sn[j];
                        x[j + 1] = x1 * cs[j] + x0 * sn[j];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
                        x[j] = lane < 16 ? x[j] * cs[j] - other * sn[j] : x[j] * cs[j] + other * sn[j];
                    }
                }
            }
            float* dst = h < Gq ? sh.q[h] : h == Gq ? sh.k : sh.v;
#pragma unroll
            for (int j = 0; j < 4; j++) dst[e0 + j] = x[j];
            // The unit covering the newest position stores its K and V.
            if (h >= Gq && it.p1 == geo.L && it.p0 <= geo.L - 1 && (it.type != IT_AO || it.s == 0)) {
                uint16_t* base = (h == Gq ? p.k_cache : p.v_cache) + (size_t)it.l * p.layer_stride +
                                 ((size_t)it.g * p.max_seq + geo.pos) * kHD;
                __half* d16 = reinterpret_cast<__half*>(base);
#pragma unroll
                for (int j = 0; j < 4; j++) d16[e0 + j] = __float2half_rn(x[j]);
            }
        }
        consumer_sync();
        const int sub = lane & 7;
#pragma unroll
        for (int h2 = 0; h2 < kMaxGq; h2++)
#pragma unroll
            for (int j = 0; j < 16; j++) qv_[h2][j] = h2 < Gq ? sh.q[h2][sub * 16 + j] : 0.f;
    }

    // One position per lane group; kf/vf are this lane's 16 dims.
    __device__ void attn_update(bool live, const float (&kf)[16], const float (&vf)[16]) {
        const float scale = 1.0f / sqrtf((float)kHD);
#pragma unroll
        for (int h = 0; h < kMaxGq; h++) {
            if (h >= geo.Gq) break;
            float d = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) d = fmaf(qv_[h][j], kf[j], d);
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            d += __shfl_xor_sync(0xffffffffu, d, 4);
            if (!live) continue;
            const float s = d * scale;
            const float mn = fmaxf(m_[h], s);
            const float corr = expf(m_[h] - mn);
            const float pr = expf(s - mn);
            l_[h] = l_[h] * corr + pr;
#pragma unroll
            for (int j = 0; j < 16; j++) o_[h][j] = fmaf(pr, vf[j], o_[h][j] * corr);
            m_[h] = mn;
        }
    }

    __device__ void attn_chunk(const Chunk& c, const unsigned char* buf) {
        const int n = c.b - c.a, sub = lane & 7;
        const __half* kb = reinterpret_cast<const __half*>(buf);
        const __half* vb = reinterpret_cast<const __half*>(buf + c.off1);
        for (int pb = warp * 4; pb < n; pb += 4 * kCWarps) {  // warp-uniform bound
            const int i = pb + (lane >> 3);
            const bool live = i < n;
            float kf[16], vf[16];
            if (live) {
                const uint4* kp = reinterpret_cast<const uint4*>(kb + (size_t)i * kHD + sub * 16);
                const uint4* vp = reinterpret_cast<const uint4*>(vb + (size_t)i * kHD + sub * 16);
                uint4 w4[4] = {kp[0], kp[1], vp[0], vp[1]};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const uint32_t* u = &w4[q].x;
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        float2 f = b2::h2_to_f2(u[t]);
                        float* d = q < 2 ? kf : vf;
                        d[(q & 1) * 8 + 2 * t] = f.x;
                        d[(q & 1) * 8 + 2 * t + 1] = f.y;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) kf[j] = vf[j] = 0.f;
            }
            attn_update(live, kf, vf);
        }
    }

    // Fold the newest position into the softmax state, merge the lane groups
    // of each warp, and leave one (m, l, o) state per warp in shared memory.
    __device__ void attn_merge_warps(const Item& it) {
        const int Gq = geo.Gq, sub = lane & 7;
        // the newest position (not in the cache stream): lane group 0 of warp 0
        if (it.p1 == geo.L && it.p0 <= geo.L - 1 && warp == 0) {
            float kf[16], vf[16];
            const bool live = (lane >> 3) == 0;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                kf[j] = live ? __half2float(__float2half_rn(sh.k[sub * 16 + j])) : 0.f;
                vf[j] = live ? __half2float(__float2half_rn(sh.v[sub * 16 + j])) : 0.f;
            }
            attn_update(live, kf, vf);
        }
        // Merge the four lane groups of this warp (lanes sub, sub^8, sub^16,
        // sub^24 hold the same 16 dims) with shuffles, then publish one state
        // per warp.
#pragma unroll
        for (int h = 0; h < kMaxGq; h++) {
            if (h >= Gq) break;
#pragma unroll
            for (int off = 8; off <= 16; off <<= 1) {
                const float mo = __shfl_xor_sync(0xffffffffu, m_[h], off);
                const float lo = __shfl_xor_sync(0xffffffffu, l_[h], off);
                const float M = fmaxf(m_[h], mo);
                const float a = (m_[h] == -INFINITY) ? 0.f : expf(m_[h] - M);
                const float b = (mo == -INFINITY) ? 0.f : expf(mo - M);
                l_[h] = l_[h] * a + lo * b;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float oo = __shfl_xor_sync(0xffffffffu, o_[h][j], off);
                    o_[h][j] = o_[h][j] * a + oo * b;
                }
                m_[h] = M;
            }
            if (lane < 8) {
                if (sub == 0) {
                    sh.gm[warp][h] = m_[h];
                    sh.gl[warp][h] = l_[h];
                }
#pragma unroll
                for (int j = 0; j < 16; j++) sh.go[warp][h][sub * 16 + j] = o_[h][j];
            }
        }
        consumer_sync();
    }

    // merged (m, l, o) of head h, dim d over the warps' states
    __device__ void attn_state(int h, int d, float& M, float& ls, float& acc) const {
        M = -INFINITY;
        for (int r = 0; r < kCWarps; r++) M = fmaxf(M, sh.gm[r][h]);
        ls = 0.f;
        acc = 0.f;
        if (M != -INFINITY)
            for (int r = 0; r < kCWarps; r++) {
                if (sh.gm[r][h] == -INFINITY) continue;
                const float w = expf(sh.gm[r][h] - M);
                ls = fmaf(sh.gl[r][h], w, ls);
                acc = fmaf(sh.go[r][h][d], w, acc);
            }
    }

    // Fused phase: the attention output of the unit's q heads, FP16-rounded,
    // as the staged input of its o_proj columns (k order of sb_mma).
    __device__ void attn_to_xs(const Item& it) {
        attn_merge_warps(it);
        for (int t = tid; t < geo.Gq * kHD; t += kConsumers) {
            float M, ls, acc;
            attn_state(t / kHD, t % kHD, M, ls, acc);
            const int pos = WT == B2_W_I4 ? (t & ~7) + ((t & 7) < 4 ? 2 * (t & 7) : 2 * ((t & 7) - 4) + 1) : t;
            xs[pos] = __float2half_rn(acc / ls);
        }
        consumer_sync();
    }

    // Split phase: write this unit's partial (m, l, o) for o_proj's combine.
    __device__ void attn_epilogue(const Item& it) {
        const int Gq = geo.Gq;
        attn_merge_warps(it);
        const size_t unit = (((size_t)it.l * p.nkv + it.g) * kMaxSplit + it.s) * Gq;
        for (int t = tid; t < Gq * kHD; t += kConsumers) {
            const int h = t / kHD, d = t % kHD;
            float M, ls, acc;
            attn_state(h, d, M, ls, acc);
            unsigned long long* rec = S.part + (unit + h) * (2 + kHD);
            ll_put(rec + 2 + d, acc, tag);
            if (d == 0) {
                ll_put(rec, M, tag);
                ll_put(rec + 1, ls, tag);
            }
        }
    }
};

template <int WT>
__global__ void __launch_bounds__(kThreads, 1) mk_decode_kernel(const __grid_constant__ B2MkPlan p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;
    __half* xs = reinterpret_cast<__half*>(smem + (size_t)kStages * kStageBytes);
    Shared& sh = *reinterpret_cast<Shared*>(smem + (size_t)kStages * kStageBytes + kMaxK * sizeof(__half));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kCWarps);
        }
        sh.abort = 0;
        sh.cabort = 0;
        sh.issued = 0;
        sh.consumed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    Scratch S = scratch_layout(p.scratch, p.n_layers, p.hidden, p.ffn, p.nq, p.nkv, p.hd, nullptr);
    Geo geo;
    geo.pos = p.state[B2_MK_POS];
    geo.L = geo.pos + 1;
    geo.G = gridDim.x;
    geo.cta = blockIdx.x;
    geo.qd = p.nq * kHD;
    geo.kvd = p.nkv * kHD;
    geo.nqkv = geo.qd + 2 * geo.kvd;
    geo.Gq = p.nq / p.nkv;
    {
        // one position range per 256 cached positions, at most one unit per CTA
        int s = (geo.L + 255) / 256;
        const int cap = min(kMaxSplit, max(1, geo.G / p.nkv));
        geo.S = max(1, min(s, cap));
    }
    // fused attention + o_proj while every unit's o_proj slice fits the prefetch buffers
    geo.R = (geo.L <= kFuseL && geo.G >= p.nkv && (p.hidden + geo.G / p.nkv - 1) / (geo.G / p.nkv) <= kResCap)
                ? geo.G / p.nkv
                : 0;
    const unsigned long long gen = (unsigned long long)(unsigned)p.state[B2_MK_GEN];

    if (warp == kCWarps) {
        if (lane == 0) {
            Producer<WT> prod{p, sh, ring};
            walk<WT>(p, geo, prod);
        }
    } else {
        const int tok = p.state[B2_MK_TOKEN];
        const float* emb_row = p.state[B2_MK_USE_EMB] ? p.staged_emb : p.emb + (size_t)tok * p.hidden;
        Consumer<WT> cons{p, geo, sh, ring, xs, S, (uint32_t)(gen + 1), emb_row, tid, lane, warp};
        {  // zero this CTA's slice of the next step's accumulators (the other
           // parity; nothing reads it during this step)
            const int per = p.hidden / 4;  // float4 per vector
            const unsigned npar = (unsigned)(gen + 2) & 1u;
            float4* z = reinterpret_cast<float4*>(S.hacc);  // [L][2][kOutCopies][per]
            const int th = p.n_layers * kOutCopies * per;
            for (int i = split_lo(th, geo.G, geo.cta) + tid; i < split_lo(th, geo.G, geo.cta + 1); i += kConsumers) {
                const int l = i / (kOutCopies * per), rest = i % (kOutCopies * per);
                z[((size_t)l * 2 + npar) * kOutCopies * per + rest] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            float4* zm = reinterpret_cast<float4*>(S.macc);  // [L][2][per]
            const int tm = p.n_layers * per;
            for (int i = split_lo(tm, geo.G, geo.cta) + tid; i < split_lo(tm, geo.G, geo.cta + 1); i += kConsumers)
                zm[((size_t)(i / per) * 2 + npar) * per + (i % per)] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        walk<WT>(p, geo, cons);
        if (!p.do_lm && geo.cta == 0 && !cons.stop()) {  // prefill-mode step: publish the final hidden
            cons.wait_counter(cons.dn_count(p.n_layers - 1), (unsigned long long)geo.G * (gen + 1));
            if (!cons.stop()) {
                float4 v[kV];
                cons.cg_gather(cons.layer_out(p.n_layers - 1), p.hidden, v, kOutCopies);
                cons.write_final(v);
            }
        }
        if (!cons.stop()) {  // FIN: the last CTA publishes the step
            consumer_sync();
            if (tid == 0) {
                unsigned long long* fin = S.cnt;
                __threadfence();
                const unsigned long long old = atom_add_acqrel(fin, 1ull);
                if (old == (unsigned long long)(geo.G - 1)) {
                    __threadfence();
                    unsigned long long* key = fin + 1;
                    int token = 0;
                    if (p.do_lm) {
                        token = (int)b2::key_index(*(volatile unsigned long long*)key);
                        p.state[B2_MK_TOKEN] = token;
                        const int step = p.state[B2_MK_STEP];
                        if (p.hist && step < p.hist_len) p.hist[step] = token;
                    }
                    p.state[B2_MK_TOKEN_OUT] = token;
                    p.state[B2_MK_POS] = geo.pos + 1;
                    p.state[B2_MK_STEP] = p.state[B2_MK_STEP] + 1;
                    p.state[B2_MK_USE_EMB] = 0;
                    *(volatile unsigned long long*)key = 0ull;
                    *(volatile unsigned long long*)fin = 0ull;
                    __threadfence();
                    p.state[B2_MK_GEN] = (int)(gen + 1);
                }
            }
        }
    }
    __syncthreads();
    // Let every copy this CTA issued land before shared memory goes away
    // (only outstanding after an abort).
    if (tid == kConsumers) {
        const int issued = *(volatile int*)&sh.issued, consumed = *(volatile int*)&sh.consumed;
        for (int k = consumed; k < issued; k++) {
            long long it = 0;
            while (!mbar_try_wait(&sh.full[k % kStages], (uint32_t)((k / kStages) & 1)) && ++it < kBarLimit) {
            }
        }
    }
}

constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kMaxK * sizeof(__half) + sizeof(Shared) + 128;
static_assert(kSmemBytes <= 232448, "dynamic shared memory above the 227 KB per-block limit");

template <int WT>
int launch(const B2MkPlan* p, cudaStream_t s) {
    auto fn = mk_decode_kernel<WT>;
    constexpr int kMaxDevices = 64;
    static thread_local int configured[kMaxDevices] = {0};
    int dev = 0;
    B2_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk_decode: device ordinal %d above %d", dev, kMaxDevices - 1);
    if (!configured[dev]) {
        B2_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        int per_sm = 0;
        B2_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, kSmemBytes));
        if (per_sm < 1) return b2_set_error(B2_ERR_CUDA, "b2_mk_decode: kernel does not fit on an SM");
        configured[dev] = 1;
    }
    int sms = 0;
    B2_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if ((p->ffn + sms - 1) / sms > kActCap)  // gate|up channels of one CTA feed its down partial
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk_decode: ffn %d needs more than %d SMs", p->ffn, p->ffn / kActCap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, *p);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_mk_decode launch: %s", cudaGetErrorString(e));
    return 0;
}

}  // namespace

extern "C" float* b2_mk_final_hidden(const B2MkPlan* p) {
    Scratch s = scratch_layout(p->scratch, p->n_layers, p->hidden, p->ffn, p->nq, p->nkv, p->hd, nullptr);
    return s.hfinal;
}

extern "C" size_t b2_mk_smem_bytes(void) { return kSmemBytes; }

extern "C" size_t b2_mk_scratch_bytes(int n_layers, int hidden, int ffn, int nq, int nkv, int hd) {
    size_t total = 0;
    scratch_layout(nullptr, n_layers, hidden, ffn, nq, nkv, hd, &total);
    return total;
}

extern "C" int b2_mk_check(const B2MkPlan* p) {
    if (!p) return B2_ERR_INVALID_ARG;
    if (p->n_layers < 1 || p->n_layers > B2_MK_MAX_LAYERS || p->hd != kHD || p->nkv < 1 || p->nkv > 8 ||
        p->nq % p->nkv != 0 || p->nq / p->nkv > kMaxGq)
        return B2_ERR_INVALID_ARG;
    // K of every matmul: a whole number of 64-byte super-blocks (the int8
    // lm_head included), and short enough to stage
    const int E = p->wtype == B2_W_F16 ? 32 : p->wtype == B2_W_I8 ? 64 : 128;
    if (p->hidden % E || p->ffn % E || (p->nq * kHD) % E || p->hidden % 64 || p->hidden > kMaxK ||
        p->ffn > kMaxK || p->nq * kHD > kMaxK || p->hidden > 4 * kConsumers)
        return B2_ERR_INVALID_ARG;
    // every streamed row range must fit one stage at least one row at a time
    if (2 * row_bytes(p->wtype, p->hidden) > (size_t)kStageBytes || row_bytes(p->wtype, p->ffn) > (size_t)kStageBytes ||
        row_bytes(p->wtype, p->nq * kHD) > (size_t)kStageBytes || (size_t)p->hidden > (size_t)kStageBytes)
        return B2_ERR_INVALID_ARG;
    if (p->do_lm && (!p->lm || !p->lm_s || !p->final_norm)) return B2_ERR_INVALID_ARG;
    if (!p->layers || !p->state || !p->scratch || !p->k_cache || !p->v_cache || !p->cos_tab || !p->sin_tab || !p->emb)
        return B2_ERR_INVALID_ARG;
    return 0;
}

extern "C" int b2_mk_decode(const B2MkPlan* p, b2_stream_t stream) {
    if (b2_mk_check(p) != 0) return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk_decode: unsupported plan");
    cudaStream_t s = (cudaStream_t)stream;
    switch (p->wtype) {
        case B2_W_F16: return launch<B2_W_F16>(p, s);
        case B2_W_I8: return launch<B2_W_I8>(p, s);
        case B2_W_I4: return launch<B2_W_I4>(p, s);
        default: return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk_decode: wtype %d", p->wtype);
    }
}
