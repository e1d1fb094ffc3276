// Persistent single-token decode kernel, second generation (b2_mk2_decode).
//
// One cooperative launch runs a whole matmul_decoder_step
// (src/matmul_decoder.c:1430-1634 of suharvest/rknn-matmul-parallel): the
// embedding row, every layer's RMSNorm / q|k|v / per-head q,k norm / RoPE /
// KV append / GQA attention / o_proj + residual / RMSNorm / gate|up SiLU /
// down + residual, then optionally the final RMSNorm, the INT8 lm_head and
// the argmax.  Numerics are those of the multi-kernel path.
//
// Structure.  One CTA per SM.  Thread 0 of the last warp (the producer)
// turns the CTA's share of the token into a stream of operations kept in
// shared-memory slots.  A data operation carries a block of weights — whole
// 16-row tiles in the tile-major layout b2_tile_relayout writes, or K/V rows
// of one kv head — copied into a 192 KB byte ring by bulk copies whose
// completion is counted on the slot's mbarrier.  A control operation has no
// data.  The producer never waits for another CTA, only for ring space, so it
// streams the next phases' weights while the consumers wait on the
// dependency chain.
//
// The eight consumer warps take the operations in order.  A dot operation's
// tiles are split over the warps by K range (each warp a slice of every
// tile's 64-byte super-blocks; FP16 x FP16 products accumulated in FP32 with
// the mixed-precision FMA); the partial sums meet in shared memory after one
// barrier.  Every barrier on this path is a vote, so a failed wait anywhere
// turns into a failed vote and the whole CTA stops together.
//
// Per layer l (the steps other CTAs depend on; the steps in brackets run at
// the start or end of the neighbouring data operation):
//   QKV      [XIN: poll the layer-(l-1) output words (LL words: an FP32 value
//            and a tag of step and layer in one 64-bit store, which readers
//            poll); RMSNorm -> FP16] tiles of q|k|v rows; results published
//            as LL words
//   unit (kv head g, o_proj row slice r), on nkv * (G / nkv) CTAs:
//     KV     [AIN: poll the q|k|v words of head group g; q/k RMSNorm, RoPE;
//            unit r = 0 appends the new K/V row to the cache] up to 120
//            cached positions of head g in one two-pass softmax step over
//            all consumer threads, the newest position folded into the last
//            one [AOUT: FP16 attention output]; above 240 cached positions
//            16 units per head split the positions [APUB: publish the
//            partial state] and AMRG merges the 16 states per unit
//     O      o_proj tiles of rows in slice r, columns of group g: partial sums
//            published as LL words (one partial per kv head and output)
//   RO       reducer: for the 8 outputs this CTA owns, the nkv partials in
//            head order plus the residual x -> h_mid words, then
//            GIN: poll every h_mid word; RMSNorm(h_mid) -> FP16
//   GU       tiles of 8 channels (gate and up rows interleaved): SiLU(g) * u
//   DN       [a barrier: every act is in] the same channels' rows of the
//            input-major down weight times SiLU(g) * u: a partial of every
//            output [DEND: the partial as LL words, one counter increment]
//   RD       reducer: once the counter shows every CTA, for the 8 outputs this
//            CTA owns every CTA's partial in CTA order plus the residual
//            h_mid -> layer-output words
// then LIN / LM / LEND (final norm, lm_head tiles, argmax keys) and the
// last CTA to finish publishes the token.
//
// Sums run in a fixed order, so a step's result does not depend on timing.
// Tags are the generation + 1 of the step that wrote the word, where the
// generation (state[B2_MK_GEN]) counts completed launches.  Every wait is
// bounded (plan->poll_limit polls): on timeout the CTA sets state[B2_MK_ERR],
// stops, lets its in-flight copies land and returns.
#include "b2_common.cuh"

namespace {

constexpr int NC = 8;                  // consumer warps
constexpr int kCons = NC * 32;
constexpr int kThreads = kCons + 32;   // + the producer warp
constexpr int kHD = 128;
constexpr int kGq = 2;                 // q heads per kv head
constexpr int kND = 64;                // operation slots
constexpr int kOpMax = 64 * 1024;      // bytes of one data operation
constexpr int kOpRows = 64;            // rows (4 tiles) of one dot operation
constexpr int kKVPos = 128;            // cached positions per K/V operation (K and V: 64 KB)
constexpr int kKVPosNew = 120;         // ... of an unsplit head, whose last operation adds the newest
constexpr int kAttMax = 128;           // positions of one attention step
constexpr int kSplit = 2 * NC;         // units of a kv head that share its positions above 2 kKVPosNew
constexpr int kMaxH = 4 * kCons;       // hidden: one float4 per consumer thread
constexpr int kMaxF = 3072;            // longest staged activation
constexpr int kMaxCh = 32;             // gate|up channels per CTA
constexpr int kOwn = 8;                // outputs each reducer CTA owns (CTAs 0 .. hidden / 8 - 1)
constexpr int kMaxG = 256;             // CTAs the partial arrays have room for
constexpr int kMaxLayers = 32;         // layers of the shared-memory pointer table
constexpr long long kDefaultPolls = 1ll << 22;
static_assert(kCons == kGq * kHD, "the attention merge gives one consumer thread per (q head, dim)");
static_assert(kKVPos <= kAttMax && kKVPosNew < kAttMax && kAttMax == kCons / kGq,
              "an attention step gives each thread one (position, head)");

enum Op : int {
    OP_XIN, OP_QKV, OP_AIN, OP_KV, OP_AOUT, OP_APUB, OP_AMRG, OP_O, OP_RO, OP_GIN, OP_GU, OP_ACT, OP_DN, OP_DEND, OP_RD,
    OP_LIN, OP_LM, OP_LEND, OP_PFIN, OP_DONE
};

struct Desc {
    int op, l, a, b;     // type, layer, tile / position / channel range
    int c, d;            // unit: kv head, row slice
    uint32_t off, bytes; // data in the ring
};

struct Sh {
    uint64_t full[kND];
    uint64_t empty[kND];
    Desc desc[kND];
    int fifo_k[kND];            // producer: data operations holding ring space, oldest first
    uint32_t fifo_end[kND];
    int abort;                  // any thread: stop the CTA
    int issued;                 // operations issued by the producer
    int pk, pfh, pft, pdead;    // producer: operations issued, fifo head / tail, stopped
    uint32_t phead, ptail;      // producer: ring bytes taken / released (monotonic)
    float red[NC];
    unsigned long long best[NC];
    float part[2][NC][kOpRows]; // per-warp partial row sums of a dot operation (two in flight)
    float sq[kGq][kHD];         // q heads of the unit (normalized, rotated)
    __half knew[kHD], vnew[kHD];  // the new K and V rows (FP16, as cached)
    float mrg_m[NC][kGq], mrg_l[NC][kGq];  // per-warp softmax state: max, sum
    float mrg_o[NC][kGq][kHD];             // ... and output
    float act[kMaxCh];          // FP16-rounded SiLU(gate) * up of this CTA's channels
    float xres[kMaxH];          // x (layer input: the h_mid residual), then h_mid (the x residual)
    __half xs[2][kMaxH];        // staged FP16 inputs: [0] q|k|v and lm_head, [1] gate|up
    __half xo[kGq * kHD];       // attention output of the unit (o_proj input)
    B2MkLayer lay[kMaxLayers];  // the per-layer pointer table (read by every operation)
};

constexpr int kRing = 192 * 1024;
// an operation never wraps around the ring end, so any operation must fit
// beside the largest wasted tail: twice the largest operation
static_assert(2 * kOpMax <= kRing, "ring smaller than two operations");
constexpr size_t kSmemBytes = (size_t)kRing + sizeof(Sh) + 128;
static_assert(kSmemBytes <= 232448, "dynamic shared memory above the 227 KB per-block limit");

// ─── scratch in global memory ───

// Every vector passed between CTAs is a set of LL words (a value and a tag
// in one 64-bit store); partial sums are reduced by the CTA that owns the
// output (outputs split evenly over the CTAs), in a fixed order.  All layers
// share one slot per vector, told apart by the tag (step generation and
// layer), so the words stay resident in L2 across layers.  A slot is reused
// only after every reader of the previous layer's words has moved on: each
// phase that writes a slot for layer l + 1 runs after XIN(l + 1), which
// needs every CTA's RD(l), which in every CTA follows its reads of layer l.
struct Scr {
    unsigned long long* cnt;   // [8]: [0] CTAs finished, [1] best key
    unsigned long long* qkv;   // LL [nqkv]
    unsigned long long* apart; // LL [nkv][kSplit][4 + 2 hd] attention partials: m, l per q head, then o
    unsigned long long* opart; // LL [nkv][H] o_proj partials, one per kv head
    unsigned long long* hmid;  // LL [H] h_mid = x + o_proj(attention)
    unsigned long long* dpart; // LL [H / kOwn][kMaxG][kOwn] down partials by reducer, then source CTA
    unsigned long long* dcnt;  // down partials published since the scratch was cleared
    unsigned long long* xout;  // LL [H] layer output = h_mid + down(act)
    float* hfinal;             // [H]
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline Scr scr_layout(void* base, int L, int H, int nqkv, int nkv, size_t* total) {
    unsigned char* p = static_cast<unsigned char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* r = p + off;
        off += align256(bytes);
        return r;
    };
    Scr s;
    s.cnt = reinterpret_cast<unsigned long long*>(take(8 * 8));
    (void)L;
    s.qkv = reinterpret_cast<unsigned long long*>(take((size_t)nqkv * 8));
    s.apart = reinterpret_cast<unsigned long long*>(take((size_t)nkv * kSplit * (4 + 2 * kHD) * 8));
    s.opart = reinterpret_cast<unsigned long long*>(take((size_t)nkv * H * 8));
    s.hmid = reinterpret_cast<unsigned long long*>(take((size_t)H * 8));
    s.dpart = reinterpret_cast<unsigned long long*>(take((size_t)kMaxG * H * 8));
    s.dcnt = reinterpret_cast<unsigned long long*>(take(8));
    s.xout = reinterpret_cast<unsigned long long*>(take((size_t)H * 8));
    s.hfinal = reinterpret_cast<float*>(take((size_t)H * 4));
    if (total) *total = off;
    return s;
}

// ─── PTX helpers ───

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
// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  Both addresses and the size are multiples of 16.
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
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory"); }
// Every barrier on the consumers' operation path is a vote (bar.red): a warp
// that stops early takes part in the next barrier of the others with a false
// vote, and everyone leaves together.  Plain bar.sync only after a
// successful run, when all warps take the same path.
__device__ __forceinline__ bool vote(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.and.pred po, 1, %2, pi;\n"
        " selp.u32 %0, 1, 0, po;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(kCons)
        : "memory");
    return r != 0;
}
// LL words: FP32 value in the low half, the step's tag in the high half.
__device__ __forceinline__ void ll_put(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_get(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ ulonglong2 ll_get2(const unsigned long long* p) {
    ulonglong2 r;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ bool ll_ok(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// ─── row dots over a tile-major 16-row tile (CUDA cores) ───
//
// A tile is [super-block][16 rows][64 bytes].  Lane (g = lane / 4, q = lane
// % 4) reads the 16 bytes at offset 16 q of rows g and g + 8 of every
// super-block; the eight lanes of one shared-memory wavefront read 128
// consecutive bytes, so the loads are conflict-free.  The products are FP16
// weight x FP16 activation, exact in FP32, added into FP32 accumulators by
// the mixed-precision fma.rn.f32.f16 (one rounding per addition, the FP32
// accumulation the reference's matmul semantics ask for).  INT8 / INT4 widen
// to FP16 exactly with byte permutes (value + 1024 in the mantissa of 1024,
// one half2 subtraction removes the bias).  Legacy mma.sync would waste 7 of
// its 8 columns on a single activation vector and runs at a fraction of the
// FMA pipes' rate on this part.

template <int WT>
__host__ __device__ constexpr int sb_k() {
    return WT == B2_W_F16 ? 32 : WT == B2_W_I8 ? 64 : 128;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// a0 += w.lo * x.lo, a1 += w.hi * x.hi (FP16 operands, FP32 accumulators)
__device__ __forceinline__ void fma2h(float& a0, float& a1, uint32_t w, uint32_t x) {
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %2;\n mov.b32 {xl, xh}, %3;\n"
        " fma.rn.f32.f16 %0, wl, xl, %0;\n fma.rn.f32.f16 %1, wh, xh, %1;\n}"
        : "+f"(a0), "+f"(a1)
        : "r"(w), "r"(x));
}

// One 16-byte chunk of weights (w) against its activations (x: 16 bytes for
// FP16, 32 for INT8, 64 for INT4, as half2 words in the matching k order).
template <int WT>
__device__ __forceinline__ void chunk_fma(float& a0, float& a1, const uint4 w, const uint32_t* x) {
    const uint32_t* u = &w.x;
    if constexpr (WT == B2_W_F16) {
#pragma unroll
        for (int t = 0; t < 4; t++) fma2h(a0, a1, u[t], x[t]);
    } else if constexpr (WT == B2_W_I8) {
        const uint32_t bias = 0x64806480u;  // half2(1152, 1152) = 1024 + 128
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint32_t b = u[t] ^ 0x80808080u;
            fma2h(a0, a1, hsub2_u32(__byte_perm(b, 0x64646464u, 0x4140), bias), x[2 * t]);
            fma2h(a0, a1, hsub2_u32(__byte_perm(b, 0x64646464u, 0x4342), bias), x[2 * t + 1]);
        }
    } else {
        const uint32_t bias = 0x64086408u;  // half2(1032, 1032) = 1024 + 8
#pragma unroll
        for (int t = 0; t < 4; t++) {
            // word t holds k = 8t + i at nibble i; half2 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7),
            // the order the INT4 activation staging uses
            const uint32_t b = u[t] ^ 0x88888888u;
#pragma unroll
            for (int j = 0; j < 4; j++)
                fma2h(a0, a1, hsub2_u32(((b >> (4 * j)) & 0x000F000Fu) | 0x64006400u, bias), x[4 * t + j]);
        }
    }
}

// Rows g and g + 8 of T (<= 4) tiles, `stride` bytes apart, over
// super-blocks [sb0, sb1) against xs.  The super-block loop is outermost, so
// each activation chunk is loaded once for all tiles, and the 4 x 2 x 2
// accumulators form independent FMA chains.  After the cross-lane
// reduction every lane holds y[t][0] (row g of tile t) and y[t][1] (row g + 8).
template <int WT>
__device__ __forceinline__ void tiles_dot(const unsigned char* base, uint32_t stride, int T, const __half* xs, int sb0,
                                          int sb1, int lane, float (&y)[4][2]) {
    constexpr int SK = sb_k<WT>(), XW = SK / 8;  // activation words (half2) per lane per super-block
    const int q = lane & 3;
    const unsigned char* pa = base + (lane >> 2) * 64 + q * 16;
    const __half* px = xs + q * (SK / 4);
    float acc[4][2][2];
#pragma unroll
    for (int t = 0; t < 4; t++) acc[t][0][0] = acc[t][0][1] = acc[t][1][0] = acc[t][1][1] = 0.f;
    for (int sb = sb0; sb < sb1; sb++) {
        uint32_t xw[XW];
#pragma unroll
        for (int i = 0; i < XW / 4; i++)
            *reinterpret_cast<uint4*>(xw + 4 * i) = *reinterpret_cast<const uint4*>(px + sb * SK + 8 * i);
#pragma unroll
        for (int t = 0; t < 4; t++)
            if (t < T) {
                const uint4 wg = *reinterpret_cast<const uint4*>(pa + (size_t)t * stride + sb * 1024);
                const uint4 wh = *reinterpret_cast<const uint4*>(pa + (size_t)t * stride + sb * 1024 + 512);
                chunk_fma<WT>(acc[t][0][0], acc[t][0][1], wg, xw);
                chunk_fma<WT>(acc[t][1][0], acc[t][1][1], wh, xw);
            }
    }
#pragma unroll
    for (int t = 0; t < 4; t++) {
        float a = acc[t][0][0] + acc[t][0][1], b = acc[t][1][0] + acc[t][1][1];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        y[t][0] = a;
        y[t][1] = b;
    }
}

__host__ __device__ inline int row_bytes(int wtype, int K) {
    return wtype == B2_W_F16 ? K * 2 : wtype == B2_W_I8 ? K : K / 2;
}
__device__ __forceinline__ int split_lo(int n, int parts, int i) { return (int)(((long long)n * i) / parts); }

// Position of element e of a staged vector in the k order of the row dots:
// natural, or for INT4 rows each group of 8 as (0 4 1 5 2 6 3 7).
template <int WT>
__device__ __forceinline__ int stage_pos(int e) {
    if constexpr (WT == B2_W_I4) return (e & ~7) + ((e & 7) < 4 ? 2 * (e & 7) : 2 * ((e & 7) - 4) + 1);
    return e;
}

// Online softmax over up to 16 positions of one warp (K and V rows of 256
// bytes; lane owns dims 4 lane .. 4 lane + 3 of both q heads).  The warp's
// softmax state (running max, sum and output per head) lives in
// sh.mrg_m / mrg_l / mrg_o.  The 32 partial scores (16 positions x 2 heads)
// are reduced across the warp in a transposed butterfly: afterwards lane l
// holds the score of position l >> 1, head l & 1.  Every loop has a
// compile-time trip count (positions past n are predicated off), so the
// chains unroll.
__device__ __forceinline__ void attend16(Sh& sh, const unsigned char* kb, const unsigned char* vb, int n, int warp,
                                         int lane) {
    const float scale = 0.08838834764831845f;  // 1/sqrt(128)
    float qv[kGq][4], ao[kGq][4], am[kGq], al[kGq];
#pragma unroll
    for (int h = 0; h < kGq; h++) {
        const float4 q = *reinterpret_cast<const float4*>(&sh.sq[h][lane * 4]);
        const float4 o = *reinterpret_cast<const float4*>(&sh.mrg_o[warp][h][lane * 4]);
        qv[h][0] = q.x, qv[h][1] = q.y, qv[h][2] = q.z, qv[h][3] = q.w;
        ao[h][0] = o.x, ao[h][1] = o.y, ao[h][2] = o.z, ao[h][3] = o.w;
        am[h] = sh.mrg_m[warp][h];
        al[h] = sh.mrg_l[warp][h];
    }
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; i++) {
        float2 k01 = make_float2(0.f, 0.f), k23 = k01;
        if (i < n) {
            const uint2 kk = *reinterpret_cast<const uint2*>(kb + i * 256 + lane * 8);
            k01 = b2::h2_to_f2(kk.x);
            k23 = b2::h2_to_f2(kk.y);
        }
#pragma unroll
        for (int h = 0; h < kGq; h++)
            v[2 * i + h] = fmaf(qv[h][0], k01.x, fmaf(qv[h][1], k01.y, fmaf(qv[h][2], k23.x, qv[h][3] * k23.y)));
    }
    // transposed butterfly: 32 sums in 31 shuffles; lane l ends with value l
#pragma unroll
    for (int step = 0; step < 5; step++) {
        const int half = 16 >> step;  // values kept after this step
        const int bit = 16 >> step;   // lane bit that selects the half
        const bool hi = (lane & bit) != 0;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            if (j >= half) break;
            const float send = hi ? v[j] : v[j + half];
            const float recv = __shfl_xor_sync(0xffffffffu, send, bit);
            v[j] = (hi ? v[j + half] : v[j]) + recv;
        }
    }
    const int i = lane >> 1, h = lane & 1;
    const float s = i < n ? v[0] * scale : -INFINITY;
    // per-head max and sum over the lanes holding that head (lane bits 1..4)
    float mc = s;
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 2));
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 4));
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 8));
    mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 16));
    const float mo = __shfl_xor_sync(0xffffffffu, mc, 1);  // the other head's chunk max
    const float mch0 = h == 0 ? mc : mo, mch1 = h == 0 ? mo : mc;
    const float mn0 = fmaxf(am[0], mch0), mn1 = fmaxf(am[1], mch1);
    const float c0 = am[0] == -INFINITY ? 0.f : expf(am[0] - mn0);
    const float c1 = am[1] == -INFINITY ? 0.f : expf(am[1] - mn1);
    const float pr = i < n ? expf(s - (h == 0 ? mn0 : mn1)) : 0.f;
    float ps = pr;
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
    const float po = __shfl_xor_sync(0xffffffffu, ps, 1);
    al[0] = al[0] * c0 + (h == 0 ? ps : po);
    al[1] = al[1] * c1 + (h == 0 ? po : ps);
    am[0] = mn0;
    am[1] = mn1;
#pragma unroll
    for (int j = 0; j < 4; j++) ao[0][j] *= c0, ao[1][j] *= c1;
#pragma unroll
    for (int ii = 0; ii < 16; ii++) {
        const float p0 = __shfl_sync(0xffffffffu, pr, 2 * ii);
        const float p1 = __shfl_sync(0xffffffffu, pr, 2 * ii + 1);
        if (ii < n) {  // (warp-uniform)
            const uint2 vv = *reinterpret_cast<const uint2*>(vb + ii * 256 + lane * 8);
            const float2 v01 = b2::h2_to_f2(vv.x), v23 = b2::h2_to_f2(vv.y);
            ao[0][0] = fmaf(p0, v01.x, ao[0][0]), ao[0][1] = fmaf(p0, v01.y, ao[0][1]);
            ao[0][2] = fmaf(p0, v23.x, ao[0][2]), ao[0][3] = fmaf(p0, v23.y, ao[0][3]);
            ao[1][0] = fmaf(p1, v01.x, ao[1][0]), ao[1][1] = fmaf(p1, v01.y, ao[1][1]);
            ao[1][2] = fmaf(p1, v23.x, ao[1][2]), ao[1][3] = fmaf(p1, v23.y, ao[1][3]);
        }
    }
#pragma unroll
    for (int hh = 0; hh < kGq; hh++)
        *reinterpret_cast<float4*>(&sh.mrg_o[warp][hh][lane * 4]) = make_float4(ao[hh][0], ao[hh][1], ao[hh][2], ao[hh][3]);
    if (lane == 0) {
        sh.mrg_m[warp][0] = am[0], sh.mrg_m[warp][1] = am[1];
        sh.mrg_l[warp][0] = al[0], sh.mrg_l[warp][1] = al[1];
    }
    __syncwarp();
}

// ─── per-CTA geometry (identical in every thread) ───

struct Geo {
    int G, cta, pos, nqkv, qd, kvd;
    int R, units, ug, ur;                // o_proj row slices per kv head; this CTA's unit (ug < 0: none)
    int split, S, a0, a1;                // split attention: S units share the positions; this unit's [a0, a1)
    int q0, q1, o0, o1, c0, c1, m0, m1;  // tile ranges: qkv, o (unit rows), gate|up (8 channels), lm
};

__device__ Geo make_geo(const B2MkPlan& p) {
    Geo g;
    g.G = gridDim.x;
    g.cta = blockIdx.x;
    g.pos = p.state[B2_MK_POS];
    g.qd = p.nq * kHD;
    g.kvd = p.nkv * kHD;
    g.nqkv = g.qd + 2 * g.kvd;
    g.R = g.G / p.nkv;
    g.units = p.nkv * g.R;
    g.ug = g.cta < g.units ? g.cta / g.R : -1;
    g.ur = g.cta < g.units ? g.cta % g.R : 0;
    // Up to 2 kKVPosNew cached positions every unit of a kv head attends over
    // all of them; beyond, the first S units split them and publish partial
    // softmax states that every unit of the head merges.
    g.split = g.pos > 2 * kKVPosNew;
    g.S = min(kSplit, g.R);
    g.a0 = g.split ? (g.ur < g.S ? split_lo(g.pos, g.S, g.ur) : 0) : 0;
    g.a1 = g.split ? (g.ur < g.S ? split_lo(g.pos, g.S, g.ur + 1) : 0) : g.pos;
    const int qt = g.nqkv / 16, ot = p.hidden / 16, ct = p.ffn / 8, mt = p.vocab / 16;
    g.q0 = split_lo(qt, g.G, g.cta);
    g.q1 = split_lo(qt, g.G, g.cta + 1);
    g.o0 = split_lo(ot, g.R, g.ur);
    g.o1 = split_lo(ot, g.R, g.ur + 1);
    g.c0 = split_lo(ct, g.G, g.cta);
    g.c1 = split_lo(ct, g.G, g.cta + 1);
    g.m0 = split_lo(mt, g.G, g.cta);
    g.m1 = split_lo(mt, g.G, g.cta + 1);
    return g;
}

__device__ __forceinline__ void set_error(const B2MkPlan& p, Sh& sh, int code) {
    *(volatile int*)&sh.abort = 1;
    atomicOr(p.state + B2_MK_ERR, code);
}

// ─── producer ───
//
// The producer's state lives in shared memory (Sh::pk, phead, ...) so the
// two routines below stay out of line: one copy of the ring bookkeeping
// instead of one per call site of the walk.

// Operation j's slot has been released by every consumer warp.
__device__ __noinline__ bool prod_wait_empty(Sh& sh, const B2MkPlan& p, int j, long long limit) {
    uint64_t* bar = &sh.empty[j % kND];
    const uint32_t parity = (uint32_t)((j / kND) & 1);
    for (long long it = 0; !mbar_try_wait(bar, parity); it++) {
        if (*(volatile int*)&sh.abort) return false;
        if (it > limit) {
            set_error(p, sh, 2);
            return false;
        }
    }
    return true;
}

// Issue one operation: n == 0 a control operation, else a data operation
// whose n (<= 4) source blocks are packed into the ring.
__device__ __noinline__ void prod_emit(Sh& sh, unsigned char* ring, const B2MkPlan& p, long long limit, Desc d, int n,
                                       const void* const* src, const uint32_t* bytes) {
    if (sh.pdead) return;
    const int k = sh.pk;
    if (k >= kND && !prod_wait_empty(sh, p, k - kND, limit)) {
        sh.pdead = 1;
        return;
    }
    const int s = k % kND;
    if (n == 0) {
        d.off = 0;
        d.bytes = 0;
        sh.desc[s] = d;
        mbar_arrive(&sh.full[s]);
    } else {
        uint32_t total = 0;
        for (int i = 0; i < n; i++) total += bytes[i];
        uint32_t head = sh.phead;
        const uint32_t pos = head % kRing;
        if (pos + total > kRing) head += kRing - pos;  // no wrap inside an operation
        while (head + total - sh.ptail > kRing) {
            if (sh.pfh == sh.pft || !prod_wait_empty(sh, p, sh.fifo_k[sh.pft % kND], limit)) {
                if (sh.pfh == sh.pft) set_error(p, sh, 4);
                sh.pdead = 1;
                return;
            }
            sh.ptail = sh.fifo_end[sh.pft % kND];
            sh.pft++;
        }
        const uint32_t off = head % kRing;
        head += total;
        sh.phead = head;
        sh.fifo_k[sh.pfh % kND] = k;
        sh.fifo_end[sh.pfh % kND] = head;
        sh.pfh++;
        d.off = off;
        d.bytes = total;
        sh.desc[s] = d;
        mbar_expect_tx(&sh.full[s], total);
        uint32_t o = off;
        for (int i = 0; i < n; i++) {
            bulk_g2s(ring + o, src[i], bytes[i], &sh.full[s]);
            o += bytes[i];
        }
    }
    sh.pk = k + 1;
    *(volatile int*)&sh.issued = k + 1;
}

template <int WT>
__device__ void produce(const B2MkPlan& p, const Geo& geo, Sh& sh, unsigned char* ring, long long limit) {
    const int H = p.hidden;
    const uint32_t rb_h = row_bytes(WT, H);
    const uint32_t tb_h = 16u * rb_h;                                           // a tile of K = hidden rows
    const uint32_t sub_o = 1024u * (uint32_t)(row_bytes(WT, kGq * kHD) / 64);  // a tile's unit columns
    const uint32_t tb_o = 16u * row_bytes(WT, geo.qd);
    auto ctl = [&](int op, int l) {
        prod_emit(sh, ring, p, limit, Desc{op, l, 0, 0, geo.ug, geo.ur, 0u, 0u}, 0, nullptr, nullptr);
    };
    auto blocks = [&](int op, int l, int a, int b, int n, const void* const* src, const uint32_t* by) {
        prod_emit(sh, ring, p, limit, Desc{op, l, a, b, geo.ug, geo.ur, 0u, 0u}, n, src, by);
    };
    // items [t0, t1) of `unit` bytes each from base, as many per operation as
    // fit (at most `cap`: four tiles fill the partial-sum buffer)
    auto stream = [&](int op, int l, const void* base, int t0, int t1, uint32_t unit, int cap) {
        const int per = max(1, min(cap, (int)(kOpMax / unit)));
        for (int a = t0; a < t1 && !sh.pdead; a += per) {
            const int b = min(t1, a + per);
            const void* src[1] = {(const unsigned char*)base + (size_t)a * unit};
            const uint32_t by[1] = {(uint32_t)(b - a) * unit};
            blocks(op, l, a, b, 1, src, by);
        }
    };
    for (int l = 0; l < p.n_layers && !sh.pdead; l++) {
        const B2MkLayer& Lw = p.layers[l];
        if (geo.q0 == geo.q1) ctl(OP_XIN, l);  // else the first q|k|v operation stages x
        stream(OP_QKV, l, Lw.qkv_t, geo.q0, geo.q1, tb_h, kOpRows / 16);
        if (geo.ug >= 0) {
            // the first K/V operation also runs AIN, the last one AOUT (or APUB)
            const bool has_kv = geo.a0 < geo.a1;
            if (!has_kv) ctl(OP_AIN, l);
            const size_t head = (size_t)l * p.layer_stride + (size_t)geo.ug * p.max_seq * kHD;
            const int per_kv = geo.split ? kKVPos : kKVPosNew;
            for (int a = geo.a0; a < geo.a1 && !sh.pdead; a += per_kv) {
                const int b = min(geo.a1, a + per_kv);
                const uint32_t by = (uint32_t)(b - a) * kHD * 2;
                const void* src[2] = {p.k_cache + head + (size_t)a * kHD, p.v_cache + head + (size_t)a * kHD};
                const uint32_t bys[2] = {by, by};
                blocks(OP_KV, l, a, b, 2, src, bys);
            }
            if (geo.split) {
                if (geo.ur < geo.S && !has_kv) ctl(OP_APUB, l);
                ctl(OP_AMRG, l);
            } else if (!has_kv) {
                ctl(OP_AOUT, l);
            }
            const int per = max(1, min(4, (int)(kOpMax / sub_o)));
            for (int a = geo.o0; a < geo.o1 && !sh.pdead; a += per) {
                const int b = min(geo.o1, a + per);
                const void* src[4];
                uint32_t bys[4];
                for (int t = a; t < b; t++) {
                    src[t - a] = (const unsigned char*)Lw.o_t + (size_t)t * tb_o + (size_t)geo.ug * sub_o;
                    bys[t - a] = sub_o;
                }
                blocks(OP_O, l, a, b, b - a, src, bys);
            }
        }
        ctl(OP_RO, l);  // RO, then GIN
        stream(OP_GU, l, Lw.gu_t, geo.c0, geo.c1, tb_h, kOpRows / 16);
        // input-major down rows of the CTA's channels (one operation: the act
        // barrier first, DEND at its end); without channels a zero partial
        if (geo.c0 == geo.c1) ctl(OP_DEND, l);
        else stream(OP_DN, l, Lw.dn_t, 8 * geo.c0, 8 * geo.c1, rb_h, kMaxCh);
        ctl(OP_RD, l);
    }
    if (p.do_lm) {
        ctl(OP_LIN, p.n_layers);
        stream(OP_LM, p.n_layers, p.lm_t, geo.m0, geo.m1, 16u * (uint32_t)H, kOpRows / 16);
        ctl(OP_LEND, p.n_layers);
    } else {
        ctl(OP_PFIN, p.n_layers);
    }
    ctl(OP_DONE, p.n_layers);
}

// ─── consumers ───

template <int WT>
struct Consumer {
    const B2MkPlan& p;
    const Geo& geo;
    Sh& sh;
    const unsigned char* ring;
    const Scr& S;
    uint32_t tag;        // generation + 1 of this step
    long long limit;
    int tid, lane, warp;
    float dacc[4];       // down partial of outputs 4 tid .. 4 tid + 3
    unsigned long long best = 0ull;

    __device__ bool abort_seen() const {
        return *(volatile int*)&sh.abort || *(volatile const int*)(p.state + B2_MK_ERR);
    }
    // Elements 4 tid .. 4 tid + 3 of an LL vector, polled until all carry
    // tag t (false after the poll limit or an abort elsewhere).
    __device__ bool poll4(const unsigned long long* src, uint32_t t, float4& v) const {
        if (4 * tid >= p.hidden) {
            v = make_float4(0.f, 0.f, 0.f, 0.f);
            return true;
        }
        for (long long it = 0;; it++) {
            const ulonglong2 a = ll_get2(src + 4 * tid), b = ll_get2(src + 4 * tid + 2);
            if (ll_ok(a.x, t) && ll_ok(a.y, t) && ll_ok(b.x, t) && ll_ok(b.y, t)) {
                v = make_float4(ll_val(a.x), ll_val(a.y), ll_val(b.x), ll_val(b.y));
                return true;
            }
            if (it > limit || ((it & 63) == 63 && abort_seen())) {
                if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                return false;
            }
            if (it > 8) __nanosleep(32);
        }
    }
    // One LL word polled until it carries `want`.
    __device__ bool poll1(const unsigned long long* w, uint32_t want, float& v) const {
        for (long long it = 0;; it++) {
            const unsigned long long x = ll_get(w);
            if (ll_ok(x, want)) {
                v = ll_val(x);
                return true;
            }
            if (it > limit || ((it & 63) == 63 && abort_seen())) {
                if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                return false;
            }
            if (it > 8) __nanosleep(32);
        }
    }
    // Tag of layer l's words: unique over 2^27 consecutive steps (a word is
    // rewritten every step, so a reader never meets one older than a step).
    __device__ uint32_t ltag(int l) const { return tag * (uint32_t)kMaxLayers + (uint32_t)l; }
    __device__ unsigned long long* opart(int g) const { return S.opart + (size_t)g * p.hidden; }
    // the kOwn words CTA c sends to reducer r
    __device__ unsigned long long* dpart(int r, int c) const { return S.dpart + ((size_t)r * kMaxG + c) * kOwn; }
    // outputs [own0, own0 + nown) this CTA reduces
    __device__ int own0() const { return kOwn * geo.cta; }
    __device__ int nown() const { return kOwn * geo.cta < p.hidden ? kOwn : 0; }

    // x at elements 4 tid .. 4 tid + 3: the embedding row (l < 0) or the
    // output of layer l
    __device__ bool load_x(int l, float4& x) const {
        if (l < 0) {
            const int e = 4 * tid;
            if (e >= p.hidden) {
                x = make_float4(0.f, 0.f, 0.f, 0.f);
                return true;
            }
            const float* row = p.state[B2_MK_USE_EMB] ? p.staged_emb : p.emb + (size_t)p.state[B2_MK_TOKEN] * p.hidden;
            x = __ldg(reinterpret_cast<const float4*>(row + e));
            return true;
        }
        return poll4(S.xout, ltag(l), x);
    }

    // RMSNorm (weights nw) of the distributed vector x (4 elements per
    // thread) and FP16 rounding into dst in the row dots' k order (int8 table
    // for the lm_head: natural order).
    __device__ float4 norm_w(const float* nw) const {
        return 4 * tid < p.hidden ? __ldg(reinterpret_cast<const float4*>(nw) + tid) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __device__ bool stage(float4 x, float4 w, __half* dst, bool perm) {
        const int e = 4 * tid;
        const bool has = e < p.hidden;
        float ss = has ? fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, x.w * x.w))) : 0.f;
        ss = b2::warp_sum(ss);
        if (lane == 0) sh.red[warp] = ss;
        if (!vote(true)) return false;
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NC; w++) t += sh.red[w];
        const float rms = 1.0f / sqrtf(t / (float)p.hidden + p.eps);
        if (has) {
            const float v[4] = {(x.x * rms) * w.x, (x.y * rms) * w.y, (x.z * rms) * w.z, (x.w * rms) * w.w};
#pragma unroll
            for (int i = 0; i < 4; i++) dst[perm ? stage_pos<WT>(e + i) : e + i] = __float2half_rn(v[i]);
        }
        return vote(true);
    }

    // ── control operations ──

    __device__ bool xin(int l) {
        const float4 w = norm_w(sh.lay[l].in_norm);  // in flight during the wait
        float4 x;
        const bool ok = load_x(l - 1, x);
        if (!vote(ok)) return false;
        if (4 * tid < p.hidden) *reinterpret_cast<float4*>(&sh.xres[4 * tid]) = x;
        return stage(x, w, sh.xs[0], true);
    }

    // The unit's q heads, new k and v: poll the LL words of head group g, then
    // per-head RMSNorm and RoPE (src/matmul_decoder.c:1495-1510); unit r = 0
    // appends K and V at this position (:1512-1516).
    __device__ bool ain(int l, int g, int r) {
        const B2MkLayer& Lw = sh.lay[l];
        const unsigned long long* qkv = S.qkv;
        const uint32_t t = ltag(l);
        const int h = warp, e0 = lane * 4;
        bool ok = true;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        // static inputs first, in flight during the poll: norm weights, RoPE angles
        const float* nwp = h < kGq ? Lw.q_norm : h == kGq ? Lw.k_norm : nullptr;
        const float4 nw = nwp ? __ldg(reinterpret_cast<const float4*>(nwp + e0)) : make_float4(1.f, 1.f, 1.f, 1.f);
        float cs[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
        if (h <= kGq) {
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
        if (h < kGq + 2) {
            const unsigned long long* src = h < kGq ? qkv + (size_t)(g * kGq + h) * kHD
                                            : h == kGq ? qkv + geo.qd + (size_t)g * kHD
                                                       : qkv + geo.qd + geo.kvd + (size_t)g * kHD;
            for (long long it = 0;; it++) {
                const ulonglong2 a = ll_get2(src + e0), b = ll_get2(src + e0 + 2);
                if (ll_ok(a.x, t) && ll_ok(a.y, t) && ll_ok(b.x, t) && ll_ok(b.y, t)) {
                    x[0] = ll_val(a.x), x[1] = ll_val(a.y), x[2] = ll_val(b.x), x[3] = ll_val(b.y);
                    break;
                }
                if (it > limit || ((it & 63) == 63 && abort_seen())) {
                    if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                    ok = false;
                    break;
                }
                if (it > 8) __nanosleep(32);
            }
        }
        if (!vote(ok)) return false;
        if (h <= kGq) {
            if (nwp) {
                float ss = fmaf(x[0], x[0], fmaf(x[1], x[1], fmaf(x[2], x[2], x[3] * x[3])));
                ss = b2::warp_sum(ss);
                const float rms = 1.0f / sqrtf(ss / (float)kHD + p.eps);
                x[0] = (x[0] * rms) * nw.x, x[1] = (x[1] * rms) * nw.y, x[2] = (x[2] * rms) * nw.z,
                x[3] = (x[3] * rms) * nw.w;
            }
            if (p.rope_style == 0) {  // interleaved pairs (2i, 2i+1) at angle i
#pragma unroll
                for (int j = 0; j < 4; j += 2) {
                    const float x0 = x[j], x1 = x[j + 1];
                    x[j] = x0 * cs[j] - x1 * sn[j];
                    x[j + 1] = x1 * cs[j] + x0 * sn[j];
                }
            } else {  // split halves (e, e + hd/2) at angle e
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
                    x[j] = lane < 16 ? x[j] * cs[j] - other * sn[j] : x[j] * cs[j] + other * sn[j];
                }
            }
        }
        if (h < kGq) {
#pragma unroll
            for (int j = 0; j < 4; j++) sh.sq[h][e0 + j] = x[j];
        } else if (h < kGq + 2) {
            __half* row = h == kGq ? sh.knew : sh.vnew;
            __half* cache = nullptr;
            if (r == 0)
                cache = reinterpret_cast<__half*>(h == kGq ? p.k_cache : p.v_cache) + (size_t)l * p.layer_stride +
                        ((size_t)g * p.max_seq + geo.pos) * kHD;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const __half v = __float2half_rn(x[j]);
                row[e0 + j] = v;
                if (cache) cache[e0 + j] = v;
            }
        }
        // every softmax state starts empty
#pragma unroll
        for (int hh = 0; hh < kGq; hh++) {
            *reinterpret_cast<float4*>(&sh.mrg_o[warp][hh][e0]) = make_float4(0.f, 0.f, 0.f, 0.f);
            if (lane == 0) {
                sh.mrg_m[warp][hh] = -INFINITY;
                sh.mrg_l[warp][hh] = 0.f;
            }
        }
        return vote(true);
    }

    // Split attention, this unit's share: the warps' softmax states merged
    // into one (max, sum, unnormalized output per q head) and published.
    __device__ bool apub(int l) {
        unsigned long long* dst = S.apart + ((size_t)geo.ug * kSplit + geo.ur) * (4 + 2 * kHD);
        const uint32_t t = ltag(l);
        // (called after a barrier that follows the last attend_op)
        if ((lane >> 3) == 0) {
            const int hv = warp >> 2, dq = (warp & 3) * 8 + (lane & 7);
            const float4 uo = *reinterpret_cast<const float4*>(&sh.mrg_o[0][hv][4 * dq]);
            unsigned long long* o = dst + 4 + hv * kHD + 4 * dq;
            ll_put(o, uo.x, t), ll_put(o + 1, uo.y, t), ll_put(o + 2, uo.z, t), ll_put(o + 3, uo.w, t);
        }
        if (tid < kGq) {
            ll_put(dst + 2 * tid, sh.mrg_m[0][tid], t);
            ll_put(dst + 2 * tid + 1, sh.mrg_l[0][tid], t);
        }
        return true;
    }

    // One unit's published state (both q heads; this lane's 4 dims), polled
    // until every word carries the tag.
    __device__ bool poll_state(const unsigned long long* src, uint32_t t, float (&m)[kGq], float (&lv)[kGq],
                               float4 (&o)[kGq]) const {
        for (long long it = 0;; it++) {
            const ulonglong2 a = ll_get2(src), b = ll_get2(src + 2);
            const ulonglong2 c = ll_get2(src + 4 + 4 * lane), e = ll_get2(src + 6 + 4 * lane);
            const ulonglong2 f = ll_get2(src + 4 + kHD + 4 * lane), g = ll_get2(src + 6 + kHD + 4 * lane);
            if (ll_ok(a.x, t) && ll_ok(a.y, t) && ll_ok(b.x, t) && ll_ok(b.y, t) && ll_ok(c.x, t) && ll_ok(c.y, t) &&
                ll_ok(e.x, t) && ll_ok(e.y, t) && ll_ok(f.x, t) && ll_ok(f.y, t) && ll_ok(g.x, t) && ll_ok(g.y, t)) {
                m[0] = ll_val(a.x), lv[0] = ll_val(a.y), m[1] = ll_val(b.x), lv[1] = ll_val(b.y);
                o[0] = make_float4(ll_val(c.x), ll_val(c.y), ll_val(e.x), ll_val(e.y));
                o[1] = make_float4(ll_val(f.x), ll_val(f.y), ll_val(g.x), ll_val(g.y));
                return true;
            }
            if (it > limit || ((it & 63) == 63 && abort_seen())) {
                if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                return false;
            }
            if (it > 8) __nanosleep(32);
        }
    }

    // Split attention, every unit of the head: warp w merges the published
    // states of units w and w + 8 (in that order), then the merge of aout adds
    // the newest position, combines the warps in warp order and normalizes.
    __device__ bool amrg(int l) {
        float4 o[kGq] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
        float m[kGq] = {-INFINITY, -INFINITY}, lv[kGq] = {0.f, 0.f};
        bool ok = true;
        const uint32_t t = ltag(l);
        for (int u = warp; u < geo.S && ok; u += NC) {
            float mu[kGq], lu[kGq];
            float4 ou[kGq];
            ok = poll_state(S.apart + ((size_t)geo.ug * kSplit + u) * (4 + 2 * kHD), t, mu, lu, ou);
            if (!ok) break;
#pragma unroll
            for (int h = 0; h < kGq; h++) {
                if (mu[h] == -INFINITY) continue;
                const float M = fmaxf(m[h], mu[h]);
                const float c1 = m[h] == -INFINITY ? 0.f : expf(m[h] - M), c2 = expf(mu[h] - M);
                lv[h] = lv[h] * c1 + lu[h] * c2;
                o[h] = make_float4(o[h].x * c1 + ou[h].x * c2, o[h].y * c1 + ou[h].y * c2, o[h].z * c1 + ou[h].z * c2,
                                   o[h].w * c1 + ou[h].w * c2);
                m[h] = M;
            }
        }
        const float4 o0 = o[0], o1 = o[1];
        const float m0 = m[0], l0 = lv[0], m1 = m[1], l1 = lv[1];
        *reinterpret_cast<float4*>(&sh.mrg_o[warp][0][4 * lane]) = o0;
        *reinterpret_cast<float4*>(&sh.mrg_o[warp][1][4 * lane]) = o1;
        if (lane == 0) {
            sh.mrg_m[warp][0] = m0, sh.mrg_l[warp][0] = l0;
            sh.mrg_m[warp][1] = m1, sh.mrg_l[warp][1] = l1;
        }
        __syncwarp();
        if (!vote(ok)) return false;
        return aout_merge();
    }

    // All consumer threads: online softmax over n <= kAttMax positions (K and V
    // rows of 256 bytes), and the newest position (sh.knew / vnew) after them
    // when with_new, into the unit's state in slot 0 of sh.mrg_m / mrg_l /
    // mrg_o.  Thread 0 writes the max and sum after the last barrier (every
    // thread reads them after the next call's first barrier); each output
    // element has one owner thread, which alone reads and writes it.
    //  1. scores: thread t takes position t >> 1, q head t & 1, the 128-dim
    //     dot product over 16-byte chunks in a per-position rotated order (the
    //     rows sit 256 bytes apart, so unrotated chunks would share banks);
    //  2. per-head maximum and exponentials (warp shuffles, then the eight
    //     warps' values through shared memory);
    //  3. P.V: thread (head warp >> 2, dims 4 dq .. + 3, quarter lane >> 3)
    //     sums a quarter of the positions; the quarters meet by shuffles.
    __device__ bool attend_op(const unsigned char* kb, const unsigned char* vb, int n, bool with_new) {
        float* pr = reinterpret_cast<float*>(sh.xs[1]);  // [kGq][kAttMax] probabilities (free during attention)
        float* wmax = pr + kGq * kAttMax;                 // [NC][kGq]
        float* wsum = wmax + NC * kGq;                    // [NC][kGq]
        const float scale = 0.08838834764831845f;         // 1/sqrt(128)
        const int i = tid >> 1, h = tid & 1, m_all = n + (with_new ? 1 : 0);
        float sc = -INFINITY;
        if (i < m_all) {
            const unsigned char* kr = i < n ? kb + (size_t)i * 256 : reinterpret_cast<const unsigned char*>(sh.knew);
            const float* q = sh.sq[h];
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 2
            for (int c = 0; c < 16; c++) {
                const int cc = (c + i) & 15;
                const uint4 kk = *reinterpret_cast<const uint4*>(kr + cc * 16);
                const float4 qa = *reinterpret_cast<const float4*>(q + cc * 8);
                const float4 qb = *reinterpret_cast<const float4*>(q + cc * 8 + 4);
                const float2 k0 = b2::h2_to_f2(kk.x), k1 = b2::h2_to_f2(kk.y);
                const float2 k2 = b2::h2_to_f2(kk.z), k3 = b2::h2_to_f2(kk.w);
                a0 = fmaf(qa.x, k0.x, fmaf(qa.y, k0.y, a0));
                a1 = fmaf(qa.z, k1.x, fmaf(qa.w, k1.y, a1));
                a2 = fmaf(qb.x, k2.x, fmaf(qb.y, k2.y, a2));
                a3 = fmaf(qb.z, k3.x, fmaf(qb.w, k3.y, a3));
            }
            sc = ((a0 + a1) + (a2 + a3)) * scale;
        }
        float m = sc;
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (lane < kGq) wmax[warp * kGq + lane] = m;  // lane h holds head h
        if (!vote(true)) return false;
        float mn[kGq], c[kGq];
#pragma unroll
        for (int hh = 0; hh < kGq; hh++) {
            const float mo = sh.mrg_m[0][hh];
            float M = mo;
#pragma unroll
            for (int w = 0; w < NC; w++) M = fmaxf(M, wmax[w * kGq + hh]);
            mn[hh] = M;
            c[hh] = mo == -INFINITY ? 0.f : expf(mo - M);
        }
        const float pe = i < m_all ? expf(sc - (h == 0 ? mn[0] : mn[1])) : 0.f;
        pr[h * kAttMax + i] = pe;
        float ps = pe;
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        if (lane < kGq) wsum[warp * kGq + lane] = ps;
        if (!vote(true)) return false;
        float lnew[kGq];
#pragma unroll
        for (int hh = 0; hh < kGq; hh++) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < NC; w++) t += wsum[w * kGq + hh];
            lnew[hh] = sh.mrg_l[0][hh] * c[hh] + t;
        }
        const int hv = warp >> 2, dq = (warp & 3) * 8 + (lane & 7), pq = lane >> 3;
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
        const float* ph = pr + hv * kAttMax + pq * (kAttMax / 4);
        const unsigned char* vr = vb + (size_t)pq * (kAttMax / 4) * 256 + dq * 8;
#pragma unroll 8
        for (int j = 0; j < kAttMax / 4; j++) {
            if (pq * (kAttMax / 4) + j >= n) break;
            const float pj = ph[j];
            const uint2 vv = *reinterpret_cast<const uint2*>(vr + (size_t)j * 256);
            const float2 v01 = b2::h2_to_f2(vv.x), v23 = b2::h2_to_f2(vv.y);
            o0 = fmaf(pj, v01.x, o0), o1 = fmaf(pj, v01.y, o1), o2 = fmaf(pj, v23.x, o2), o3 = fmaf(pj, v23.y, o3);
        }
        if (with_new && pq == 0) {  // the newest position, from shared memory
            const float pj = pr[hv * kAttMax + n];
            const uint2 vv = *reinterpret_cast<const uint2*>(reinterpret_cast<const unsigned char*>(sh.vnew) + dq * 8);
            const float2 v01 = b2::h2_to_f2(vv.x), v23 = b2::h2_to_f2(vv.y);
            o0 = fmaf(pj, v01.x, o0), o1 = fmaf(pj, v01.y, o1), o2 = fmaf(pj, v23.x, o2), o3 = fmaf(pj, v23.y, o3);
        }
        o0 += __shfl_xor_sync(0xffffffffu, o0, 8), o1 += __shfl_xor_sync(0xffffffffu, o1, 8);
        o2 += __shfl_xor_sync(0xffffffffu, o2, 8), o3 += __shfl_xor_sync(0xffffffffu, o3, 8);
        o0 += __shfl_xor_sync(0xffffffffu, o0, 16), o1 += __shfl_xor_sync(0xffffffffu, o1, 16);
        o2 += __shfl_xor_sync(0xffffffffu, o2, 16), o3 += __shfl_xor_sync(0xffffffffu, o3, 16);
        if (pq == 0) {
            const float cv = hv == 0 ? c[0] : c[1];
            float4* uo = reinterpret_cast<float4*>(&sh.mrg_o[0][hv][4 * dq]);
            const float4 u = *uo;
            *uo = make_float4(fmaf(u.x, cv, o0), fmaf(u.y, cv, o1), fmaf(u.z, cv, o2), fmaf(u.w, cv, o3));
        }
        if (!vote(true)) return false;  // the state and probabilities are read before they change
        if (tid == 0) {
#pragma unroll
            for (int hh = 0; hh < kGq; hh++) sh.mrg_m[0][hh] = mn[hh], sh.mrg_l[0][hh] = lnew[hh];
        }
        return true;
    }

    // Non-split attention without cached positions: the newest position alone.
    __device__ bool aout() { return attend_op(nullptr, nullptr, 0, true) && finish_out(); }

    // xo = output / sum of the unit's state (after the last attention step).
    __device__ bool finish_out() {
        if (!vote(true)) return false;  // thread 0's sums are in
        if ((lane >> 3) == 0) {
            const int hv = warp >> 2, dq = (warp & 3) * 8 + (lane & 7);
            const float inv = 1.0f / sh.mrg_l[0][hv];
            const float4 uo = *reinterpret_cast<const float4*>(&sh.mrg_o[0][hv][4 * dq]);
            const float v[4] = {uo.x, uo.y, uo.z, uo.w};
#pragma unroll
            for (int j = 0; j < 4; j++) sh.xo[stage_pos<WT>(hv * kHD + 4 * dq + j)] = __float2half_rn(v[j] * inv);
        }
        return vote(true);
    }

    // The newest position (warp 0), then the merge of the warps' softmax
    // states into the FP16 attention output xo (the o_proj input).
    __device__ bool aout_merge() {
        if (warp == 0)
            attend16(sh, reinterpret_cast<const unsigned char*>(sh.knew), reinterpret_cast<const unsigned char*>(sh.vnew),
                    1, warp, lane);
        if (!vote(true)) return false;
        {
            const int h = tid / kHD, d = tid % kHD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NC; w++) M = fmaxf(M, sh.mrg_m[w][h]);
            float den = 0.f, num = 0.f;
#pragma unroll
            for (int w = 0; w < NC; w++) {
                const float m = sh.mrg_m[w][h];
                if (m == -INFINITY) continue;
                const float c = expf(m - M);
                den = fmaf(sh.mrg_l[w][h], c, den);
                num = fmaf(sh.mrg_o[w][h][d], c, num);
            }
            sh.xo[stage_pos<WT>(tid)] = __float2half_rn(num / den);
        }
        return vote(true);
    }

    __device__ bool gin(int l) {
        const float4 w = norm_w(sh.lay[l].post_norm);
        float4 h;
        const bool ok = poll4(S.hmid, ltag(l), h);
        if (!vote(ok)) return false;  // (also: every RO of this CTA read xres as x)
        if (4 * tid < p.hidden) *reinterpret_cast<float4*>(&sh.xres[4 * tid]) = h;  // the residual of RD
#pragma unroll
        for (int i = 0; i < 4; i++) dacc[i] = 0.f;
        return stage(h, w, sh.xs[1], true);
    }

    // h_mid of the outputs this CTA owns: the nkv o_proj partials (fixed
    // order) plus the residual x.
    __device__ bool ro(int l) {
        const int o0 = own0(), n = nown();
        float* red = &sh.mrg_o[0][0][0];  // [nkv][kOwn] (free outside attention)
        bool ok = true;
        if (tid < n * p.nkv) {  // every partial polled at once, one per thread
            const int g = tid / n, j = tid - g * n;
            float v;
            ok = poll1(opart(g) + o0 + j, ltag(l), v);
            red[g * kOwn + j] = v;
        }
        if (!vote(ok)) return false;
        if (tid < n) {
            float acc = 0.f;
            for (int g = 0; g < p.nkv; g++) acc += red[g * kOwn + tid];
            ll_put(S.hmid + o0 + tid, acc + sh.xres[o0 + tid], ltag(l));
        }
        return vote(true);  // the partials are read before the next use of mrg_o
    }

    // Layer output of the outputs this CTA owns: every CTA's down partial
    // (summed in CTA order) plus the residual h_mid.  The partials are polled
    // only once the publication counter says all CTAs have sent theirs, which
    // keeps early reducers from loading L2 while the last CTAs still stream
    // their down weights; the tags still decide what is read.
    __device__ bool rd(int l) {
        const int o0 = own0(), n = nown();
        if (n == 0) return true;
        float* red = &sh.mrg_o[0][0][0];  // [kMaxG][kOwn] partial sums by source CTA (free here)
        bool ok = true;
        if (tid == 0) {
            const unsigned long long target =
                ((unsigned long long)(tag - 1) * p.n_layers + l + 1) * (unsigned long long)geo.G;
            for (long long it = 0;; it++) {
                unsigned long long c;
                asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(c) : "l"(S.dcnt) : "memory");
                if (c >= target) break;
                if (it > limit || ((it & 63) == 63 && abort_seen())) {
                    if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                    ok = false;
                    break;
                }
                if (it > 8) __nanosleep(32);
            }
        }
        if (!vote(ok)) return false;
        const uint32_t t = ltag(l);
        for (int c = tid; c < geo.G && ok; c += kCons) {
            const unsigned long long* src = dpart(geo.cta, c);
            for (long long it = 0;; it++) {
                const ulonglong2 a = ll_get2(src), b = ll_get2(src + 2), e = ll_get2(src + 4), f = ll_get2(src + 6);
                if (ll_ok(a.x, t) && ll_ok(a.y, t) && ll_ok(b.x, t) && ll_ok(b.y, t) && ll_ok(e.x, t) &&
                    ll_ok(e.y, t) && ll_ok(f.x, t) && ll_ok(f.y, t)) {
                    float4* dst = reinterpret_cast<float4*>(red + c * kOwn);
                    dst[0] = make_float4(ll_val(a.x), ll_val(a.y), ll_val(b.x), ll_val(b.y));
                    dst[1] = make_float4(ll_val(e.x), ll_val(e.y), ll_val(f.x), ll_val(f.y));
                    break;
                }
                if (it > limit || ((it & 63) == 63 && abort_seen())) {
                    if (it > limit) atomicOr(p.state + B2_MK_ERR, 1);
                    ok = false;
                    break;
                }
                if (it > 8) __nanosleep(32);
            }
        }
        if (!vote(ok)) return false;
        if (tid < n) {
            float acc = 0.f;
            for (int c = 0; c < geo.G; c++) acc += red[c * kOwn + tid];
            ll_put(S.xout + o0 + tid, acc + sh.xres[o0 + tid], t);
        }
        return vote(true);  // the partial area is read before the next use of mrg_o
    }

    // This CTA's down partial (its channels' contribution to every output,
    // times the per-output scale) as LL words for the reducers.
    __device__ bool dend(int l) {
        const int n = 4 * tid;
        if (n < p.hidden) {
            const float* ds = sh.lay[l].dn_s;
            float4 d = make_float4(dacc[0], dacc[1], dacc[2], dacc[3]);
            if (ds) {
                const float4 sc = __ldg(reinterpret_cast<const float4*>(ds + n));
                d.x *= sc.x, d.y *= sc.y, d.z *= sc.z, d.w *= sc.w;
            }
            // outputs n .. n + 3 are half (tid & 1) of reducer tid / 2's words
            unsigned long long* dst = dpart(tid >> 1, geo.cta) + 4 * (tid & 1);
            const unsigned long long t = (unsigned long long)ltag(l) << 32;
            const ulonglong2 a = make_ulonglong2(t | __float_as_uint(d.x), t | __float_as_uint(d.y));
            const ulonglong2 b = make_ulonglong2(t | __float_as_uint(d.z), t | __float_as_uint(d.w));
            asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a.x), "l"(a.y) : "memory");
            asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(b.x), "l"(b.y) : "memory");
        }
        // count this CTA's publication (a hint for the reducers' polling: the
        // other warps' words may still be in flight, their tags decide)
        if (tid == 0) asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(S.dcnt) : "memory");
        return true;
    }

    __device__ bool lin() {
        const float4 w = norm_w(p.final_norm);
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        bool ok = true;
        if (p.stall_test) {  // a word no CTA writes with this tag: the wait runs out
            float v;
            ok = poll1(S.xout, ltag(p.n_layers), v);  // (the next layer's tag: never written)
        }
        ok = ok && load_x(p.n_layers - 1, x);
        if (!vote(ok)) return false;
        if (geo.cta == 0 && 4 * tid < p.hidden) reinterpret_cast<float4*>(S.hfinal)[tid] = x;
        best = 0ull;
        return stage(x, w, sh.xs[0], false);  // int8 table: natural k order
    }

    __device__ bool pfin() {  // prefill-mode step: publish the final hidden state
        float4 x;
        const bool ok = geo.cta != 0 || load_x(p.n_layers - 1, x);
        if (!vote(ok)) return false;
        if (geo.cta == 0 && 4 * tid < p.hidden) reinterpret_cast<float4*>(S.hfinal)[tid] = x;
        return true;
    }

    __device__ bool lend() {
        const unsigned long long b = b2::warp_max_u64(best);  // threads < 64 hold keys
        if (lane == 0) sh.best[warp] = b;
        if (!vote(true)) return false;
        if (tid == 0) {
            unsigned long long m = 0ull;
            for (int w = 0; w < NC; w++) m = sh.best[w] > m ? sh.best[w] : m;
            atomicMax(S.cnt + 1, m);
        }
        return true;
    }

    // ── data operations ──

    // Row dots of the operation's T (<= 4) tiles, `stride` bytes apart, nsb
    // super-blocks each: warp w takes its slice of every tile's super-blocks,
    // the partial sums meet in sh.part, and after the barrier thread r < 16 T
    // holds row r (tile r / 16, row r % 16) in the return value.
    __device__ float op_dots(const unsigned char* buf, uint32_t stride, int T, int nsb, const __half* xs, bool int8,
                             int pb, bool& ok) {
        const int s0 = split_lo(nsb, NC, warp), s1 = split_lo(nsb, NC, warp + 1);
        const int g = lane >> 2;
        float y[4][2];
        if (int8) tiles_dot<B2_W_I8>(buf, stride, T, xs, s0, s1, lane, y);
        else tiles_dot<WT>(buf, stride, T, xs, s0, s1, lane, y);
        if ((lane & 3) == 0)
#pragma unroll
            for (int t = 0; t < 4; t++)
                if (t < T) {
                    sh.part[pb][warp][16 * t + g] = y[t][0];
                    sh.part[pb][warp][16 * t + g + 8] = y[t][1];
                }
        ok = vote(true);
        float v = 0.f;
        if (ok && tid < 16 * T)
#pragma unroll
            for (int w = 0; w < NC; w++) v += sh.part[pb][w][tid];
        return v;
    }

    __device__ bool qkv_tiles(const Desc& d, const unsigned char* buf, int pb) {
        const int T = d.b - d.a, nsb = row_bytes(WT, p.hidden) / 64;
        const int r = 16 * d.a + tid;
        const float* sc = sh.lay[d.l].qkv_s;
        const float s = (sc && tid < 16 * T) ? __ldg(sc + r) : 1.f;
        bool ok;
        const float v = op_dots(buf, 16u * row_bytes(WT, p.hidden), T, nsb, sh.xs[0], false, pb, ok);
        if (ok && tid < 16 * T) ll_put(S.qkv + r, v * s, ltag(d.l));
        return ok;
    }

    // The operation's positions (K rows, then V rows), and the newest one
    // after the last operation of an unsplit head.
    __device__ bool kv_op(const Desc& d, const unsigned char* buf, bool with_new) {
        const int n = d.b - d.a;
        return attend_op(buf, buf + (size_t)n * 256, n, with_new);
    }

    __device__ bool o_tiles(const Desc& d, const unsigned char* buf, int pb) {
        const int T = d.b - d.a, nsb = row_bytes(WT, kGq * kHD) / 64;
        const int r = 16 * d.a + tid;
        const float* sc = sh.lay[d.l].o_s;
        const float s = (sc && tid < 16 * T) ? __ldg(sc + r) : 1.f;
        bool ok;
        const float v = op_dots(buf, 1024u * (uint32_t)nsb, T, nsb, sh.xo, false, pb, ok);
        if (ok && tid < 16 * T) ll_put(opart(d.c) + r, v * s, ltag(d.l));
        return ok;
    }

    // Tiles of 8 channels, rows gate(c), up(c) interleaved: thread j < 8 T
    // gets channel j's SiLU(gate) * up, FP16-rounded as the down input.
    __device__ bool gu_tiles(const Desc& d, const unsigned char* buf, int pb) {
        const int T = d.b - d.a, nsb = row_bytes(WT, p.hidden) / 64;
        const float* sc = sh.lay[d.l].gu_ts;
        const float s = (sc && tid < 16 * T) ? __ldg(sc + 16 * d.a + tid) : 1.f;
        bool ok;
        const float v = op_dots(buf, 16u * row_bytes(WT, p.hidden), T, nsb, sh.xs[1], false, pb, ok) * s;
        const float u = __shfl_down_sync(0xffffffffu, v, 1);
        if (ok && tid < 16 * T && (tid & 1) == 0)
            sh.act[8 * (d.a - geo.c0) + tid / 2] = __half2float(__float2half_rn((v / (1.0f + expf(-v))) * u));
        return ok;
    }

    // Down partial: outputs 4 tid .. 4 tid + 3 over channels [a, b) of the
    // input-major down weight (exact widening, FP32 sums; the per-output
    // scale is applied in dend).
    __device__ void dn_rows(const Desc& d, const unsigned char* buf) {
        const int n = 4 * tid;
        if (n >= p.hidden) return;
        const int rb = row_bytes(WT, p.hidden), base = 8 * geo.c0;
#pragma unroll 8
        for (int jj = 0; jj < kMaxCh; jj++) {
            const int j = d.a + jj;
            if (j >= d.b) break;
            const float a = sh.act[j - base];
            const unsigned char* row = buf + (size_t)jj * rb;
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
            for (int i = 0; i < 4; i++) dacc[i] = fmaf(a, w[i], dacc[i]);
        }
    }

    __device__ bool lm_tiles(const Desc& d, const unsigned char* buf, int pb) {
        const int T = d.b - d.a, r = 16 * d.a + tid;
        const float s = tid < 16 * T ? __ldg(p.lm_s + r) : 0.f;
        bool ok;
        const float v = op_dots(buf, 16u * (uint32_t)p.hidden, T, p.hidden / 64, sh.xs[0], true, pb, ok);
        if (ok && tid < 16 * T) {
            const float logit = v * s;
            if (p.logits) p.logits[r] = logit;
            const unsigned long long k = b2::argmax_key(logit, (uint32_t)r);
            best = k > best ? k : best;
        }
        return ok;
    }

    // Runs the operation stream; true when it reached OP_DONE.
    __device__ bool run() {
        int pb = 0;  // partial-sum buffer of the next dot operation (alternates)
        for (int k = 0;; k++) {
            const int s = k % kND;
            const uint32_t parity = (uint32_t)((k / kND) & 1);
            bool got = true;
            for (long long it = 0; !mbar_try_wait(&sh.full[s], parity); it++) {
                if (*(volatile int*)&sh.abort) {
                    got = false;
                    break;
                }
                if (it > limit) {
                    set_error(p, sh, 3);
                    got = false;
                    break;
                }
            }
            if (!got) {
                vote(false);  // pairs with the next vote of the other warps
                return false;
            }
            const Desc d = sh.desc[s];
            const unsigned char* buf = ring + d.off;
            bool ok = true;
            switch (d.op) {
                case OP_XIN: ok = xin(d.l); break;
                case OP_QKV:
                    pb ^= 1;
                    ok = (d.a != geo.q0 || xin(d.l)) && qkv_tiles(d, buf, pb);
                    break;
                case OP_AIN: ok = vote(true) && ain(d.l, d.c, d.d); break;
                case OP_KV:
                    ok = d.a != geo.a0 || (vote(true) && ain(d.l, d.c, d.d));
                    ok = ok && kv_op(d, buf, d.b == geo.a1 && !geo.split);
                    if (ok && d.b == geo.a1) ok = geo.split ? (vote(true) && apub(d.l)) : finish_out();
                    break;
                case OP_AOUT: ok = vote(true) && aout(); break;
                case OP_APUB: ok = vote(true) && apub(d.l); break;
                case OP_AMRG: ok = vote(true) && amrg(d.l); break;  // (apub's reads of the warp states are done)
                case OP_O: ok = o_tiles(d, buf, pb ^= 1); break;
                case OP_RO: ok = vote(true) && ro(d.l) && gin(d.l); break;
                case OP_GIN: ok = gin(d.l); break;
                case OP_GU: ok = gu_tiles(d, buf, pb ^= 1); break;
                case OP_ACT: ok = vote(true); break;
                case OP_DN:
                    ok = d.a != 8 * geo.c0 || vote(true);  // every channel's act is in shared memory
                    if (ok) dn_rows(d, buf);
                    if (ok && d.b == 8 * geo.c1) ok = dend(d.l);
                    break;
                case OP_DEND: ok = vote(true) && dend(d.l); break;
                case OP_RD: ok = vote(true) && rd(d.l); break;
                case OP_LIN: ok = lin(); break;
                case OP_LM: ok = lm_tiles(d, buf, pb ^= 1); break;
                case OP_LEND: ok = vote(true) && lend(); break;
                case OP_PFIN: ok = pfin(); break;
                case OP_DONE: ok = vote(true); break;
                default: ok = vote(false); break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.empty[s]);
            if (!ok) {
                if (tid == 0) *(volatile int*)&sh.abort = 1;
                return false;
            }
            if (d.op == OP_DONE) return true;
        }
    }
};

template <int WT>
__global__ void __launch_bounds__(kThreads, 1) mk2_kernel(const __grid_constant__ B2MkPlan p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;
    Sh& sh = *reinterpret_cast<Sh*>(smem + kRing);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long limit = p.poll_limit > 0 ? p.poll_limit : kDefaultPolls;

    if (tid == 0) {
        for (int s = 0; s < kND; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], NC);
        }
        sh.abort = 0;
        sh.issued = 0;
        sh.pk = sh.pfh = sh.pft = sh.pdead = 0;
        sh.phead = sh.ptail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const Geo geo = make_geo(p);
    const Scr S = scr_layout(p.scratch, p.n_layers, p.hidden, geo.nqkv, p.nkv, nullptr);
    const unsigned long long gen = (unsigned long long)(unsigned)p.state[B2_MK_GEN];

    if (warp == NC) {
        if (lane == 0) produce<WT>(p, geo, sh, ring, limit);
    } else {
        for (int i = tid; i < p.n_layers * (int)(sizeof(B2MkLayer) / 8); i += kCons)
            reinterpret_cast<unsigned long long*>(sh.lay)[i] = reinterpret_cast<const unsigned long long*>(p.layers)[i];
        consumer_sync();
        Consumer<WT> cons{p, geo, sh, ring, S, (uint32_t)(gen + 1), limit, tid, lane, warp};
        if (cons.run()) {  // FIN: the last CTA to arrive publishes the step
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
    // (outstanding only after an abort).  Operations older than the last kND
    // were consumed before their slot was reused.
    if (tid == kCons) {
        const int issued = *(volatile int*)&sh.issued;
        for (int k = max(0, issued - kND); k < issued; k++) {
            const int s = k % kND;
            if (sh.desc[s].bytes == 0) continue;
            for (long long it = 0; !mbar_try_wait(&sh.full[s], (uint32_t)((k / kND) & 1)) && it < limit; it++) {
            }
        }
    }
}

// ─── tile-major relayout (one-time) ───

__global__ void relayout_kernel(uint4* dst, const uint4* src, int rows, int rb16, int pair_half, float* dst_s,
                                const float* src_s) {
    // one thread per 16-byte unit of the destination, in the order
    // tile T, super-block s, row i, 16-byte part j
    const long long total = (long long)rows * rb16;
    const long long per_tile = 16ll * rb16;
    for (long long u = blockIdx.x * (long long)blockDim.x + threadIdx.x; u < total; u += (long long)gridDim.x * blockDim.x) {
        const int T = (int)(u / per_tile);
        const int rem = (int)(u % per_tile);
        const int s = rem / 64, i = (rem % 64) / 4, j = rem % 4;
        const int r = 16 * T + i;
        const int sr = pair_half > 0 ? ((i & 1) ? pair_half : 0) + 8 * T + i / 2 : r;
        dst[u] = src[(long long)sr * rb16 + s * 4 + j];
        if (dst_s && s == 0 && j == 0) dst_s[r] = src_s[sr];
    }
}

template <int WT>
int launch(const B2MkPlan* p, cudaStream_t s) {
    auto fn = mk2_kernel<WT>;
    static int configured[64] = {0};
    int dev = 0;
    B2_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk2_decode: device %d", dev);
    if (!configured[dev]) {
        B2_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        int per_sm = 0;
        B2_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, kSmemBytes));
        if (per_sm < 1) return b2_set_error(B2_ERR_CUDA, "b2_mk2_decode: kernel does not fit on an SM");
        configured[dev] = 1;
    }
    int sms = 0;
    B2_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (sms < p->nkv || sms > kMaxG)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk2_decode: %d SMs (kv heads %d, at most %d SMs)", sms, p->nkv, kMaxG);
    if ((p->hidden + kOwn - 1) / kOwn > sms)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk2_decode: hidden %d needs more SMs", p->hidden);
    if (8 * ((p->ffn / 8 + sms - 1) / sms) > kMaxCh)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk2_decode: ffn %d needs more SMs", p->ffn);
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
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_mk2_decode launch: %s", cudaGetErrorString(e));
    return 0;
}

}  // namespace

extern "C" int b2_mk2_max_context(void) { return 1 << 30; }  // any context: long ones split over units

extern "C" size_t b2_mk2_scratch_bytes(int n_layers, int hidden, int ffn, int nq, int nkv, int hd) {
    (void)ffn;
    size_t total = 0;
    scr_layout(nullptr, n_layers, hidden, nq * hd + 2 * nkv * hd, nkv, &total);
    return total;
}

extern "C" float* b2_mk2_final_hidden(const B2MkPlan* p) {
    Scr s = scr_layout(p->scratch, p->n_layers, p->hidden, p->nq * p->hd + 2 * p->nkv * p->hd, p->nkv, nullptr);
    return s.hfinal;
}

extern "C" int b2_mk2_check(const B2MkPlan* p) {
    if (!p) return B2_ERR_INVALID_ARG;
    if (p->n_layers < 1 || p->n_layers > kMaxLayers || p->hd != kHD || p->nkv < 1 || p->nq != kGq * p->nkv)
        return B2_ERR_INVALID_ARG;
    // every matmul a whole number of 16-row tiles of 64-byte super-blocks
    if (p->hidden != kMaxH || p->ffn % 8 || p->ffn > kMaxF || p->vocab % 16 || (p->nq * kHD + 2 * p->nkv * kHD) % 16)
        return B2_ERR_INVALID_ARG;
    if (p->wtype != B2_W_F16 && p->wtype != B2_W_I8 && p->wtype != B2_W_I4) return B2_ERR_INVALID_ARG;
    const int rb_h = row_bytes(p->wtype, p->hidden), rb_o = row_bytes(p->wtype, kGq * kHD);
    if (rb_h % 128 || rb_o % 128 || 16 * rb_h > kOpMax || p->hidden * 16 > kOpMax || rb_h * kMaxCh > kOpMax)
        return B2_ERR_INVALID_ARG;
    if (p->do_lm && (!p->lm_t || !p->lm_s || !p->final_norm)) return B2_ERR_INVALID_ARG;
    if (!p->layers || !p->state || !p->scratch || !p->k_cache || !p->v_cache || !p->cos_tab || !p->sin_tab || !p->emb)
        return B2_ERR_INVALID_ARG;
    return 0;
}

extern "C" int b2_mk2_decode(const B2MkPlan* p, b2_stream_t stream) {
    if (b2_mk2_check(p) != 0) return b2_set_error(B2_ERR_INVALID_ARG, "b2_mk2_decode: unsupported plan");
    cudaStream_t s = (cudaStream_t)stream;
    switch (p->wtype) {
        case B2_W_F16: return launch<B2_W_F16>(p, s);
        case B2_W_I8: return launch<B2_W_I8>(p, s);
        default: return launch<B2_W_I4>(p, s);
    }
}

extern "C" int b2_tile_relayout(void* dst, const void* src, int rows, int row_bytes, int pair_half, float* dst_s,
                                const float* src_s, b2_stream_t stream) {
    if (!dst || !src || rows <= 0 || rows % 16 || row_bytes <= 0 || row_bytes % 64 ||
        ((uintptr_t)dst | (uintptr_t)src) % 16 || (dst_s && !src_s) || (pair_half > 0 && rows != 2 * pair_half))
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_tile_relayout: bad arguments");
    const long long units = (long long)rows * (row_bytes / 16);
    const int threads = 256;
    const int blocks = (int)min((units + threads - 1) / threads, 148ll * 16);
    relayout_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>((uint4*)dst, (const uint4*)src, rows, row_bytes / 16,
                                                                  pair_half, dst_s, src_s);
    return b2_check_launch("b2_tile_relayout");
}
