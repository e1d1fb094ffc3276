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
constexpr int kStages = 6;
constexpr int kStageBytes = 32 * 1024;
constexpr int kHD = 128;
constexpr int kMaxK = 4096;        // longest activation staged as FP16
constexpr int kMaxSplit = 32;      // attention position ranges per kv head
constexpr int kCntPerLayer = 32;   // u64 counters per layer
constexpr int kMaxGq = 2;          // q heads per kv head handled by one attention unit
constexpr long long kPollLimit = 1ll << 23;
constexpr long long kBarLimit = 1ll << 22;

enum { C_QKV = 0, C_ATTN = 8, C_ATTN_DONE = 16, C_O = 17, C_GU = 18, C_DN = 19 };
enum { IT_QKV, IT_ATTN, IT_O, IT_GU, IT_DN, IT_LM };

struct Scratch {
    unsigned long long* cnt;  // [L][kCntPerLayer] + [8] globals
    float* hbuf;              // [L+1][H]
    float* hmid;              // [L][H]
    float* qkv;               // [L][qd + 2 kvd]
    float* attn;              // [L][qd]
    float* act;               // [L][F]
    float* part;              // [L][nkv][kMaxSplit][Gq][2 + hd]
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline Scratch scratch_layout(void* base, int L, int H, int F, int nq, int nkv, int hd,
                                                  size_t* total) {
    unsigned char* p = static_cast<unsigned char*>(base);
    size_t off = 0;
    Scratch s;
    const size_t qd = (size_t)nq * hd, kvd = (size_t)nkv * hd;
    s.cnt = reinterpret_cast<unsigned long long*>(p + off);
    off += align256(((size_t)L * kCntPerLayer + 8) * 8);
    s.hbuf = reinterpret_cast<float*>(p + off);
    off += align256((size_t)(L + 1) * H * 4);
    s.hmid = reinterpret_cast<float*>(p + off);
    off += align256((size_t)L * H * 4);
    s.qkv = reinterpret_cast<float*>(p + off);
    off += align256((size_t)L * (qd + 2 * kvd) * 4);
    s.attn = reinterpret_cast<float*>(p + off);
    off += align256((size_t)L * qd * 4);
    s.act = reinterpret_cast<float*>(p + off);
    off += align256((size_t)L * F * 4);
    s.part = reinterpret_cast<float*>(p + off);
    off += align256((size_t)L * nkv * kMaxSplit * (nq / nkv) * (2 + hd) * 4);
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

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long atom_add_acqrel(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
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

// ─── dot products from shared memory ───

template <int WT>
__device__ __forceinline__ void expand8(const uint4 wv, int g, float (&w)[8]) {
    const uint32_t* u = &wv.x;
    if constexpr (WT == B2_W_F16) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = b2::h2_to_f2(u[i]);
            w[2 * i] = f.x;
            w[2 * i + 1] = f.y;
        }
    } else if constexpr (WT == B2_W_I8) {
        const uint32_t a = u[2 * g], b = u[2 * g + 1];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[i] = (float)(int8_t)(a >> (8 * i));
            w[4 + i] = (float)(int8_t)(b >> (8 * i));
        }
    } else {
        const uint32_t a = u[g];
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (float)(((int32_t)(a << (28 - 4 * i))) >> 28);
    }
}

template <int WT>
__host__ __device__ constexpr int elems16() {
    return WT == B2_W_F16 ? 8 : WT == B2_W_I8 ? 16 : 32;
}

// Warp-collective dots of NR weight rows (rows[i], i < nvalid) in shared
// memory with the FP16 activation xs[K]; every lane gets the NR sums (rows at
// i >= nvalid re-read row 0 and their sums are meaningless).  All NR
// rows' 16-byte words of one step are loaded before any arithmetic, and each
// activation word is converted once for all rows, so a warp keeps NR loads in
// flight and spends its issue slots on FMAs.
template <int WT, int NR>
__device__ __forceinline__ void rows_dot(const unsigned char* const (&rows)[NR], int nvalid, const __half* xs,
                                         int K, int lane, float (&out)[NR]) {
    constexpr int E = elems16<WT>();
    const int nch = K / E;
    float acc[NR];
    const unsigned char* rp[NR];
#pragma unroll
    for (int i = 0; i < NR; i++) {
        acc[i] = 0.f;
        rp[i] = i < nvalid ? rows[i] : rows[0];
    }
#pragma unroll 2
    for (int c = lane; c < nch; c += 32) {
        uint4 wv[NR];
#pragma unroll
        for (int i = 0; i < NR; i++)
            wv[i] = *reinterpret_cast<const uint4*>(rp[i] + (size_t)c * 16);
#pragma unroll
        for (int g = 0; g < E / 8; g++) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + c * E + g * 8);
            float xf[8];
            const uint32_t* xu = &xv.x;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const float2 f = b2::h2_to_f2(xu[t]);
                xf[2 * t] = f.x;
                xf[2 * t + 1] = f.y;
            }
#pragma unroll
            for (int i = 0; i < NR; i++) {
                float w[8];
                expand8<WT>(wv[i], g, w);
#pragma unroll
                for (int t = 0; t < 8; t++) acc[i] = fmaf(xf[t], w[t], acc[i]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < NR; i++) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
    for (int i = 0; i < NR; i++) out[i] = acc[i];
}

__host__ __device__ inline size_t row_bytes(int wtype, int K) {
    return wtype == B2_W_F16 ? (size_t)K * 2 : wtype == B2_W_I8 ? (size_t)K : (size_t)K / 2;
}

__device__ __forceinline__ int split_lo(int n, int parts, int i) { return (int)(((long long)n * i) / parts); }

// ─── the per-CTA schedule, shared by producer and consumers ───

struct Geo {
    int L, pos, S, G, cta, qd, kvd, nqkv, Gq;
};

struct Chunk {
    int type, l, a, b, g, s;
    const void* src0;
    uint32_t bytes0;
    const void* src1;
    uint32_t bytes1;
    uint32_t off1;
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
    const int cap_h = kStageBytes / (int)rb_h, cap_q = kStageBytes / (int)rb_q, cap_f = kStageBytes / (int)rb_f;
    const int cap_pair = kStageBytes / (2 * (int)rb_h);
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
        {  // gate|up channel pairs
            Item it{IT_GU, l, split_lo(F, geo.G, geo.cta), split_lo(F, geo.G, geo.cta + 1), 0, 0, 0, 0};
            v.begin(it);
            for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_pair) {
                const int b = min(it.r1, a + cap_pair);
                const uint32_t bytes = (uint32_t)((b - a) * rb_h);
                Chunk c{IT_GU, l, a, b, 0, 0, (const unsigned char*)Lw.gu + a * rb_h, bytes,
                        (const unsigned char*)Lw.gu + (size_t)(F + a) * rb_h, bytes, bytes};
                v.chunk(c);
            }
            v.end(it);
        }
        if (v.stop()) return;
        {  // down rows
            Item it{IT_DN, l, split_lo(H, geo.G, geo.cta), split_lo(H, geo.G, geo.cta + 1), 0, 0, 0, 0};
            v.begin(it);
            for (int a = it.r0; a < it.r1 && !v.stop(); a += cap_f) {
                const int b = min(it.r1, a + cap_f);
                Chunk c{IT_DN, l, a, b, 0, 0, (const unsigned char*)Lw.dn + a * rb_f, (uint32_t)((b - a) * rb_f),
                        nullptr, 0, 0};
                v.chunk(c);
            }
            v.end(it);
        }
    }
    if (p.do_lm && !v.stop()) {
        Item it{IT_LM, p.n_layers, split_lo(p.vocab, geo.G, geo.cta), split_lo(p.vocab, geo.G, geo.cta + 1), 0, 0,
                0, 0};
        v.begin(it);
        const int cap = kStageBytes / H;  // int8 rows
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
    int cabort;                 // consumers' decision, written by consumer 0 before a barrier
    int issued, consumed;
    int last;                   // this CTA was the last arriver of a group
    float red[kCWarps];
    unsigned long long best[kCWarps];
    float q[kMaxGq][kHD];                  // normalized + rotated q heads of the group
    float k[kHD], v[kHD];                  // new k (rotated) and v of the kv head
    float gm[kCWarps][kMaxGq], gl[kCWarps][kMaxGq];  // per-warp softmax state
    float go[kCWarps][kMaxGq][kHD];                   // per-warp partial outputs
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
        mbar_expect_tx(&sh.full[stage], c.bytes0 + c.bytes1);
        bulk_g2s(dst, c.src0, c.bytes0, &sh.full[stage]);
        if (c.bytes1) bulk_g2s(dst + c.off1, c.src1, c.bytes1, &sh.full[stage]);
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
    unsigned long long target;  // per-CTA counter target multiplier: gen + 1
    const float* emb_row;
    int tid, lane, warp;
    int n = 0;
    // attention state of this thread's lane group (positions of group grp)
    float m_[kMaxGq], l_[kMaxGq], o_[kMaxGq][16], qv_[kMaxGq][16];
    unsigned long long best = 0ull;
    bool aborted = false;  // identical in every consumer thread (set only at barriers)

    __device__ bool stop() const { return aborted; }

    // Consumer 0 waits until *cnt >= want (or gives up); the decision reaches
    // every consumer through shared memory across a barrier.
    __device__ void wait_counter(const unsigned long long* cnt, unsigned long long want) {
        if (tid == 0) {
            long long it = 0;
            unsigned ns = 32;
            while (ld_acquire(cnt) < want) {
                if (*(volatile int*)&sh.abort || *(volatile int*)(p.state + B2_MK_ERR)) {
                    sh.cabort = 1;
                    break;
                }
                if (++it > kPollLimit) {
                    sh.cabort = 1;
                    atomicOr(p.state + B2_MK_ERR, 1);
                    break;
                }
                if (it > 64) __nanosleep(ns);
                if (ns < 128) ns <<= 1;
            }
        }
        consumer_sync();
        aborted = *(volatile int*)&sh.cabort != 0;
    }

    // After a CTA barrier, consumer 0's release publishes every consumer's
    // prior stores (release is cumulative over what the barrier ordered).
    __device__ void signal(unsigned long long* cnt, unsigned long long amount) {
        consumer_sync();
        if (tid == 0) red_release(cnt, amount);
    }

    // Stage src[0..K) (global, written by other CTAs) as FP16, optionally
    // RMS-normalized.  K <= kMaxK and K % 8 == 0 (b2_mk_check), so each thread
    // holds at most four float4 of src in registers: one L2 round trip.
    __device__ void stage_x(const float* src, int K, const float* norm_w) {
        constexpr int kV = kMaxK / (4 * kConsumers);
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4 v[kV];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kV; j++) {
            const int q = tid + j * kConsumers;
            v[j] = q * 4 < K ? __ldcg(s4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
        }
        float rms = 1.f;
        if (norm_w) {
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
            if (norm_w) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w) + q);
                x.x = (x.x * rms) * w.x;
                x.y = (x.y * rms) * w.y;
                x.z = (x.z * rms) * w.z;
                x.w = (x.w * rms) * w.w;
            }
            __half2* d = reinterpret_cast<__half2*>(xs + q * 4);
            d[0] = __floats2half2_rn(x.x, x.y);
            d[1] = __floats2half2_rn(x.z, x.w);
        }
        consumer_sync();
    }

    __device__ const float* hidden_in(int l) const { return l == 0 ? emb_row : S.hbuf + (size_t)l * p.hidden; }

    __device__ unsigned long long* cnt(int l, int c) const { return S.cnt + (size_t)l * kCntPerLayer + c; }

    __device__ void begin(const Item& it) {
        const int H = p.hidden;
        switch (it.type) {
            case IT_QKV:
                if (it.l > 0) wait_counter(cnt(it.l - 1, C_DN), (unsigned long long)geo.G * target);
                if (!stop()) stage_x(hidden_in(it.l), H, p.layers[it.l].in_norm);
                break;
            case IT_ATTN: {
                wait_counter(cnt(it.l, C_QKV + it.g), (unsigned long long)(geo.Gq + 2) * kHD * target);
                if (stop()) return;
                attn_prologue(it);
                break;
            }
            case IT_O:
                wait_counter(cnt(it.l, C_ATTN_DONE), (unsigned long long)p.nkv * target);
                if (!stop()) stage_x(S.attn + (size_t)it.l * geo.qd, geo.qd, nullptr);
                break;
            case IT_GU:
                wait_counter(cnt(it.l, C_O), (unsigned long long)geo.G * target);
                if (!stop()) stage_x(S.hmid + (size_t)it.l * H, H, p.layers[it.l].post_norm);
                break;
            case IT_DN:
                wait_counter(cnt(it.l, C_GU), (unsigned long long)geo.G * target);
                if (!stop()) stage_x(S.act + (size_t)it.l * p.ffn, p.ffn, nullptr);
                break;
            case IT_LM:
                wait_counter(cnt(p.n_layers - 1, C_DN), (unsigned long long)geo.G * target);
                if (!stop()) stage_x(S.hbuf + (size_t)p.n_layers * H, H, p.final_norm);
                best = 0ull;
                break;
        }
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
        const unsigned char* buf = ring + (size_t)stage * kStageBytes;
        switch (c.type) {
            case IT_QKV: rows_qkv(c, buf); break;
            case IT_ATTN: attn_chunk(c, buf); break;
            case IT_O: rows_resid(c, buf, geo.qd, p.layers[c.l].o, p.layers[c.l].o_s, S.hmid); break;
            case IT_GU: rows_gu(c, buf); break;
            case IT_DN: rows_resid(c, buf, p.ffn, p.layers[c.l].dn, p.layers[c.l].dn_s, S.hbuf); break;
            case IT_LM: rows_lm(c, buf); break;
        }
        __syncwarp();  // this warp is done reading the stage
        if (lane == 0) mbar_arrive(&sh.empty[stage]);
        if (tid == 0) *(volatile int*)&sh.consumed = n + 1;
        n++;
    }

    __device__ void end(const Item& it) {
        if (stop()) return;
        switch (it.type) {
            case IT_QKV: {
                // rows of kv group g: q heads [g*Gq, (g+1)*Gq), k head g, v head g
                consumer_sync();
                if (tid == 0) {
                    for (int g = 0; g < p.nkv; g++) {
                        const int q0 = g * geo.Gq * kHD, q1 = q0 + geo.Gq * kHD;
                        const int k0 = geo.qd + g * kHD, v0 = geo.qd + geo.kvd + g * kHD;
                        int n_rows = max(0, min(it.r1, q1) - max(it.r0, q0)) +
                                     max(0, min(it.r1, k0 + kHD) - max(it.r0, k0)) +
                                     max(0, min(it.r1, v0 + kHD) - max(it.r0, v0));
                        if (n_rows) red_release(cnt(it.l, C_QKV + g), (unsigned long long)n_rows);
                    }
                }
                break;
            }
            case IT_ATTN: attn_epilogue(it); break;
            case IT_O: signal(cnt(it.l, C_O), 1); break;
            case IT_GU: signal(cnt(it.l, C_GU), 1); break;
            case IT_DN: signal(cnt(it.l, C_DN), 1); break;
            case IT_LM: {
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
                    atomicMax(S.cnt + (size_t)p.n_layers * kCntPerLayer + 1, m);
                }
                break;
            }
        }
    }

    // ── row kernels ──

    __device__ float scale_of(const float* s, int r) const { return s ? s[r] : 1.f; }

    __device__ void rows_qkv(const Chunk& c, const unsigned char* buf) {
        const size_t rb = row_bytes(WT, p.hidden);
        const float* sc = p.layers[c.l].qkv_s;
        float* out = S.qkv + (size_t)c.l * geo.nqkv;
        const int n = c.b - c.a;
        for (int r0 = warp * 4; r0 < n; r0 += 4 * kCWarps) {
            const unsigned char* rows[4] = {buf + (size_t)r0 * rb, buf + (size_t)(r0 + 1) * rb,
                                            buf + (size_t)(r0 + 2) * rb, buf + (size_t)(r0 + 3) * rb};
            float d[4];
            rows_dot<WT, 4>(rows, min(4, n - r0), xs, p.hidden, lane, d);
            if (lane < 4 && r0 + lane < n) {
                const int r = c.a + r0 + lane;
                const float v = lane == 0 ? d[0] : lane == 1 ? d[1] : lane == 2 ? d[2] : d[3];
                out[r] = sc ? v * sc[r] : v;
            }
        }
    }

    // out[r] = resid[r] + s[r] * dot(row r, xs)  (o_proj into hmid, down into hbuf[l+1]);
    // these chunks hold few long rows, so one row per warp.
    __device__ void rows_resid(const Chunk& c, const unsigned char* buf, int K, const void*, const float* sc,
                               float* dst_base) {
        const size_t rb = row_bytes(WT, K);
        const int H = p.hidden;
        const float* resid = c.type == IT_O ? hidden_in(c.l) : S.hmid + (size_t)c.l * H;
        float* dst = c.type == IT_O ? S.hmid + (size_t)c.l * H : S.hbuf + (size_t)(c.l + 1) * H;
        (void)dst_base;
        for (int r = c.a + warp; r < c.b; r += kCWarps) {
            const unsigned char* rows[1] = {buf + (size_t)(r - c.a) * rb};
            float d[1];
            rows_dot<WT, 1>(rows, 1, xs, K, lane, d);
            if (lane == 0) dst[r] = __ldcg(resid + r) + (sc ? d[0] * sc[r] : d[0]);
        }
    }

    __device__ void rows_gu(const Chunk& c, const unsigned char* buf) {
        const size_t rb = row_bytes(WT, p.hidden);
        const float* sc = p.layers[c.l].gu_s;
        float* act = S.act + (size_t)c.l * p.ffn;
        const int n = c.b - c.a;
        for (int j0 = warp * 2; j0 < n; j0 += 2 * kCWarps) {
            const int j1 = min(j0 + 1, n - 1);
            const unsigned char* rows[4] = {buf + (size_t)j0 * rb, buf + c.off1 + (size_t)j0 * rb,
                                            buf + (size_t)j1 * rb, buf + c.off1 + (size_t)j1 * rb};
            float d[4];
            rows_dot<WT, 4>(rows, j0 + 1 < n ? 4 : 2, xs, p.hidden, lane, d);
            if (lane < 2 && j0 + lane < n) {
                const int j = c.a + j0 + lane;
                float g = lane == 0 ? d[0] : d[2], u = lane == 0 ? d[1] : d[3];
                if (sc) {
                    g = g * sc[j];
                    u = u * sc[p.ffn + j];
                }
                const float sig = 1.0f / (1.0f + expf(-g));
                act[j] = (g * sig) * u;
            }
        }
    }

    __device__ void rows_lm(const Chunk& c, const unsigned char* buf) {
        const int n = c.b - c.a;
        const size_t rb = (size_t)p.hidden;
        for (int r0 = warp * 4; r0 < n; r0 += 4 * kCWarps) {
            const unsigned char* rows[4] = {buf + (size_t)r0 * rb, buf + (size_t)(r0 + 1) * rb,
                                            buf + (size_t)(r0 + 2) * rb, buf + (size_t)(r0 + 3) * rb};
            float d[4];
            const int nv = min(4, n - r0);
            rows_dot<B2_W_I8, 4>(rows, nv, xs, p.hidden, lane, d);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (i >= nv) break;
                const int r = c.a + r0 + i;
                const float logit = d[i] * p.lm_s[r];
                if (lane == i && p.logits) p.logits[r] = logit;
                const unsigned long long k = b2::argmax_key(logit, (uint32_t)r);
                best = k > best ? k : best;
            }
        }
    }

    // ── attention: one (kv head g, position range) unit ──

    __device__ void attn_prologue(const Item& it) {
        const int Gq = geo.Gq;
        const float* qkv = S.qkv + (size_t)it.l * geo.nqkv;
        const B2MkLayer& Lw = p.layers[it.l];
        const int h = warp;  // warps 0..Gq-1: q heads, Gq: k head, Gq+1: v head
        if (h <= Gq + 1) {
            const int e0 = lane * 4;
            const float* src = h < Gq ? qkv + (size_t)(it.g * Gq + h) * kHD
                                      : h == Gq ? qkv + geo.qd + (size_t)it.g * kHD
                                                : qkv + geo.qd + geo.kvd + (size_t)it.g * kHD;
            float x[4];
#pragma unroll
            for (int j = 0; j < 4; j++) x[j] = __ldcg(src + e0 + j);
            if (h <= Gq) {
                const float* nw = h < Gq ? Lw.q_norm : Lw.k_norm;
                if (nw) {
                    float ss = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; j++) ss = fmaf(x[j], x[j], ss);
                    ss = b2::warp_sum(ss);
                    const float rms = 1.0f / sqrtf(ss / (float)kHD + p.eps);
#pragma unroll
                    for (int j = 0; j < 4; j++) x[j] = (x[j] * rms) * nw[e0 + j];
                }
                const float* cs = p.cos_tab + (size_t)geo.pos * (kHD / 2);
                const float* sn = p.sin_tab + (size_t)geo.pos * (kHD / 2);
                if (p.rope_style == 0) {
#pragma unroll
                    for (int j = 0; j < 4; j += 2) {
                        const int i = (e0 + j) >> 1;
                        const float x0 = x[j], x1 = x[j + 1];
                        x[j] = x0 * cs[i] - x1 * sn[i];
                        x[j + 1] = x1 * cs[i] + x0 * sn[i];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
                        const int e = e0 + j;
                        const int i = lane < 16 ? e : e - kHD / 2;
                        const float c0 = cs[i], s0 = sn[i];
                        x[j] = lane < 16 ? x[j] * c0 - other * s0 : x[j] * c0 + other * s0;
                    }
                }
            }
            float* dst = h < Gq ? sh.q[h] : h == Gq ? sh.k : sh.v;
#pragma unroll
            for (int j = 0; j < 4; j++) dst[e0 + j] = x[j];
            // The unit covering the newest position stores its K and V.
            if (h >= Gq && it.p1 == geo.L && it.p0 <= geo.L - 1) {
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
        for (int h2 = 0; h2 < kMaxGq; h2++) {
            m_[h2] = -INFINITY;
            l_[h2] = 0.f;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                o_[h2][j] = 0.f;
                qv_[h2][j] = h2 < Gq ? sh.q[h2][sub * 16 + j] : 0.f;
            }
        }
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

    __device__ void attn_epilogue(const Item& it) {
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
        // merge the per-warp states into this unit's partial (thread = (head, dim))
        const size_t unit = (((size_t)it.l * p.nkv + it.g) * kMaxSplit + it.s) * Gq;
        for (int t = tid; t < Gq * kHD; t += kConsumers) {
            const int h = t / kHD, d = t % kHD;
            float M = -INFINITY;
            for (int r = 0; r < kCWarps; r++) M = fmaxf(M, sh.gm[r][h]);
            float ls = 0.f, acc = 0.f;
            if (M != -INFINITY)
                for (int r = 0; r < kCWarps; r++) {
                    if (sh.gm[r][h] == -INFINITY) continue;
                    const float w = expf(sh.gm[r][h] - M);
                    ls = fmaf(sh.gl[r][h], w, ls);
                    acc = fmaf(sh.go[r][h][d], w, acc);
                }
            float* part = S.part + (unit + h) * (2 + kHD);
            part[2 + d] = acc;
            if (d == 0) {
                part[0] = M;
                part[1] = ls;
            }
        }
        consumer_sync();
        if (tid == 0) {
            __threadfence();
            const unsigned long long old = atom_add_acqrel(cnt(it.l, C_ATTN + it.g), 1ull);
            sh.last = old == (unsigned long long)(geo.S - 1) ? 1 : 0;
            __threadfence();
        }
        consumer_sync();
        if (!sh.last) return;
        // last unit of kv head g: merge the S position ranges of its q heads
        for (int t = tid; t < Gq * kHD; t += kConsumers) {
            const int h = t / kHD, d = t % kHD;
            float M = -INFINITY;
            for (int s = 0; s < geo.S; s++) {
                const float* part = S.part + ((((size_t)it.l * p.nkv + it.g) * kMaxSplit + s) * Gq + h) * (2 + kHD);
                M = fmaxf(M, __ldcg(part));
            }
            float num = 0.f, den = 0.f;
            for (int s = 0; s < geo.S; s++) {
                const float* part = S.part + ((((size_t)it.l * p.nkv + it.g) * kMaxSplit + s) * Gq + h) * (2 + kHD);
                const float ms = __ldcg(part);
                if (ms == -INFINITY) continue;
                const float w = expf(ms - M);
                den = fmaf(__ldcg(part + 1), w, den);
                num = fmaf(__ldcg(part + 2 + d), w, num);
            }
            S.attn[(size_t)it.l * geo.qd + (size_t)(it.g * Gq + h) * kHD + d] = num / den;
        }
        consumer_sync();
        if (tid == 0) {
            *(volatile unsigned long long*)cnt(it.l, C_ATTN + it.g) = 0ull;  // reset for the next step
            __threadfence();
            red_release(cnt(it.l, C_ATTN_DONE), 1ull);
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
        int s = (geo.L + 63) / 64;
        const int cap = min(kMaxSplit, max(1, geo.G / p.nkv));
        geo.S = max(1, min(s, cap));
    }
    const unsigned long long gen = (unsigned long long)(unsigned)p.state[B2_MK_GEN];

    if (warp == kCWarps) {
        if (lane == 0) {
            Producer<WT> prod{p, sh, ring};
            walk<WT>(p, geo, prod);
        }
    } else {
        const int tok = p.state[B2_MK_TOKEN];
        const float* emb_row = p.state[B2_MK_USE_EMB] ? p.staged_emb : p.emb + (size_t)tok * p.hidden;
        Consumer<WT> cons{p, geo, sh, ring, xs, S, gen + 1, emb_row, tid, lane, warp};
        walk<WT>(p, geo, cons);
        if (!cons.stop()) {  // FIN: the last CTA publishes the step
            consumer_sync();
            if (tid == 0) {
                unsigned long long* fin = S.cnt + (size_t)p.n_layers * kCntPerLayer;
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

template <int WT>
int launch(const B2MkPlan* p, cudaStream_t s) {
    auto fn = mk_decode_kernel<WT>;
    static thread_local int configured[8] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 7]) {
        B2_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        int per_sm = 0;
        B2_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, kSmemBytes));
        if (per_sm < 1) return b2_set_error(B2_ERR_CUDA, "b2_mk_decode: kernel does not fit on an SM");
        configured[dev & 7] = 1;
    }
    int sms = 0;
    B2_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
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
    return s.hbuf + (size_t)p->n_layers * p->hidden;
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
    const int E = p->wtype == B2_W_F16 ? 8 : p->wtype == B2_W_I8 ? 16 : 32;
    if (p->hidden % E || p->ffn % E || (p->nq * kHD) % E || p->hidden > kMaxK || p->ffn > kMaxK ||
        p->nq * kHD > kMaxK || p->hidden % 16)
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
