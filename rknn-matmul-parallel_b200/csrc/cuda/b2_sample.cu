// On-device token sampling after the lm_head (b2_sample_token).
//
// Semantics of matmul_sample_token (csrc/host/md_generate.c), which extends
// the reference's greedy matmul_sample_token (src/matmul_decoder.c:2316-2323)
// and top_k_sample_f32 (src/cpu_ops.c:593-647) with top-p and a repeat
// penalty:
//   1. repeat penalty, applied once per occurrence in the list, in list
//      order: x > 0 ? x / penalty : x * penalty
//   2. top_k == 1: the first index of the largest x (no temperature)
//   3. v = x / temperature (IEEE division; temperature <= 0 means 1)
//   4. the K = top_k largest v (all when top_k <= 0 or > V), ordered by v
//      descending and index ascending; w_i = exp(v_i - v_max), the
//      exponential in FP32 and every sum of weights in FP64
//   5. top_p in (0, 1): keep the shortest prefix of that order whose mass
//      reaches top_p of the K-set's mass
//   6. draw a token from the kept set with probability w_i / sum(w)
// The draw uses a counter-based generator (SplitMix64 of seed and counter),
// so a (seed, counter) pair always gives the same token; the host sampler's
// rand() stream is not reproduced, only its distribution.
//
// Structure.  One cluster of kCl CTAs (distributed shared memory).  Each CTA
// holds a contiguous slice of the vocabulary in shared memory, each thread a
// contiguous run of that slice, so every scan is in index order.  The K-th
// largest key and the top-p cut are found by radix selection on the 32-bit
// orderable keys of v, 8 bits per round, with per-CTA histograms (counts,
// then masses) that every CTA sums over the cluster through DSMEM.  Ties at a
// threshold go to the lowest indices, as in the sorted order of step 4.
// Mass sums in a different order than the host's sorted prefix sums, so a
// top-p cut that the host decides within rounding can differ by one token.
#include <cooperative_groups.h>

#include "b2_common.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int kCl = 8;                    // CTAs of the cluster
constexpr int kT = 1024;                  // threads per CTA
constexpr int kW = kT / 32;
constexpr int kMaxSlice = 54 * 1024;      // vocabulary entries per CTA (216 KB)
// Histogram masses are summed as 64-bit fixed point (weights <= 1 times
// 2^40; 2^18 entries cannot overflow): integer shared-memory atomics, where
// FP64 ones contended on the few busiest digits, and sums that do not depend
// on the order of the additions.
constexpr double kMassOne = 1099511627776.0;  // 2^40

struct Shared {
    unsigned int hist[2][256];            // radix counts (double-buffered across rounds)
    unsigned long long mass[2][256];      // radix masses, fixed point (kMassOne = 1.0)
    unsigned int tot[256];                // cluster-wide counts of the current round
    double totm[256];                     // cluster-wide masses of the current round
    unsigned long long wkey[kW];          // warp partials of (key, index) maxima
    unsigned long long wkey2[kW];
    double wd[kW];                        // warp partials of doubles
    unsigned int wu[kW];                  // warp partials of counts
    unsigned long long ckey;              // this CTA's (key, index) maximum
    unsigned long long ckey2;
    double cd;                            // this CTA's double total
    unsigned int cu;                      // this CTA's count total
    unsigned int sel_digit;               // digit chosen by the current radix round
    unsigned int sel_above;               // count above the chosen digit
    double sel_mass_above;                // mass above the chosen digit
};

__device__ __forceinline__ float key_value(uint32_t u) {  // inverse of float_order for non-NaN keys
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
    // SplitMix64 (G. Steele, D. Lea, C. Flood, "Fast splittable pseudorandom
    // number generators", OOPSLA 2014)
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Weight of a logit: exp(v - v_max) in FP32 (the FP64 exponential made the
// radix rounds FP64-bound on the cluster's 8 SMs), summed in FP64 by callers.
// (A NaN logit weighs nothing.)
__device__ __forceinline__ double wgt(float v, float vmax) {
    const float e = expf(v - vmax);
    return e == e ? (double)e : 0.0;
}

// Block-wide sums / maxima with every thread receiving the result.
__device__ double block_sum_d(Shared& sh, double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh.wd[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < kW; i++) t += sh.wd[i];  // fixed order
    __syncthreads();
    return t;
}

__device__ unsigned int block_sum_u(Shared& sh, unsigned int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh.wu[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned int t = 0;
    for (int i = 0; i < kW; i++) t += sh.wu[i];
    __syncthreads();
    return t;
}

// Exclusive prefix over the threads of the block (thread order = index
// order) plus the block's total.
__device__ unsigned int block_excl_u(Shared& sh, unsigned int v, unsigned int& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) sh.wu[w] = inc;
    __syncthreads();
    unsigned int before = 0;
    total = 0;
    for (int i = 0; i < kW; i++) {
        if (i < w) before += sh.wu[i];
        total += sh.wu[i];
    }
    __syncthreads();
    return before + inc - v;
}

__device__ double block_excl_d(Shared& sh, double v, double& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) sh.wd[w] = inc;
    __syncthreads();
    double before = 0.0;
    total = 0.0;
    for (int i = 0; i < kW; i++) {
        if (i < w) before += sh.wd[i];
        total += sh.wd[i];
    }
    __syncthreads();
    return before + inc - v;
}

struct Ctx {
    cg::cluster_group cl;
    Shared& sh;
    const float* v;       // this CTA's slice (shared memory)
    int n;                // entries in the slice
    int base;             // vocabulary index of the slice's first entry
    int r0, r1;           // this thread's run [r0, r1) within the slice
    unsigned rank;

    // cluster-wide sum of a per-CTA value (every thread gets it, plus the
    // sum over the CTAs before this one)
    __device__ unsigned int cluster_u(unsigned int cta_total, unsigned int& before) {
        if (threadIdx.x == 0) sh.cu = cta_total;
        cl.sync();
        unsigned int t = 0;
        before = 0;
        for (unsigned c = 0; c < kCl; c++) {
            const unsigned int x = *cl.map_shared_rank(&sh.cu, c);
            if (c < rank) before += x;
            t += x;
        }
        cl.sync();
        return t;
    }
    __device__ double cluster_d(double cta_total, double& before) {
        if (threadIdx.x == 0) sh.cd = cta_total;
        cl.sync();
        double t = 0.0;
        before = 0.0;
        for (unsigned c = 0; c < kCl; c++) {
            const double x = *cl.map_shared_rank(&sh.cd, c);
            if (c < rank) before += x;
            t += x;
        }
        cl.sync();
        return t;
    }

    // Rank, among all entries with key T in index order, of this thread's
    // first such entry.
    __device__ unsigned int eq_rank0(uint32_t T) {
        unsigned int mine = 0;
        for (int i = r0; i < r1; i++) mine += b2::float_order(v[i]) == T;
        unsigned int cta_total;
        const unsigned int in_cta = block_excl_u(sh, mine, cta_total);
        unsigned int before;
        cluster_u(cta_total, before);
        return before + in_cta;
    }

    // One radix round over the entries selected by sel(i, u): the digit d of
    // key bits [shift, shift + 8) where the running count (from the largest
    // digit down) first reaches `want`.  Returns d; `above` = the count of
    // larger digits.
    template <class Sel>
    __device__ unsigned int count_round(int buf, int shift, uint32_t prefix, uint32_t mask, unsigned int want,
                                        unsigned int& above, Sel sel) {
        for (int i = threadIdx.x; i < 256; i += kT) sh.hist[buf][i] = 0;
        __syncthreads();
        for (int i = r0; i < r1; i++) {
            const uint32_t u = b2::float_order(v[i]);
            if ((u & mask) == prefix && sel(i, u)) atomicAdd(&sh.hist[buf][(u >> shift) & 255u], 1u);
        }
        cl.sync();  // every CTA's histogram complete
        if (threadIdx.x < 256) {  // one digit per thread, the 8 remote reads in flight together
            unsigned int v[kCl];
#pragma unroll
            for (unsigned c = 0; c < kCl; c++) v[c] = cl.map_shared_rank(&sh.hist[buf][0], c)[threadIdx.x];
            unsigned int t = 0;
#pragma unroll
            for (unsigned c = 0; c < kCl; c++) t += v[c];
            sh.tot[threadIdx.x] = t;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane l takes digits 255 - 8 l .. 248 - 8 l
            const int lane = threadIdx.x;
            unsigned int c8[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                c8[j] = sh.tot[255 - 8 * lane - j];
                s += c8[j];
            }
            unsigned int inc = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const unsigned int ex = inc - s;
            // the lane whose range holds the crossing
            const unsigned hit = __ballot_sync(0xffffffffu, ex < want && want <= inc);
            const int hl = hit ? __ffs(hit) - 1 : 31;
            if (lane == hl) {
                unsigned int run = ex;
                int dsel = 255 - 8 * lane - 7;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (run + c8[j] >= want) {
                        dsel = 255 - 8 * lane - j;
                        break;
                    }
                    run += c8[j];
                }
                // (no crossing: want exceeds the selected count; take digit 0)
                sh.sel_digit = hit ? (unsigned)dsel : 0u;
                sh.sel_above = hit ? run : inc;
            }
        }
        __syncthreads();
        above = sh.sel_above;
        return sh.sel_digit;
    }

    // Same with masses: the digit where the running mass first reaches want.
    template <class Sel>
    __device__ unsigned int mass_round(int buf, int shift, uint32_t prefix, uint32_t mask, double want, float vmax,
                                       double& above, Sel sel) {
        for (int i = threadIdx.x; i < 256; i += kT) sh.mass[buf][i] = 0ull;
        __syncthreads();
        for (int i = r0; i < r1; i++) {
            const uint32_t u = b2::float_order(v[i]);
            if ((u & mask) == prefix && sel(i, u))
                atomicAdd(&sh.mass[buf][(u >> shift) & 255u],
                          (unsigned long long)__double2ll_rn(wgt(v[i], vmax) * kMassOne));
        }
        cl.sync();
        if (threadIdx.x < 256) {
            unsigned long long v[kCl];
#pragma unroll
            for (unsigned c = 0; c < kCl; c++) v[c] = cl.map_shared_rank(&sh.mass[buf][0], c)[threadIdx.x];
            unsigned long long t = 0ull;
#pragma unroll
            for (unsigned c = 0; c < kCl; c++) t += v[c];
            sh.totm[threadIdx.x] = (double)t / kMassOne;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            double m8[8], s = 0.0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                m8[j] = sh.totm[255 - 8 * lane - j];
                s += m8[j];
            }
            double inc = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const double ex = inc - s;
            const unsigned hit = __ballot_sync(0xffffffffu, ex < want && want <= inc && s > 0.0);
            // no crossing (rounding left want above the total): the lowest digit with mass
            const unsigned nz = __ballot_sync(0xffffffffu, s > 0.0);
            const int hl = hit ? __ffs(hit) - 1 : (nz ? 31 - __clz(nz) : 0);
            if (lane == hl) {
                double run = ex;
                int dsel = -1;
                int last_nz = -1;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (m8[j] > 0.0) last_nz = 255 - 8 * lane - j;
                    if (dsel < 0 && hit && m8[j] > 0.0 && run + m8[j] >= want) {
                        dsel = 255 - 8 * lane - j;
                        break;
                    }
                    if (dsel < 0) run += m8[j];
                }
                if (dsel < 0) {  // fall back to the lowest digit with mass in this lane
                    dsel = last_nz >= 0 ? last_nz : 0;
                    run = ex;
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (255 - 8 * lane - j > dsel) run += m8[j];
                }
                sh.sel_digit = (unsigned)dsel;
                sh.sel_mass_above = run;
            }
        }
        __syncthreads();
        above = sh.sel_mass_above;
        return sh.sel_digit;
    }
};

// Largest (key, lowest index) over the cluster.
__device__ unsigned long long cluster_argmax(Ctx& c) {
    unsigned long long k = 0ull;
    for (int i = c.r0; i < c.r1; i++) {
        const unsigned long long x = b2::argmax_key(c.v[i], (uint32_t)(c.base + i));
        k = x > k ? x : k;
    }
    k = b2::warp_max_u64(k);
    if ((threadIdx.x & 31) == 0) c.sh.wkey[threadIdx.x >> 5] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0ull;
        for (int i = 0; i < kW; i++) m = c.sh.wkey[i] > m ? c.sh.wkey[i] : m;
        c.sh.ckey = m;
    }
    c.cl.sync();
    unsigned long long m = 0ull;
    for (unsigned r = 0; r < kCl; r++) {
        const unsigned long long x = *c.cl.map_shared_rank(&c.sh.ckey, r);
        m = x > m ? x : m;
    }
    c.cl.sync();
    return m;
}

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kT, 1)
    sample_kernel(const float* __restrict__ logits, int V, int slice, const int* __restrict__ rep, int n_rep,
                  float penalty, int top_k, float top_p, float temperature, unsigned long long seed,
                  unsigned long long counter, int* __restrict__ token, int* __restrict__ info) {
    extern __shared__ __align__(16) unsigned char smem[];
    Shared& sh = *reinterpret_cast<Shared*>(smem);
    float* v = reinterpret_cast<float*>(smem + ((sizeof(Shared) + 15) & ~(size_t)15));
    cg::cluster_group cl = cg::this_cluster();
    const unsigned rank = cl.block_rank();
    const int base = (int)rank * slice;
    const int n = max(0, min(slice, V - base));
    const int per = (n + kT - 1) / kT;
    Ctx c{cl, sh, v, n, base, min(n, (int)threadIdx.x * per), min(n, ((int)threadIdx.x + 1) * per), rank};

    b2::pdl_wait();
    for (int i = threadIdx.x; i < n; i += kT) v[i] = logits[base + i];
    __syncthreads();
    if (threadIdx.x == 0 && penalty != 1.0f)
        for (int j = 0; j < n_rep; j++) {  // in list order: a repeated token is penalized again
            const int t = rep[j] - base;
            if (t >= 0 && t < n) v[t] = v[t] > 0.f ? v[t] / penalty : v[t] * penalty;
        }
    __syncthreads();
    if (top_k == 1) {  // greedy: first index of the largest penalized logit
        const unsigned long long k = cluster_argmax(c);
        if (rank == 0 && threadIdx.x == 0) {
            *token = (int)b2::key_index(k);
            if (info) info[0] = 1, info[1] = 1, info[2] = (int)(k >> 32), info[3] = 1;
        }
        return;
    }
    const float temp = temperature > 0.f ? temperature : 1.0f;
    for (int i = threadIdx.x; i < n; i += kT) v[i] = __fdiv_rn(v[i], temp);
    __syncthreads();
    const unsigned long long kmax = cluster_argmax(c);
    const float vmaxf = key_value((uint32_t)(kmax >> 32));
    const unsigned int K = (top_k <= 0 || top_k > V) ? (unsigned)V : (unsigned)top_k;

    // ── top-K threshold: key T and how many entries equal to T (lowest
    // indices first) belong to the set ──
    uint32_t T = 0u;
    unsigned int needT = 0;  // entries with key T in the set
    unsigned int eq0 = 0;    // cluster rank of this thread's first entry with key T
    const auto all = [](int, uint32_t) { return true; };
    if (K < (unsigned)V) {
        uint32_t prefix = 0u, mask = 0u;
        unsigned int want = K;
        for (int r = 0; r < 4; r++) {
            const int shift = 24 - 8 * r;
            unsigned int above;
            const unsigned int d = c.count_round(r & 1, shift, prefix, mask, want, above, all);
            prefix |= d << shift;
            mask |= 255u << shift;
            want -= above;
        }
        T = prefix;
        needT = want;
        eq0 = c.eq_rank0(T);
    } else {
        needT = 0xFFFFFFFFu;  // every entry
        eq0 = 0;
    }
    // membership of entry i (visited in index order, `seen` = entries with
    // key T met so far by this thread)
    const auto in_k = [&](uint32_t u, unsigned int seen) {
        return K >= (unsigned)V || u > T || (u == T && eq0 + seen < needT);
    };

    // ── mass of the K-set ──
    double mine = 0.0;
    {
        unsigned int seen = 0;
        for (int i = c.r0; i < c.r1; i++) {
            const uint32_t u = b2::float_order(v[i]);
            if (in_k(u, seen)) mine += wgt(v[i], vmaxf);
            seen += u == T;
        }
    }
    double before;
    const double sumK = c.cluster_d(block_sum_d(sh, mine), before);

    // ── top-p cut within the K-set: key P and the count of its entries kept ──
    uint32_t P = T;
    unsigned int needP = needT, eqP0 = eq0;
    if (top_p > 0.f && top_p < 1.0f) {
        const double want = (double)top_p * sumK;
        uint32_t prefix = 0u, mask = 0u;
        double above_total = 0.0;
        for (int r = 0; r < 4; r++) {
            const int shift = 24 - 8 * r;
            double above;
            // entries of the K-set: by key, except the ties at T (resolved
            // below), which are all counted; a cut at key T keeps at most needT
            const auto sel = [&](int, uint32_t u) { return K >= (unsigned)V || u >= T; };
            const unsigned int d = c.mass_round(r & 1, shift, prefix, mask, want - above_total, vmaxf, above, sel);
            above_total += above;
            prefix |= d << shift;
            mask |= 255u << shift;
        }
        P = prefix;
        const double w = wgt(key_value(P), vmaxf);
        // smallest j with above_total + j w >= want
        double j = w > 0.0 ? ceil((want - above_total) / w) : 1.0;
        j = j < 1.0 ? 1.0 : j;
        needP = j > 4.0e9 ? 0xFFFFFFFFu : (unsigned int)j;
        if (K < (unsigned)V && P == T) needP = min(needP, needT);
        eqP0 = P == T ? eq0 : c.eq_rank0(P);
    }
    const auto kept = [&](uint32_t u, unsigned int seenP) {
        if (K < (unsigned)V && (u < T)) return false;
        return u > P || (u == P && eqP0 + seenP < needP);
    };

    // ── draw: r uniform in [0, total) over the kept entries in index order ──
    double wm = 0.0;
    unsigned int nk = 0;
    int last = -1;
    {
        unsigned int seen = 0;
        for (int i = c.r0; i < c.r1; i++) {
            const uint32_t u = b2::float_order(v[i]);
            if (kept(u, seen)) {
                wm += wgt(v[i], vmaxf);
                nk++;
                last = i;
            }
            seen += u == P;
        }
    }
    double cta_total;
    const double in_cta = block_excl_d(sh, wm, cta_total);
    double cta_before;
    const double total = c.cluster_d(cta_total, cta_before);
    unsigned int nk_before;
    const unsigned int nk_total = c.cluster_u(block_sum_u(sh, nk), nk_before);
    const unsigned long long z = splitmix64(seed ^ splitmix64(counter));
    const double r = (double)(z >> 11) * 0x1.0p-53 * total;
    const double t0 = cta_before + in_cta;
    // The thread whose range holds r walks its run.  Ranges come from
    // rounded prefix sums, so two neighbours may both claim r (the lower
    // index wins) or neither (the last kept entry is taken, as when rounding
    // leaves r at the total).
    unsigned long long pick = ~0ull;
    if (wm > 0.0 && r >= t0 && r < t0 + wm) {
        double acc = t0;
        unsigned int seen = 0;
        int at = last;
        for (int i = c.r0; i < c.r1; i++) {
            const uint32_t u = b2::float_order(v[i]);
            if (kept(u, seen)) {
                acc += wgt(v[i], vmaxf);
                if (r < acc) {
                    at = i;
                    break;
                }
            }
            seen += u == P;
        }
        pick = (unsigned long long)(base + at);
    }
    const unsigned long long lk = last >= 0 ? (unsigned long long)(base + last) : 0ull;
    unsigned long long pmin = pick, lmax = lk;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long a = __shfl_xor_sync(0xffffffffu, pmin, o), b = __shfl_xor_sync(0xffffffffu, lmax, o);
        pmin = a < pmin ? a : pmin;
        lmax = b > lmax ? b : lmax;
    }
    if ((threadIdx.x & 31) == 0) sh.wkey[threadIdx.x >> 5] = pmin, sh.wkey2[threadIdx.x >> 5] = lmax;
    __syncthreads();
    if (threadIdx.x == 0) {
        pmin = ~0ull, lmax = 0ull;
        for (int i = 0; i < kW; i++) {
            pmin = sh.wkey[i] < pmin ? sh.wkey[i] : pmin;
            lmax = sh.wkey2[i] > lmax ? sh.wkey2[i] : lmax;
        }
        sh.ckey = pmin;
        sh.ckey2 = lmax;
    }
    cl.sync();
    if (rank == 0 && threadIdx.x == 0) {
        pmin = ~0ull, lmax = 0ull;
        for (unsigned q = 0; q < kCl; q++) {
            const unsigned long long x = *cl.map_shared_rank(&sh.ckey, q), y = *cl.map_shared_rank(&sh.ckey2, q);
            pmin = x < pmin ? x : pmin;
            lmax = y > lmax ? y : lmax;
        }
        *token = (int)(pmin != ~0ull ? pmin : lmax);
        if (info) info[0] = (int)nk_total, info[1] = (int)K, info[2] = (int)P, info[3] = (int)needP;
    }
    cl.sync();  // remote reads done before any CTA exits
}

}  // namespace

extern "C" size_t b2_sample_max_vocab(void) { return (size_t)kCl * kMaxSlice; }

extern "C" int b2_sample_token(const float* logits, int V, const int* repeat_tokens, int n_repeat,
                               float repeat_penalty, int top_k, float top_p, float temperature,
                               unsigned long long seed, unsigned long long counter, int* token, int* info,
                               b2_stream_t stream) {
    if (!logits || !token || V <= 0 || n_repeat < 0 || (n_repeat > 0 && !repeat_tokens))
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_sample_token: bad arguments (V=%d n_repeat=%d)", V, n_repeat);
    if ((size_t)V > b2_sample_max_vocab())
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_sample_token: vocabulary %d above %zu", V, b2_sample_max_vocab());
    if (!(repeat_penalty > 0.f)) return b2_set_error(B2_ERR_INVALID_ARG, "b2_sample_token: repeat_penalty must be > 0");
    const int slice = (((V + kCl - 1) / kCl) + 3) & ~3;
    const size_t smem = ((sizeof(Shared) + 15) & ~(size_t)15) + (size_t)slice * 4;
    static int configured[64] = {0};
    int dev = 0;
    B2_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return b2_set_error(B2_ERR_INVALID_ARG, "b2_sample_token: device %d", dev);
    if (!configured[dev]) {
        const size_t most = ((sizeof(Shared) + 15) & ~(size_t)15) + (size_t)kMaxSlice * 4;
        B2_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)most));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kCl);
        cfg.blockDim = dim3(kT);
        cfg.dynamicSmemBytes = most;
        int clusters = 0;
        B2_TRY(cudaOccupancyMaxActiveClusters(&clusters, sample_kernel, &cfg));
        if (clusters < 1) return b2_set_error(B2_ERR_CUDA, "b2_sample_token: no room for a cluster of %d CTAs", kCl);
        configured[dev] = 1;
    }
    const cudaError_t e = b2::launch_pdl(sample_kernel, dim3(kCl), dim3(kT), smem, (cudaStream_t)stream, logits, V,
                                         slice, repeat_tokens, n_repeat, repeat_penalty, top_k, top_p, temperature,
                                         seed, counter, token, info);
    if (e != cudaSuccess) return b2_set_error(B2_ERR_CUDA, "b2_sample_token: %s", cudaGetErrorString(e));
    return 0;
}
