/*
 * ref_ops.c — CPU ORACLE (test infrastructure, never the product).
 *
 * Scalar restatement of the reference decoder's CPU arithmetic.  Each function
 * cites the reference file:line it follows (paths within
 * suharvest/rknn-matmul-parallel).  The reference's NEON lane structure is
 * mirrored where it fixes a summation order (RMSNorm's 4-lane sum, the
 * attention dot product's 4-wide partial sums); the oracle is compiled with
 * -ffp-contract=off so products and sums round separately, as the reference's
 * separate vmulq/vaddq intrinsics do.
 */
#include "ref_ops.h"
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* FP32 <-> FP16 with round-to-nearest-even: vec_fp32_to_fp16 / vec_fp16_to_fp32
 * (src/cpu_ops.c:383-406; vcvt_f16_f32 rounds to nearest even). */
uint16_t ref_f32_to_f16(float x) {
    _Float16 h = (_Float16)x;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

float ref_f16_to_f32(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

void ref_vec_f32_to_f16(uint16_t* dst, const float* src, int n) {
    for (int i = 0; i < n; i++) dst[i] = ref_f32_to_f16(src[i]);
}

void ref_vec_f16_to_f32(float* dst, const uint16_t* src, int n) {
    for (int i = 0; i < n; i++) dst[i] = ref_f16_to_f32(src[i]);
}

/* rms_norm_f32 (src/cpu_ops.c:18-55): four lane accumulators fed 8 elements
 * per iteration, lanes folded pairwise ((l0+l1)+(l2+l3)), scalar tail, then
 * out = (x * rms) * w with rms = 1 / sqrtf(sum/dim + eps). */
void ref_rms_norm(float* out, const float* x, const float* w, int dim, float eps) {
    float lane[4] = {0.f, 0.f, 0.f, 0.f};
    int i = 0;
    for (; i <= dim - 8; i += 8) {
        for (int j = 0; j < 4; j++) lane[j] = lane[j] + x[i + j] * x[i + j];
        for (int j = 0; j < 4; j++) lane[j] = lane[j] + x[i + 4 + j] * x[i + 4 + j];
    }
    float sum = (lane[0] + lane[1]) + (lane[2] + lane[3]);
    for (; i < dim; i++) sum = sum + x[i] * x[i];
    float rms = 1.0f / sqrtf(sum / (float)dim + eps);
    for (int k = 0; k < dim; k++) out[k] = (x[k] * rms) * w[k];
}

/* precompute_rope_tables (src/matmul_decoder.c:620-631):
 * freq = 1 / powf(theta, 2i/hd), angle = pos * freq. */
void ref_rope_tables(float* cos_tab, float* sin_tab, int max_seq, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int pos = 0; pos < max_seq; pos++) {
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (2.0f * (float)i) / (float)head_dim);
            float angle = (float)pos * freq;
            cos_tab[pos * half + i] = cosf(angle);
            sin_tab[pos * half + i] = sinf(angle);
        }
    }
}

/* apply_rope_f32 (src/cpu_ops.c:109-155).  style 0 rotates (x[2i], x[2i+1]);
 * style 1 rotates (x[i], x[i+half]); both use cos/sin[i] of this position. */
void ref_apply_rope(float* x, const float* c, const float* s, int num_heads, int head_dim,
                    int style) {
    int half = head_dim / 2;
    for (int h = 0; h < num_heads; h++) {
        float* hx = x + h * head_dim;
        for (int i = 0; i < half; i++) {
            int a = style == 0 ? 2 * i : i;
            int b = style == 0 ? 2 * i + 1 : i + half;
            float x0 = hx[a], x1 = hx[b];
            hx[a] = x0 * c[i] - x1 * s[i];
            hx[b] = x1 * c[i] + x0 * s[i];
        }
    }
}

/* 4-wide partial dot as in attention_f32's `dot += vaddvq_f32(vmulq_f32(q,k))`
 * (src/cpu_ops.c:226-230), with a scalar tail as in src/cpu_ops.c:493-500. */
static float dot4(const float* q, const float* k, int n) {
    float dot = 0.f;
    int d = 0;
    for (; d <= n - 4; d += 4) {
        float p0 = q[d] * k[d], p1 = q[d + 1] * k[d + 1];
        float p2 = q[d + 2] * k[d + 2], p3 = q[d + 3] * k[d + 3];
        dot = dot + ((p0 + p1) + (p2 + p3));
    }
    for (; d < n; d++) dot = dot + q[d] * k[d];
    return dot;
}

/* attention_f32 (src/cpu_ops.c:202-264): GQA kv_h = h / (nq/nkv); scores =
 * dot * (1/sqrtf(hd)); max from -1e30; expf(s - max); sum; *= 1/sum;
 * out = sum_s p_s * v_s.  Cache layout [pos][nkv][hd]. */
void ref_attention(float* out, const float* q, const float* kc, const float* vc,
                   int nq, int nkv, int hd, int L) {
    float scale = 1.0f / sqrtf((float)hd);
    int groups = nq / nkv;
    int stride = nkv * hd;
    float* sc = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
    for (int h = 0; h < nq; h++) {
        int g = h / groups;
        const float* qh = q + h * hd;
        float mx = -1e30f;
        for (int t = 0; t < L; t++) {
            sc[t] = dot4(qh, kc + (size_t)t * stride + g * hd, hd) * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        float sum = 0.f;
        for (int t = 0; t < L; t++) {
            sc[t] = expf(sc[t] - mx);
            sum = sum + sc[t];
        }
        float inv = 1.0f / sum;
        for (int t = 0; t < L; t++) sc[t] = sc[t] * inv;
        float* oh = out + h * hd;
        for (int d = 0; d < hd; d++) oh[d] = 0.f;
        for (int t = 0; t < L; t++) {
            const float* vs = vc + (size_t)t * stride + g * hd;
            for (int d = 0; d < hd; d++) oh[d] = oh[d] + vs[d] * sc[t];
        }
    }
    free(sc);
}

/* attention_batch_causal_f32 (src/cpu_ops.c:459-571): token t attends to the
 * cache [0, cache_len) then to batch tokens [0, t]; same softmax as above. */
void ref_attention_batch_causal(float* out, const float* q, const float* kb, const float* vb,
                                const float* kc, const float* vc, int M, int nq, int nkv,
                                int hd, int cache_len) {
    float scale = 1.0f / sqrtf((float)hd);
    int groups = nq / nkv;
    int kvs = nkv * hd, qs = nq * hd;
    float* sc = (float*)malloc(sizeof(float) * (size_t)(cache_len + M));
    for (int t = 0; t < M; t++) {
        int len = cache_len + t + 1;
        for (int h = 0; h < nq; h++) {
            int g = h / groups;
            const float* qh = q + (size_t)t * qs + h * hd;
            float mx = -1e30f;
            for (int s = 0; s < cache_len; s++) {
                sc[s] = dot4(qh, kc + (size_t)s * kvs + g * hd, hd) * scale;
                if (sc[s] > mx) mx = sc[s];
            }
            for (int b = 0; b <= t; b++) {
                sc[cache_len + b] = dot4(qh, kb + (size_t)b * kvs + g * hd, hd) * scale;
                if (sc[cache_len + b] > mx) mx = sc[cache_len + b];
            }
            float sum = 0.f;
            for (int s = 0; s < len; s++) {
                sc[s] = expf(sc[s] - mx);
                sum = sum + sc[s];
            }
            float inv = 1.0f / sum;
            for (int s = 0; s < len; s++) sc[s] = sc[s] * inv;
            float* oh = out + (size_t)t * qs + h * hd;
            for (int d = 0; d < hd; d++) oh[d] = 0.f;
            for (int s = 0; s < cache_len; s++) {
                const float* vs = vc + (size_t)s * kvs + g * hd;
                for (int d = 0; d < hd; d++) oh[d] = oh[d] + sc[s] * vs[d];
            }
            for (int b = 0; b <= t; b++) {
                const float* vs = vb + (size_t)b * kvs + g * hd;
                for (int d = 0; d < hd; d++) oh[d] = oh[d] + sc[cache_len + b] * vs[d];
            }
        }
    }
    free(sc);
}

/* silu_mul_f32 (src/cpu_ops.c:296-319): 4-wide part computes
 * (g * (1/(1+expf(-g)))) * u; the tail computes (g/(1+expf(-g))) * u. */
void ref_silu_mul(float* out, const float* g, const float* u, int n) {
    int body = n - (n % 4);
    for (int i = 0; i < body; i++) {
        float sig = 1.0f / (1.0f + expf(-g[i]));
        out[i] = (g[i] * sig) * u[i];
    }
    for (int i = body; i < n; i++) out[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* vec_add_f32 (src/cpu_ops.c:350-359). */
void ref_vec_add(float* dst, const float* src, int n) {
    for (int i = 0; i < n; i++) dst[i] = dst[i] + src[i];
}

/* argmax_f32 (src/cpu_ops.c:575-586): strict '>' keeps the first maximum. */
int ref_argmax(const float* x, int n) {
    float mv = x[0];
    int mi = 0;
    for (int i = 1; i < n; i++) {
        if (x[i] > mv) {
            mv = x[i];
            mi = i;
        }
    }
    return mi;
}

/* ───────── GEMM with the reference matmul semantics ─────────
 * run_persistent_matmul (src/matmul_decoder.c:382-445) and run_batch_matmul
 * (:1841-1899): the FP32 input row is rounded to FP16 (:395, :1845), the
 * multiply accumulates in FP32 (matmul type FLOAT16_MM_{FLOAT16,INT8}_TO_FLOAT32,
 * :179-195) and per-column scales multiply the FP32 result (:408-420). */
static inline float w_at(const void* W, int wtype, int N, int k, int n) {
    if (wtype == REF_W_F16) return ref_f16_to_f32(((const uint16_t*)W)[(size_t)k * N + n]);
    if (wtype == REF_W_I8) return (float)((const int8_t*)W)[(size_t)k * N + n];
    uint8_t b = ((const uint8_t*)W)[(size_t)k * (N / 2) + n / 2];
    int v = (n & 1) ? (b >> 4) : (b & 15);
    return (float)(v >= 8 ? v - 16 : v);
}

typedef struct {
    float* Y;
    const uint16_t* X16;
    int M, K, N, n0, n1, wtype;
    const void* W;
    const float* scales;
} GemmJob;

static void* gemm_worker(void* arg) {
    GemmJob* j = (GemmJob*)arg;
    int width = j->n1 - j->n0;
    float* acc = (float*)malloc(sizeof(float) * (size_t)(width > 0 ? width : 1));
    float* wrow = (float*)malloc(sizeof(float) * (size_t)(width > 0 ? width : 1));
    for (int m = 0; m < j->M; m++) {
        for (int n = 0; n < width; n++) acc[n] = 0.f;
        for (int k = 0; k < j->K; k++) {
            float xv = ref_f16_to_f32(j->X16[(size_t)m * j->K + k]);
            if (j->wtype == REF_W_F16) {
                const _Float16* wr = (const _Float16*)j->W + (size_t)k * j->N + j->n0;
                for (int n = 0; n < width; n++) wrow[n] = (float)wr[n];
            } else if (j->wtype == REF_W_I8) {
                const int8_t* wr = (const int8_t*)j->W + (size_t)k * j->N + j->n0;
                for (int n = 0; n < width; n++) wrow[n] = (float)wr[n];
            } else {
                for (int n = 0; n < width; n++) wrow[n] = w_at(j->W, j->wtype, j->N, k, j->n0 + n);
            }
            for (int n = 0; n < width; n++) acc[n] = acc[n] + xv * wrow[n];
        }
        for (int n = 0; n < width; n++) {
            float v = acc[n];
            if (j->scales) v = v * j->scales[j->n0 + n];
            j->Y[(size_t)m * j->N + j->n0 + n] = v;
        }
    }
    free(acc);
    free(wrow);
    return NULL;
}

void ref_gemm(float* Y, const float* X, int M, const void* W, const float* scales, int K, int N,
              int wtype, int nthreads) {
    uint16_t* X16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * K);
    ref_vec_f32_to_f16(X16, X, M * K);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    int step = (N + nthreads - 1) / nthreads;
    if (wtype == REF_W_I4) step = (step + 1) & ~1;
    GemmJob jobs[64];
    pthread_t th[64];
    int nj = 0;
    for (int n0 = 0; n0 < N; n0 += step) {
        GemmJob* j = &jobs[nj];
        j->Y = Y; j->X16 = X16; j->M = M; j->K = K; j->N = N; j->wtype = wtype;
        j->W = W; j->scales = scales; j->n0 = n0; j->n1 = n0 + step < N ? n0 + step : N;
        nj++;
    }
    if (nj == 1) {
        gemm_worker(&jobs[0]);
    } else {
        for (int i = 0; i < nj; i++) pthread_create(&th[i], NULL, gemm_worker, &jobs[i]);
        for (int i = 0; i < nj; i++) pthread_join(th[i], NULL);
    }
    free(X16);
}

/* ───────── Quantisers (bit-exact) ─────────
 * Per-column rule of the lm_head quantiser (src/matmul_decoder.c:1216-1244):
 * max = max|w| over the column, scale = max / qmax, inv = max > 0 ? qmax/max : 0,
 * q = clamp((int)roundf(w * inv), qmin, qmax).  The reference applies it with
 * qmax = 127 only; bits = 4 uses qmax = 7 with the FP16-rounded scale. */
void ref_quantize_cols(const uint16_t* w, int K, int N, int bits, uint8_t* q, float* scales) {
    float qmax = bits == 8 ? 127.0f : 7.0f;
    int qlo = bits == 8 ? -128 : -8, qhi = bits == 8 ? 127 : 7;
    if (bits == 4) memset(q, 0, (size_t)K * (N / 2));
    for (int n = 0; n < N; n++) {
        float mx = 0.f;
        for (int k = 0; k < K; k++) {
            float v = fabsf(ref_f16_to_f32(w[(size_t)k * N + n]));
            if (v > mx) mx = v;
        }
        float sc = mx / qmax;
        if (bits == 4) sc = ref_f16_to_f32(ref_f32_to_f16(sc));
        scales[n] = sc;
        float inv = (mx > 0) ? qmax / mx : 0;
        for (int k = 0; k < K; k++) {
            int v = (int)roundf(ref_f16_to_f32(w[(size_t)k * N + n]) * inv);
            if (v < qlo) v = qlo;
            if (v > qhi) v = qhi;
            if (bits == 8) {
                q[(size_t)k * N + n] = (uint8_t)(int8_t)v;
            } else {
                uint8_t nib = (uint8_t)(v & 15);
                q[(size_t)k * (N / 2) + n / 2] |= (n & 1) ? (uint8_t)(nib << 4) : nib;
            }
        }
    }
}

/* INT8 NPU lm_head build (src/matmul_decoder.c:1186-1248): tiles of tile_n
 * vocab columns; the FP16 [V][K] table is transposed to [K][tile_n] per tile,
 * padding columns stay 0 (scale 0). */
void ref_quantize_lm_head(const uint16_t* table, int V, int K, int tile_n, int8_t* q,
                          float* scales) {
    int n_tiles = (V + tile_n - 1) / tile_n;
    memset(q, 0, (size_t)n_tiles * K * tile_n);
    memset(scales, 0, sizeof(float) * (size_t)n_tiles * tile_n);
    for (int t = 0; t < n_tiles; t++) {
        int v0 = t * tile_n;
        int cnt = V - v0 < tile_n ? V - v0 : tile_n;
        int8_t* qt = q + (size_t)t * K * tile_n;
        for (int n = 0; n < cnt; n++) {
            const uint16_t* row = table + (size_t)(v0 + n) * K;
            float mx = 0.f;
            for (int k = 0; k < K; k++) {
                float v = fabsf(ref_f16_to_f32(row[k]));
                if (v > mx) mx = v;
            }
            scales[v0 + n] = mx / 127.0f;
            float inv = (mx > 0) ? 127.0f / mx : 0;
            for (int k = 0; k < K; k++) {
                int v = (int)roundf(ref_f16_to_f32(row[k]) * inv);
                if (v < -128) v = -128;
                if (v > 127) v = 127;
                qt[(size_t)k * tile_n + n] = (int8_t)v;
            }
        }
    }
}

typedef struct {
    float* logits;
    const uint16_t* x16;
    const float* x32;
    const void* tab;
    const float* scales;
    int K, V, tile_n, v0, v1, kind;
} LmJob;

static void* lm_worker(void* arg) {
    LmJob* j = (LmJob*)arg;
    if (j->kind == 0) { /* int8 tiles: per tile column n, k loop */
        for (int v = j->v0; v < j->v1; v++) {
            int t = v / j->tile_n, n = v % j->tile_n;
            const int8_t* qt = (const int8_t*)j->tab + (size_t)t * j->K * j->tile_n;
            float acc = 0.f;
            for (int k = 0; k < j->K; k++)
                acc = acc + ref_f16_to_f32(j->x16[k]) * (float)qt[(size_t)k * j->tile_n + n];
            j->logits[v] = acc * j->scales[v];
        }
    } else { /* fp16 rows [V][K] with FP32 input */
        for (int v = j->v0; v < j->v1; v++) {
            const uint16_t* row = (const uint16_t*)j->tab + (size_t)v * j->K;
            float acc = 0.f;
            for (int k = 0; k < j->K; k++) acc = acc + j->x32[k] * ref_f16_to_f32(row[k]);
            j->logits[v] = acc;
        }
    }
    return NULL;
}

static void lm_run(LmJob proto, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    int step = (proto.V + nthreads - 1) / nthreads;
    LmJob jobs[64];
    pthread_t th[64];
    int nj = 0;
    for (int v0 = 0; v0 < proto.V; v0 += step) {
        jobs[nj] = proto;
        jobs[nj].v0 = v0;
        jobs[nj].v1 = v0 + step < proto.V ? v0 + step : proto.V;
        nj++;
    }
    for (int i = 0; i < nj; i++) pthread_create(&th[i], NULL, lm_worker, &jobs[i]);
    for (int i = 0; i < nj; i++) pthread_join(th[i], NULL);
}

/* NPU lm_head run (src/matmul_decoder.c:1569-1605): FP16-rounded input
 * (:1577), FP32 result per tile times the column scale (:1590-1598). */
void ref_lm_head_int8(float* logits, const float* x, const int8_t* q, const float* scales,
                      int K, int V, int tile_n, int nthreads) {
    uint16_t* x16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)K);
    ref_vec_f32_to_f16(x16, x, K);
    LmJob p = {logits, x16, x, q, scales, K, V, tile_n, 0, V, 0};
    lm_run(p, nthreads);
    free(x16);
}

/* gemv_f16_neon (src/matmul_decoder.c:572-616): FP32 input, FP16 rows. */
void ref_lm_head_f16(float* logits, const float* x, const uint16_t* table, int V, int K,
                     int nthreads) {
    LmJob p = {logits, NULL, x, table, NULL, K, V, 0, 0, V, 1};
    lm_run(p, nthreads);
}

/* gemv_f32_neon (src/matmul_decoder.c:511-566), used by step_head. */
void ref_lm_head_f32(float* logits, const float* x, const float* table, int V, int K) {
    for (int v = 0; v < V; v++) {
        const float* row = table + (size_t)v * K;
        float acc = 0.f;
        for (int k = 0; k < K; k++) acc = acc + x[k] * row[k];
        logits[v] = acc;
    }
}

/* ───────── Layer step ─────────
 * Per-layer body of matmul_decoder_step (src/matmul_decoder.c:1464-1546):
 * residual save, input RMSNorm, q/k/v GEMV, per-head q/k RMSNorm (:1495-1504),
 * RoPE at pos (:1507-1510), K/V store at pos BEFORE attention (:1512-1516),
 * attention over pos+1 positions, o_proj + residual, post-attn RMSNorm,
 * gate/up, SiLU*mul, down + residual. */
void ref_layer_decode(float* hidden, const RefLayer* L, const RefDims* d, float* kc, float* vc,
                      int pos, const float* cos_tab, const float* sin_tab, int nth) {
    int H = d->hidden, qd = d->nq * d->hd, kvd = d->nkv * d->hd, F = d->ffn;
    float* resid = (float*)malloc(sizeof(float) * H);
    float* normed = (float*)malloc(sizeof(float) * H);
    float* q = (float*)malloc(sizeof(float) * qd);
    float* k = (float*)malloc(sizeof(float) * kvd);
    float* v = (float*)malloc(sizeof(float) * kvd);
    float* att = (float*)malloc(sizeof(float) * qd);
    float* g = (float*)malloc(sizeof(float) * F);
    float* u = (float*)malloc(sizeof(float) * F);
    float* dn = (float*)malloc(sizeof(float) * H);

    memcpy(resid, hidden, sizeof(float) * H);
    ref_rms_norm(normed, hidden, L->in_norm, H, d->eps);
    ref_gemm(q, normed, 1, L->w[0], L->s[0], H, qd, d->wtype, nth);
    ref_gemm(k, normed, 1, L->w[1], L->s[1], H, kvd, d->wtype, nth);
    ref_gemm(v, normed, 1, L->w[2], L->s[2], H, kvd, d->wtype, nth);
    if (d->has_qk_norm && L->q_norm && L->k_norm) {
        for (int h = 0; h < d->nq; h++)
            ref_rms_norm(q + h * d->hd, q + h * d->hd, L->q_norm, d->hd, d->eps);
        for (int h = 0; h < d->nkv; h++)
            ref_rms_norm(k + h * d->hd, k + h * d->hd, L->k_norm, d->hd, d->eps);
    }
    const float* c = cos_tab + (size_t)pos * (d->hd / 2);
    const float* s = sin_tab + (size_t)pos * (d->hd / 2);
    ref_apply_rope(q, c, s, d->nq, d->hd, d->rope_style);
    ref_apply_rope(k, c, s, d->nkv, d->hd, d->rope_style);
    memcpy(kc + (size_t)pos * kvd, k, sizeof(float) * kvd);
    memcpy(vc + (size_t)pos * kvd, v, sizeof(float) * kvd);
    ref_attention(att, q, kc, vc, d->nq, d->nkv, d->hd, pos + 1);
    ref_gemm(hidden, att, 1, L->w[3], L->s[3], qd, H, d->wtype, nth);
    ref_vec_add(hidden, resid, H);
    ref_rms_norm(normed, hidden, L->post_norm, H, d->eps);
    ref_gemm(g, normed, 1, L->w[4], L->s[4], H, F, d->wtype, nth);
    ref_gemm(u, normed, 1, L->w[5], L->s[5], H, F, d->wtype, nth);
    ref_silu_mul(g, g, u, F);
    ref_gemm(dn, g, 1, L->w[6], L->s[6], F, H, d->wtype, nth);
    ref_vec_add(hidden, dn, H);

    free(resid); free(normed); free(q); free(k); free(v); free(att); free(g); free(u); free(dn);
}

/* Per-layer body of matmul_decoder_prefill_batch (src/matmul_decoder.c:1970-2061),
 * with apply_rope_batch_f32's per-position table (src/cpu_ops.c:417-445) and
 * the K/V store AFTER attention (:2026-2034). */
void ref_layer_prefill(float* hidden, int M, const RefLayer* L, const RefDims* d, float* kc,
                       float* vc, int start, float theta, int nth) {
    int H = d->hidden, qd = d->nq * d->hd, kvd = d->nkv * d->hd, F = d->ffn, half = d->hd / 2;
    size_t m = (size_t)M;
    float* resid = (float*)malloc(sizeof(float) * m * H);
    float* normed = (float*)malloc(sizeof(float) * m * H);
    float* q = (float*)malloc(sizeof(float) * m * qd);
    float* k = (float*)malloc(sizeof(float) * m * kvd);
    float* v = (float*)malloc(sizeof(float) * m * kvd);
    float* att = (float*)malloc(sizeof(float) * m * qd);
    float* g = (float*)malloc(sizeof(float) * m * F);
    float* u = (float*)malloc(sizeof(float) * m * F);
    float* dn = (float*)malloc(sizeof(float) * m * H);
    float* cs = (float*)malloc(sizeof(float) * half);
    float* sn = (float*)malloc(sizeof(float) * half);

    memcpy(resid, hidden, sizeof(float) * m * H);
    for (int t = 0; t < M; t++)
        ref_rms_norm(normed + (size_t)t * H, hidden + (size_t)t * H, L->in_norm, H, d->eps);
    ref_gemm(q, normed, M, L->w[0], L->s[0], H, qd, d->wtype, nth);
    ref_gemm(k, normed, M, L->w[1], L->s[1], H, kvd, d->wtype, nth);
    ref_gemm(v, normed, M, L->w[2], L->s[2], H, kvd, d->wtype, nth);
    for (int t = 0; t < M; t++) {
        float* qt = q + (size_t)t * qd;
        float* kt = k + (size_t)t * kvd;
        if (d->has_qk_norm && L->q_norm && L->k_norm) {
            for (int h = 0; h < d->nq; h++)
                ref_rms_norm(qt + h * d->hd, qt + h * d->hd, L->q_norm, d->hd, d->eps);
            for (int h = 0; h < d->nkv; h++)
                ref_rms_norm(kt + h * d->hd, kt + h * d->hd, L->k_norm, d->hd, d->eps);
        }
        int pos = start + t;
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (2.0f * (float)i) / (float)d->hd);
            float angle = (float)pos * freq;
            cs[i] = cosf(angle);
            sn[i] = sinf(angle);
        }
        ref_apply_rope(qt, cs, sn, d->nq, d->hd, d->rope_style);
        ref_apply_rope(kt, cs, sn, d->nkv, d->hd, d->rope_style);
    }
    ref_attention_batch_causal(att, q, k, v, kc, vc, M, d->nq, d->nkv, d->hd, start);
    memcpy(kc + (size_t)start * kvd, k, sizeof(float) * m * kvd);
    memcpy(vc + (size_t)start * kvd, v, sizeof(float) * m * kvd);
    ref_gemm(hidden, att, M, L->w[3], L->s[3], qd, H, d->wtype, nth);
    ref_vec_add(hidden, resid, M * H);
    for (int t = 0; t < M; t++)
        ref_rms_norm(normed + (size_t)t * H, hidden + (size_t)t * H, L->post_norm, H, d->eps);
    ref_gemm(g, normed, M, L->w[4], L->s[4], H, F, d->wtype, nth);
    ref_gemm(u, normed, M, L->w[5], L->s[5], H, F, d->wtype, nth);
    ref_silu_mul(g, g, u, M * F);
    ref_gemm(dn, g, M, L->w[6], L->s[6], F, H, d->wtype, nth);
    ref_vec_add(hidden, dn, M * H);

    free(resid); free(normed); free(q); free(k); free(v); free(att); free(g); free(u); free(dn);
    free(cs); free(sn);
}
