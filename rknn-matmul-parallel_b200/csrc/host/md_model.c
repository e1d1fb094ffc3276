/*
 * Model loading and upload to the device arena.
 *
 * Reads the reference on-disk layout (load_layer_weights,
 * src/matmul_decoder.c:698-826, with its alternate file names; embeddings,
 * lm_head and final norm, :862-926 and :1155-1168) and uploads it once:
 *
 *   - projections are re-laid out from the file's [K][N] (int4: [K][N/2],
 *     column pairs per byte) to one K-contiguous row per output column, the
 *     layout the streaming GEMV reads with 16-byte loads (int4: [N][K/2],
 *     k pairs per byte, even k in the low nibble);
 *   - q/k/v are concatenated into one [qd + 2 kvd] x K matrix and gate/up into
 *     one [2 ffn] x K matrix (the reference's disabled QKV merge, :1037-1142,
 *     is always on here);
 *   - the lm_head (tied to the embeddings or lm_head.bin) is rounded to FP16
 *     and quantized to INT8 per vocab row with the reference rule
 *     (:917-926, :1216-1244), or kept FP16 when disable_npu_lm_head is set;
 *   - multi-head models load lm_head_NN.bin FP32 tables (:885-901);
 *   - RoPE tables use the reference formula (precompute_rope_tables, :620-631).
 *
 * Unlike the reference, which prints and continues past a missing layer file
 * (:1033-1035), a missing or short file fails creation.  A missing final_norm
 * falls back to the last layer's post-attention norm as the reference does
 * (:1162-1165).  A quantized type whose {proj}_weight.bin is absent uses the
 * FP16 {proj}.bin quantized at load with the same per-column rule (the
 * reference would run that projection in FP16 instead; a fused matrix needs
 * one encoding).
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include "md_internal.h"

#define ALIGN_UP(x) (((x) + 255u) & ~(size_t)255u)

void* md_arena_alloc(DevArena* a, size_t bytes) {
    size_t need = ALIGN_UP(bytes ? bytes : 1);
    if (a->off + need > a->size) {
        MD_LOG("device arena exhausted (%zu + %zu > %zu)\n", a->off, need, a->size);
        return NULL;
    }
    void* p = a->base + a->off;
    a->off += need;
    return p;
}

static size_t row_bytes(int wtype, int K) {
    return wtype == B2_W_F16 ? (size_t)K * 2 : wtype == B2_W_I8 ? (size_t)K : (size_t)K / 2;
}

static size_t proj_bytes(int wtype, int rows, int K) {
    return ALIGN_UP(row_bytes(wtype, K) * rows) + (wtype == B2_W_F16 ? 0 : ALIGN_UP((size_t)rows * 4));
}

size_t md_model_bytes(const MatmulDecoderConfig* c, int wtype, int max_seq, int n_lm_heads) {
    const size_t H = c->hidden_dim, V = c->vocab_size, F = c->ffn_dim;
    const int qd = c->num_q_heads * c->head_dim, kvd = c->num_kv_heads * c->head_dim;
    size_t t = ALIGN_UP(V * H * 4) + ALIGN_UP(H * 4);
    if (n_lm_heads > 1) {
        const size_t vh = c->lm_head_vocab_size > 0 ? (size_t)c->lm_head_vocab_size : V;
        t += (size_t)n_lm_heads * ALIGN_UP(vh * H * 4);
    } else if (c->disable_npu_lm_head) {
        t += ALIGN_UP(V * H * 2);
    } else {
        t += ALIGN_UP(V * H) + ALIGN_UP(V * 4);
    }
    size_t per_layer = proj_bytes(wtype, qd + 2 * kvd, (int)H) + proj_bytes(wtype, (int)H, qd) +
                       proj_bytes(wtype, (int)(2 * F), (int)H) + 2 * proj_bytes(wtype, (int)H, (int)F) +
                       2 * ALIGN_UP(H * 4) + 2 * ALIGN_UP((size_t)c->head_dim * 4);
    t += per_layer * (size_t)c->num_layers;
    t += 2 * ALIGN_UP((size_t)max_seq * (c->head_dim / 2) * 4);
    return t + 4096;
}

/* ─── file helpers ─── */

static void* read_file_exact(const char* path, size_t bytes) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    void* buf = malloc(bytes ? bytes : 1);
    if (!buf) {
        fclose(f);
        return NULL;
    }
    size_t got = fread(buf, 1, bytes, f);
    fclose(f);
    if (got != bytes) {
        MD_LOG("%s: expected %zu bytes, read %zu\n", path, bytes, got);
        free(buf);
        return NULL;
    }
    return buf;
}

static void* read_first(const char* dir, const char* const* names, size_t bytes, char* used) {
    char path[1024];
    for (int i = 0; names[i]; i++) {
        snprintf(path, sizeof(path), "%s/%s", dir, names[i]);
        void* p = read_file_exact(path, bytes);
        if (p) {
            if (used) snprintf(used, 1024, "%s", path);
            return p;
        }
    }
    return NULL;
}

static int is_dir(const char* p) {
    struct stat st;
    return stat(p, &st) == 0 && S_ISDIR(st.st_mode);
}

static const char* kProj[7] = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"};

static void proj_shape(const MatmulDecoderConfig* c, int i, int* K, int* N) {
    const int H = c->hidden_dim, qd = c->num_q_heads * c->head_dim, kvd = c->num_kv_heads * c->head_dim;
    const int F = c->ffn_dim;
    const int ks[7] = {H, H, H, qd, H, H, F};
    const int ns[7] = {qd, kvd, kvd, H, F, F, H};
    *K = ks[i];
    *N = ns[i];
}

static void free_host_layer(HostLayer* L) {
    for (int i = 0; i < 7; i++) {
        free(L->w[i]);
        free(L->s[i]);
    }
    free(L->in_norm);
    free(L->post_norm);
    free(L->q_norm);
    free(L->k_norm);
    memset(L, 0, sizeof(*L));
}

static int load_host_layer(HostLayer* L, const char* dir, const MatmulDecoderConfig* c, int target) {
    memset(L, 0, sizeof(*L));
    const size_t H = c->hidden_dim, hd = c->head_dim;
    static const char* in_names[] = {"input_norm.bin", "input_norm_weight.bin", NULL};
    static const char* post_names[] = {"post_attn_norm.bin", "post_norm.bin", "post_attn_norm_weight.bin", NULL};
    static const char* qn_names[] = {"q_norm.bin", "q_norm_weight.bin", NULL};
    static const char* kn_names[] = {"k_norm.bin", "k_norm_weight.bin", NULL};
    L->in_norm = (float*)read_first(dir, in_names, H * 4, NULL);
    L->post_norm = (float*)read_first(dir, post_names, H * 4, NULL);
    if (!L->in_norm || !L->post_norm) {
        MD_LOG("Failed to load norm weights from %s\n", dir);
        return MATMUL_DECODER_ERR_FILE_IO;
    }
    if (c->has_qk_norm) {
        L->q_norm = (float*)read_first(dir, qn_names, hd * 4, NULL);
        L->k_norm = (float*)read_first(dir, kn_names, hd * 4, NULL);
        if (!L->q_norm || !L->k_norm) {
            MD_LOG("Failed to load QK norm weights from %s\n", dir);
            return MATMUL_DECODER_ERR_FILE_IO;
        }
    }
    char path[1024];
    for (int i = 0; i < 7; i++) {
        int K, N;
        proj_shape(c, i, &K, &N);
        if (target != B2_W_F16) {
            size_t qb = target == B2_W_I8 ? (size_t)K * N : (size_t)K * N / 2;
            snprintf(path, sizeof(path), "%s/%s_weight.bin", dir, kProj[i]);
            L->w[i] = read_file_exact(path, qb);
            if (L->w[i]) {
                snprintf(path, sizeof(path), "%s/%s_scales.bin", dir, kProj[i]);
                L->s[i] = (float*)read_file_exact(path, (size_t)N * 4);
                if (!L->s[i]) {
                    MD_LOG("Missing scales %s\n", path);
                    return MATMUL_DECODER_ERR_FILE_IO;
                }
                L->wt[i] = target;
                continue;
            }
        }
        snprintf(path, sizeof(path), "%s/%s.bin", dir, kProj[i]);
        L->w[i] = read_file_exact(path, (size_t)K * N * 2);
        if (!L->w[i]) {
            MD_LOG("Failed to load %s\n", path);
            return MATMUL_DECODER_ERR_FILE_IO;
        }
        L->wt[i] = B2_W_F16;
    }
    return MATMUL_DECODER_OK;
}

/* ─── relayout into device rows ─── */

/* Write projection i (file layout, encoding wt) as rows [row0, row0+N) of a
 * device-layout staging matrix with K columns and encoding `target`. */
static int stage_rows(unsigned char* dst, float* dst_scales, int row0, int target, const void* src,
                      const float* src_scales, int wt, int K, int N) {
    const void* use = src;
    const float* use_s = src_scales;
    uint8_t* tmpq = NULL;
    float* tmps = NULL;
    if (wt != target) {
        if (wt != B2_W_F16) return MATMUL_DECODER_ERR_UNSUPPORTED;
        const int bits = target == B2_W_I8 ? 8 : 4;
        tmpq = (uint8_t*)malloc(bits == 8 ? (size_t)K * N : (size_t)K * N / 2);
        tmps = (float*)malloc((size_t)N * 4);
        if (!tmpq || !tmps) {
            free(tmpq);
            free(tmps);
            return MATMUL_DECODER_ERR_MEMORY;
        }
        md_quantize_cols((const uint16_t*)src, K, N, bits, tmpq, tmps);
        use = tmpq;
        use_s = tmps;
    }
    const size_t rb = row_bytes(target, K);
    for (int n0 = 0; n0 < N; n0 += 64) {
        const int n1 = n0 + 64 < N ? n0 + 64 : N;
        for (int k = 0; k < K; k++) {
            for (int n = n0; n < n1; n++) {
                unsigned char* row = dst + (size_t)(row0 + n) * rb;
                if (target == B2_W_F16) {
                    ((uint16_t*)row)[k] = ((const uint16_t*)use)[(size_t)k * N + n];
                } else if (target == B2_W_I8) {
                    row[k] = ((const uint8_t*)use)[(size_t)k * N + n];
                } else {
                    const uint8_t b = ((const uint8_t*)use)[(size_t)k * (N / 2) + n / 2];
                    const uint8_t nib = (n & 1) ? (uint8_t)(b >> 4) : (uint8_t)(b & 15);
                    if (k & 1) row[k / 2] = (uint8_t)((row[k / 2] & 0x0F) | (nib << 4));
                    else row[k / 2] = (uint8_t)((row[k / 2] & 0xF0) | nib);
                }
            }
        }
    }
    if (dst_scales && use_s) memcpy(dst_scales + row0, use_s, (size_t)N * 4);
    free(tmpq);
    free(tmps);
    return MATMUL_DECODER_OK;
}

static int upload_proj(DevModel* m, DevProj* P, int rows, int K, const int* parts, int nparts,
                       const HostLayer* L) {
    const int target = m->wtype;
    const size_t rb = row_bytes(target, K);
    unsigned char* stage = (unsigned char*)calloc((size_t)rows, rb);
    float* sstage = target == B2_W_F16 ? NULL : (float*)calloc((size_t)rows, 4);
    if (!stage || (target != B2_W_F16 && !sstage)) {
        free(stage);
        free(sstage);
        return MATMUL_DECODER_ERR_MEMORY;
    }
    int row0 = 0, rc = 0;
    for (int i = 0; i < nparts && !rc; i++) {
        int k, n;
        proj_shape(&m->cfg, parts[i], &k, &n);
        if (L->wt[parts[i]] != target && L->wt[parts[i]] == B2_W_F16)
            MD_LOG("%s: no quantized file, quantizing the FP16 weight at load\n", kProj[parts[i]]);
        rc = stage_rows(stage, sstage, row0, target, L->w[parts[i]], L->s[parts[i]], L->wt[parts[i]], k, n);
        row0 += n;
    }
    if (!rc) {
        P->rows = rows;
        P->K = K;
        P->wtype = target;
        P->w = md_arena_alloc(&m->arena, rb * rows);
        P->s = target == B2_W_F16 ? NULL : (float*)md_arena_alloc(&m->arena, (size_t)rows * 4);
        if (!P->w || (target != B2_W_F16 && !P->s)) rc = MATMUL_DECODER_ERR_MEMORY;
    }
    if (!rc) rc = b2_memcpy_h2d(P->w, stage, rb * rows, NULL);
    if (!rc && sstage) rc = b2_memcpy_h2d(P->s, sstage, (size_t)rows * 4, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    if (rc) MD_LOG("upload failed: %s\n", b2_last_error());
    free(stage);
    free(sstage);
    return rc;
}

/* Projection i in its file layout ([K][N], int4 [K][N/2]) in the model's
 * encoding, quantized at load like stage_rows when only FP16 exists.  The
 * persistent decode kernel streams down_proj this way: one row per input
 * channel with the output columns contiguous. */
static int upload_file_layout(DevModel* m, void** dst, int proj, const HostLayer* L) {
    int K, N;
    proj_shape(&m->cfg, proj, &K, &N);
    const int target = m->wtype, wt = L->wt[proj];
    const void* use = L->w[proj];
    uint8_t* tmpq = NULL;
    float* tmps = NULL;
    if (wt != target) {
        if (wt != B2_W_F16) return MATMUL_DECODER_ERR_UNSUPPORTED;
        const int bits = target == B2_W_I8 ? 8 : 4;
        tmpq = (uint8_t*)malloc(bits == 8 ? (size_t)K * N : (size_t)K * N / 2);
        tmps = (float*)malloc((size_t)N * 4);
        if (!tmpq || !tmps) {
            free(tmpq);
            free(tmps);
            return MATMUL_DECODER_ERR_MEMORY;
        }
        md_quantize_cols((const uint16_t*)use, K, N, bits, tmpq, tmps);
        use = tmpq;
    }
    const size_t bytes = target == B2_W_F16 ? (size_t)K * N * 2 : target == B2_W_I8 ? (size_t)K * N : (size_t)K * N / 2;
    int rc = 0;
    *dst = md_arena_alloc(&m->arena, bytes);
    if (!*dst) rc = MATMUL_DECODER_ERR_MEMORY;
    if (!rc) rc = b2_memcpy_h2d(*dst, use, bytes, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    free(tmpq);
    free(tmps);
    return rc;
}

static float* upload_f32(DevModel* m, const float* src, size_t n) {
    float* d = (float*)md_arena_alloc(&m->arena, n * 4);
    if (!d) return NULL;
    if (b2_memcpy_h2d(d, src, n * 4, NULL) || b2_stream_sync(NULL)) {
        MD_LOG("upload failed: %s\n", b2_last_error());
        return NULL;
    }
    return d;
}

static int wtype_of(QuantizationType q) {
    return q == QUANT_INT8 ? B2_W_I8 : (q == QUANT_INT4 || q == QUANT_INT4_G128) ? B2_W_I4 : B2_W_F16;
}

static int arena_init(DevModel* m, size_t extra) {
    const int nh = m->cfg.num_lm_heads > 1 ? m->cfg.num_lm_heads : 0;
    m->arena.size = md_model_bytes(&m->cfg, m->wtype, m->max_seq, nh) + extra;
    void* p = NULL;
    if (b2_malloc(&p, m->arena.size)) {
        MD_LOG("device arena of %.1f MB: %s\n", m->arena.size / 1e6, b2_last_error());
        return MATMUL_DECODER_ERR_MEMORY;
    }
    m->arena.base = (unsigned char*)p;
    m->arena.off = 0;
    return 0;
}

static int upload_lm_head(DevModel* m, const float* table) {
    const size_t V = m->cfg.vocab_size, H = m->cfg.hidden_dim;
    uint16_t* t16 = (uint16_t*)malloc(V * H * 2);
    if (!t16) return MATMUL_DECODER_ERR_MEMORY;
    for (size_t i = 0; i < V * H; i++) t16[i] = md_f32_to_f16(table[i]);
    int rc = 0;
    if (m->cfg.disable_npu_lm_head) {
        m->lm_wtype = B2_W_F16;
        m->lm = md_arena_alloc(&m->arena, V * H * 2);
        rc = m->lm ? b2_memcpy_h2d(m->lm, t16, V * H * 2, NULL) : MATMUL_DECODER_ERR_MEMORY;
    } else {
        m->lm_wtype = B2_W_I8;
        int8_t* q = (int8_t*)malloc(V * H);
        float* s = (float*)malloc(V * 4);
        if (!q || !s) rc = MATMUL_DECODER_ERR_MEMORY;
        if (!rc) {
            md_quantize_rows_i8(t16, (int)V, (int)H, q, s);
            m->lm = md_arena_alloc(&m->arena, V * H);
            m->lm_scales = (float*)md_arena_alloc(&m->arena, V * 4);
            if (!m->lm || !m->lm_scales) rc = MATMUL_DECODER_ERR_MEMORY;
        }
        if (!rc) rc = b2_memcpy_h2d(m->lm, q, V * H, NULL);
        if (!rc) rc = b2_memcpy_h2d(m->lm_scales, s, V * 4, NULL);
        free(q);
        free(s);
    }
    if (!rc) rc = b2_stream_sync(NULL);
    free(t16);
    return rc;
}

static int upload_common(DevModel* m, const float* emb, const float* lm_head, float** lm_heads,
                         const float* final_norm, const HostLayer* layers) {
    const MatmulDecoderConfig* c = &m->cfg;
    const size_t V = c->vocab_size, H = c->hidden_dim;
    const int qd = c->num_q_heads * c->head_dim, kvd = c->num_kv_heads * c->head_dim;
    m->emb = upload_f32(m, emb, V * H);
    if (!m->emb) return MATMUL_DECODER_ERR_MEMORY;
    if (m->n_lm_heads > 1) {
        m->lm_heads = (float**)calloc((size_t)m->n_lm_heads, sizeof(float*));
        for (int i = 0; i < m->n_lm_heads; i++) {
            m->lm_heads[i] = upload_f32(m, lm_heads[i], (size_t)m->lm_vocab * H);
            if (!m->lm_heads[i]) return MATMUL_DECODER_ERR_MEMORY;
        }
    } else {
        int rc = upload_lm_head(m, lm_head ? lm_head : emb);
        if (rc) return rc;
    }
    m->layers = (DevLayer*)calloc((size_t)c->num_layers, sizeof(DevLayer));
    if (!m->layers) return MATMUL_DECODER_ERR_MEMORY;
    for (int l = 0; l < c->num_layers; l++) {
        const HostLayer* L = &layers[l];
        DevLayer* D = &m->layers[l];
        static const int qkv[3] = {0, 1, 2}, o[1] = {3}, gu[2] = {4, 5}, dn[1] = {6};
        int rc = upload_proj(m, &D->qkv, qd + 2 * kvd, (int)H, qkv, 3, L);
        if (!rc) rc = upload_proj(m, &D->o, (int)H, qd, o, 1, L);
        if (!rc) rc = upload_proj(m, &D->gu, 2 * c->ffn_dim, (int)H, gu, 2, L);
        if (!rc) rc = upload_proj(m, &D->down, (int)H, c->ffn_dim, dn, 1, L);
        if (!rc) rc = upload_file_layout(m, &D->down_t, 6, L);
        if (rc) return rc;
        D->in_norm = upload_f32(m, L->in_norm, H);
        D->post_norm = upload_f32(m, L->post_norm, H);
        if (!D->in_norm || !D->post_norm) return MATMUL_DECODER_ERR_MEMORY;
        if (c->has_qk_norm && L->q_norm && L->k_norm) {
            D->q_norm = upload_f32(m, L->q_norm, c->head_dim);
            D->k_norm = upload_f32(m, L->k_norm, c->head_dim);
            if (!D->q_norm || !D->k_norm) return MATMUL_DECODER_ERR_MEMORY;
        }
    }
    m->final_norm = final_norm ? upload_f32(m, final_norm, H) : m->layers[c->num_layers - 1].post_norm;
    if (!m->final_norm) return MATMUL_DECODER_ERR_MEMORY;
    /* RoPE tables, precompute_rope_tables (src/matmul_decoder.c:620-631). */
    const int half = c->head_dim / 2;
    float* ct = (float*)malloc((size_t)m->max_seq * half * 4);
    float* st = (float*)malloc((size_t)m->max_seq * half * 4);
    if (!ct || !st) {
        free(ct);
        free(st);
        return MATMUL_DECODER_ERR_MEMORY;
    }
    for (int pos = 0; pos < m->max_seq; pos++)
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(c->rope_theta, (2.0f * (float)i) / (float)c->head_dim);
            float angle = (float)pos * freq;
            ct[(size_t)pos * half + i] = cosf(angle);
            st[(size_t)pos * half + i] = sinf(angle);
        }
    m->cos_tab = upload_f32(m, ct, (size_t)m->max_seq * half);
    m->sin_tab = upload_f32(m, st, (size_t)m->max_seq * half);
    free(ct);
    free(st);
    return (m->cos_tab && m->sin_tab) ? 0 : MATMUL_DECODER_ERR_MEMORY;
}

static int model_init_common(DevModel* m, const MatmulDecoderConfig* cfg, QuantizationType q, int max_seq) {
    memset(m, 0, sizeof(*m));
    m->cfg = *cfg;
    snprintf(m->name, sizeof(m->name), "%s", cfg->name ? cfg->name : "");
    m->cfg.name = m->name;
    m->cfg.max_seq_len = max_seq;
    m->quant = q;
    m->wtype = wtype_of(q);
    m->max_seq = max_seq;
    m->n_lm_heads = cfg->num_lm_heads > 1 ? cfg->num_lm_heads : 0;
    m->lm_vocab = cfg->lm_head_vocab_size > 0 ? cfg->lm_head_vocab_size : cfg->vocab_size;
    int rc = md_config_validate(cfg);
    if (rc) MD_LOG("unsupported or invalid config (code %d)\n", rc);
    return rc;
}

int md_model_from_host(DevModel* m, const MatmulDecoderConfig* cfg, QuantizationType q, int max_seq,
                       const float* emb, const float* lm_head, const HostLayer* layers, size_t extra) {
    int rc = model_init_common(m, cfg, q, max_seq);
    if (rc) return rc;
    if (m->n_lm_heads > 1) return MATMUL_DECODER_ERR_UNSUPPORTED;
    rc = arena_init(m, extra);
    if (rc) return rc;
    return upload_common(m, emb, lm_head, NULL, NULL, layers);
}

int md_model_load_dir(DevModel* m, const char* dir, const MatmulDecoderConfig* cfg, QuantizationType q,
                      int max_seq, size_t extra) {
    int rc = model_init_common(m, cfg, q, max_seq);
    if (rc) return rc;
    const size_t V = cfg->vocab_size, H = cfg->hidden_dim;
    char path[1024];
    float* emb = NULL;
    float* lm = NULL;
    float** heads = NULL;
    float* fnorm = NULL;
    HostLayer* layers = (HostLayer*)calloc((size_t)cfg->num_layers, sizeof(HostLayer));
    if (!layers) return MATMUL_DECODER_ERR_MEMORY;

    snprintf(path, sizeof(path), "%s/embeddings.bin", dir);
    emb = (float*)read_file_exact(path, V * H * 4);
    if (!emb) {
        MD_LOG("Failed to load embeddings from %s\n", path);
        rc = MATMUL_DECODER_ERR_FILE_IO;
        goto done;
    }
    if (m->n_lm_heads > 1) {
        heads = (float**)calloc((size_t)m->n_lm_heads, sizeof(float*));
        for (int i = 0; i < m->n_lm_heads && !rc; i++) {
            snprintf(path, sizeof(path), "%s/lm_head_%02d.bin", dir, i);
            heads[i] = (float*)read_file_exact(path, (size_t)m->lm_vocab * H * 4);
            if (!heads[i]) {
                MD_LOG("Failed to load %s\n", path);
                rc = MATMUL_DECODER_ERR_FILE_IO;
            }
        }
        if (rc) goto done;
    } else {
        snprintf(path, sizeof(path), "%s/lm_head.bin", dir);
        lm = (float*)read_file_exact(path, V * H * 4);
        if (!lm && !cfg->tie_word_embeddings) {
            MD_LOG("Failed to load lm_head from %s\n", path);
            rc = MATMUL_DECODER_ERR_FILE_IO;
            goto done;
        }
    }
    {
        static const char* fn_names[] = {"final_norm.bin", "model_norm.bin", NULL};
        fnorm = (float*)read_first(dir, fn_names, H * 4, NULL);
        if (!fnorm) MD_LOG("WARNING: final_norm.bin not found, using last layer post_norm\n");
    }
    for (int l = 0; l < cfg->num_layers; l++) {
        char ld[1024];
        snprintf(ld, sizeof(ld), "%s/layers/layer_%02d", dir, l);
        if (!is_dir(ld)) snprintf(ld, sizeof(ld), "%s/layer_%02d", dir, l);
        rc = load_host_layer(&layers[l], ld, cfg, m->wtype);
        if (rc) {
            MD_LOG("Failed to load layer %d weights\n", l);
            goto done;
        }
    }
    rc = arena_init(m, extra);
    if (!rc) rc = upload_common(m, emb, lm, heads, fnorm, layers);
done:
    free(emb);
    free(lm);
    if (heads) {
        for (int i = 0; i < m->n_lm_heads; i++) free(heads[i]);
        free(heads);
    }
    free(fnorm);
    for (int l = 0; l < cfg->num_layers; l++) free_host_layer(&layers[l]);
    free(layers);
    return rc;
}

void md_model_free(DevModel* m) {
    if (m->arena.base) b2_free(m->arena.base);
    free(m->layers);
    free(m->lm_heads);
    memset(m, 0, sizeof(*m));
}
