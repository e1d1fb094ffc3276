/*
 * Decoder context: create / step / prefill / KV / stats (the reference C API,
 * src/matmul_decoder.c:830-2180 of suharvest/rknn-matmul-parallel).
 *
 * Device residency: weights, the FP16 KV cache [layer][kv_head][pos][hd],
 * RoPE tables and every activation live in one device arena.  A decode step
 * is one CUDA graph replay: a host->device copy of a small pinned parameter
 * block (token id, "use embedding" flag, position, optional embedding), the
 * embedding gather, all layers, then (unless in prefill mode) the final norm,
 * the lm_head and the on-device argmax, and a 4-byte device->host copy of the
 * token.  The graph reads the position from device memory, so one graph
 * serves every position.  Logits cross to the host only when the caller
 * passes a logits buffer.
 *
 * When the shapes allow it (INT8 lm_head, GQA group <= 2, head_dim 128), a
 * single-token step runs instead as ONE launch of the persistent decode
 * kernel (b2_mk_decode), which streams the whole token's weights from one
 * CTA per SM; B2_DECODE_KERNEL=graph in the environment at create time keeps
 * the graph of per-op kernels.  Batch prefill always uses the multi-kernel
 * pass.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "md_internal.h"

#define PARAMS_INTS 8 /* [0] token, [1] use_embedding, [4] position */

/* Context length up to which a single-token step uses the persistent kernel:
 * beyond it the graph path's split-KV attention is faster (B200, W8A16:
 * persistent 0.84 / 1.11 / 1.79 ms and graph 1.22 / 1.33 / 1.44 ms per token
 * at 128 / 1024 / 4096 cached positions).  B2_MK_MAX_CONTEXT overrides it at
 * create time. */
#define MD_MK_MAX_CONTEXT 2048

struct MatmulDecoderContext {
    DevModel model;
    MatmulDecoderConfig config;
    int device, max_seq, seq_len, rows_cap, split_decode;
    int hidden_row; /* row of `hidden` holding the most recent token */
    b2_stream_t stream;
    uint16_t *k_cache, *v_cache;
    long long layer_stride;
    float *hidden, *qkv, *attn, *act, *logits;
    uint16_t* x16; /* [rows_cap][max(H, qd, ffn)] FP16 rows for the prefill tensor-core GEMM */
    uint16_t* x16b; /* [rows_cap][ffn] FP16 gate|up output for the down-projection GEMM */
    int* d_blk;    /* PARAMS_INTS ints then hidden_dim floats */
    int* d_pos;    /* [rows_cap] prefill positions */
    int* d_tok;
    int* d_loop;   /* device greedy loop: [0] token, [1] position, [2] step */
    int* d_hist;   /* [max_seq] tokens produced by the device loop */
    void *attn_work, *lm_work;
    int* h_blk;    /* pinned mirror of d_blk */
    int* h_tok;    /* pinned */
    int* h_pos;    /* pinned [rows_cap] */
    int* h_loop;   /* pinned [4] */
    b2_graph_t g_head, g_nohead, g_loop;
    int use_mk;       /* persistent decode kernel selected */
    int mk_max_ctx;   /* ... for steps below this many cached positions */
    int hidden_mk;    /* last token's hidden lives in a persistent kernel's scratch (1: first, 2: second) */
    B2MkPlan mk;
    B2MkLayer* d_mk_layers; /* device copy of the per-layer pointer table */
    int* d_mk_state;  /* B2_MK_STATE_INTS */
    int* h_mk_state;  /* pinned mirror */
    void* mk_scratch;
    /* second-generation persistent kernel: its own plan, state block and scratch */
    int use_mk2;
    B2MkPlan mk2;
    B2MkLayer* d_mk2_layers;
    int* d_mk2_state;
    int* h_mk2_state;
    void* mk2_buf;    /* tile-major weights, lm_head tiles, scratch and state (one allocation) */
    int test_hooks;   /* B2_MK_POLL_LIMIT was set at create: B2_MK_STALL_TEST is read per step */
    size_t mk2_scratch_bytes;
    /* on-device sampling: draw i of this context uses (sample_seed, sample_counter = i) */
    unsigned long long sample_seed, sample_counter;
    int* d_sample;    /* [8]: [0] token, [1..4] sampler info, then the repeat list */
    int d_sample_cap; /* repeat-list entries d_sample has room for */
    b2_event_t ev[3];
    MatmulDecoderStats stats;
};

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

static int fail(const char* what, int rc) {
    MD_LOG("%s failed (%d): %s\n", what, rc, b2_last_error());
    return rc;
}

/* ─── creation ─── */

static size_t ctx_bytes(const MatmulDecoderConfig* c, int max_seq, int rows_cap, int split_decode) {
    const size_t H = c->hidden_dim, hd = c->head_dim, qd = (size_t)c->num_q_heads * hd;
    const size_t kvd = (size_t)c->num_kv_heads * hd, F = c->ffn_dim;
    size_t vmax = c->vocab_size;
    if (c->num_lm_heads > 1 && (size_t)c->lm_head_vocab_size > vmax) vmax = c->lm_head_vocab_size;
    size_t t = 2 * (size_t)c->num_layers * kvd * (size_t)max_seq * 2;   /* KV cache */
    t += (size_t)rows_cap * (H + qd + 2 * kvd + qd + F) * 4 + 8 * 256;   /* activations */
    t += (size_t)rows_cap * (H > qd ? (H > F ? H : F) : (qd > F ? qd : F)) * 2 + 256; /* FP16 GEMM rows */
    t += (size_t)rows_cap * F * 2 + 256;                                  /* FP16 gate|up output */
    t += vmax * 4 + (PARAMS_INTS + H) * 4 + (size_t)rows_cap * 4 + 1024;
    size_t aw1 = b2_attention_workspace(1, c->num_q_heads, (int)hd, split_decode);
    size_t aw2 = b2_attention_workspace(rows_cap, c->num_q_heads, (int)hd, 1);
    t += (aw1 > aw2 ? aw1 : aw2) + b2_lm_head_workspace(1, (int)vmax) + 1024;
    t += 256 + (size_t)max_seq * 4 + 256;
    t += 256 + b2_mk_scratch_bytes(c->num_layers, (int)H, (int)F, c->num_q_heads, c->num_kv_heads, (int)hd) + 256;
    t += sizeof(B2MkLayer) * (size_t)c->num_layers + 256;
    return t;
}

static int ctx_alloc(MatmulDecoderContext* ctx) {
    DevModel* m = &ctx->model;
    const MatmulDecoderConfig* c = &m->cfg;
    const size_t H = c->hidden_dim, hd = c->head_dim, qd = (size_t)c->num_q_heads * hd;
    const size_t kvd = (size_t)c->num_kv_heads * hd, F = c->ffn_dim;
    size_t vmax = c->vocab_size;
    if (c->num_lm_heads > 1 && (size_t)c->lm_head_vocab_size > vmax) vmax = c->lm_head_vocab_size;
    ctx->layer_stride = (long long)kvd * ctx->max_seq;
    const size_t kv_bytes = (size_t)c->num_layers * kvd * ctx->max_seq * 2;
    ctx->k_cache = (uint16_t*)md_arena_alloc(&m->arena, kv_bytes);
    ctx->v_cache = (uint16_t*)md_arena_alloc(&m->arena, kv_bytes);
    ctx->hidden = (float*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * H * 4);
    ctx->qkv = (float*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * (qd + 2 * kvd) * 4);
    ctx->attn = (float*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * qd * 4);
    ctx->act = (float*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * F * 4);
    {
        const size_t kmax = H > qd ? (H > F ? H : F) : (qd > F ? qd : F);
        ctx->x16 = (uint16_t*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * kmax * 2);
        ctx->x16b = (uint16_t*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * F * 2);
        if (!ctx->x16 || !ctx->x16b) return MATMUL_DECODER_ERR_MEMORY;
    }
    ctx->logits = (float*)md_arena_alloc(&m->arena, vmax * 4);
    ctx->d_blk = (int*)md_arena_alloc(&m->arena, (PARAMS_INTS + H) * 4);
    ctx->d_pos = (int*)md_arena_alloc(&m->arena, (size_t)ctx->rows_cap * 4);
    ctx->d_tok = (int*)md_arena_alloc(&m->arena, 64);
    size_t aw1 = b2_attention_workspace(1, c->num_q_heads, (int)hd, ctx->split_decode);
    size_t aw2 = b2_attention_workspace(ctx->rows_cap, c->num_q_heads, (int)hd, 1);
    ctx->attn_work = md_arena_alloc(&m->arena, aw1 > aw2 ? aw1 : aw2);
    ctx->lm_work = md_arena_alloc(&m->arena, b2_lm_head_workspace(1, (int)vmax));
    ctx->d_loop = (int*)md_arena_alloc(&m->arena, 64);
    ctx->d_hist = (int*)md_arena_alloc(&m->arena, (size_t)ctx->max_seq * 4);
    if (!ctx->d_loop || !ctx->d_hist) return MATMUL_DECODER_ERR_MEMORY;
    const size_t mk_bytes =
        b2_mk_scratch_bytes(c->num_layers, (int)H, (int)F, c->num_q_heads, c->num_kv_heads, (int)hd);
    ctx->d_mk_state = (int*)md_arena_alloc(&m->arena, B2_MK_STATE_INTS * 4);
    ctx->d_mk_layers = (B2MkLayer*)md_arena_alloc(&m->arena, sizeof(B2MkLayer) * (size_t)c->num_layers);
    if (!ctx->d_mk_layers) return MATMUL_DECODER_ERR_MEMORY;
    ctx->mk_scratch = md_arena_alloc(&m->arena, mk_bytes);
    if (!ctx->d_mk_state || !ctx->mk_scratch) return MATMUL_DECODER_ERR_MEMORY;
    if (b2_memset(ctx->d_mk_state, 0, B2_MK_STATE_INTS * 4, NULL) || b2_memset(ctx->mk_scratch, 0, mk_bytes, NULL))
        return MATMUL_DECODER_ERR_RKNN;
    if (!ctx->k_cache || !ctx->v_cache || !ctx->hidden || !ctx->qkv || !ctx->attn || !ctx->act ||
        !ctx->logits || !ctx->d_blk || !ctx->d_pos || !ctx->d_tok || !ctx->attn_work || !ctx->lm_work)
        return MATMUL_DECODER_ERR_MEMORY;
    int rc = b2_memset(ctx->k_cache, 0, kv_bytes, NULL);
    if (!rc) rc = b2_memset(ctx->v_cache, 0, kv_bytes, NULL);
    if (!rc) rc = b2_memset(ctx->d_blk, 0, (PARAMS_INTS + H) * 4, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    if (!rc) rc = b2_stream_create(&ctx->stream);
    for (int i = 0; i < 3 && !rc; i++) rc = b2_event_create(&ctx->ev[i]);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_blk, (PARAMS_INTS + H) * 4);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_tok, 64);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_pos, (size_t)ctx->rows_cap * 4);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_loop, 64);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_mk_state, B2_MK_STATE_INTS * 4);
    if (!rc) memset(ctx->h_blk, 0, (PARAMS_INTS + H) * 4);
    return rc;
}

static MatmulDecoderContext* ctx_new(const MatmulDecoderConfig* cfg, int max_seq) {
    MatmulDecoderContext* ctx = (MatmulDecoderContext*)calloc(1, sizeof(*ctx));
    if (!ctx) return NULL;
    ctx->max_seq = max_seq;
    ctx->rows_cap = 512;
    int sm = 148;
    b2_sm_count(&sm);
    ctx->split_decode = (2 * sm + cfg->num_kv_heads - 1) / cfg->num_kv_heads;
    if (ctx->split_decode > 64) ctx->split_decode = 64;
    b2_get_device(&ctx->device);
    return ctx;
}

/* Fill the persistent-kernel plan; selects it when the shapes are supported. */
static void mk_setup(MatmulDecoderContext* ctx) {
    const char* env = getenv("B2_DECODE_KERNEL");
    DevModel* m = &ctx->model;
    const MatmulDecoderConfig* c = &m->cfg;
    if ((env && strcmp(env, "graph") == 0) || m->n_lm_heads > 1 || m->lm_wtype != B2_W_I8 ||
        c->num_layers > B2_MK_MAX_LAYERS)
        return;
    B2MkPlan* p = &ctx->mk;
    memset(p, 0, sizeof(*p));
    p->n_layers = c->num_layers;
    p->hidden = c->hidden_dim;
    p->nq = c->num_q_heads;
    p->nkv = c->num_kv_heads;
    p->hd = c->head_dim;
    p->ffn = c->ffn_dim;
    p->vocab = c->vocab_size;
    p->max_seq = ctx->max_seq;
    p->rope_style = c->rope_style;
    p->wtype = m->wtype;
    p->eps = c->rms_eps;
    p->emb = m->emb;
    p->lm = m->lm;
    p->lm_s = m->lm_scales;
    p->final_norm = m->final_norm;
    p->cos_tab = m->cos_tab;
    p->sin_tab = m->sin_tab;
    p->k_cache = ctx->k_cache;
    p->v_cache = ctx->v_cache;
    p->layer_stride = ctx->layer_stride;
    p->state = ctx->d_mk_state;
    p->staged_emb = (const float*)(ctx->d_blk + PARAMS_INTS);
    p->logits = ctx->logits;
    p->hist = ctx->d_hist;
    p->hist_len = ctx->max_seq;
    p->do_lm = 1;
    p->scratch = ctx->mk_scratch;
    B2MkLayer* table = (B2MkLayer*)calloc((size_t)c->num_layers, sizeof(B2MkLayer));
    if (!table) return;
    for (int l = 0; l < c->num_layers; l++) {
        const DevLayer* L = &m->layers[l];
        B2MkLayer* d = &table[l];
        d->qkv = L->qkv.w;
        d->qkv_s = L->qkv.s;
        d->o = L->o.w;
        d->o_s = L->o.s;
        d->gu = L->gu.w;
        d->gu_s = L->gu.s;
        d->dn = L->down.w;
        d->dn_s = L->down.s;
        d->dn_t = L->down_t;
        d->in_norm = L->in_norm;
        d->post_norm = L->post_norm;
        const int qk = c->has_qk_norm && L->q_norm && L->k_norm;
        d->q_norm = qk ? L->q_norm : NULL;
        d->k_norm = qk ? L->k_norm : NULL;
    }
    int rc = b2_memcpy_h2d(ctx->d_mk_layers, table, sizeof(B2MkLayer) * (size_t)c->num_layers, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    free(table);
    p->layers = ctx->d_mk_layers;
    ctx->use_mk = !rc && b2_mk_check(p) == 0;
    const char* mx = getenv("B2_MK_MAX_CONTEXT");
    ctx->mk_max_ctx = mx && atoi(mx) > 0 ? atoi(mx) : MD_MK_MAX_CONTEXT;
}

/* The second-generation persistent kernel: tile-major copies of the layer
 * weights and of the INT8 lm_head (b2_tile_relayout), its own state block and
 * scratch, in one device allocation.  Selected when the first plan is valid
 * and the shapes fit (B2_DECODE_KERNEL=mk1 keeps the first kernel). */
static void mk2_setup(MatmulDecoderContext* ctx) {
    const char* env = getenv("B2_DECODE_KERNEL");
    if (!ctx->use_mk || (env && (strcmp(env, "mk1") == 0 || strcmp(env, "graph") == 0))) return;
    DevModel* m = &ctx->model;
    const MatmulDecoderConfig* c = &m->cfg;
    B2MkPlan* p = &ctx->mk2;
    *p = ctx->mk;
    const int L = c->num_layers, H = c->hidden_dim, F = c->ffn_dim;
    const int qd = c->num_q_heads * c->head_dim, nqkv = qd + 2 * c->num_kv_heads * c->head_dim;
    const int wt = m->wtype;
    const size_t rb_h = wt == B2_W_F16 ? (size_t)H * 2 : wt == B2_W_I8 ? (size_t)H : (size_t)H / 2;
    const size_t rb_o = wt == B2_W_F16 ? (size_t)qd * 2 : wt == B2_W_I8 ? (size_t)qd : (size_t)qd / 2;
#define MK2_AL(x) (((x) + 255) & ~(size_t)255)
    const size_t per_layer = MK2_AL((size_t)nqkv * rb_h) + MK2_AL((size_t)H * rb_o) + MK2_AL((size_t)2 * F * rb_h) +
                             MK2_AL((size_t)2 * F * 4);
    const size_t lm_bytes = MK2_AL((size_t)c->vocab_size * H);
    ctx->mk2_scratch_bytes = MK2_AL(b2_mk2_scratch_bytes(L, H, F, c->num_q_heads, c->num_kv_heads, c->head_dim));
    const size_t total = per_layer * L + lm_bytes + ctx->mk2_scratch_bytes + MK2_AL(sizeof(B2MkLayer) * L) +
                         MK2_AL(B2_MK_STATE_INTS * 4);
    unsigned char* base = NULL;
    if (b2_malloc((void**)&base, total)) {
        MD_LOG("second persistent kernel disabled: %s\n", b2_last_error());
        return;
    }
    ctx->mk2_buf = base;
    size_t off = 0;
#define MK2_TAKE(n) (off += MK2_AL(n), base + off - MK2_AL(n))
    B2MkLayer* table = (B2MkLayer*)calloc((size_t)L, sizeof(B2MkLayer));
    int rc = table ? b2_memcpy_d2h(table, ctx->d_mk_layers, sizeof(B2MkLayer) * (size_t)L, NULL) : -1;
    if (!rc) rc = b2_stream_sync(NULL);
    for (int l = 0; l < L && !rc; l++) {
        const DevLayer* D = &m->layers[l];
        void* qkv_t = MK2_TAKE((size_t)nqkv * rb_h);
        void* o_t = MK2_TAKE((size_t)H * rb_o);
        void* gu_t = MK2_TAKE((size_t)2 * F * rb_h);
        float* gu_ts = (float*)MK2_TAKE((size_t)2 * F * 4);
        rc = b2_tile_relayout(qkv_t, D->qkv.w, nqkv, (int)rb_h, 0, NULL, NULL, NULL);
        if (!rc) rc = b2_tile_relayout(o_t, D->o.w, H, (int)rb_o, 0, NULL, NULL, NULL);
        if (!rc) rc = b2_tile_relayout(gu_t, D->gu.w, 2 * F, (int)rb_h, F, D->gu.s ? gu_ts : NULL, D->gu.s, NULL);
        table[l].qkv_t = qkv_t;
        table[l].o_t = o_t;
        table[l].gu_t = gu_t;
        table[l].gu_ts = D->gu.s ? gu_ts : NULL;
    }
    void* lm_t = MK2_TAKE((size_t)c->vocab_size * H);
    if (!rc) rc = b2_tile_relayout(lm_t, m->lm, c->vocab_size, H, 0, NULL, NULL, NULL);
    p->scratch = MK2_TAKE(ctx->mk2_scratch_bytes);
    ctx->d_mk2_layers = (B2MkLayer*)MK2_TAKE(sizeof(B2MkLayer) * L);
    ctx->d_mk2_state = (int*)MK2_TAKE(B2_MK_STATE_INTS * 4);
#undef MK2_TAKE
#undef MK2_AL
    if (!rc) rc = b2_memcpy_h2d(ctx->d_mk2_layers, table, sizeof(B2MkLayer) * (size_t)L, NULL);
    if (!rc) rc = b2_memset(p->scratch, 0, ctx->mk2_scratch_bytes, NULL);
    if (!rc) rc = b2_memset(ctx->d_mk2_state, 0, B2_MK_STATE_INTS * 4, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    if (!rc) rc = b2_host_alloc((void**)&ctx->h_mk2_state, B2_MK_STATE_INTS * 4);
    free(table);
    p->layers = ctx->d_mk2_layers;
    p->lm_t = lm_t;
    p->state = ctx->d_mk2_state;
    {
        /* test-only: a short poll limit, and a wait that never completes, for
         * the tests of the timed-out-wait path */
        const char* pl = getenv("B2_MK_POLL_LIMIT");
        p->poll_limit = pl && atoll(pl) > 0 ? atoll(pl) : 0;
        ctx->test_hooks = p->poll_limit > 0;
        p->stall_test = 0;
    }
    ctx->use_mk2 = !rc && b2_mk2_check(p) == 0;
    if (rc) MD_LOG("second persistent kernel disabled (%d): %s\n", rc, b2_last_error());
}

static MatmulDecoderContext* ctx_finish(MatmulDecoderContext* ctx) {
    int rc = ctx_alloc(ctx);
    if (rc) {
        fail("context allocation", rc);
        matmul_decoder_destroy(ctx);
        return NULL;
    }
    mk_setup(ctx);
    mk2_setup(ctx);
    ctx->config = ctx->model.cfg;
    /* the draws follow the C library's generator, as the host sampler does */
    ctx->sample_seed = ((unsigned long long)(unsigned)rand() << 32) ^ (unsigned long long)(unsigned)rand();
    printf("[MatmulDecoder] Ready: %d layers, hidden=%d, heads=%d/%d, ffn=%d, vocab=%d, quant=%d, "
           "max_seq=%d, arena %.1f MB, decode kernel: %s\n",
           ctx->config.num_layers, ctx->config.hidden_dim, ctx->config.num_q_heads,
           ctx->config.num_kv_heads, ctx->config.ffn_dim, ctx->config.vocab_size, ctx->model.quant,
           ctx->max_seq, ctx->model.arena.size / 1e6,
           ctx->use_mk2 ? "persistent (tile stream below 512 cached positions)" : ctx->use_mk ? "persistent" : "graph");
    return ctx;
}

MatmulDecoderContext* matmul_decoder_create(const char* model_dir, const MatmulDecoderConfig* config,
                                            QuantizationType quant_type, int max_seq_len) {
    if (!model_dir) return NULL;
    MatmulDecoderConfig cfg;
    if (config) {
        cfg = *config;
    } else {
        char path[1024];
        snprintf(path, sizeof(path), "%s/config.json", model_dir);
        if (matmul_decoder_load_config(path, &cfg) != 0) {
            MD_LOG("Failed to load config from %s\n", path);
            return NULL;
        }
    }
    if (max_seq_len <= 0) max_seq_len = cfg.max_seq_len > 0 ? cfg.max_seq_len : 4096;
    MatmulDecoderContext* ctx = ctx_new(&cfg, max_seq_len);
    if (!ctx) return NULL;
    int rc = md_model_load_dir(&ctx->model, model_dir, &cfg, quant_type, max_seq_len,
                               ctx_bytes(&cfg, max_seq_len, ctx->rows_cap, ctx->split_decode));
    if (rc) {
        MD_LOG("Failed to create decoder from %s (%d)\n", model_dir, rc);
        matmul_decoder_destroy(ctx);
        return NULL;
    }
    return ctx_finish(ctx);
}

MatmulDecoderContext* matmul_decoder_create_from_weights(const MatmulDecoderConfig* config,
                                                         const float* embeddings,
                                                         const LayerWeights* layers,
                                                         const float* lm_head, QuantizationType quant_type,
                                                         int max_seq_len) {
    if (!config || !embeddings || !layers) return NULL;
    if (config->num_lm_heads > 1) {
        MD_LOG("create_from_weights: multi-head models load from a directory\n");
        return NULL;
    }
    if (max_seq_len <= 0) max_seq_len = config->max_seq_len > 0 ? config->max_seq_len : 4096;
    HostLayer* hl = (HostLayer*)calloc((size_t)config->num_layers, sizeof(HostLayer));
    if (!hl) return NULL;
    for (int l = 0; l < config->num_layers; l++) {
        const ProjectionWeight* p[7] = {&layers[l].q_proj, &layers[l].k_proj, &layers[l].v_proj,
                                        &layers[l].o_proj, &layers[l].gate_proj, &layers[l].up_proj,
                                        &layers[l].down_proj};
        for (int i = 0; i < 7; i++) {
            hl[l].w[i] = p[i]->data;
            hl[l].s[i] = p[i]->scales;
            hl[l].wt[i] = p[i]->quant_type == QUANT_INT8 ? B2_W_I8
                          : (p[i]->quant_type == QUANT_INT4 || p[i]->quant_type == QUANT_INT4_G128) ? B2_W_I4
                                                                                                 : B2_W_F16;
        }
        hl[l].in_norm = layers[l].input_norm_weight;
        hl[l].post_norm = layers[l].post_attn_norm_weight;
        hl[l].q_norm = layers[l].q_norm_weight;
        hl[l].k_norm = layers[l].k_norm_weight;
    }
    MatmulDecoderContext* ctx = ctx_new(config, max_seq_len);
    int rc = ctx ? md_model_from_host(&ctx->model, config, quant_type, max_seq_len, embeddings,
                                      config->tie_word_embeddings ? NULL : lm_head, hl,
                                      ctx_bytes(config, max_seq_len, ctx->rows_cap, ctx->split_decode))
                 : MATMUL_DECODER_ERR_MEMORY;
    free(hl);
    if (rc) {
        MD_LOG("create_from_weights failed (%d)\n", rc);
        matmul_decoder_destroy(ctx);
        return NULL;
    }
    return ctx_finish(ctx);
}

void matmul_decoder_destroy(MatmulDecoderContext* ctx) {
    if (!ctx) return;
    b2_set_device(ctx->device);
    if (ctx->stream) b2_stream_sync(ctx->stream);
    b2_graph_destroy(ctx->g_head);
    b2_graph_destroy(ctx->g_nohead);
    b2_graph_destroy(ctx->g_loop);
    for (int i = 0; i < 3; i++) b2_event_destroy(ctx->ev[i]);
    b2_stream_destroy(ctx->stream);
    b2_host_free(ctx->h_blk);
    b2_host_free(ctx->h_tok);
    b2_host_free(ctx->h_pos);
    b2_host_free(ctx->h_loop);
    b2_host_free(ctx->h_mk_state);
    b2_host_free(ctx->h_mk2_state);
    if (ctx->mk2_buf) b2_free(ctx->mk2_buf);
    if (ctx->d_sample) b2_free(ctx->d_sample);
    md_model_free(&ctx->model);
    free(ctx);
}

/* ─── the decode step ─── */

static B2KVRef kv_ref(const MatmulDecoderContext* ctx, const int* pos) {
    B2KVRef kv;
    kv.k_base = ctx->k_cache;
    kv.v_base = ctx->v_cache;
    kv.seq_stride = 0;
    kv.layer_stride = ctx->layer_stride;
    kv.layer = 0;
    kv.max_seq = ctx->max_seq;
    kv.rows_seq = NULL;
    kv.pos = pos;
    kv.n_seqs = 1;
    return kv;
}

/* Kernels of one token: embed, layers, and (head != NULL) lm_head + argmax
 * with the given table.  Shared by graph capture and the uncaptured path. */
static int enqueue_token(MatmulDecoderContext* ctx, int with_head, const void* table, const float* scales,
                         int wtype, int vocab, int copy_params) {
    DevModel* m = &ctx->model;
    const int H = m->cfg.hidden_dim;
    b2_stream_t s = ctx->stream;
    int rc = 0;
    if (copy_params) rc = b2_memcpy_h2d(ctx->d_blk, ctx->h_blk, (PARAMS_INTS + H) * 4, s);
    if (!rc) rc = b2_event_record(ctx->ev[0], s);
    if (!rc)
        rc = b2_embed(ctx->hidden, m->emb, ctx->d_blk, ctx->d_blk + 1, (const float*)(ctx->d_blk + PARAMS_INTS),
                      1, H, s);
    B2KVRef kv = kv_ref(ctx, ctx->d_blk + 4);
    LayerBuffers lb = {ctx->hidden, ctx->qkv, ctx->attn, ctx->act, ctx->attn_work, ctx->split_decode, NULL, NULL, -1, 0, NULL};
    if (!rc) rc = md_enqueue_layers(m, &lb, 1, &kv, s);
    if (!rc) rc = b2_event_record(ctx->ev[1], s);
    if (!rc && with_head) {
        rc = b2_lm_head_argmax(ctx->hidden, H, 1, H, vocab, table, scales, wtype, m->final_norm,
                               m->cfg.rms_eps, ctx->logits, vocab, ctx->d_tok, ctx->lm_work, s);
        if (!rc) rc = b2_memcpy_d2h(ctx->h_tok, ctx->d_tok, 4, s);
    }
    if (!rc) rc = b2_event_record(ctx->ev[2], s);
    return rc;
}

static int build_graph(MatmulDecoderContext* ctx, int with_head, b2_graph_t* g) {
    int rc = b2_graph_begin(ctx->stream);
    if (rc) return rc;
    DevModel* m = &ctx->model;
    int rc2 = enqueue_token(ctx, with_head, m->lm, m->lm_scales, m->lm_wtype, m->cfg.vocab_size, 1);
    b2_graph_t tmp = NULL;
    rc = b2_graph_end(ctx->stream, &tmp);
    if (rc2) {
        b2_graph_destroy(tmp);
        return rc2;
    }
    if (rc) return rc;
    *g = tmp;
    return 0;
}

static int check_step_args(MatmulDecoderContext* ctx, int token_id, const float* embedding, int vocab) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (!embedding && (token_id < 0 || token_id >= vocab)) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (ctx->seq_len >= ctx->max_seq) {
        MD_LOG("KV cache full: seq_len=%d >= max=%d\n", ctx->seq_len, ctx->max_seq);
        return MATMUL_DECODER_ERR_INVALID_ARG;
    }
    return 0;
}

static void stage_params(MatmulDecoderContext* ctx, int token_id, const float* embedding) {
    const int H = ctx->model.cfg.hidden_dim;
    ctx->h_blk[0] = embedding ? 0 : token_id;
    ctx->h_blk[1] = embedding ? 1 : 0;
    ctx->h_blk[4] = ctx->seq_len;
    if (embedding) memcpy(ctx->h_blk + PARAMS_INTS, embedding, (size_t)H * 4);
}

static void record_stats(MatmulDecoderContext* ctx, double t0, double t_copy, int with_head) {
    float layers_ms = 0.f, head_ms = 0.f;
    b2_event_elapsed_ms(&layers_ms, ctx->ev[0], ctx->ev[1]);
    if (with_head) b2_event_elapsed_ms(&head_ms, ctx->ev[1], ctx->ev[2]);
    ctx->stats.total_ms = (float)(now_ms() - t0);
    ctx->stats.matmul_ms = layers_ms;
    ctx->stats.rebind_ms = 0.f;
    ctx->stats.convert_ms = (float)t_copy;
    ctx->stats.cpu_ops_ms = 0.f;
    ctx->stats.lm_head_ms = head_ms;
    ctx->stats.n_steps++;
}

/* Which persistent kernel runs tokens at positions [pos, pos + n): 2 = the
 * tile-stream kernel, 1 = the first kernel, 0 = none (graph of per-op kernels). */
static int mk_kind(const MatmulDecoderContext* ctx, int pos, int n) {
    if (ctx->use_mk2 && pos + n <= b2_mk2_max_context()) return 2;
    if (ctx->use_mk && pos + n <= ctx->mk_max_ctx) return 1;
    return 0;
}

static B2MkPlan* mk_plan(MatmulDecoderContext* ctx, int kind) { return kind == 2 ? &ctx->mk2 : &ctx->mk; }
static int* mk_dstate(MatmulDecoderContext* ctx, int kind) { return kind == 2 ? ctx->d_mk2_state : ctx->d_mk_state; }
static int* mk_hstate(MatmulDecoderContext* ctx, int kind) { return kind == 2 ? ctx->h_mk2_state : ctx->h_mk_state; }
static int mk_launch(MatmulDecoderContext* ctx, int kind) {
    return kind == 2 ? b2_mk2_decode(&ctx->mk2, ctx->stream) : b2_mk_decode(&ctx->mk, ctx->stream);
}

/* A persistent-kernel wait timed out: clear its scratch (counters, flags,
 * accumulators) and state block so the next step starts from a consistent
 * state, and report a runtime error. */
static int mk_recover(MatmulDecoderContext* ctx, int kind, int code) {
    MD_LOG("persistent decode kernel reported error %d (timed-out wait); state reset\n", code);
    const MatmulDecoderConfig* c = &ctx->model.cfg;
    if (kind == 2) {
        b2_memset(ctx->mk2.scratch, 0, ctx->mk2_scratch_bytes, ctx->stream);
    } else {
        const size_t bytes = b2_mk_scratch_bytes(c->num_layers, c->hidden_dim, c->ffn_dim, c->num_q_heads,
                                                 c->num_kv_heads, c->head_dim);
        b2_memset(ctx->mk_scratch, 0, bytes, ctx->stream);
    }
    b2_memset(mk_dstate(ctx, kind), 0, B2_MK_STATE_INTS * 4, ctx->stream);
    b2_stream_sync(ctx->stream);
    return MATMUL_DECODER_ERR_RKNN;
}

static int mk_step(MatmulDecoderContext* ctx, int kind, int token_id, const float* embedding, int with_head,
                   float* logits_out) {
    const double t0 = now_ms();
    const int H = ctx->model.cfg.hidden_dim;
    int* st = mk_hstate(ctx, kind);
    int* dst = mk_dstate(ctx, kind);
    st[B2_MK_TOKEN] = embedding ? 0 : token_id;
    st[B2_MK_POS] = ctx->seq_len;
    st[B2_MK_STEP] = 0;
    st[B2_MK_USE_EMB] = embedding ? 1 : 0;
    b2_stream_t s = ctx->stream;
    int rc = b2_memcpy_h2d(dst, st, 4 * 4, s);
    if (!rc && embedding) {
        memcpy(ctx->h_blk + PARAMS_INTS, embedding, (size_t)H * 4);
        rc = b2_memcpy_h2d(ctx->d_blk + PARAMS_INTS, ctx->h_blk + PARAMS_INTS, (size_t)H * 4, s);
    }
    mk_plan(ctx, kind)->do_lm = with_head;
    if (ctx->test_hooks) {
        const char* stall = getenv("B2_MK_STALL_TEST");
        ctx->mk2.stall_test = stall && atoi(stall) > 0;
    }
    if (!rc) rc = b2_event_record(ctx->ev[0], s);
    if (!rc) rc = mk_launch(ctx, kind);
    if (!rc) rc = b2_event_record(ctx->ev[2], s);
    if (!rc) rc = b2_memcpy_d2h(st + B2_MK_ERR, dst + B2_MK_ERR, 2 * 4, s);
    if (!rc) rc = b2_stream_sync(s);
    if (rc) return fail("persistent decode step", rc);
    if (st[B2_MK_ERR]) return mk_recover(ctx, kind, st[B2_MK_ERR]);
    double t_copy = 0;
    if (with_head && logits_out) {
        const double tc = now_ms();
        if ((rc = b2_memcpy_d2h(logits_out, ctx->logits, (size_t)ctx->model.cfg.vocab_size * 4, s)) ||
            (rc = b2_stream_sync(s)))
            return fail("logits copy", rc);
        t_copy = now_ms() - tc;
    }
    ctx->seq_len++;
    ctx->hidden_mk = kind;
    float ms = 0.f;
    b2_event_elapsed_ms(&ms, ctx->ev[0], ctx->ev[2]);
    ctx->stats.total_ms = (float)(now_ms() - t0);
    ctx->stats.matmul_ms = ms;
    ctx->stats.rebind_ms = 0.f;
    ctx->stats.convert_ms = (float)t_copy;
    ctx->stats.cpu_ops_ms = 0.f;
    ctx->stats.lm_head_ms = 0.f;
    ctx->stats.n_steps++;
    return with_head ? st[B2_MK_TOKEN_OUT] : 0;
}

/* with_head: run final norm + lm_head + argmax; logits_out: optional host copy. */
static int step_impl(MatmulDecoderContext* ctx, int token_id, const float* embedding, int with_head,
                     float* logits_out) {
    int rc = check_step_args(ctx, token_id, embedding, ctx ? ctx->model.cfg.vocab_size : 0);
    if (rc) return rc;
    b2_set_device(ctx->device);
    const int kind = mk_kind(ctx, ctx->seq_len, 1);
    if (kind) return mk_step(ctx, kind, token_id, embedding, with_head, logits_out);
    const double t0 = now_ms();
    b2_graph_t* g = with_head ? &ctx->g_head : &ctx->g_nohead;
    if (!*g && (rc = build_graph(ctx, with_head, g))) return fail("graph capture", rc);
    stage_params(ctx, token_id, embedding);
    if ((rc = b2_graph_launch(*g, ctx->stream)) || (rc = b2_stream_sync(ctx->stream)))
        return fail("decode step", rc);
    double t_copy = 0;
    if (with_head && logits_out) {
        const double tc = now_ms();
        if ((rc = b2_memcpy_d2h(logits_out, ctx->logits, (size_t)ctx->model.cfg.vocab_size * 4, ctx->stream)) ||
            (rc = b2_stream_sync(ctx->stream)))
            return fail("logits copy", rc);
        t_copy = now_ms() - tc;
    }
    ctx->seq_len++;
    ctx->hidden_row = 0;
    ctx->hidden_mk = 0;
    record_stats(ctx, t0, t_copy, with_head);
    return with_head ? ctx->h_tok[0] : 0;
}

int matmul_decoder_step(MatmulDecoderContext* ctx, int token_id, const float* embedding,
                        float* output_logits) {
    /* NULL logits = prefill mode (src/matmul_decoder.c:1551-1561). */
    return step_impl(ctx, token_id, embedding, output_logits != NULL, output_logits);
}

int matmul_decoder_step_get_logits(MatmulDecoderContext* ctx, int token_id, const float* embedding,
                                   float* logits_out) {
    if (!logits_out) return MATMUL_DECODER_ERR_INVALID_ARG;
    return step_impl(ctx, token_id, embedding, 1, logits_out);
}

int matmul_decoder_step_token(MatmulDecoderContext* ctx, int token_id, const float* embedding) {
    return step_impl(ctx, token_id, embedding, 1, NULL);
}

int matmul_decoder_set_seed(MatmulDecoderContext* ctx, unsigned long long seed) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    ctx->sample_seed = seed;
    ctx->sample_counter = 0;
    return MATMUL_DECODER_OK;
}

/* One step whose logits stay on the device, then b2_sample_token on the same
 * stream: only the token crosses to the host. */
int matmul_decoder_step_sample(MatmulDecoderContext* ctx, int token_id, const float* embedding,
                               const SamplingParams* params) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    const SamplingParams p = params ? *params : sampling_params_greedy();
    const int penalize = p.repeat_penalty != 1.0f && p.repeat_tokens && p.n_repeat_tokens > 0;
    if (p.n_repeat_tokens < 0 || (penalize && !(p.repeat_penalty > 0.f))) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (p.top_k == 1 && !penalize) return step_impl(ctx, token_id, embedding, 1, NULL);
    const int n_rep = penalize ? p.n_repeat_tokens : 0;
    b2_set_device(ctx->device);
    int rc = 0;
    if (!ctx->d_sample || ctx->d_sample_cap < n_rep) {
        if (ctx->d_sample) b2_free(ctx->d_sample);
        ctx->d_sample = NULL;
        const int cap = 2 * n_rep > 256 ? 2 * n_rep : 256;  /* room to grow with a generation's history */
        if ((rc = b2_malloc((void**)&ctx->d_sample, (size_t)(8 + cap) * 4))) return fail("sampler buffer", rc);
        ctx->d_sample_cap = cap;
    }
    const int r = step_impl(ctx, token_id, embedding, 1, NULL);
    if (r < 0) return r;
    b2_stream_t s = ctx->stream;
    if (n_rep && (rc = b2_memcpy_h2d(ctx->d_sample + 8, p.repeat_tokens, (size_t)n_rep * 4, s)))
        return fail("repeat list copy", rc);
    rc = b2_sample_token(ctx->logits, ctx->model.cfg.vocab_size, ctx->d_sample + 8, n_rep,
                         penalize ? p.repeat_penalty : 1.0f, p.top_k, p.top_p, p.temperature, ctx->sample_seed,
                         ctx->sample_counter, ctx->d_sample, ctx->d_sample + 1, s);
    if (!rc) rc = b2_memcpy_d2h(ctx->h_tok, ctx->d_sample, 4, s);
    if (!rc) rc = b2_stream_sync(s);
    if (rc) return fail("on-device sampling", rc);
    ctx->sample_counter++;
    return ctx->h_tok[0];
}

int matmul_decoder_step_head(MatmulDecoderContext* ctx, int token_id, const float* embedding,
                             int lm_head_idx, float* output_logits) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    DevModel* m = &ctx->model;
    if (m->n_lm_heads <= 1) return matmul_decoder_step(ctx, token_id, embedding, output_logits);
    if (lm_head_idx < 0 || lm_head_idx >= m->n_lm_heads) return MATMUL_DECODER_ERR_INVALID_ARG;
    int rc = check_step_args(ctx, token_id, embedding, m->cfg.vocab_size);
    if (rc) return rc;
    const double t0 = now_ms();
    b2_set_device(ctx->device);
    stage_params(ctx, token_id, embedding);
    /* Multi-head steps run uncaptured: the table differs per call. */
    rc = enqueue_token(ctx, 1, m->lm_heads[lm_head_idx], NULL, B2_W_F32, m->lm_vocab, 1);
    if (!rc) rc = b2_stream_sync(ctx->stream);
    if (rc) return fail("step_head", rc);
    double t_copy = 0;
    if (output_logits) {
        const double tc = now_ms();
        if ((rc = b2_memcpy_d2h(output_logits, ctx->logits, (size_t)m->lm_vocab * 4, ctx->stream)) ||
            (rc = b2_stream_sync(ctx->stream)))
            return fail("logits copy", rc);
        t_copy = now_ms() - tc;
    }
    ctx->seq_len++;
    ctx->hidden_row = 0;
    ctx->hidden_mk = 0;
    record_stats(ctx, t0, t_copy, 1);
    return ctx->h_tok[0];
}

/* ─── device-resident greedy loop ─── */

static int build_loop_graph(MatmulDecoderContext* ctx) {
    DevModel* m = &ctx->model;
    const int H = m->cfg.hidden_dim;
    b2_stream_t s = ctx->stream;
    int rc = b2_graph_begin(s);
    if (rc) return rc;
    int rc2 = b2_embed(ctx->hidden, m->emb, ctx->d_loop, NULL, NULL, 1, H, s);
    B2KVRef kv = kv_ref(ctx, ctx->d_loop + 1);
    LayerBuffers lb = {ctx->hidden, ctx->qkv, ctx->attn, ctx->act, ctx->attn_work, ctx->split_decode, NULL, NULL, -1, 0, NULL};
    if (!rc2) rc2 = md_enqueue_layers(m, &lb, 1, &kv, s);
    if (!rc2)
        rc2 = b2_lm_head_argmax(ctx->hidden, H, 1, H, m->cfg.vocab_size, m->lm, m->lm_scales, m->lm_wtype,
                                m->final_norm, m->cfg.rms_eps, ctx->logits, m->cfg.vocab_size, ctx->d_loop,
                                ctx->lm_work, s);
    if (!rc2) rc2 = b2_loop_advance(ctx->d_loop, ctx->d_hist, ctx->max_seq, s);
    b2_graph_t g = NULL;
    rc = b2_graph_end(s, &g);
    if (rc2 || rc) {
        b2_graph_destroy(g);
        return rc2 ? rc2 : rc;
    }
    ctx->g_loop = g;
    return 0;
}

int matmul_decoder_decode_greedy(MatmulDecoderContext* ctx, int first_token, int n_tokens, int* tokens_out,
                                 float* device_ms) {
    if (!ctx || !tokens_out || n_tokens <= 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (ctx->model.n_lm_heads > 1) return MATMUL_DECODER_ERR_UNSUPPORTED;
    if (first_token < 0 || first_token >= ctx->model.cfg.vocab_size) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (ctx->seq_len + n_tokens > ctx->max_seq) {
        MD_LOG("decode_greedy: seq_len=%d + %d > max=%d\n", ctx->seq_len, n_tokens, ctx->max_seq);
        return MATMUL_DECODER_ERR_INVALID_ARG;
    }
    const double t0 = now_ms();
    b2_set_device(ctx->device);
    int rc = 0;
    const int kind = mk_kind(ctx, ctx->seq_len, n_tokens);
    if (kind) {
        int* st = mk_hstate(ctx, kind);
        int* dst = mk_dstate(ctx, kind);
        st[B2_MK_TOKEN] = first_token;
        st[B2_MK_POS] = ctx->seq_len;
        st[B2_MK_STEP] = 0;
        st[B2_MK_USE_EMB] = 0;
        mk_plan(ctx, kind)->do_lm = 1;
        if (ctx->test_hooks) {
            const char* stall = getenv("B2_MK_STALL_TEST");
            ctx->mk2.stall_test = stall && atoi(stall) > 0;
        }
        rc = b2_memcpy_h2d(dst, st, 4 * 4, ctx->stream);
        if (!rc) rc = b2_event_record(ctx->ev[0], ctx->stream);
        for (int i = 0; i < n_tokens && !rc; i++) rc = mk_launch(ctx, kind);
        if (!rc) rc = b2_event_record(ctx->ev[2], ctx->stream);
        if (!rc) rc = b2_memcpy_d2h(tokens_out, ctx->d_hist, (size_t)n_tokens * 4, ctx->stream);
        if (!rc) rc = b2_memcpy_d2h(st + B2_MK_ERR, dst + B2_MK_ERR, 4, ctx->stream);
        if (!rc) rc = b2_stream_sync(ctx->stream);
        if (rc) return fail("decode_greedy", rc);
        if (st[B2_MK_ERR]) return mk_recover(ctx, kind, st[B2_MK_ERR]);
        float ms = 0.f;
        b2_event_elapsed_ms(&ms, ctx->ev[0], ctx->ev[2]);
        if (device_ms) *device_ms = ms;
        ctx->seq_len += n_tokens;
        ctx->hidden_mk = kind;
        ctx->stats.total_ms = (float)(now_ms() - t0);
        ctx->stats.matmul_ms = ms;
        ctx->stats.lm_head_ms = 0.f;
        ctx->stats.n_steps += n_tokens;
        return n_tokens;
    }
    if (!ctx->g_loop && (rc = build_loop_graph(ctx))) return fail("loop graph capture", rc);
    ctx->h_loop[0] = first_token;
    ctx->h_loop[1] = ctx->seq_len;
    ctx->h_loop[2] = 0;
    ctx->h_loop[3] = 0;
    rc = b2_memcpy_h2d(ctx->d_loop, ctx->h_loop, 16, ctx->stream);
    if (!rc) rc = b2_event_record(ctx->ev[0], ctx->stream);
    for (int i = 0; i < n_tokens && !rc; i++) rc = b2_graph_launch(ctx->g_loop, ctx->stream);
    if (!rc) rc = b2_event_record(ctx->ev[2], ctx->stream);
    if (!rc) rc = b2_memcpy_d2h(tokens_out, ctx->d_hist, (size_t)n_tokens * 4, ctx->stream);
    if (!rc) rc = b2_stream_sync(ctx->stream);
    if (rc) return fail("decode_greedy", rc);
    float ms = 0.f;
    b2_event_elapsed_ms(&ms, ctx->ev[0], ctx->ev[2]);
    if (device_ms) *device_ms = ms;
    ctx->seq_len += n_tokens;
    ctx->hidden_row = 0;
    ctx->hidden_mk = 0;
    ctx->stats.total_ms = (float)(now_ms() - t0);
    ctx->stats.matmul_ms = ms;
    ctx->stats.lm_head_ms = 0.f;
    ctx->stats.n_steps += n_tokens;
    return n_tokens;
}

/* ─── batch prefill ─── */

int matmul_decoder_prefill_batch(MatmulDecoderContext* ctx, const float* embeddings, int M) {
    if (!ctx || !embeddings || M <= 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (ctx->seq_len + M > ctx->max_seq) {
        fprintf(stderr, "[BatchPrefill] KV cache overflow: seq_len=%d + M=%d > max=%d\n", ctx->seq_len, M,
                ctx->max_seq);
        return MATMUL_DECODER_ERR_INVALID_ARG;
    }
    b2_set_device(ctx->device);
    DevModel* m = &ctx->model;
    const int H = m->cfg.hidden_dim;
    const double t0 = now_ms();
    float dev_ms = 0.f;
    for (int off = 0; off < M; off += ctx->rows_cap) {
        const int rows = M - off < ctx->rows_cap ? M - off : ctx->rows_cap;
        for (int i = 0; i < rows; i++) ctx->h_pos[i] = ctx->seq_len + i;
        int rc = b2_memcpy_h2d(ctx->hidden, embeddings + (size_t)off * H, (size_t)rows * H * 4, ctx->stream);
        if (!rc) rc = b2_memcpy_h2d(ctx->d_pos, ctx->h_pos, (size_t)rows * 4, ctx->stream);
        B2KVRef kv = kv_ref(ctx, ctx->d_pos);
        int split = (296 + rows * m->cfg.num_kv_heads - 1) / (rows * m->cfg.num_kv_heads);
        if (split < 1) split = 1;
        if (split > ctx->split_decode) split = ctx->split_decode;
        LayerBuffers lb = {ctx->hidden, ctx->qkv, ctx->attn, ctx->act, ctx->attn_work, split, ctx->x16,
                           ctx->x16b, ctx->seq_len, 0, NULL};
        if (!rc) rc = b2_event_record(ctx->ev[0], ctx->stream);
        if (!rc) rc = md_enqueue_layers(m, &lb, rows, &kv, ctx->stream);
        if (!rc) rc = b2_event_record(ctx->ev[1], ctx->stream);
        if (!rc) rc = b2_stream_sync(ctx->stream);
        float ms = 0.f;
        if (!rc) rc = b2_event_elapsed_ms(&ms, ctx->ev[0], ctx->ev[1]);
        if (rc) return fail("prefill_batch", rc);
        dev_ms += ms;
        ctx->seq_len += rows;
        ctx->hidden_row = rows - 1;
        ctx->hidden_mk = 0;
    }
    /* stats of the call: wall time, and the device time of the layer stack */
    ctx->stats.total_ms = (float)(now_ms() - t0);
    ctx->stats.matmul_ms = dev_ms;
    ctx->stats.lm_head_ms = 0.f;
    return MATMUL_DECODER_OK;
}

/* ─── state queries ─── */

int matmul_decoder_uses_persistent_kernel(const MatmulDecoderContext* ctx) {
    return ctx && (ctx->use_mk || ctx->use_mk2) ? 1 : 0;
}

int matmul_decoder_step_kernel(const MatmulDecoderContext* ctx, int n_cached) {
    if (!ctx || n_cached < 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    return mk_kind(ctx, n_cached, 1);
}

void matmul_decoder_clear_kv_cache(MatmulDecoderContext* ctx) {
    if (ctx) ctx->seq_len = 0;
}

int matmul_decoder_get_seq_len(const MatmulDecoderContext* ctx) { return ctx ? ctx->seq_len : 0; }

const MatmulDecoderConfig* matmul_decoder_get_config(const MatmulDecoderContext* ctx) {
    return ctx ? &ctx->config : NULL;
}

void matmul_decoder_get_stats(const MatmulDecoderContext* ctx, MatmulDecoderStats* stats) {
    if (ctx && stats) *stats = ctx->stats;
}

int matmul_decoder_set_seq_len(MatmulDecoderContext* ctx, int n) {
    if (!ctx || n < 0 || n > ctx->max_seq) return MATMUL_DECODER_ERR_INVALID_ARG;
    ctx->seq_len = n;
    return MATMUL_DECODER_OK;
}

int matmul_decoder_get_hidden(MatmulDecoderContext* ctx, float* hidden_out) {
    if (!ctx || !hidden_out) return MATMUL_DECODER_ERR_INVALID_ARG;
    b2_set_device(ctx->device);
    const size_t H = (size_t)ctx->model.cfg.hidden_dim;
    const float* src = ctx->hidden_mk == 2   ? b2_mk2_final_hidden(&ctx->mk2)
                       : ctx->hidden_mk == 1 ? b2_mk_final_hidden(&ctx->mk)
                                             : ctx->hidden + (size_t)ctx->hidden_row * H;
    int rc = b2_memcpy_d2h(hidden_out, src, H * 4, ctx->stream);
    if (!rc) rc = b2_stream_sync(ctx->stream);
    return rc ? fail("get_hidden", rc) : MATMUL_DECODER_OK;
}

int matmul_decoder_build_embed(MatmulDecoderContext* ctx, const int* prefix_ids, int n_pre,
                               const float* audio_embd, int n_audio, const int* suffix_ids, int n_suf,
                               float* embed_out) {
    if (!ctx || !embed_out || n_pre < 0 || n_audio < 0 || n_suf < 0 || (n_pre && !prefix_ids) ||
        (n_audio && !audio_embd) || (n_suf && !suffix_ids))
        return MATMUL_DECODER_ERR_INVALID_ARG;
    const int V = ctx->model.cfg.vocab_size, H = ctx->model.cfg.hidden_dim;
    for (int i = 0; i < n_pre; i++)
        if (prefix_ids[i] < 0 || prefix_ids[i] >= V) return MATMUL_DECODER_ERR_INVALID_ARG;
    for (int i = 0; i < n_suf; i++)
        if (suffix_ids[i] < 0 || suffix_ids[i] >= V) return MATMUL_DECODER_ERR_INVALID_ARG;
    const int total = n_pre + n_audio + n_suf;
    if (total == 0) return 0;
    b2_set_device(ctx->device);
    const size_t ids_bytes = (((size_t)n_pre + n_suf) * 4 + 255) & ~(size_t)255;
    const size_t a_bytes = ((size_t)n_audio * H * 4 + 255) & ~(size_t)255;
    unsigned char* buf = NULL;
    int rc = b2_malloc((void**)&buf, ids_bytes + a_bytes + (size_t)total * H * 4);
    if (rc) return MATMUL_DECODER_ERR_MEMORY;
    int* d_ids = (int*)buf;
    float* d_audio = (float*)(buf + ids_bytes);
    float* d_out = (float*)(buf + ids_bytes + a_bytes);
    b2_stream_t s = ctx->stream;
    if (!rc && n_pre) rc = b2_memcpy_h2d(d_ids, prefix_ids, (size_t)n_pre * 4, s);
    if (!rc && n_suf) rc = b2_memcpy_h2d(d_ids + n_pre, suffix_ids, (size_t)n_suf * 4, s);
    if (!rc && n_audio) rc = b2_memcpy_h2d(d_audio, audio_embd, (size_t)n_audio * H * 4, s);
    if (!rc)
        rc = b2_build_embed(ctx->model.emb, V, H, d_ids, n_pre, d_audio, n_audio, d_ids + n_pre, n_suf, d_out, s);
    if (!rc) rc = b2_memcpy_d2h(embed_out, d_out, (size_t)total * H * 4, s);
    if (!rc) rc = b2_stream_sync(s);
    b2_free(buf);
    return rc ? fail("build_embed", rc) : total;
}

/* Host [len][nkv][hd] <-> device [nkv][max_seq][hd] for one layer. */
static int kv_transfer(MatmulDecoderContext* ctx, int layer, int start, int len, uint16_t* kh, uint16_t* vh,
                       int to_device) {
    const MatmulDecoderConfig* c = &ctx->model.cfg;
    if (layer < 0 || layer >= c->num_layers || start < 0 || len <= 0 || start + len > ctx->max_seq || !kh ||
        !vh)
        return MATMUL_DECODER_ERR_INVALID_ARG;
    b2_set_device(ctx->device);
    const int nkv = c->num_kv_heads, hd = c->head_dim;
    uint16_t* tmp = (uint16_t*)malloc((size_t)len * nkv * hd * 2);
    if (!tmp) return MATMUL_DECODER_ERR_MEMORY;
    int rc = 0;
    for (int which = 0; which < 2 && !rc; which++) {
        uint16_t* host = which ? vh : kh;
        uint16_t* dev = (which ? ctx->v_cache : ctx->k_cache) + (size_t)layer * ctx->layer_stride;
        if (to_device)
            for (int g = 0; g < nkv; g++)
                for (int p = 0; p < len; p++)
                    memcpy(tmp + ((size_t)g * len + p) * hd, host + ((size_t)p * nkv + g) * hd, (size_t)hd * 2);
        for (int g = 0; g < nkv && !rc; g++) {
            uint16_t* d = dev + ((size_t)g * ctx->max_seq + start) * hd;
            rc = to_device ? b2_memcpy_h2d(d, tmp + (size_t)g * len * hd, (size_t)len * hd * 2, ctx->stream)
                           : b2_memcpy_d2h(tmp + (size_t)g * len * hd, d, (size_t)len * hd * 2, ctx->stream);
        }
        if (!rc) rc = b2_stream_sync(ctx->stream);
        if (!rc && !to_device)
            for (int g = 0; g < nkv; g++)
                for (int p = 0; p < len; p++)
                    memcpy(host + ((size_t)p * nkv + g) * hd, tmp + ((size_t)g * len + p) * hd, (size_t)hd * 2);
    }
    free(tmp);
    return rc ? fail("kv transfer", rc) : MATMUL_DECODER_OK;
}

int matmul_decoder_set_kv(MatmulDecoderContext* ctx, int layer, int start, int len, const uint16_t* k_fp16,
                          const uint16_t* v_fp16) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    return kv_transfer(ctx, layer, start, len, (uint16_t*)k_fp16, (uint16_t*)v_fp16, 1);
}

int matmul_decoder_get_kv(MatmulDecoderContext* ctx, int layer, int start, int len, uint16_t* k_fp16,
                          uint16_t* v_fp16) {
    if (!ctx) return MATMUL_DECODER_ERR_INVALID_ARG;
    return kv_transfer(ctx, layer, start, len, k_fp16, v_fp16, 0);
}
