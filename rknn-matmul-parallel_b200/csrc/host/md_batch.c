/*
 * Batched multi-sequence decode (ADDITIVE entry points of matmul_decoder.h).
 *
 * The reference decodes one sequence per context (matmul_decoder_step,
 * src/matmul_decoder.c:1430-1634).  Here n_seqs independent sequences share
 * one device copy of the weights; each has its own FP16 KV cache
 * [layer][kv_head][pos][hd] and position.  One step is one CUDA graph replay
 * over all sequences as the rows of a skinny GEMM: the weights stream once
 * per step for every sequence, attention reads each row's own cache up to its
 * own position, and the lm_head + argmax produce one token per sequence.
 * Token ids and positions travel in a small pinned block per step.
 */
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "md_internal.h"

struct MatmulDecoderBatch {
    DevModel model;
    int device, n, max_seq, split;
    int attn_block; /* > 0: attention in blocks of this many positions (b2_attention_blocks) */
    int ws_split;   /* position ranges the attention workspace is sized for */
    b2_stream_t stream;
    uint16_t *k_cache, *v_cache;
    long long seq_stride, layer_stride;
    float *hidden, *qkv, *attn, *act, *logits;
    uint16_t* x16;                /* [n][max(H, qd, ffn)] FP16 rows for the tensor-core GEMMs */
    uint16_t* x16b;               /* [n][ffn] FP16 gate|up output for the down-projection GEMM */
    unsigned long long* lm_keys;  /* per-CTA argmax keys of the tensor-core lm_head */
    int *d_blk;   /* [0,n) tokens, [n,2n) positions, [2n,3n) row->sequence */
    int *d_tok;   /* [0,n) next tokens, [n] attention error flag */
    void *attn_work, *lm_work;
    int *h_blk, *h_tok;
    int* seq_len;
    b2_graph_t graph;
    b2_event_t ev[3];
    MatmulDecoderStats stats;
    /* vocab-sharded lm_head (matmul_decoder_batch_shard_vocab) */
    int world, rank, rows;          /* ranks, this rank, rows each rank contributes (>= n) */
    int v0, v1;                     /* this rank's vocabulary slice */
    ncclComm_t comm;
    void* shard_buf;                /* one allocation for the buffers below */
    uint16_t* g_x16;                /* [world * rows][H] final-normed FP16 rows of every rank */
    unsigned long long* g_keys;     /* lm_head GEMM keys [world * rows][parts] */
    unsigned long long* m_keys;     /* merged keys [world * rows] (global indices) */
    int* g_tok;                     /* tokens of the local GEMM (unused) */
};

/* ─── NCCL, loaded at run time ───
 * libnccl.so.2 is opened when the first sharded decoder is set up; in a
 * process that already uses NCCL (torch.distributed) this is that library. */
static struct {
    void* h;
    ncclResult_t (*get_id)(ncclUniqueId*);
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*destroy)(ncclComm_t);
    ncclResult_t (*abort_)(ncclComm_t);
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*);
    const char* (*error_string)(ncclResult_t);
} g_nccl;

static int nccl_load(void) {
    if (g_nccl.h) return 0;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        MD_LOG("NCCL not found: %s\n", dlerror());
        return MATMUL_DECODER_ERR_UNSUPPORTED;
    }
#define NCCL_SYM(field, name)                                    \
    *(void**)&g_nccl.field = dlsym(h, name);                     \
    if (!g_nccl.field) {                                         \
        MD_LOG("NCCL symbol %s missing\n", name);                \
        return MATMUL_DECODER_ERR_UNSUPPORTED;                   \
    }
    NCCL_SYM(get_id, "ncclGetUniqueId");
    NCCL_SYM(init_rank, "ncclCommInitRank");
    NCCL_SYM(all_gather, "ncclAllGather");
    NCCL_SYM(all_reduce, "ncclAllReduce");
    NCCL_SYM(destroy, "ncclCommDestroy");
    NCCL_SYM(abort_, "ncclCommAbort");
    NCCL_SYM(async_error, "ncclCommGetAsyncError");
    NCCL_SYM(error_string, "ncclGetErrorString");
#undef NCCL_SYM
    g_nccl.h = h;
    return 0;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

static size_t batch_bytes(const MatmulDecoderConfig* c, int n, int max_seq, int split) {
    const size_t H = c->hidden_dim, hd = c->head_dim, qd = (size_t)c->num_q_heads * hd;
    const size_t kvd = (size_t)c->num_kv_heads * hd, F = c->ffn_dim;
    size_t t = 2 * (size_t)n * c->num_layers * kvd * (size_t)max_seq * 2;
    t += (size_t)n * (H + qd + 2 * kvd + qd + F) * 4 + (size_t)n * c->vocab_size * 4 + 16 * 256;
    t += (size_t)n * 3 * 4 + 1024;
    t += b2_attention_workspace(n, c->num_q_heads, (int)hd, split) + b2_lm_head_workspace(n, c->vocab_size);
    const size_t kmax = H > qd ? (H > F ? H : F) : (qd > F ? qd : F);
    t += (size_t)n * kmax * 2 + (size_t)n * F * 2 + b2_gemm_argmax_keys(n, c->vocab_size) + 768;
    return t + 4096;
}

void matmul_decoder_batch_destroy(MatmulDecoderBatch* b) {
    if (!b) return;
    b2_set_device(b->device);
    if (b->stream) b2_stream_sync(b->stream);
    b2_graph_destroy(b->graph);
    for (int i = 0; i < 3; i++) b2_event_destroy(b->ev[i]);
    b2_stream_destroy(b->stream);
    b2_host_free(b->h_blk);
    b2_host_free(b->h_tok);
    if (b->comm) g_nccl.destroy(b->comm);
    if (b->shard_buf) b2_free(b->shard_buf);
    free(b->seq_len);
    md_model_free(&b->model);
    free(b);
}

MatmulDecoderBatch* matmul_decoder_batch_create(const char* model_dir, const MatmulDecoderConfig* config,
                                                QuantizationType quant_type, int max_seq_len, int n_seqs) {
    if (!model_dir || n_seqs <= 0 || n_seqs > 4096) return NULL;
    MatmulDecoderConfig cfg;
    if (config) {
        cfg = *config;
    } else {
        char path[1024];
        snprintf(path, sizeof(path), "%s/config.json", model_dir);
        if (matmul_decoder_load_config(path, &cfg) != 0) return NULL;
    }
    if (cfg.num_lm_heads > 1) {
        MD_LOG("batched decode supports single-head models\n");
        return NULL;
    }
    if (max_seq_len <= 0) max_seq_len = cfg.max_seq_len > 0 ? cfg.max_seq_len : 4096;
    MatmulDecoderBatch* b = (MatmulDecoderBatch*)calloc(1, sizeof(*b));
    if (!b) return NULL;
    b->n = n_seqs;
    b->max_seq = max_seq_len;
    int sm = 148;
    b2_sm_count(&sm);
    /* attention position ranges per (sequence, kv head): about eight CTAs per
     * SM, so the long sequences do not leave a tail of idle SMs
     * (B2_BATCH_SPLIT overrides) */
    b->split = (8 * sm + n_seqs * cfg.num_kv_heads - 1) / (n_seqs * cfg.num_kv_heads);
    const char* es = getenv("B2_BATCH_SPLIT");
    if (es && atoi(es) > 0) b->split = atoi(es);
    if (b->split < 1) b->split = 1;
    if (b->split > 64) b->split = 64;
    /* Attention in fixed blocks of positions streamed by bulk copies: the
     * work per CTA does not depend on the sequence lengths (B2_BATCH_BLOCK,
     * a multiple of 64; 0 keeps the per-sequence ranges above). */
    b->attn_block = 512;
    const char* eb = getenv("B2_BATCH_BLOCK");
    if (eb) b->attn_block = atoi(eb);
    if (b->attn_block < 0 || b->attn_block % 64) b->attn_block = 512;
    if (n_seqs > 512) b->attn_block = 0; /* b2_attention_blocks takes up to 512 rows */
    b->ws_split = b->split;
    if (b->attn_block > 0) {
        const int bs = b2_attention_blocks_split(max_seq_len, b->attn_block);
        if (bs > b->ws_split) b->ws_split = bs;
    }
    b2_get_device(&b->device);
    b->seq_len = (int*)calloc((size_t)n_seqs, sizeof(int));
    int rc = b->seq_len ? 0 : MATMUL_DECODER_ERR_MEMORY;
    if (!rc)
        rc = md_model_load_dir(&b->model, model_dir, &cfg, quant_type, max_seq_len,
                               batch_bytes(&cfg, n_seqs, max_seq_len, b->ws_split));
    if (rc) {
        MD_LOG("batch_create failed (%d)\n", rc);
        matmul_decoder_batch_destroy(b);
        return NULL;
    }
    DevModel* m = &b->model;
    const MatmulDecoderConfig* c = &m->cfg;
    const size_t H = c->hidden_dim, hd = c->head_dim, qd = (size_t)c->num_q_heads * hd;
    const size_t kvd = (size_t)c->num_kv_heads * hd, F = c->ffn_dim, n = (size_t)n_seqs;
    b->layer_stride = (long long)kvd * max_seq_len;
    b->seq_stride = b->layer_stride * c->num_layers;
    const size_t kv_bytes = n * c->num_layers * kvd * (size_t)max_seq_len * 2;
    b->k_cache = (uint16_t*)md_arena_alloc(&m->arena, kv_bytes);
    b->v_cache = (uint16_t*)md_arena_alloc(&m->arena, kv_bytes);
    b->hidden = (float*)md_arena_alloc(&m->arena, n * H * 4);
    b->qkv = (float*)md_arena_alloc(&m->arena, n * (qd + 2 * kvd) * 4);
    b->attn = (float*)md_arena_alloc(&m->arena, n * qd * 4);
    b->act = (float*)md_arena_alloc(&m->arena, n * F * 4);
    b->logits = (float*)md_arena_alloc(&m->arena, n * c->vocab_size * 4);
    b->d_blk = (int*)md_arena_alloc(&m->arena, n * 3 * 4);
    b->d_tok = (int*)md_arena_alloc(&m->arena, (n + 1) * 4);
    b->attn_work = md_arena_alloc(&m->arena, b2_attention_workspace(n_seqs, c->num_q_heads, (int)hd, b->ws_split));
    b->lm_work = md_arena_alloc(&m->arena, b2_lm_head_workspace(n_seqs, c->vocab_size));
    {
        const size_t kmax = H > qd ? (H > F ? H : F) : (qd > F ? qd : F);
        b->x16 = (uint16_t*)md_arena_alloc(&m->arena, n * kmax * 2);
        b->x16b = (uint16_t*)md_arena_alloc(&m->arena, n * F * 2);
        b->lm_keys = (unsigned long long*)md_arena_alloc(&m->arena, b2_gemm_argmax_keys(n_seqs, c->vocab_size));
    }
    if (!b->k_cache || !b->v_cache || !b->hidden || !b->qkv || !b->attn || !b->act || !b->logits || !b->d_blk ||
        !b->d_tok || !b->attn_work || !b->lm_work || !b->x16 || !b->x16b || !b->lm_keys)
        rc = MATMUL_DECODER_ERR_MEMORY;
    if (!rc) rc = b2_memset(b->k_cache, 0, kv_bytes, NULL);
    if (!rc) rc = b2_memset(b->v_cache, 0, kv_bytes, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    if (!rc) rc = b2_stream_create(&b->stream);
    for (int i = 0; i < 3 && !rc; i++) rc = b2_event_create(&b->ev[i]);
    if (!rc) rc = b2_host_alloc((void**)&b->h_blk, n * 3 * 4);
    if (!rc) rc = b2_host_alloc((void**)&b->h_tok, (n + 1) * 4);
    if (!rc) rc = b2_memset(b->d_tok, 0, (n + 1) * 4, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    if (rc) {
        MD_LOG("batch_create allocation failed (%d): %s\n", rc, b2_last_error());
        matmul_decoder_batch_destroy(b);
        return NULL;
    }
    for (int i = 0; i < n_seqs; i++) b->h_blk[2 * n_seqs + i] = i;
    printf("[MatmulDecoder] Batch ready: %d sequences, max_seq=%d, arena %.1f GB\n", n_seqs, max_seq_len,
           m->arena.size / 1e9);
    return b;
}

int matmul_decoder_batch_set_kv(MatmulDecoderBatch* b, int seq, int layer, int start, int len,
                                const uint16_t* k_fp16, const uint16_t* v_fp16) {
    if (!b || seq < 0 || seq >= b->n) return MATMUL_DECODER_ERR_INVALID_ARG;
    const MatmulDecoderConfig* c = &b->model.cfg;
    if (layer < 0 || layer >= c->num_layers || start < 0 || len <= 0 || start + len > b->max_seq || !k_fp16 ||
        !v_fp16)
        return MATMUL_DECODER_ERR_INVALID_ARG;
    b2_set_device(b->device);
    const int nkv = c->num_kv_heads, hd = c->head_dim;
    uint16_t* tmp = (uint16_t*)malloc((size_t)len * nkv * hd * 2);
    if (!tmp) return MATMUL_DECODER_ERR_MEMORY;
    int rc = 0;
    for (int which = 0; which < 2 && !rc; which++) {
        const uint16_t* host = which ? v_fp16 : k_fp16;
        uint16_t* dev = (which ? b->v_cache : b->k_cache) + seq * b->seq_stride + layer * b->layer_stride;
        for (int g = 0; g < nkv; g++)
            for (int p = 0; p < len; p++)
                memcpy(tmp + ((size_t)g * len + p) * hd, host + ((size_t)p * nkv + g) * hd, (size_t)hd * 2);
        for (int g = 0; g < nkv && !rc; g++)
            rc = b2_memcpy_h2d(dev + ((size_t)g * b->max_seq + start) * hd, tmp + (size_t)g * len * hd,
                               (size_t)len * hd * 2, b->stream);
        if (!rc) rc = b2_stream_sync(b->stream);
    }
    free(tmp);
    return rc;
}

int matmul_decoder_batch_set_seq_len(MatmulDecoderBatch* b, int seq, int n) {
    if (!b || seq < 0 || seq >= b->n || n < 0 || n > b->max_seq) return MATMUL_DECODER_ERR_INVALID_ARG;
    b->seq_len[seq] = n;
    return MATMUL_DECODER_OK;
}

int matmul_decoder_batch_get_seq_len(const MatmulDecoderBatch* b, int seq) {
    if (!b || seq < 0 || seq >= b->n) return MATMUL_DECODER_ERR_INVALID_ARG;
    return b->seq_len[seq];
}

static int batch_enqueue(MatmulDecoderBatch* b) {
    DevModel* m = &b->model;
    const MatmulDecoderConfig* c = &m->cfg;
    const int H = c->hidden_dim, n = b->n;
    b2_stream_t s = b->stream;
    int rc = b2_memcpy_h2d(b->d_blk, b->h_blk, (size_t)n * 3 * 4, s);
    if (!rc) rc = b2_event_record(b->ev[0], s);
    if (!rc) rc = b2_embed(b->hidden, m->emb, b->d_blk, NULL, NULL, n, H, s);
    B2KVRef kv = {b->k_cache, b->v_cache, b->seq_stride, b->layer_stride, 0, b->max_seq, b->d_blk + 2 * n,
                  b->d_blk + n, n};
    LayerBuffers lb = {b->hidden, b->qkv, b->attn, b->act, b->attn_work, b->split, b->x16, b->x16b, -1,
                       b->attn_block, b->d_tok + n};
    if (!rc) rc = md_enqueue_layers(m, &lb, n, &kv, s);
    if (!rc) rc = b2_event_record(b->ev[1], s);
    if (!rc && b->comm) {
        /* sharded lm_head: this rank's final-normed rows into its slot of the
         * gathered buffer; the collectives run outside the graph */
        return b2_rows_to_f16(b->g_x16 + (size_t)b->rank * b->rows * H, H, b->hidden, H, n, H, m->final_norm,
                              c->rms_eps, s);
    }
    if (!rc && b->x16 && n >= 16 && (m->lm_wtype == B2_W_I8 || m->lm_wtype == B2_W_F16) && H % 64 == 0) {
        /* many sequences: the lm_head is a GEMM on the tensor cores with the argmax in its epilogue */
        rc = b2_rows_to_f16(b->x16, H, b->hidden, H, n, H, m->final_norm, c->rms_eps, s);
        B2GemmArgs g = {b->logits, c->vocab_size, b->x16, H, n, H, c->vocab_size, m->lm,
                        m->lm_wtype == B2_W_I8 ? m->lm_scales : NULL, m->lm_wtype, B2_EPI_ARGMAX, b->lm_keys, b->d_tok, NULL, 0};
        if (!rc) rc = b2_gemm(&g, s);
    } else if (!rc) {
        rc = b2_lm_head_argmax(b->hidden, H, n, H, c->vocab_size, m->lm, m->lm_scales, m->lm_wtype, m->final_norm,
                               c->rms_eps, b->logits, c->vocab_size, b->d_tok, b->lm_work, s);
    }
    if (!rc) rc = b2_memcpy_d2h(b->h_tok, b->d_tok, (size_t)(n + 1) * 4, s);
    if (!rc) rc = b2_event_record(b->ev[2], s);
    return rc;
}

/* Sharded lm_head tail of a step (enqueued after the graph):
 *   all-gather of every rank's final-normed FP16 rows,
 *   the INT8 (or FP16) lm_head GEMM over this rank's vocab slice for all rows,
 *   per-row merge of the GEMM's keys with global vocab indices,
 *   all-reduce MAX of the keys over the ranks, and this rank's tokens.
 * Then a bounded wait: the stream is polled together with the communicator's
 * asynchronous error state, and a wait longer than B2_NCCL_TIMEOUT_S seconds
 * (default 120) aborts the communicator instead of hanging. */
static int shard_head(MatmulDecoderBatch* b) {
    DevModel* m = &b->model;
    const MatmulDecoderConfig* c = &m->cfg;
    const int H = c->hidden_dim, M = b->world * b->rows, Nv = b->v1 - b->v0;
    cudaStream_t cs = (cudaStream_t)b->stream;
    ncclResult_t nr = g_nccl.all_gather(b->g_x16 + (size_t)b->rank * b->rows * H, b->g_x16, (size_t)b->rows * H * 2,
                                        ncclUint8, b->comm, cs);
    if (nr != ncclSuccess) {
        MD_LOG("ncclAllGather: %s\n", g_nccl.error_string(nr));
        return MATMUL_DECODER_ERR_RKNN;
    }
    const size_t wrow = m->lm_wtype == B2_W_I8 ? (size_t)H : (size_t)H * 2;
    B2GemmArgs g = {NULL, 0, b->g_x16, H, M, H, Nv, (const unsigned char*)m->lm + (size_t)b->v0 * wrow,
                    m->lm_wtype == B2_W_I8 ? m->lm_scales + b->v0 : NULL, m->lm_wtype, B2_EPI_ARGMAX, b->g_keys,
                    b->g_tok, NULL, 0};
    int rc = b2_gemm(&g, b->stream);
    if (!rc) rc = b2_argmax_keys_merge(b->g_keys, M, (Nv + 127) / 128, (unsigned)b->v0, b->m_keys, b->stream);
    if (rc) return rc;
    nr = g_nccl.all_reduce(b->m_keys, b->m_keys, (size_t)M, ncclUint64, ncclMax, b->comm, cs);
    if (nr != ncclSuccess) {
        MD_LOG("ncclAllReduce: %s\n", g_nccl.error_string(nr));
        return MATMUL_DECODER_ERR_RKNN;
    }
    rc = b2_keys_tokens(b->m_keys + (size_t)b->rank * b->rows, b->n, b->d_tok, b->stream);
    if (!rc) rc = b2_memcpy_d2h(b->h_tok, b->d_tok, (size_t)(b->n + 1) * 4, b->stream);
    if (!rc) rc = b2_event_record(b->ev[2], b->stream);
    if (rc) return rc;
    const char* to = getenv("B2_NCCL_TIMEOUT_S");
    const double limit_ms = (to && atof(to) > 0 ? atof(to) : 120.0) * 1e3, t0 = now_ms();
    for (;;) {
        const int q = b2_stream_query(b->stream);
        if (q == 0) return 0;
        if (q < 0) return q;
        ncclResult_t ae = ncclSuccess;
        g_nccl.async_error(b->comm, &ae);
        if ((ae != ncclSuccess && ae != ncclInProgress) || now_ms() - t0 > limit_ms) {
            MD_LOG("sharded lm_head: %s; aborting the communicator\n",
                   ae != ncclSuccess ? g_nccl.error_string(ae) : "timed out");
            g_nccl.abort_(b->comm);
            b->comm = NULL;
            return MATMUL_DECODER_ERR_RKNN;
        }
        usleep(20);
    }
}

int matmul_decoder_nccl_unique_id(void* id_out) {
    if (!id_out) return MATMUL_DECODER_ERR_INVALID_ARG;
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    const ncclResult_t nr = g_nccl.get_id(&id);
    if (nr != ncclSuccess) {
        MD_LOG("ncclGetUniqueId: %s\n", g_nccl.error_string(nr));
        return MATMUL_DECODER_ERR_RKNN;
    }
    memcpy(id_out, &id, sizeof(id));
    return MATMUL_DECODER_OK;
}

int matmul_decoder_batch_shard_vocab(MatmulDecoderBatch* b, int rank, int world, const void* nccl_id,
                                     int rows_per_rank) {
    if (!b || !nccl_id || world < 1 || rank < 0 || rank >= world || rows_per_rank < b->n || b->comm)
        return MATMUL_DECODER_ERR_INVALID_ARG;
    DevModel* m = &b->model;
    const MatmulDecoderConfig* c = &m->cfg;
    const int H = c->hidden_dim, V = c->vocab_size;
    if ((m->lm_wtype != B2_W_I8 && m->lm_wtype != B2_W_F16) || H % 64 || (long long)world * rows_per_rank > 4096)
        return MATMUL_DECODER_ERR_UNSUPPORTED;
    int rc = nccl_load();
    if (rc) return rc;
    b2_set_device(b->device);
    b->world = world;
    b->rank = rank;
    b->rows = rows_per_rank;
    b->v0 = (int)((long long)V * rank / world);
    b->v1 = (int)((long long)V * (rank + 1) / world);
    const size_t M = (size_t)world * rows_per_rank, parts = (size_t)(b->v1 - b->v0 + 127) / 128;
    const size_t bx = (M * H * 2 + 255) & ~(size_t)255, bk = (M * parts * 8 + 255) & ~(size_t)255;
    const size_t bm = (M * 8 + 255) & ~(size_t)255;
    rc = b2_malloc(&b->shard_buf, bx + bk + bm + M * 4 + 256);
    if (rc) return MATMUL_DECODER_ERR_MEMORY;
    unsigned char* p = (unsigned char*)b->shard_buf;
    b->g_x16 = (uint16_t*)p;
    b->g_keys = (unsigned long long*)(p + bx);
    b->m_keys = (unsigned long long*)(p + bx + bk);
    b->g_tok = (int*)(p + bx + bk + bm);
    rc = b2_memset(b->g_x16, 0, bx, NULL);  /* pad rows stay zero */
    if (!rc) rc = b2_stream_sync(NULL);
    if (rc) return rc;
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t nr = g_nccl.init_rank(&b->comm, world, id, rank);
    if (nr != ncclSuccess) {
        MD_LOG("ncclCommInitRank: %s\n", g_nccl.error_string(nr));
        b->comm = NULL;
        return MATMUL_DECODER_ERR_RKNN;
    }
    /* the step graph changes: recapture without the replicated lm_head */
    b2_graph_destroy(b->graph);
    b->graph = NULL;
    printf("[MatmulDecoder] Batch lm_head sharded: rank %d of %d, vocab [%d, %d), %d rows per rank\n", rank, world,
           b->v0, b->v1, rows_per_rank);
    return MATMUL_DECODER_OK;
}

int matmul_decoder_batch_step(MatmulDecoderBatch* b, const int* tokens_in, int* tokens_out, float* logits_out) {
    if (!b || !tokens_in || !tokens_out) return MATMUL_DECODER_ERR_INVALID_ARG;
    const MatmulDecoderConfig* c = &b->model.cfg;
    for (int i = 0; i < b->n; i++) {
        if (tokens_in[i] < 0 || tokens_in[i] >= c->vocab_size) return MATMUL_DECODER_ERR_INVALID_ARG;
        if (b->seq_len[i] >= b->max_seq) {
            MD_LOG("KV cache full for sequence %d\n", i);
            return MATMUL_DECODER_ERR_INVALID_ARG;
        }
    }
    const double t0 = now_ms();
    b2_set_device(b->device);
    int rc = 0;
    if (!b->graph) {
        rc = b2_graph_begin(b->stream);
        if (rc) return rc;
        int rc2 = batch_enqueue(b);
        b2_graph_t g = NULL;
        rc = b2_graph_end(b->stream, &g);
        if (rc2 || rc) {
            b2_graph_destroy(g);
            MD_LOG("batch graph capture failed: %s\n", b2_last_error());
            return rc2 ? rc2 : rc;
        }
        b->graph = g;
    }
    for (int i = 0; i < b->n; i++) {
        b->h_blk[i] = tokens_in[i];
        b->h_blk[b->n + i] = b->seq_len[i];
    }
    if (logits_out && b->comm) return MATMUL_DECODER_ERR_UNSUPPORTED;  /* a rank holds one vocab slice */
    rc = b2_graph_launch(b->graph, b->stream);
    if (!rc && b->comm) rc = shard_head(b);
    if (!rc) rc = b2_stream_sync(b->stream);
    if (rc) {
        MD_LOG("batch step failed: %s\n", b2_last_error());
        return rc;
    }
    if (b->h_tok[b->n]) {  /* a bulk copy of the attention did not arrive in time */
        MD_LOG("batch step: attention wait limit reached\n");
        b2_memset(b->d_tok + b->n, 0, 4, b->stream);
        b2_stream_sync(b->stream);
        return MATMUL_DECODER_ERR_RKNN;
    }
    double t_copy = 0;
    if (logits_out) {
        const double tc = now_ms();
        rc = b2_memcpy_d2h(logits_out, b->logits, (size_t)b->n * c->vocab_size * 4, b->stream);
        if (!rc) rc = b2_stream_sync(b->stream);
        if (rc) return rc;
        t_copy = now_ms() - tc;
    }
    for (int i = 0; i < b->n; i++) {
        tokens_out[i] = b->h_tok[i];
        b->seq_len[i]++;
    }
    float lay = 0, head = 0;
    b2_event_elapsed_ms(&lay, b->ev[0], b->ev[1]);
    b2_event_elapsed_ms(&head, b->ev[1], b->ev[2]);
    b->stats.total_ms = (float)(now_ms() - t0);
    b->stats.matmul_ms = lay;
    b->stats.lm_head_ms = head;
    b->stats.convert_ms = (float)t_copy;
    b->stats.rebind_ms = 0;
    b->stats.cpu_ops_ms = 0;
    b->stats.n_steps++;
    return MATMUL_DECODER_OK;
}

void matmul_decoder_batch_get_stats(const MatmulDecoderBatch* b, MatmulDecoderStats* stats) {
    if (b && stats) *stats = b->stats;
}
