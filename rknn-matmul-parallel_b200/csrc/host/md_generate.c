/*
 * Sampling, generation and the stand-alone KV-cache object.
 *
 * matmul_sample_token (ref include/matmul_decoder.h:422) is greedy argmax for
 * top_k == 1, the reference's only implemented mode (src/matmul_decoder.c:
 * 2316-2324 returns argmax for every setting).  Here the other settings work:
 * repetition penalty on the listed tokens (logit / p if positive, * p if not),
 * temperature, top-k, then top-p over the top-k survivors, sampled with
 * rand() like the reference's top_k_sample_f32 (src/cpu_ops.c:593-652).
 *
 * matmul_decoder_generate is declared by the reference but never defined; here
 * it feeds the prompt (all but the last token in prefill mode), then feeds every
 * produced token back — the loop the reference's pybind generate() gets wrong by
 * passing token -1 (src/pybind_matmul_decoder.cpp:266).
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "md_internal.h"

static int argmax_first(const float* x, int n) {
    float mv = x[0];
    int mi = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > mv) {
            mv = x[i];
            mi = i;
        }
    return mi;
}

typedef struct {
    float v;
    int i;
} Cand;

static int cand_desc(const void* a, const void* b) {
    const Cand* x = (const Cand*)a;
    const Cand* y = (const Cand*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return x->i - y->i;
}

int matmul_sample_token(const float* logits, int vocab_size, SamplingParams* params) {
    if (!logits || vocab_size <= 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    SamplingParams p = params ? *params : sampling_params_greedy();
    const int penalize = p.repeat_penalty != 1.0f && p.repeat_tokens && p.n_repeat_tokens > 0;
    if (p.top_k == 1 && !penalize) return argmax_first(logits, vocab_size);
    float* x = (float*)malloc((size_t)vocab_size * sizeof(float));
    if (!x) return MATMUL_DECODER_ERR_MEMORY;
    memcpy(x, logits, (size_t)vocab_size * sizeof(float));
    if (penalize)
        for (int i = 0; i < p.n_repeat_tokens; i++) {
            int t = p.repeat_tokens[i];
            if (t >= 0 && t < vocab_size) x[t] = x[t] > 0 ? x[t] / p.repeat_penalty : x[t] * p.repeat_penalty;
        }
    if (p.top_k == 1) {
        int r = argmax_first(x, vocab_size);
        free(x);
        return r;
    }
    int k = p.top_k <= 0 || p.top_k > vocab_size ? vocab_size : p.top_k;
    Cand* c = (Cand*)malloc((size_t)vocab_size * sizeof(Cand));
    if (!c) {
        free(x);
        return MATMUL_DECODER_ERR_MEMORY;
    }
    const float temp = p.temperature > 0 ? p.temperature : 1.0f;
    for (int i = 0; i < vocab_size; i++) {
        c[i].v = x[i] / temp;
        c[i].i = i;
    }
    qsort(c, (size_t)vocab_size, sizeof(Cand), cand_desc);
    double sum = 0;
    for (int i = 0; i < k; i++) sum += exp((double)c[i].v - c[0].v);
    int keep = k;
    if (p.top_p > 0 && p.top_p < 1.0f) {
        double cum = 0;
        for (int i = 0; i < k; i++) {
            cum += exp((double)c[i].v - c[0].v) / sum;
            if (cum >= p.top_p) {
                keep = i + 1;
                break;
            }
        }
    }
    double tot = 0;
    for (int i = 0; i < keep; i++) tot += exp((double)c[i].v - c[0].v);
    double r = (double)rand() / RAND_MAX * tot, acc = 0;
    int out = c[keep - 1].i;
    for (int i = 0; i < keep; i++) {
        acc += exp((double)c[i].v - c[0].v);
        if (r < acc) {
            out = c[i].i;
            break;
        }
    }
    free(c);
    free(x);
    return out;
}

int matmul_decoder_generate(MatmulDecoderContext* ctx, const int* prompt_tokens, int n_prompt,
                            int max_new_tokens, SamplingParams* params, GenerateCallback callback,
                            void* user_data) {
    if (!ctx || !prompt_tokens || n_prompt <= 0 || max_new_tokens < 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    for (int i = 0; i < n_prompt - 1; i++) {
        int rc = matmul_decoder_step(ctx, prompt_tokens[i], NULL, NULL);
        if (rc < 0) return rc;
    }
    if (max_new_tokens == 0) return 0;
    /* every produced token is drawn on the device (greedy steps run the
     * argmax there): no logits are copied to the host */
    int tok = prompt_tokens[n_prompt - 1], produced = 0;
    for (int i = 0; i < max_new_tokens; i++) {
        const int next = matmul_decoder_step_sample(ctx, tok, NULL, params);
        if (next < 0) return produced > 0 ? produced : next;
        produced++;
        if (callback) callback(next, NULL, user_data);
        tok = next;
    }
    return produced;
}

/* ─── stand-alone KV cache (ref src/matmul_decoder.c:449-502) ───
 * A host FP32 [layers][max_seq][kv_heads][hd] cache object with a length
 * counter, as the reference exports it.  Decoder contexts keep their own
 * device cache and do not use this type. */
struct MatmulKVCache {
    float* k_cache;
    float* v_cache;
    int num_layers, num_kv_heads, head_dim, max_seq_len, seq_len;
};

MatmulKVCache* matmul_kv_cache_create(int num_layers, int num_kv_heads, int head_dim, int max_seq_len) {
    if (num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_seq_len <= 0) return NULL;
    MatmulKVCache* c = (MatmulKVCache*)calloc(1, sizeof(*c));
    if (!c) return NULL;
    const size_t n = (size_t)num_layers * max_seq_len * num_kv_heads * head_dim;
    c->k_cache = (float*)calloc(n, sizeof(float));
    c->v_cache = (float*)calloc(n, sizeof(float));
    if (!c->k_cache || !c->v_cache) {
        free(c->k_cache);
        free(c->v_cache);
        free(c);
        return NULL;
    }
    c->num_layers = num_layers;
    c->num_kv_heads = num_kv_heads;
    c->head_dim = head_dim;
    c->max_seq_len = max_seq_len;
    return c;
}

void matmul_kv_cache_clear(MatmulKVCache* cache) {
    if (cache) cache->seq_len = 0;
}

int matmul_kv_cache_get_seq_len(const MatmulKVCache* cache) { return cache ? cache->seq_len : 0; }

void matmul_kv_cache_destroy(MatmulKVCache* cache) {
    if (!cache) return;
    free(cache->k_cache);
    free(cache->v_cache);
    free(cache);
}

/* ─── ASR front end (ADDITIVE) ───
 * The log-mel features on the current device: the waveform and the filters
 * go up, the (128, T) features come back. */
int matmul_log_mel(const float* audio, int n_samples, const float* filters, float* mel_out) {
    if (!audio || !filters || !mel_out || n_samples <= 200) return MATMUL_DECODER_ERR_INVALID_ARG;
    const int T = n_samples / 160;
    const size_t wbytes = b2_log_mel_workspace(n_samples);
    const size_t a_bytes = ((size_t)n_samples * 4 + 255) & ~(size_t)255;
    const size_t f_bytes = ((size_t)201 * 128 * 4 + 255) & ~(size_t)255;
    const size_t o_bytes = ((size_t)T * 128 * 4 + 255) & ~(size_t)255;
    unsigned char* buf = NULL;
    int rc = b2_malloc((void**)&buf, a_bytes + f_bytes + o_bytes + wbytes);
    if (rc) return MATMUL_DECODER_ERR_MEMORY;
    float* d_audio = (float*)buf;
    float* d_filters = (float*)(buf + a_bytes);
    float* d_out = (float*)(buf + a_bytes + f_bytes);
    void* d_work = buf + a_bytes + f_bytes + o_bytes;
    if (!rc) rc = b2_memcpy_h2d(d_audio, audio, (size_t)n_samples * 4, NULL);
    if (!rc) rc = b2_memcpy_h2d(d_filters, filters, (size_t)201 * 128 * 4, NULL);
    if (!rc) rc = b2_log_mel(d_audio, n_samples, d_filters, d_out, d_work, NULL);
    if (!rc && T > 0) rc = b2_memcpy_d2h(mel_out, d_out, (size_t)T * 128 * 4, NULL);
    if (!rc) rc = b2_stream_sync(NULL);
    b2_free(buf);
    if (rc) {
        MD_LOG("log-mel failed (%d): %s\n", rc, b2_last_error());
        return rc;
    }
    return T;
}
