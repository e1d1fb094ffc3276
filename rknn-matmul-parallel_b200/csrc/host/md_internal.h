/*
 * Internal structures of the host runtime (libmatmul_decoder.so).
 *
 * The reference keeps per-projection NPU contexts and rebinds weight buffers
 * before every matmul (PersistentMatmul / MatmulPoolEntry,
 * src/matmul_decoder.c:38-65).  Here every weight, the KV cache, the RoPE
 * tables and all activations live in one device arena allocated at create
 * time; kernels get raw device pointers and nothing is rebound.
 */
#ifndef MD_INTERNAL_H
#define MD_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "b2_kernels.h"
#include "matmul_decoder.h"

#define MD_LOG(...) fprintf(stderr, "[MatmulDecoder] " __VA_ARGS__)

/* One fused projection in device layout: `rows` output rows of K weights. */
typedef struct {
    void* w;
    float* s;      /* per-row scales (quantized) or NULL */
    int rows, K, wtype;
} DevProj;

typedef struct {
    DevProj qkv;   /* rows: q (nq*hd) | k (nkv*hd) | v (nkv*hd) */
    DevProj o;     /* rows: hidden, K = nq*hd */
    DevProj gu;    /* rows: gate (ffn) | up (ffn) */
    DevProj down;  /* rows: hidden, K = ffn */
    void* down_t;  /* down_proj in its file layout [ffn][hidden] (input-channel rows), same encoding */
    float *in_norm, *post_norm, *q_norm, *k_norm;
} DevLayer;

/* Bump allocator over one device allocation (the device-buffer pool). */
typedef struct {
    unsigned char* base;
    size_t size, off;
} DevArena;

/* Device-resident model weights shared by decoder contexts of one device. */
typedef struct {
    MatmulDecoderConfig cfg;
    char name[128];
    QuantizationType quant;
    int wtype;             /* B2_W_F16 / B2_W_I8 / B2_W_I4 for the layers */
    DevArena arena;
    float* emb;            /* [V][H] FP32 */
    void* lm;              /* [V][H] int8 (with lm_scales) or FP16 */
    float* lm_scales;
    int lm_wtype;
    float** lm_heads;      /* multi-head: [n][Vh][H] FP32 */
    int n_lm_heads, lm_vocab;
    float* final_norm;
    DevLayer* layers;
    float *cos_tab, *sin_tab;  /* [max_seq][hd/2] */
    int max_seq;
} DevModel;

/* Host-side tensors of one layer in the reference on-disk layout. */
typedef struct {
    void* w[7];            /* q k v o gate up down: FP16 [K][N], int8 [K][N], int4 [K][N/2] */
    float* s[7];
    int wt[7];             /* per-projection encoding of w[] */
    float *in_norm, *post_norm, *q_norm, *k_norm;
} HostLayer;

/* md_config.c */
void md_config_defaults(MatmulDecoderConfig* c);
int md_config_validate(const MatmulDecoderConfig* c);

/* md_model.c */
int md_model_load_dir(DevModel* m, const char* dir, const MatmulDecoderConfig* cfg,
                      QuantizationType q, int max_seq, size_t extra_bytes);
int md_model_from_host(DevModel* m, const MatmulDecoderConfig* cfg, QuantizationType q, int max_seq,
                       const float* emb, const float* lm_head, const HostLayer* layers,
                       size_t extra_bytes);
void md_model_free(DevModel* m);
void* md_arena_alloc(DevArena* a, size_t bytes);
size_t md_model_bytes(const MatmulDecoderConfig* c, int wtype, int max_seq, int n_lm_heads);

/* md_quant.c (bit-exact host quantisers) */
uint16_t md_f32_to_f16(float x);
float md_f16_to_f32(uint16_t h);
void md_quantize_cols(const uint16_t* w_kn, int K, int N, int bits, uint8_t* q, float* scales);
void md_quantize_rows_i8(const uint16_t* t_vk, int V, int K, int8_t* q_vk, float* scales);

/* md_layers.c: enqueue one decode/prefill pass of all layers on a stream. */
typedef struct {
    float* hidden;   /* [M][H] */
    float* qkv;      /* [M][qd + 2 kvd] */
    float* attn;     /* [M][qd] */
    float* act;      /* [M][ffn] */
    void* attn_work;
    int attn_split;
    uint16_t* x16;   /* [M][max(H, qd, ffn)] FP16 staging for the tensor-core GEMM, or NULL */
    uint16_t* x16b;  /* [M][ffn] FP16 gate|up output = down-projection input, or NULL */
    int prefill_base; /* >= 0: the M rows are one sequence at positions prefill_base + m (flash attention) */
    int attn_block;   /* > 0: attention in fixed blocks of this many positions (b2_attention_blocks) */
    int* attn_err;    /* device flag for b2_attention_blocks */
} LayerBuffers;
int md_enqueue_layers(const DevModel* m, const LayerBuffers* b, int M, const B2KVRef* kv_proto,
                      b2_stream_t s);

#endif
