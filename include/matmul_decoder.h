/*
 * matmul_decoder.h — public C API of the B200 decoder runtime.
 *
 * This header is the drop-in boundary: every type, enum value, field order and
 * function signature below matches the reference interface
 * include/matmul_decoder.h of suharvest/rknn-matmul-parallel (cited per item as
 * "ref include/matmul_decoder.h:LINE"), so a caller compiled against the
 * reference header links against libmatmul_decoder.so unchanged.  The
 * implementation behind it keeps all weights, the KV cache and all
 * activations resident in B200 HBM and runs the decode step as sm_100a
 * kernels; host pointers passed in and out are ordinary host memory.
 *
 * Entry points marked ADDITIVE have no counterpart in the reference header;
 * they exist for seeded-KV benchmarking, batched multi-sequence decode and
 * multi-GPU sharding.  No reference signature was changed to add them.
 */
#ifndef MATMUL_DECODER_H
#define MATMUL_DECODER_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Version (ref include/matmul_decoder.h:25-27). */
#define MATMUL_DECODER_VERSION_MAJOR 1
#define MATMUL_DECODER_VERSION_MINOR 0
#define MATMUL_DECODER_VERSION_PATCH 0

/* Error codes (ref include/matmul_decoder.h:30-37).  ERR_RKNN is kept at its
 * value; here it reports a CUDA runtime failure (the device-side analogue of
 * an NPU runtime failure). */
typedef enum {
    MATMUL_DECODER_OK = 0,
    MATMUL_DECODER_ERR_INVALID_ARG = -1,
    MATMUL_DECODER_ERR_MEMORY = -2,
    MATMUL_DECODER_ERR_FILE_IO = -3,
    MATMUL_DECODER_ERR_RKNN = -4,
    MATMUL_DECODER_ERR_UNSUPPORTED = -5,
} MatmulDecoderError;

/* Execution mode (ref include/matmul_decoder.h:41-44).  Accepted and stored;
 * a single B200 runs the whole step either way. */
typedef enum {
    EXEC_SINGLE_CORE = 0,
    EXEC_DUAL_CORE = 1,
} ExecutionMode;

/* Model configuration (ref include/matmul_decoder.h:52-114); identical field
 * order so the struct is layout-compatible. */
typedef struct {
    const char* name;
    int hidden_dim;
    int num_q_heads;
    int num_kv_heads;
    int head_dim;
    int ffn_dim;
    int num_layers;
    int vocab_size;
    int max_seq_len;
    float rms_eps;
    float rope_theta;
    int tie_word_embeddings;
    float rope_scaling_factor;   /* declared, unused (as in the reference) */
    int rope_scaling_type;       /* declared, unused */
    int norm_type;               /* 0 = RMSNorm (only value supported) */
    int rope_style;              /* 0 = interleaved pairs (2i,2i+1); 1 = split-half (i,i+hd/2) */
    int ffn_act_type;            /* 0 = SwiGLU (only value supported) */
    int has_qk_norm;             /* per-head RMSNorm on q and k after projection */
    int num_lm_heads;            /* >1 selects multi-head mode (step_head) */
    int lm_head_vocab_size;      /* per-head vocab in multi-head mode */
    int context_pool_mode;       /* NPU-only in the reference; accepted, ignored */
    int iommu_domain_id;         /* NPU-only in the reference; accepted, ignored */
    ExecutionMode exec_mode;
    int disable_npu_lm_head;     /* 1 = FP16 lm_head instead of the INT8 one */
    int max_batch_prefill;       /* reference chunk size for prefill_batch (0 = 64) */
} MatmulDecoderConfig;

/* Preset for Qwen3-0.6B-shaped decoders (ref include/matmul_decoder.h:119-144). */
static inline MatmulDecoderConfig matmul_decoder_config_qwen3_0_6b(void) {
    MatmulDecoderConfig c;
    c.name = "qwen3-asr-0.6b";
    c.hidden_dim = 1024;
    c.num_q_heads = 16;
    c.num_kv_heads = 8;
    c.head_dim = 128;
    c.ffn_dim = 3072;
    c.num_layers = 28;
    c.vocab_size = 151936;
    c.max_seq_len = 4096;
    c.rms_eps = 1e-6f;
    c.rope_theta = 1000000.0f;
    c.tie_word_embeddings = 1;
    c.rope_scaling_factor = 1.0f;
    c.rope_scaling_type = 0;
    c.norm_type = 0;
    c.rope_style = 0;
    c.ffn_act_type = 0;
    c.has_qk_norm = 1;
    c.num_lm_heads = 0;
    c.lm_head_vocab_size = 0;
    c.context_pool_mode = 0;
    c.iommu_domain_id = 1;
    c.exec_mode = EXEC_DUAL_CORE;
    c.disable_npu_lm_head = 0;
    c.max_batch_prefill = 64;
    return c;
}

/* Single-core variant (ref include/matmul_decoder.h:149-153). */
static inline MatmulDecoderConfig matmul_decoder_config_qwen3_0_6b_single_core(void) {
    MatmulDecoderConfig c = matmul_decoder_config_qwen3_0_6b();
    c.exec_mode = EXEC_SINGLE_CORE;
    return c;
}

/* 15-head code-predictor preset (ref include/matmul_decoder.h:159-184). */
static inline MatmulDecoderConfig matmul_decoder_config_qwen3_tts_cp(void) {
    MatmulDecoderConfig c = matmul_decoder_config_qwen3_0_6b();
    c.name = "qwen3-tts-cp";
    c.num_layers = 5;
    c.vocab_size = 2048;
    c.max_seq_len = 20;
    c.tie_word_embeddings = 0;
    c.num_lm_heads = 15;
    c.lm_head_vocab_size = 2048;
    return c;
}

/* Quantization type (ref include/matmul_decoder.h:188-193).
 *   QUANT_FP16      FP16 weights.
 *   QUANT_INT8      int8 per-output-column symmetric (W8A16).
 *   QUANT_INT4      int4 per-output-column symmetric, two per byte (W4A16).
 *   QUANT_INT4_G128 accepted; loads the same per-column INT4 files. */
typedef enum {
    QUANT_FP16 = 0,
    QUANT_INT8 = 1,
    QUANT_INT4 = 2,
    QUANT_INT4_G128 = 3,
} QuantizationType;

/* In-memory weights (ref include/matmul_decoder.h:201-231).  `data` is host
 * memory in the on-disk layout: FP16 [K][N] row-major, int8 [K][N], or int4
 * [K][N/2] bytes (low nibble = even column).  `scales` is FP32 [N] or NULL. */
typedef struct {
    void* data;
    float* scales;
    int K;
    int N;
    QuantizationType quant_type;
} ProjectionWeight;

typedef struct {
    ProjectionWeight q_proj;
    ProjectionWeight k_proj;
    ProjectionWeight v_proj;
    ProjectionWeight o_proj;
    ProjectionWeight gate_proj;
    ProjectionWeight up_proj;
    ProjectionWeight down_proj;
    float* input_norm_weight;
    float* post_attn_norm_weight;
    float* q_norm_weight;
    float* k_norm_weight;
} LayerWeights;

/* ─── KV cache (ref include/matmul_decoder.h:235-262) ───
 * A stand-alone cache object.  The decoder owns its own device-resident cache;
 * this object is the host-side bookkeeping type the reference exports. */
typedef struct MatmulKVCache MatmulKVCache;

MatmulKVCache* matmul_kv_cache_create(int num_layers, int num_kv_heads,
                                      int head_dim, int max_seq_len);
void matmul_kv_cache_clear(MatmulKVCache* cache);
int matmul_kv_cache_get_seq_len(const MatmulKVCache* cache);
void matmul_kv_cache_destroy(MatmulKVCache* cache);

/* ─── Decoder context (ref include/matmul_decoder.h:266-387) ─── */
typedef struct MatmulDecoderContext MatmulDecoderContext;

/* Load a model directory in the reference's on-disk format and upload it to
 * the current CUDA device (ref :286-289).  config == NULL reads
 * model_dir/config.json.  Returns NULL on any failure (missing or short weight
 * file, CUDA error); the message goes to stderr with a [MatmulDecoder] prefix. */
MatmulDecoderContext* matmul_decoder_create(const char* model_dir,
                                            const MatmulDecoderConfig* config,
                                            QuantizationType quant_type,
                                            int max_seq_len);

/* Build a decoder from host arrays (ref :294-301). */
MatmulDecoderContext* matmul_decoder_create_from_weights(
    const MatmulDecoderConfig* config,
    const float* embeddings,
    const LayerWeights* layers,
    const float* lm_head,
    QuantizationType quant_type,
    int max_seq_len);

/* One decode step (ref :312-315).  Returns the greedy token id (>= 0), or 0
 * when output_logits == NULL (prefill mode: no final norm, no lm_head), or a
 * negative MatmulDecoderError. */
int matmul_decoder_step(MatmulDecoderContext* ctx,
                        int token_id,
                        const float* embedding,
                        float* output_logits);

/* Same step, logits always produced (ref :320-323; declared but never
 * defined by the reference). */
int matmul_decoder_step_get_logits(MatmulDecoderContext* ctx,
                                   int token_id,
                                   const float* embedding,
                                   float* logits_out);

/* Step with lm_head number lm_head_idx in multi-head mode (ref :335-339). */
int matmul_decoder_step_head(MatmulDecoderContext* ctx,
                             int token_id,
                             const float* embedding,
                             int lm_head_idx,
                             float* output_logits);

/* Run M embeddings [M][hidden_dim] through all layers causally, filling the
 * KV cache; no lm_head (ref :351-352). */
int matmul_decoder_prefill_batch(MatmulDecoderContext* ctx,
                                 const float* embeddings, int M);

void matmul_decoder_clear_kv_cache(MatmulDecoderContext* ctx);
int matmul_decoder_get_seq_len(const MatmulDecoderContext* ctx);
const MatmulDecoderConfig* matmul_decoder_get_config(const MatmulDecoderContext* ctx);

/* Per-step timing (ref :372-382).  On the B200: matmul_ms is GPU time of the
 * weight GEMVs, rebind_ms is always 0, convert_ms is host<->device copy time,
 * cpu_ops_ms is GPU time of norm/RoPE/attention, lm_head_ms is GPU time of
 * the lm_head and argmax, total_ms is wall time of the step. */
typedef struct {
    float total_ms;
    float matmul_ms;
    float rebind_ms;
    float convert_ms;
    float cpu_ops_ms;
    float lm_head_ms;
    int n_steps;
} MatmulDecoderStats;

void matmul_decoder_get_stats(const MatmulDecoderContext* ctx, MatmulDecoderStats* stats);
void matmul_decoder_destroy(MatmulDecoderContext* ctx);

/* ─── Sampling (ref include/matmul_decoder.h:391-422) ─── */
typedef struct {
    int top_k;
    float top_p;
    float temperature;
    float repeat_penalty;
    const int* repeat_tokens;
    int n_repeat_tokens;
} SamplingParams;

static inline SamplingParams sampling_params_greedy(void) {
    SamplingParams p;
    p.top_k = 1;
    p.top_p = 1.0f;
    p.temperature = 1.0f;
    p.repeat_penalty = 1.0f;
    p.repeat_tokens = NULL;
    p.n_repeat_tokens = 0;
    return p;
}

/* Pick a token from host logits (ref :422).  top_k == 1 is greedy argmax
 * (first index holding the maximum). */
int matmul_sample_token(const float* logits, int vocab_size, SamplingParams* params);

/* ─── Generation (ref include/matmul_decoder.h:434-454; undefined in the
 * reference).  Feeds the prompt, then feeds each produced token back. ─── */
typedef void (*GenerateCallback)(int token_id, const char* token_text, void* user_data);

int matmul_decoder_generate(MatmulDecoderContext* ctx,
                            const int* prompt_tokens,
                            int n_prompt,
                            int max_new_tokens,
                            SamplingParams* params,
                            GenerateCallback callback,
                            void* user_data);

/* ─── Utilities (ref include/matmul_decoder.h:461-467) ─── */
int matmul_decoder_load_config(const char* json_path, MatmulDecoderConfig* config);

/* Returns MATMUL_DECODER_ERR_UNSUPPORTED: HF export needs the HF checkpoint
 * tooling, which this runtime does not ship (the reference never defined it). */
int matmul_decoder_export_hf_model(const char* hf_model_path,
                                   const char* output_dir,
                                   QuantizationType quant_type);

/* ═══════════════════════ ADDITIVE entry points ═══════════════════════ */

/* ADDITIVE.  Greedy step that returns only the token id: runs the lm_head and
 * the on-device argmax but copies no logits to the host (4 bytes come back). */
int matmul_decoder_step_token(MatmulDecoderContext* ctx, int token_id,
                              const float* embedding);

/* ADDITIVE.  One decode step, then the token drawn on the device from its
 * logits (b2_sample_token) with the semantics of matmul_sample_token:
 * repeat penalty per listed occurrence, top_k == 1 greedy, temperature,
 * top-k, top-p, then a draw with probability proportional to
 * exp(v - v_max).  Only the token crosses to the host.  Draw i of a context
 * is a function of (seed, i): the seed comes from rand() at creation (so
 * srand() before create fixes it) or from matmul_decoder_set_seed, which also
 * restarts i at 0.  top_k == 1 without a penalty is the greedy step
 * (matmul_decoder_step_token).  matmul_decoder_generate draws every token
 * this way.  Returns the token or a negative error. */
int matmul_decoder_step_sample(MatmulDecoderContext* ctx, int token_id, const float* embedding,
                               const SamplingParams* params);
int matmul_decoder_set_seed(MatmulDecoderContext* ctx, unsigned long long seed);

/* ADDITIVE.  ASR front end on the GPU (the reference does it in numpy,
 * examples/qwen3_asr/mel.py:52-67 and engine.py:255-314).
 * matmul_log_mel: host FP32 waveform audio[n_samples] at 16 kHz (n_samples
 * > 200) and mel filters [201][128] -> host mel_out [128][n_samples / 160],
 * the Whisper-style log-mel features (returns the frame count or an error).
 * matmul_decoder_build_embed: host token ids and host audio embeddings
 * [n_audio][hidden_dim] -> host embed_out [n_pre + n_audio + n_suf][hidden],
 * token rows taken from the context's embedding table on the device
 * (returns the row count or an error; ids outside [0, vocab) are rejected). */
int matmul_log_mel(const float* audio, int n_samples, const float* filters, float* mel_out);
int matmul_decoder_build_embed(MatmulDecoderContext* ctx, const int* prefix_ids, int n_pre,
                               const float* audio_embd, int n_audio, const int* suffix_ids, int n_suf,
                               float* embed_out);

/* ADDITIVE.  Greedy decode of n_tokens tokens with the token feedback kept on
 * the device: step i consumes the token produced by step i-1 (step 0 consumes
 * first_token), so the host neither copies a token nor synchronizes between
 * steps.  tokens_out (host, n_tokens) gets the produced tokens; device_ms
 * (optional) gets the GPU time of the n_tokens steps measured with CUDA
 * events on the decoder's stream.  Returns n_tokens or a negative error. */
int matmul_decoder_decode_greedy(MatmulDecoderContext* ctx, int first_token, int n_tokens,
                                 int* tokens_out, float* device_ms);

/* ADDITIVE.  Write positions [start, start+len) of one layer's KV cache from
 * host FP16 bits laid out [len][num_kv_heads][head_dim] (the reference cache's
 * position-major order).  Does not change seq_len. */
int matmul_decoder_set_kv(MatmulDecoderContext* ctx, int layer, int start, int len,
                          const uint16_t* k_fp16, const uint16_t* v_fp16);

/* ADDITIVE.  Read the same range back (FP16 bits, same layout). */
int matmul_decoder_get_kv(MatmulDecoderContext* ctx, int layer, int start, int len,
                          uint16_t* k_fp16, uint16_t* v_fp16);

/* ADDITIVE.  Set the current sequence length (0 <= n <= max_seq_len), e.g.
 * after seeding the cache with set_kv. */
int matmul_decoder_set_seq_len(MatmulDecoderContext* ctx, int n);

/* ADDITIVE.  Copy the residual-stream hidden state after the last layer of
 * the most recent token (the step's token, or the last row of the last
 * prefill_batch), before the final norm, to host FP32 [hidden_dim]. */
int matmul_decoder_get_hidden(MatmulDecoderContext* ctx, float* hidden_out);

/* ADDITIVE.  1 when single-token steps run as the persistent decode kernel
 * (one launch per token), 0 when they replay the graph of per-op kernels
 * (B2_DECODE_KERNEL=graph at create time, or shapes the kernel does not
 * cover). */
int matmul_decoder_uses_persistent_kernel(const MatmulDecoderContext* ctx);

/* ADDITIVE.  Which kernel a single-token step with n_cached positions already
 * in the cache runs: 2 = the tile-stream persistent kernel (b2_mk2_decode),
 * 1 = the first persistent kernel (b2_mk_decode), 0 = the CUDA graph of
 * per-op kernels. */
int matmul_decoder_step_kernel(const MatmulDecoderContext* ctx, int n_cached);

/* ADDITIVE.  Quantize one FP16 [K][N] weight on the host into the on-disk
 * quantized layout: bits = 8 writes int8 [K][N]; bits = 4 writes int4 [K][N/2]
 * (low nibble = even column).  scales_out gets FP32 [N].  Bit-exact with the
 * reference's per-column rule (max|col| / qmax, roundf, clamp). */
int matmul_decoder_quantize_weight(const uint16_t* w_fp16, int K, int N, int bits,
                                   uint8_t* q_out, float* scales_out);

/* ADDITIVE.  The INT8 lm_head the decoder builds at create time, computed on
 * the host: the FP32 [V][K] table is rounded to FP16, then each vocab row is
 * quantized with the reference rule (max|row| / 127, roundf, clamp to
 * [-128, 127]).  q_out gets int8 [V][K]; scales_out gets FP32 [V]. */
int matmul_decoder_quantize_lm_head(const float* table, int V, int K, int8_t* q_out,
                                    float* scales_out);

/* ─── ADDITIVE: batched multi-sequence decode ───
 * n_seqs independent sequences share one copy of the weights; each has its own
 * KV cache and position.  One batch step advances every active sequence by one
 * greedy token. */
typedef struct MatmulDecoderBatch MatmulDecoderBatch;

MatmulDecoderBatch* matmul_decoder_batch_create(const char* model_dir,
                                                const MatmulDecoderConfig* config,
                                                QuantizationType quant_type,
                                                int max_seq_len, int n_seqs);
int matmul_decoder_batch_set_kv(MatmulDecoderBatch* b, int seq, int layer, int start, int len,
                                const uint16_t* k_fp16, const uint16_t* v_fp16);
int matmul_decoder_batch_set_seq_len(MatmulDecoderBatch* b, int seq, int n);
int matmul_decoder_batch_get_seq_len(const MatmulDecoderBatch* b, int seq);
/* tokens_in[n_seqs] -> tokens_out[n_seqs]; logits_out (optional, host) gets
 * [n_seqs][vocab_size]. */
int matmul_decoder_batch_step(MatmulDecoderBatch* b, const int* tokens_in, int* tokens_out,
                              float* logits_out);
void matmul_decoder_batch_get_stats(const MatmulDecoderBatch* b, MatmulDecoderStats* stats);
void matmul_decoder_batch_destroy(MatmulDecoderBatch* b);

/* ─── ADDITIVE: vocab-sharded lm_head over ranks (one GPU each) ───
 * The sequences of a batch are split over ranks; each rank runs its own
 * MatmulDecoderBatch on its GPU.  After sharding, each rank keeps the lm_head
 * rows of one slice of the vocabulary: a step gathers every rank's final
 * hidden rows (NCCL all-gather over NVLink), scores all rows against the
 * local slice, and an NCCL all-reduce MAX of packed (value, index) keys gives
 * every row its global argmax (lowest index on ties).  Every rank must call
 * matmul_decoder_batch_step the same number of times.  logits_out is not
 * available on a sharded decoder (MATMUL_DECODER_ERR_UNSUPPORTED). */

/* 128-byte NCCL unique id: made once (rank 0) and passed to every rank. */
int matmul_decoder_nccl_unique_id(void* id_out);
/* Collective over the `world` ranks (each calls it with its rank).
 * rows_per_rank >= the decoder's n_seqs and equal on every rank. */
int matmul_decoder_batch_shard_vocab(MatmulDecoderBatch* b, int rank, int world, const void* nccl_id,
                                     int rows_per_rank);

#ifdef __cplusplus
}
#endif

#endif /* MATMUL_DECODER_H */
