/*
 * b2_kernels.h — thin C-ABI over the sm_100a kernels and the CUDA runtime.
 *
 * The host C runtime (libmatmul_decoder.so) reaches the GPU only through these
 * functions; none of them takes a torch or CUDA C++ type.  Every pointer
 * documented "device" is device memory of the current CUDA device; "host" is
 * ordinary or pinned host memory.  Every function returns 0 on success or a
 * negative MatmulDecoderError (ERR_RKNN = -4 for a CUDA failure,
 * ERR_INVALID_ARG = -1 for a bad shape); b2_last_error() gives the message.
 *
 * Reference interfaces these replace (suharvest/rknn-matmul-parallel):
 *   b2_gemv            run_persistent_matmul / run_batch_matmul
 *                      (src/matmul_decoder.c:382-445, :1841-1899) plus the
 *                      RMSNorm before it and the residual add / SiLU*mul after
 *                      it (src/cpu_ops.c:18-55, :296-319, :350-359)
 *   b2_qk_rope_kv      per-head q/k RMSNorm, RoPE, KV store
 *                      (src/matmul_decoder.c:1495-1516, src/cpu_ops.c:109-155)
 *   b2_attention       attention_f32 / attention_batch_causal_f32
 *                      (src/cpu_ops.c:202-264, :459-571)
 *   b2_lm_head_argmax  final RMSNorm + tiled INT8 lm_head / FP16 / FP32 GEMV
 *                      + argmax (src/matmul_decoder.c:1563-1633,
 *                      :1722-1741, src/cpu_ops.c:575-586)
 *   b2_embed           embedding row copy (src/matmul_decoder.c:1446-1454)
 *   b2_malloc/...      the NPU buffer pool (rknn_create_mem,
 *                      src/npu_buffer_pool.c:52-87) becomes a device arena
 */
#ifndef B2_KERNELS_H
#define B2_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2_stream_s* b2_stream_t;
typedef struct b2_event_s* b2_event_t;
typedef struct b2_graph_s* b2_graph_t;

/* Weight encodings in device layout: one row per output column n, K
 * contiguous.  F16: uint16 [rows][K]; I8: int8 [rows][K]; I4: uint8
 * [rows][K/2] with element k in byte k/2, low nibble for even k,
 * two's-complement int4.  I8/I4 rows carry an FP32 scale per row. */
enum { B2_W_F16 = 0, B2_W_I8 = 1, B2_W_I4 = 2, B2_W_F32 = 3 };

/* GEMV epilogues. */
enum {
    B2_EPI_STORE = 0,     /* y[m][n] = acc * s[n]                                   */
    B2_EPI_ADD = 1,       /* y[m][n] += acc * s[n]   (residual add)                 */
    B2_EPI_SILU_PAIR = 2, /* rows n and N+n: y[m][n] = silu(g) * u                  */
    B2_EPI_ARGMAX = 3,    /* b2_gemm only: tokens[m] = argmax_n acc * s[n]           */
};

/* ─── runtime ─── */
const char* b2_last_error(void);
int b2_device_count(int* n);
int b2_set_device(int dev);
int b2_get_device(int* dev);
int b2_sm_count(int* n);
int b2_malloc(void** ptr, size_t bytes);
int b2_free(void* ptr);
int b2_host_alloc(void** ptr, size_t bytes);   /* pinned host memory */
int b2_host_free(void* ptr);
int b2_mem_get_info(size_t* free_bytes, size_t* total_bytes);
int b2_memcpy_h2d(void* dst, const void* src, size_t bytes, b2_stream_t s);
int b2_memcpy_d2h(void* dst, const void* src, size_t bytes, b2_stream_t s);
int b2_memcpy_d2d(void* dst, const void* src, size_t bytes, b2_stream_t s);
int b2_memset(void* dst, int value, size_t bytes, b2_stream_t s);
int b2_stream_create(b2_stream_t* s);
int b2_stream_destroy(b2_stream_t s);
int b2_stream_sync(b2_stream_t s);
/* 0 when all work of the stream has completed, 1 while some is pending,
 * negative on an error (lets a caller bound its wait). */
int b2_stream_query(b2_stream_t s);
int b2_event_create(b2_event_t* e);
int b2_event_destroy(b2_event_t e);
int b2_event_record(b2_event_t e, b2_stream_t s);
int b2_event_elapsed_ms(float* ms, b2_event_t start, b2_event_t stop);
int b2_graph_begin(b2_stream_t s);
int b2_graph_end(b2_stream_t s, b2_graph_t* g);
int b2_graph_launch(b2_graph_t g, b2_stream_t s);
int b2_graph_destroy(b2_graph_t g);

/* ─── kernels ─── */

/* Weight-only GEMV/skinny GEMM: y[m][n] = epi( s[n] * sum_k f16(xn[m][k]) * W[n][k] )
 * for m < M, where xn = x, or RMSNorm(x; norm_w, eps) when norm_w != NULL
 * (computed as (x * rms) * w, rms = 1/sqrtf(mean(x^2) + eps)).  The
 * activation is rounded to FP16 (round-to-nearest-even) before the multiply
 * and products accumulate in FP32, like the reference's FP16-input NPU
 * matmul.  w is the device layout above with N rows (2N for SILU_PAIR, gate
 * rows first); scales is NULL for F16.  x, y device FP32 with row strides
 * ldx, ldy (elements). */
typedef struct {
    float* y;
    int ldy;
    const float* x;
    int ldx;
    int M, K, N;
    const void* w;
    const float* scales;
    int wtype;
    const float* norm_w;
    float eps;
    int epilogue;
} B2GemvArgs;
int b2_gemv(const B2GemvArgs* a, b2_stream_t s);

/* Rows to FP16 for the tensor-core GEMM: y16[m][k] = f16(xn[m][k]) for
 * m < M, with xn = x or RMSNorm(x; norm_w, eps) exactly as in b2_gemv's
 * prologue.  y16 is device FP16 (uint16_t bits) with row stride ldy
 * (elements, a multiple of 8). */
int b2_rows_to_f16(uint16_t* y16, int ldy, const float* x, int ldx, int M, int K, const float* norm_w,
                   float eps, b2_stream_t s);

/* Tensor-core GEMM for M > 1 (batch prefill, batched decode, batched
 * lm_head): y[m][n] = epi( s[n] * sum_k x16[m][k] * W[n][k] ) with the
 * epilogues of b2_gemv (SILU_PAIR: rows n and N+n) or ARGMAX (tokens[m] =
 * the first n of the largest acc * s[n]; y, when not NULL, receives the
 * logits).  x16 comes from b2_rows_to_f16; W is FP16, INT8 or INT4 in the
 * device layout above (INT8/INT4 rows are widened exactly to FP16 on chip);
 * the sum runs on the 5th-generation tensor cores (tcgen05.mma, operands
 * staged by TMA, FP32 accumulator in tensor memory), so the numerics equal
 * b2_gemv's up to the FP32 summation order.  Shapes: K a multiple of 64, N a
 * multiple of 128 (any N for ARGMAX), ldx a multiple of 8; x16 and W 16-byte
 * aligned.  ARGMAX needs keys: device scratch of b2_gemm_argmax_keys(M, N)
 * bytes, and tokens: device int[M].  Same role as b2_gemv in the reference
 * map (run_batch_matmul, src/matmul_decoder.c:1841-1899). */
typedef struct {
    float* y;
    int ldy;
    const uint16_t* x16;
    int ldx;
    int M, K, N;
    const void* w;
    const float* scales;
    int wtype;
    int epilogue;
    unsigned long long* keys;
    int* tokens;
    uint16_t* y16; /* STORE / SILU_PAIR: when not NULL, the output as FP16 rows
                      (stride ldy) instead of y, e.g. the next GEMM's x16 */
    int split_k;   /* CTAs (a thread-block cluster) sharing one output tile's K
                      range: 0 = chosen from the grid and SM count, else 1, 2,
                      4 or 8 (<= K / 64) */
} B2GemmArgs;
size_t b2_gemm_argmax_keys(int M, int N);
int b2_gemm(const B2GemmArgs* a, b2_stream_t s);

/* Embedding: for row m, hidden[m] = use_staged && *use_staged ? staged[m]
 * : table[tokens[m]].  tokens, use_staged, staged are device pointers
 * (use_staged/staged may be NULL). */
int b2_embed(float* hidden, const float* table, const int* tokens, const int* use_staged,
             const float* staged, int M, int dim, b2_stream_t s);

/* KV cache addressing: the cache of (sequence q, layer l) starts at
 * base + q * seq_stride + l * layer_stride elements and is laid out
 * [num_kv_heads][max_seq][head_dim] FP16.  rows[m] gives the sequence of
 * row m (NULL = sequence 0) and pos[m] its position.  A row whose position is
 * outside [0, max_seq) or whose sequence is outside [0, n_seqs) is skipped by
 * the kernels (no cache access; its attention output is NaN). */
typedef struct {
    uint16_t* k_base;
    uint16_t* v_base;
    long long seq_stride;
    long long layer_stride;
    int layer;
    int max_seq;
    const int* rows_seq;
    const int* pos;
    int n_seqs;
} B2KVRef;

/* Per-head q/k RMSNorm (q_norm_w/k_norm_w may be NULL), RoPE from tables
 * cos/sin [max_seq][hd/2] at pos[m] (style 0 interleaved, 1 split-half),
 * then K and V of row m stored as FP16 at pos[m].  qkv: device FP32
 * [M][ldqkv] = [q (nq*hd) | k (nkv*hd) | v (nkv*hd)]; q is updated in place. */
int b2_qk_rope_kv(float* qkv, int ldqkv, int M, int nq, int nkv, int hd,
                  const float* q_norm_w, const float* k_norm_w, float eps,
                  const float* cos_tab, const float* sin_tab, int rope_style,
                  const B2KVRef* kv, b2_stream_t s);

/* Causal flash attention of M consecutive rows of one sequence at positions
 * base .. base + M - 1 whose K and V are already stored: row m attends cache
 * positions [0, base + m].  Same inputs and output layout as b2_attention
 * (kv->rows_seq must be NULL, head_dim 128, nq = 2 nkv); scores and P.V run
 * on the tensor cores with FP16 Q and P and FP32 accumulation and softmax.
 * With out16 (not NULL) the output is written as FP16 [M][nq*hd] instead of
 * out: the o_proj GEMM's input rows. */
int b2_attention_prefill(float* out, uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv, int hd,
                         const B2KVRef* kv, int base, b2_stream_t s);

/* GQA attention of row m over cache positions [0, pos[m]] (inclusive).
 * q device FP32 [M][ldq] (first nq*hd), out device FP32 [M][nq*hd].
 * work: device scratch of at least b2_attention_workspace(M, nq, hd, nsplit)
 * bytes; nsplit <= 0 picks a split count. */
size_t b2_attention_workspace(int M, int nq, int hd, int nsplit);
int b2_attention(float* out, const float* q, int ldq, int M, int nq, int nkv, int hd,
                 const B2KVRef* kv, void* work, int nsplit, b2_stream_t s);
/* b2_attention writing FP16 [M][nq*hd] rows (the o_proj GEMM's input). */
int b2_attention_f16(uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv, int hd,
                     const B2KVRef* kv, void* work, int nsplit, b2_stream_t s);

/* b2_attention for many sequences of different lengths: the cache positions
 * [0, max_seq) are cut into fixed blocks of `block` positions (a multiple of
 * 64) and each CTA streams one block of one (row, kv head) into shared memory
 * by TMA, with scores and P.V on the tensor cores (FP16 Q and P, FP32 sums);
 * blocks past a row's pos[m] are empty.  Persistent: two CTAs per SM walk the
 * rows' blocks, so the grid does not depend on the lengths.  M <= 512; strides
 * multiples of 128 elements.  Writes out (FP32)
 * or, when out16 is not NULL, FP16 rows instead.  work: device scratch of
 * b2_attention_workspace(M, nq, hd, b2_attention_blocks_split(max_seq, block))
 * bytes; K and V caches 16-byte aligned.  A bulk copy that does not arrive
 * within the wait limit sets *err (device int) to 1 and leaves its rows
 * unfinished. */
int b2_attention_blocks_split(int max_seq, int block);
int b2_attention_blocks(float* out, uint16_t* out16, const float* q, int ldq, int M, int nq, int nkv, int hd,
                        const B2KVRef* kv, void* work, int block, int* err, b2_stream_t s);

/* lm_head + argmax over V rows of `table` (int8 [V][K] with FP32 scales,
 * F16 [V][K], or F32 [V][K]).  Input row m is RMSNorm(x[m]; norm_w, eps)
 * (norm_w may be NULL), rounded to FP16 for the int8 table (the reference's
 * NPU path) and kept FP32 for the F16/F32 tables (its CPU GEMV path).
 * logits (device, may be NULL) get [M][ldl]; tokens (device int32 [M]) get
 * the first index of the maximum.  work: b2_lm_head_workspace(M, V) bytes. */
size_t b2_lm_head_workspace(int M, int V);
int b2_lm_head_argmax(const float* x, int ldx, int M, int K, int V, const void* table,
                      const float* scales, int wtype, const float* norm_w, float eps,
                      float* logits, int ldl, int* tokens, void* work, b2_stream_t s);

/* No counterpart in the reference.  b2_lm_head_argmax for callers that cannot
 * allocate device memory: code running inside a host that owns all HBM in
 * its own pool, or enqueueing work while another framework captures the
 * stream into a CUDA graph (cudaMalloc is not capturable and may synchronize
 * the device).  Same arguments and results as b2_lm_head_argmax without
 * `work`: the per-CTA argmax keys live in a fixed 1 MiB device array inside
 * this library (b2_lm_head_noalloc_max_keys() keys), which every device that
 * loads the library holds until exit.  Sizes with M x ceil(V / rows per CTA)
 * above that (rows per CTA: 32 int8, 16 F16, 8 F32) are rejected with
 * ERR_INVALID_ARG.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  The looked-up address is cached per device ordinal for the life
 * of the process and belongs to the device's primary context: after
 * cudaDeviceReset (or any other teardown of that context) the cached address
 * is stale, so the entry point must not be called again in that process.
 * All calls on one device share its array and it keeps the last
 * call's contents: calls that may overlap on the GPU (e.g. on two streams of
 * the same device) race and must be serialized by the caller.  Every key a
 * call reads is written by the same call, so nothing needs clearing between
 * calls. */
size_t b2_lm_head_noalloc_max_keys(void);
int b2_lm_head_argmax_noalloc(const float* x, int ldx, int M, int K, int V, const void* table,
                              const float* scales, int wtype, const float* norm_w, float eps,
                              float* logits, int ldl, int* tokens, b2_stream_t s);

/* Vocab-sharded lm_head: keys [M][parts] from b2_gemm(B2_EPI_ARGMAX) over a
 * vocab slice starting at index_offset -> out[M], each row's largest key with
 * its index rewritten as a global vocab index (an all-reduce MAX of these
 * over the ranks gives the global argmax, lowest index on ties). */
int b2_argmax_keys_merge(const unsigned long long* keys, int M, int parts, unsigned index_offset,
                         unsigned long long* out, b2_stream_t s);
/* tokens[i] = vocab index of keys[i], i < n. */
int b2_keys_tokens(const unsigned long long* keys, int n, int* tokens, b2_stream_t s);

/* Token drawn from device logits[V] (FP32) after the lm_head, with the
 * semantics of matmul_sample_token (csrc/host/md_generate.c; the reference's
 * samplers are src/matmul_decoder.c:2316-2323 and src/cpu_ops.c:593-672):
 * repeat_tokens (device, n_repeat entries) penalized once per occurrence,
 * top_k == 1 greedy (first maximum, no temperature), else temperature, the
 * top_k largest (all when top_k <= 0), the top_p prefix of those (top_p in
 * (0, 1)), and a draw with weights exp(v - v_max) from the counter-based
 * generator SplitMix64(seed, counter).  token (device int) gets the draw;
 * info (device int[4], optional) gets [kept entries, K, threshold key, ties
 * kept at the threshold].  One 8-CTA cluster; V <= b2_sample_max_vocab(). */
size_t b2_sample_max_vocab(void);
int b2_sample_token(const float* logits, int V, const int* repeat_tokens, int n_repeat, float repeat_penalty,
                    int top_k, float top_p, float temperature, unsigned long long seed, unsigned long long counter,
                    int* token, int* info, b2_stream_t s);

/* ASR front end (examples/qwen3_asr/mel.py:6-67): the (128, T = n / 160)
 * log-mel spectrogram of a 16 kHz FP32 waveform audio[n] (n > 200), reflect
 * padding, periodic Hann window, 400-point DFT power, mel = filters^T . power
 * with filters [201][128], log10 clamped at its maximum - 8, (x + 4) / 4.
 * out is device FP32 [128][T]; work holds b2_log_mel_workspace(n) bytes. */
size_t b2_log_mel_workspace(int n_samples);
int b2_log_mel(const float* audio, int n_samples, const float* filters, float* out, void* work, b2_stream_t s);
/* Decoder input rows (examples/qwen3_asr/engine.py:255-314): out[total][H] =
 * table rows of prefix_ids, then the audio rows, then table rows of
 * suffix_ids (all device pointers; ids must lie in [0, V)). */
int b2_build_embed(const float* table, int V, int H, const int* prefix_ids, int n_pre, const float* audio,
                   int n_audio, const int* suffix_ids, int n_suf, float* out, b2_stream_t s);

/* Device-side greedy loop bookkeeping, run once per step after the argmax:
 * hist[loop[2]] = loop[0] (the token just produced, which is also the next
 * step's input), then loop[1] (position) and loop[2] (step counter) advance.
 * loop and hist are device int32. */
int b2_loop_advance(int* loop, int* hist, int hist_len, b2_stream_t s);

/* ─── persistent single-token decode (one launch = one token) ───
 * The whole decode step — embedding, every layer, and optionally final norm +
 * INT8 lm_head + argmax — as one cooperative kernel with one CTA per SM.  A
 * producer warp per CTA streams that CTA's weight rows (and K/V positions
 * written by earlier steps) through a shared-memory ring with bulk copies;
 * the other warps compute and order the dependent phases with device-scope
 * acquire/release counters.  Every wait is bounded: on timeout the kernel
 * sets state[B2_MK_ERR], drains its copies and returns.
 *
 * Device state block (int32): */
enum {
    B2_MK_TOKEN = 0,     /* in: token id of this step (ignored when USE_EMB) */
    B2_MK_POS = 1,       /* in/out: position; +1 per completed step          */
    B2_MK_STEP = 2,      /* in/out: step counter (index into hist)           */
    B2_MK_USE_EMB = 3,   /* in: 1 = take the input row from staged_emb       */
    B2_MK_ERR = 4,       /* out: nonzero after a timed-out wait              */
    B2_MK_TOKEN_OUT = 5, /* out: argmax of this step (also written to TOKEN) */
    B2_MK_GEN = 6,       /* device-owned generation count; host leaves it    */
    B2_MK_STATE_INTS = 16
};
#define B2_MK_MAX_LAYERS 48

typedef struct {
    const void* qkv;       /* [nq*hd + 2*nkv*hd][hidden] rows               */
    const float* qkv_s;
    const void* o;         /* [hidden][nq*hd]                               */
    const float* o_s;
    const void* gu;        /* [2*ffn][hidden]: gate rows then up rows       */
    const float* gu_s;
    const void* dn;        /* [hidden][ffn]                                 */
    const float* dn_s;
    const float* in_norm;
    const float* post_norm;
    const float* q_norm;   /* NULL when the model has no q/k norm           */
    const float* k_norm;
    const void* dn_t;      /* down_proj by input channel: [ffn][hidden]
                              (FP16 / int8, or int4 [ffn][hidden/2] with
                              the even output column in the low nibble);
                              scales are dn_s                               */
    /* Tile-major copies read by b2_mk2_decode (b2_tile_relayout of the row
     * arrays above): 16-row tiles, each stored as [64-byte super-block][16
     * rows][64 bytes], so one tile is one contiguous block whose shared-memory
     * image the tensor-core row dots read without bank conflicts. */
    const void* qkv_t;     /* tiles of the qkv rows                         */
    const void* o_t;       /* tiles of the o rows                           */
    const void* gu_t;      /* tiles of 8 channels: rows gate(c), up(c), ... */
    const float* gu_ts;    /* per-row scales of gu_t (interleaved), or NULL */
} B2MkLayer;

typedef struct {
    int n_layers, hidden, nq, nkv, hd, ffn, vocab, max_seq, rope_style, wtype;
    float eps;
    const float* emb;          /* [vocab][hidden] FP32                        */
    const void* lm;            /* [vocab][hidden] int8                        */
    const float* lm_s;
    const float* final_norm;
    const float* cos_tab;      /* [max_seq][hd/2]                             */
    const float* sin_tab;
    uint16_t* k_cache;         /* [layer][nkv][max_seq][hd] FP16              */
    uint16_t* v_cache;
    long long layer_stride;    /* elements per layer of k_cache / v_cache     */
    int* state;                /* B2_MK_STATE_INTS ints                       */
    const float* staged_emb;   /* [hidden] input row when USE_EMB             */
    float* logits;             /* [vocab] or NULL                             */
    int* hist;                 /* tokens by step (device loop), or NULL       */
    int hist_len;
    int do_lm;                 /* 0 = prefill-mode step (no final norm/lm_head) */
    void* scratch;             /* b2_mk_scratch_bytes() bytes, zeroed once    */
    const B2MkLayer* layers;   /* device array [n_layers] (kept off the kernel
                                  parameter block, which stays small)         */
    const void* lm_t;          /* tile-major int8 lm_head (b2_mk2_decode)      */
    long long poll_limit;      /* polls before a wait gives up (0: default)   */
    int stall_test;            /* 1: the lm_head phase waits for a flag value
                                  that never comes (tests the timed-out-wait
                                  path of b2_mk2_decode)                      */
} B2MkPlan;

/* 0 when the plan's shapes are supported by the persistent kernel. */
int b2_mk_check(const B2MkPlan* plan);
size_t b2_mk_scratch_bytes(int n_layers, int hidden, int ffn, int nq, int nkv, int hd);
int b2_mk_decode(const B2MkPlan* plan, b2_stream_t s);
/* Device address of the residual stream after the last layer of the most
 * recent step (inside plan->scratch). */
float* b2_mk_final_hidden(const B2MkPlan* plan);
/* Dynamic shared memory of one CTA of the persistent kernel. */
size_t b2_mk_smem_bytes(void);

/* Second-generation persistent decode kernel (same plan, same state block
 * layout; give it its own state block and scratch).  One producer thread per
 * CTA turns the CTA's share of the token into a stream of operations in
 * shared memory: data operations carry a block of tile-major weight rows (or
 * K/V positions) copied in by bulk copies, control operations stage the input
 * of the next phase.  The consumer warps take the stream in order and split
 * every 16-row tile's dot products over their K ranges.  Attention and o_proj
 * run fused per (kv head, row slice) unit: up to 240 cached positions every
 * unit attends over all of the head's positions; beyond, 16 units per kv head
 * split them and publish partial softmax states that every unit of the head
 * merges.  The host routes contexts up to b2_mk2_max_context() cached
 * positions here (any length the cache holds). */
int b2_mk2_check(const B2MkPlan* plan);
int b2_mk2_max_context(void);
size_t b2_mk2_scratch_bytes(int n_layers, int hidden, int ffn, int nq, int nkv, int hd);
int b2_mk2_decode(const B2MkPlan* plan, b2_stream_t s);
float* b2_mk2_final_hidden(const B2MkPlan* plan);

/* Tile-major relayout (one-time, at load): dst gets rows [0, rows) of the
 * row-major src (row_bytes per row; rows % 16 == 0, row_bytes % 64 == 0) as
 * 16-row tiles [row_bytes/64][16][64 bytes].  pair_half > 0 interleaves two
 * halves of src: tile t row 2j is src row 8t + j and row 2j+1 is src row
 * pair_half + 8t + j (gate and up of one channel).  When src_s is non-NULL,
 * dst_s[r] = src_s[source row of r]. */
int b2_tile_relayout(void* dst, const void* src, int rows, int row_bytes, int pair_half, float* dst_s,
                     const float* src_s, b2_stream_t s);

#ifdef __cplusplus
}
#endif
#endif
