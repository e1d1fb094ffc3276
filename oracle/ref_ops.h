/*
 * ref_ops.h — CPU ORACLE (test infrastructure, never the product).
 *
 * Scalar C restatement of the reference decoder's arithmetic:
 *   - src/cpu_ops.c (RMSNorm, RoPE, attention, SiLU*mul, vec add, argmax,
 *     batch causal attention) of suharvest/rknn-matmul-parallel;
 *   - src/matmul_decoder.c run_persistent_matmul / run_batch_matmul semantics
 *     (input rounded FP32->FP16 round-to-nearest-even, FP32 accumulation of
 *     FP16/INT8/INT4 weight products, FP32 per-column scale applied after),
 *     the INT8 lm_head quantiser and 4096-column tiling, the RoPE table
 *     formula and the per-layer step order.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 * Weight layouts are the reference's on-disk layouts: FP16 [K][N], int8
 * [K][N], int4 [K][N/2] (low nibble = even column, two's complement).
 */
#ifndef REF_OPS_H
#define REF_OPS_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { REF_W_F16 = 0, REF_W_I8 = 1, REF_W_I4 = 2 };

uint16_t ref_f32_to_f16(float x);
float ref_f16_to_f32(uint16_t h);
void ref_vec_f32_to_f16(uint16_t* dst, const float* src, int n);
void ref_vec_f16_to_f32(float* dst, const uint16_t* src, int n);

void ref_rms_norm(float* out, const float* x, const float* w, int dim, float eps);
void ref_rope_tables(float* cos_tab, float* sin_tab, int max_seq, int head_dim, float theta);
void ref_apply_rope(float* x, const float* cos_row, const float* sin_row,
                    int num_heads, int head_dim, int style);
void ref_attention(float* out, const float* q, const float* k_cache, const float* v_cache,
                   int num_q_heads, int num_kv_heads, int head_dim, int seq_len);
void ref_attention_batch_causal(float* out, const float* q, const float* kb, const float* vb,
                                const float* k_cache, const float* v_cache, int M,
                                int num_q_heads, int num_kv_heads, int head_dim, int cache_len);
void ref_silu_mul(float* out, const float* gate, const float* up, int n);
void ref_vec_add(float* dst, const float* src, int n);
int ref_argmax(const float* x, int n);

/* Y[M][N] = scale[n] * sum_k f16(X[m][k]) * W[k][n]; nthreads >= 1 splits N. */
void ref_gemm(float* Y, const float* X, int M, const void* W, const float* scales,
              int K, int N, int wtype, int nthreads);

/* Per-column symmetric quantiser on an FP16 [K][N] matrix.  bits = 8:
 * scale = max/127, q = clamp(roundf(w*127/max), -128, 127) stored int8 [K][N].
 * bits = 4: scale = fp16(max/7) stored FP32, q = clamp(roundf(w*7/max), -8, 7)
 * packed [K][N/2]. */
void ref_quantize_cols(const uint16_t* w_kn, int K, int N, int bits,
                       uint8_t* q_out, float* scales_out);

/* INT8 lm_head from the FP16 [V][K] table, tiled 4096 columns per tile with
 * zero padding: q_out [n_tiles][K][tile_n] int8, scales_out [n_tiles*tile_n]. */
void ref_quantize_lm_head(const uint16_t* table_vk, int V, int K, int tile_n,
                          int8_t* q_out, float* scales_out);
/* logits[v] = scale[v] * sum_k f16(x[k]) * q[tile][k][col]; only V logits. */
void ref_lm_head_int8(float* logits, const float* x, const int8_t* q_tiles,
                      const float* scales, int K, int V, int tile_n, int nthreads);
/* CPU fallback lm_head: FP32 x times FP16 table rows [V][K] (no input rounding). */
void ref_lm_head_f16(float* logits, const float* x, const uint16_t* table_vk, int V, int K,
                     int nthreads);
/* Multi-head lm_head: FP32 x times FP32 rows [V][K]. */
void ref_lm_head_f32(float* logits, const float* x, const float* table_vk, int V, int K);

typedef struct {
    int hidden, nq, nkv, hd, ffn, max_seq, rope_style, has_qk_norm, wtype;
    float eps;
} RefDims;

typedef struct {
    const void* w[7];       /* q k v o gate up down, on-disk layouts */
    const float* s[7];      /* per-column scales or NULL */
    const float* in_norm;
    const float* post_norm;
    const float* q_norm;
    const float* k_norm;
} RefLayer;

/* One layer of matmul_decoder_step for one token at position pos.  hidden is
 * updated in place; k/v for pos are written into k_cache/v_cache (FP32
 * [max_seq][nkv][hd]) before attention over [0, pos]. */
void ref_layer_decode(float* hidden, const RefLayer* L, const RefDims* d,
                      float* k_cache, float* v_cache, int pos,
                      const float* cos_tab, const float* sin_tab, int nthreads);

/* One layer of matmul_decoder_prefill_batch for M tokens at positions
 * [start, start+M): attention over cache [0,start) plus batch [0..t], then
 * the batch K/V are stored. */
void ref_layer_prefill(float* hidden, int M, const RefLayer* L, const RefDims* d,
                       float* k_cache, float* v_cache, int start,
                       float theta, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
