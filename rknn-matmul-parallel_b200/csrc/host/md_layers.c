/*
 * One pass of M rows through every layer, as a sequence of fused kernels on
 * one stream (captured into a CUDA graph by the callers).
 *
 * Per layer this is the body of matmul_decoder_step / prefill_batch
 * (src/matmul_decoder.c:1464-1546, :1970-2061) regrouped into five kernels
 * plus the attention combine:
 *   1. RMSNorm(input_norm) + fused q|k|v GEMV                       (b2_gemv)
 *   2. per-head q/k RMSNorm + RoPE + K/V store at pos              (b2_qk_rope_kv)
 *   3. GQA attention over [0, pos] (split-KV + combine)            (b2_attention;
 *      causal flash attention b2_attention_prefill for prefill rows)
 *   4. o_proj GEMV + residual add into hidden                       (b2_gemv ADD)
 *   5. RMSNorm(post_attn_norm) + gate|up GEMV + SiLU*mul            (b2_gemv SILU_PAIR)
 *   6. down GEMV + residual add into hidden                         (b2_gemv ADD)
 * With M >= MD_GEMM_MIN_ROWS rows, steps 1, 4, 5 and 6 run
 * as b2_rows_to_f16 (RMSNorm + FP16 rounding) + b2_gemm (tcgen05 tensor cores).
 * K/V of the current rows are stored before attention for decode and
 * prefill alike; the reference stores them after attention in prefill
 * (:2026-2034) but reads the same values from its batch buffers, so the
 * attended set is identical.
 */
#include <stdio.h>
#include <stdlib.h>

#include "md_internal.h"

/* Rows from which a matmul runs on the tensor cores (b2_rows_to_f16 +
 * b2_gemm) instead of the GEMV; B2_PREFILL_GEMM=0 keeps every M on the GEMV. */
#define MD_GEMM_MIN_ROWS 16

static int gemm_enabled(void) {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("B2_PREFILL_GEMM");
        v = !(e && e[0] == '0');
    }
    return v;
}

/* Whether an [M] x K -> N matmul with this weight type runs on the tensor cores. */
static int on_tensor_cores(const LayerBuffers* b, int M, int wtype, int K, int N) {
    return b->x16 && M >= MD_GEMM_MIN_ROWS && wtype != B2_W_F32 && K % 64 == 0 && N % 128 == 0 &&
           gemm_enabled();
}

/* One matmul of the layer: the GEMV, or for M >= MD_GEMM_MIN_ROWS rows the
 * same operation on the tensor cores (FP16, INT8 or INT4 weights).  On the
 * tensor cores the input comes from x16_in (FP16 rows of stride K, written
 * by the previous kernel) when given, else from a->x through b2_rows_to_f16;
 * with y16 the output is written as FP16 rows of stride a->ldy instead of
 * a->y (the next matmul's input). */
static int linear(const LayerBuffers* b, const B2GemvArgs* a, const uint16_t* x16_in, uint16_t* y16,
                  b2_stream_t s) {
    if (on_tensor_cores(b, a->M, a->wtype, a->K, a->N)) {
        const uint16_t* x16 = x16_in;
        if (!x16) {
            int rc = b2_rows_to_f16(b->x16, a->K, a->x, a->ldx, a->M, a->K, a->norm_w, a->eps, s);
            if (rc) return rc;
            x16 = b->x16;
        }
        B2GemmArgs g = {y16 ? NULL : a->y, a->ldy, x16, a->K, a->M, a->K, a->N, a->w, a->scales, a->wtype,
                        a->epilogue, NULL, NULL, y16, 0};
        return b2_gemm(&g, s);
    }
    return b2_gemv(a, s);
}

int md_enqueue_layers(const DevModel* m, const LayerBuffers* b, int M, const B2KVRef* kv_proto,
                      b2_stream_t s) {
    const MatmulDecoderConfig* c = &m->cfg;
    const int H = c->hidden_dim, hd = c->head_dim, nq = c->num_q_heads, nkv = c->num_kv_heads;
    const int qd = nq * hd, kvd = nkv * hd, F = c->ffn_dim, ldqkv = qd + 2 * kvd;
    for (int l = 0; l < c->num_layers; l++) {
        const DevLayer* L = &m->layers[l];
        B2GemvArgs a = {b->qkv, ldqkv, b->hidden, H, M, H, ldqkv, L->qkv.w, L->qkv.s, L->qkv.wtype,
                        L->in_norm, c->rms_eps, B2_EPI_STORE};
        int rc = linear(b, &a, NULL, NULL, s);
        if (rc) return rc;
        B2KVRef kv = *kv_proto;
        kv.layer = l;
        const int qk = c->has_qk_norm && L->q_norm && L->k_norm;
        rc = b2_qk_rope_kv(b->qkv, ldqkv, M, nq, nkv, hd, qk ? L->q_norm : NULL, qk ? L->k_norm : NULL,
                           c->rms_eps, m->cos_tab, m->sin_tab, c->rope_style, &kv, s);
        if (rc) return rc;
        /* When o_proj runs on the tensor cores, attention writes its FP16
         * input rows directly (the rounding b2_rows_to_f16 would apply). */
        const int o_tc = on_tensor_cores(b, M, L->o.wtype, qd, H);
        float* attn32 = o_tc ? NULL : b->attn;
        uint16_t* attn16 = o_tc ? b->x16 : NULL;
        if (b->prefill_base >= 0 && M >= MD_GEMM_MIN_ROWS && nq == 2 * nkv && hd == 128 && !kv.rows_seq)
            rc = b2_attention_prefill(attn32, attn16, b->qkv, ldqkv, M, nq, nkv, hd, &kv, b->prefill_base, s);
        else if (b->attn_block > 0)
            rc = b2_attention_blocks(attn32, attn16, b->qkv, ldqkv, M, nq, nkv, hd, &kv, b->attn_work, b->attn_block,
                                     b->attn_err, s);
        else if (o_tc)
            rc = b2_attention_f16(attn16, b->qkv, ldqkv, M, nq, nkv, hd, &kv, b->attn_work, b->attn_split, s);
        else
            rc = b2_attention(b->attn, b->qkv, ldqkv, M, nq, nkv, hd, &kv, b->attn_work, b->attn_split, s);
        if (rc) return rc;
        B2GemvArgs o = {b->hidden, H, b->attn, qd, M, qd, H, L->o.w, L->o.s, L->o.wtype, NULL, 0.f,
                        B2_EPI_ADD};
        rc = linear(b, &o, attn16, NULL, s);
        if (rc) return rc;
        /* gate|up writes the down projection's FP16 input when both run on
         * the tensor cores. */
        const int dn_tc = b->x16b && on_tensor_cores(b, M, L->gu.wtype, H, F) &&
                          on_tensor_cores(b, M, L->down.wtype, F, H);
        B2GemvArgs gu = {b->act, F, b->hidden, H, M, H, F, L->gu.w, L->gu.s, L->gu.wtype, L->post_norm,
                         c->rms_eps, B2_EPI_SILU_PAIR};
        rc = linear(b, &gu, NULL, dn_tc ? b->x16b : NULL, s);
        if (rc) return rc;
        B2GemvArgs dn = {b->hidden, H, b->act, F, M, F, H, L->down.w, L->down.s, L->down.wtype, NULL, 0.f,
                         B2_EPI_ADD};
        rc = linear(b, &dn, dn_tc ? b->x16b : NULL, NULL, s);
        if (rc) return rc;
    }
    return 0;
}
