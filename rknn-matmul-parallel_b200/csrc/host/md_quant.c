/*
 * Host quantisers (bit-exact).
 *
 * The reference quantises only its lm_head (src/matmul_decoder.c:1216-1244):
 * per output column, max = max|w| over the FP16 values, scale = max / 127.0f,
 * inv = max > 0 ? 127.0f / max : 0, q = clamp((int)roundf(w * inv), -128, 127).
 * Layer weights arrive pre-quantized on disk ({proj}_weight.bin +
 * {proj}_scales.bin, :763-796), with no tool in the reference to write them;
 * md_quantize_cols applies the same rule to an FP16 [K][N] matrix so the
 * runtime and the model_format tool produce those files.  INT4 uses qmax = 7,
 * range [-8, 7], and a scale rounded to FP16 (stored as FP32); two columns
 * per byte, the even column in the low nibble.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "md_internal.h"

uint16_t md_f32_to_f16(float x) {
    _Float16 h = (_Float16)x;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

float md_f16_to_f32(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

void md_quantize_cols(const uint16_t* w, int K, int N, int bits, uint8_t* q, float* scales) {
    const float qmax = bits == 8 ? 127.0f : 7.0f;
    const int lo = bits == 8 ? -128 : -8, hi = bits == 8 ? 127 : 7;
    float* mx = (float*)calloc((size_t)N, sizeof(float));
    float* inv = (float*)malloc((size_t)N * sizeof(float));
    if (bits == 4) memset(q, 0, (size_t)K * (size_t)(N / 2));
    /* Two row-major sweeps (the column maxima, then the values) instead of a
     * column walk: the same per-column rule, cache-friendly on [K][N]. */
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) {
            float v = fabsf(md_f16_to_f32(w[(size_t)k * N + n]));
            if (v > mx[n]) mx[n] = v;
        }
    for (int n = 0; n < N; n++) {
        float sc = mx[n] / qmax;
        if (bits == 4) sc = md_f16_to_f32(md_f32_to_f16(sc));
        scales[n] = sc;
        inv[n] = (mx[n] > 0) ? qmax / mx[n] : 0;
    }
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) {
            int v = (int)roundf(md_f16_to_f32(w[(size_t)k * N + n]) * inv[n]);
            if (v < lo) v = lo;
            if (v > hi) v = hi;
            if (bits == 8) {
                q[(size_t)k * N + n] = (uint8_t)(int8_t)v;
            } else {
                uint8_t nib = (uint8_t)(v & 15);
                q[(size_t)k * (N / 2) + n / 2] |= (n & 1) ? (uint8_t)(nib << 4) : nib;
            }
        }
    free(mx);
    free(inv);
}

/* lm_head: the same rule applied to each vocab row of the FP16 [V][K] table
 * (a row of the table is a column of the reference's transposed tiles). */
void md_quantize_rows_i8(const uint16_t* t, int V, int K, int8_t* q, float* scales) {
    for (int v = 0; v < V; v++) {
        const uint16_t* row = t + (size_t)v * K;
        float mx = 0.f;
        for (int k = 0; k < K; k++) {
            float a = fabsf(md_f16_to_f32(row[k]));
            if (a > mx) mx = a;
        }
        scales[v] = mx / 127.0f;
        const float inv = (mx > 0) ? 127.0f / mx : 0;
        for (int k = 0; k < K; k++) {
            int x = (int)roundf(md_f16_to_f32(row[k]) * inv);
            if (x < -128) x = -128;
            if (x > 127) x = 127;
            q[(size_t)v * K + k] = (int8_t)x;
        }
    }
}

int matmul_decoder_quantize_weight(const uint16_t* w_fp16, int K, int N, int bits, uint8_t* q_out,
                                   float* scales_out) {
    if (!w_fp16 || !q_out || !scales_out || K <= 0 || N <= 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (bits != 8 && bits != 4) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (bits == 4 && (N % 2) != 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    md_quantize_cols(w_fp16, K, N, bits, q_out, scales_out);
    return MATMUL_DECODER_OK;
}

int matmul_decoder_quantize_lm_head(const float* table, int V, int K, int8_t* q_out, float* scales_out) {
    if (!table || !q_out || !scales_out || V <= 0 || K <= 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    uint16_t* t16 = (uint16_t*)malloc((size_t)V * K * 2);
    if (!t16) return MATMUL_DECODER_ERR_MEMORY;
    for (size_t i = 0; i < (size_t)V * K; i++) t16[i] = md_f32_to_f16(table[i]);
    md_quantize_rows_i8(t16, V, K, q_out, scales_out);
    free(t16);
    return MATMUL_DECODER_OK;
}
