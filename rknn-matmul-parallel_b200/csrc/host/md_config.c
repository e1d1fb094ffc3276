/*
 * config.json parsing (matmul_decoder_load_config).
 *
 * Follows the reference scanner (src/matmul_decoder.c:2182-2312): defaults
 * from the Qwen3-0.6B preset, then every "key": value pair whose key is known
 * overrides the default.  Keys: hidden_dim, num_q_heads, num_kv_heads,
 * head_dim, ffn_dim, num_layers, vocab_size, max_seq_len, rms_eps, rope_theta,
 * has_qk_norm (number or boolean), tie_word_embeddings (boolean).  Additions:
 * rope_style is parsed (the reference never sets it, leaving interleaved RoPE),
 * numbers may carry an exponent (the reference reads "1e-06" as 1), and keys
 * match exactly rather than by prefix.
 */
#include <ctype.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "md_internal.h"

void md_config_defaults(MatmulDecoderConfig* c) { *c = matmul_decoder_config_qwen3_0_6b(); }

int md_config_validate(const MatmulDecoderConfig* c) {
    if (c->hidden_dim <= 0 || c->num_q_heads <= 0 || c->num_kv_heads <= 0 || c->head_dim <= 0 ||
        c->ffn_dim <= 0 || c->num_layers <= 0 || c->vocab_size <= 0)
        return MATMUL_DECODER_ERR_INVALID_ARG;
    if (c->num_q_heads % c->num_kv_heads != 0) return MATMUL_DECODER_ERR_INVALID_ARG;
    if (c->head_dim != 128) return MATMUL_DECODER_ERR_UNSUPPORTED;
    if (c->hidden_dim % 32 != 0 || c->ffn_dim % 32 != 0) return MATMUL_DECODER_ERR_UNSUPPORTED;
    if (c->norm_type != 0 || c->ffn_act_type != 0) return MATMUL_DECODER_ERR_UNSUPPORTED;
    return MATMUL_DECODER_OK;
}

static int key_is(const char* k, size_t n, const char* want) {
    return strlen(want) == n && strncmp(k, want, n) == 0;
}

int matmul_decoder_load_config(const char* json_path, MatmulDecoderConfig* config) {
    if (!json_path || !config) return MATMUL_DECODER_ERR_INVALID_ARG;
    FILE* f = fopen(json_path, "rb");
    if (!f) {
        MD_LOG("Cannot open config: %s\n", json_path);
        return MATMUL_DECODER_ERR_FILE_IO;
    }
    fseek(f, 0, SEEK_END);
    long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (size < 0) {
        fclose(f);
        return MATMUL_DECODER_ERR_FILE_IO;
    }
    char* buf = (char*)malloc((size_t)size + 1);
    if (!buf) {
        fclose(f);
        return MATMUL_DECODER_ERR_MEMORY;
    }
    size_t got = fread(buf, 1, (size_t)size, f);
    buf[got] = '\0';
    fclose(f);

    md_config_defaults(config);
    char* p = buf;
    while (*p) {
        if (*p != '"') {
            p++;
            continue;
        }
        char* key = ++p;
        while (*p && *p != '"') p++;
        if (!*p) break;
        size_t klen = (size_t)(p - key);
        p++;
        while (*p && isspace((unsigned char)*p)) p++;
        if (*p != ':') continue; /* a string value, not a key */
        p++;
        while (*p && isspace((unsigned char)*p)) p++;
        if (*p == '"') { /* string value: skip */
            p++;
            while (*p && *p != '"') p++;
            if (*p) p++;
            continue;
        }
        if (*p == 't' || *p == 'f') {
            int v = (*p == 't');
            if (key_is(key, klen, "tie_word_embeddings")) config->tie_word_embeddings = v;
            else if (key_is(key, klen, "has_qk_norm")) config->has_qk_norm = v;
            p += v ? 4 : 5;
            continue;
        }
        if (*p == '-' || *p == '+' || *p == '.' || isdigit((unsigned char)*p)) {
            char* end = NULL;
            double d = strtod(p, &end);
            if (end == p) {
                p++;
                continue;
            }
            p = end;
            int iv = (int)d;
            if (key_is(key, klen, "hidden_dim")) config->hidden_dim = iv;
            else if (key_is(key, klen, "num_q_heads")) config->num_q_heads = iv;
            else if (key_is(key, klen, "num_kv_heads")) config->num_kv_heads = iv;
            else if (key_is(key, klen, "head_dim")) config->head_dim = iv;
            else if (key_is(key, klen, "ffn_dim")) config->ffn_dim = iv;
            else if (key_is(key, klen, "num_layers")) config->num_layers = iv;
            else if (key_is(key, klen, "vocab_size")) config->vocab_size = iv;
            else if (key_is(key, klen, "max_seq_len")) config->max_seq_len = iv;
            else if (key_is(key, klen, "rms_eps")) config->rms_eps = (float)d;
            else if (key_is(key, klen, "rope_theta")) config->rope_theta = (float)d;
            else if (key_is(key, klen, "has_qk_norm")) config->has_qk_norm = iv;
            else if (key_is(key, klen, "rope_style")) config->rope_style = iv;
            else if (key_is(key, klen, "num_lm_heads")) config->num_lm_heads = iv;
            else if (key_is(key, klen, "lm_head_vocab_size")) config->lm_head_vocab_size = iv;
            continue;
        }
    }
    free(buf);
    printf("[MatmulDecoder] Loaded config: hidden=%d, layers=%d, heads=%d/%d, vocab=%d, rope_style=%d\n",
           config->hidden_dim, config->num_layers, config->num_q_heads, config->num_kv_heads,
           config->vocab_size, config->rope_style);
    return MATMUL_DECODER_OK;
}

int matmul_decoder_export_hf_model(const char* hf_model_path, const char* output_dir,
                                   QuantizationType quant_type) {
    (void)hf_model_path;
    (void)output_dir;
    (void)quant_type;
    MD_LOG("export_hf_model is not provided by this runtime; write the .bin layout with the "
           "Python model_format tool\n");
    return MATMUL_DECODER_ERR_UNSUPPORTED;
}
