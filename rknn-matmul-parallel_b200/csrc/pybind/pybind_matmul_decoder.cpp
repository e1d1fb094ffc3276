// Python module `matmul_decoder` over the C API of libmatmul_decoder.so.
//
// Same module name, class, method names, keyword arguments and defaults as
// the reference binding (src/pybind_matmul_decoder.cpp:294-386 of
// suharvest/rknn-matmul-parallel): MatmulDecoder(model_dir, max_seq_len=4096,
// quant_type="int4", exec_mode="dual_core", disable_npu_lm_head=False) with
// step / prefill / prefill_batch / step_get_token / clear_kv_cache / generate
// and read-only seq_len, config, stats; config_qwen3_0_6b[_single_core]();
// __version__ "1.0.0".  Differences: step() raises on an error code instead
// of returning an unfilled array, step_get_token() does not copy logits to
// the host (only the token id returns), and generate() feeds every produced
// token back (the reference passes token -1, :266).  Additive members:
// step_head, set_kv / get_kv, set_seq_len, hidden, and class BatchDecoder.
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "matmul_decoder.h"

namespace py = pybind11;
using farr = py::array_t<float, py::array::c_style | py::array::forcecast>;
using harr = py::array_t<uint16_t, py::array::c_style | py::array::forcecast>;

static QuantizationType parse_quant(const std::string& q) {
    if (q == "fp16") return QUANT_FP16;
    if (q == "int8") return QUANT_INT8;
    if (q == "int4_g128") return QUANT_INT4_G128;
    return QUANT_INT4;
}

static py::dict config_dict(const MatmulDecoderConfig& c) {
    return py::dict(py::arg("name") = std::string(c.name ? c.name : ""), py::arg("hidden_dim") = c.hidden_dim,
                    py::arg("num_q_heads") = c.num_q_heads, py::arg("num_kv_heads") = c.num_kv_heads,
                    py::arg("head_dim") = c.head_dim, py::arg("ffn_dim") = c.ffn_dim,
                    py::arg("num_layers") = c.num_layers, py::arg("vocab_size") = c.vocab_size,
                    py::arg("max_seq_len") = c.max_seq_len, py::arg("rms_eps") = c.rms_eps,
                    py::arg("rope_theta") = c.rope_theta, py::arg("tie_word_embeddings") = c.tie_word_embeddings,
                    py::arg("has_qk_norm") = c.has_qk_norm, py::arg("rope_style") = c.rope_style,
                    py::arg("exec_mode") = (c.exec_mode == EXEC_DUAL_CORE) ? "dual_core" : "single_core");
}

static py::dict stats_dict(const MatmulDecoderStats& s) {
    return py::dict(py::arg("total_ms") = s.total_ms, py::arg("matmul_ms") = s.matmul_ms,
                    py::arg("rebind_ms") = s.rebind_ms, py::arg("convert_ms") = s.convert_ms,
                    py::arg("cpu_ops_ms") = s.cpu_ops_ms, py::arg("lm_head_ms") = s.lm_head_ms,
                    py::arg("n_steps") = s.n_steps);
}

class PyMatmulDecoder {
   public:
    PyMatmulDecoder(const std::string& model_dir, int max_seq_len, const std::string& quant_type,
                    const std::string& exec_mode, bool disable_npu_lm_head) {
        MatmulDecoderConfig cfg;
        if (matmul_decoder_load_config((model_dir + "/config.json").c_str(), &cfg) != 0)
            throw std::runtime_error("Failed to load config.json from " + model_dir);
        cfg.exec_mode = exec_mode == "single_core" ? EXEC_SINGLE_CORE : EXEC_DUAL_CORE;
        cfg.max_seq_len = max_seq_len;
        cfg.disable_npu_lm_head = disable_npu_lm_head ? 1 : 0;
        {
            py::gil_scoped_release nogil;
            ctx_ = matmul_decoder_create(model_dir.c_str(), &cfg, parse_quant(quant_type), max_seq_len);
        }
        if (!ctx_) throw std::runtime_error("Failed to create MatmulDecoder from " + model_dir);
        cfg_ = *matmul_decoder_get_config(ctx_);
    }
    ~PyMatmulDecoder() {
        if (ctx_) matmul_decoder_destroy(ctx_);
    }

    const float* emb_ptr(py::object embedding, farr& keep) {
        if (embedding.is_none()) return nullptr;
        keep = embedding.cast<farr>();
        if (keep.size() != cfg_.hidden_dim)
            throw std::invalid_argument("embedding must have hidden_dim elements");
        return keep.data();
    }

    py::array_t<float> step(int token_id, py::object embedding) {
        farr keep;
        const float* e = emb_ptr(embedding, keep);
        py::array_t<float> logits(cfg_.vocab_size);
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = matmul_decoder_step(ctx_, token_id, e, logits.mutable_data());
        }
        if (rc < 0) throw std::runtime_error("step failed with error code " + std::to_string(rc));
        return logits;
    }

    void prefill_batch(farr embeddings) {
        py::buffer_info b = embeddings.request();
        if (b.ndim != 2) throw std::runtime_error("prefill_batch: embeddings must be 2D [M, hidden_dim]");
        if (b.shape[1] != cfg_.hidden_dim) throw std::runtime_error("prefill_batch: second dim must be hidden_dim");
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = matmul_decoder_prefill_batch(ctx_, embeddings.data(), (int)b.shape[0]);
        }
        if (rc != 0) throw std::runtime_error("prefill_batch failed with error code " + std::to_string(rc));
    }

    void prefill(int token_id, py::object embedding) {
        if (!embedding.is_none()) {
            farr arr = embedding.cast<farr>();
            if (arr.ndim() == 2) {
                prefill_batch(arr);
                return;
            }
        }
        farr keep;
        const float* e = emb_ptr(embedding, keep);
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = matmul_decoder_step(ctx_, token_id, e, nullptr);
        }
        if (rc < 0) throw std::runtime_error("prefill failed with error code " + std::to_string(rc));
    }

    int step_get_token(int token_id, py::object embedding) {
        farr keep;
        const float* e = emb_ptr(embedding, keep);
        py::gil_scoped_release nogil;
        return matmul_decoder_step_token(ctx_, token_id, e);
    }

    int step_head(int token_id, py::object embedding, int lm_head_idx) {
        farr keep;
        const float* e = emb_ptr(embedding, keep);
        py::gil_scoped_release nogil;
        return matmul_decoder_step_head(ctx_, token_id, e, lm_head_idx, nullptr);
    }

    void clear_kv_cache() { matmul_decoder_clear_kv_cache(ctx_); }
    int seq_len() const { return matmul_decoder_get_seq_len(ctx_); }
    py::dict config() const { return config_dict(cfg_); }
    py::dict stats() const {
        MatmulDecoderStats s{};
        matmul_decoder_get_stats(ctx_, &s);
        return stats_dict(s);
    }

    void set_seq_len(int n) {
        if (matmul_decoder_set_seq_len(ctx_, n) != 0) throw std::invalid_argument("set_seq_len: out of range");
    }

    void set_kv(int layer, int start, harr k, harr v) {
        const py::ssize_t per = (py::ssize_t)cfg_.num_kv_heads * cfg_.head_dim;
        if (k.size() != v.size() || k.size() % per != 0) throw std::invalid_argument("set_kv: shape mismatch");
        int rc = matmul_decoder_set_kv(ctx_, layer, start, (int)(k.size() / per), k.data(), v.data());
        if (rc != 0) throw std::runtime_error("set_kv failed with error code " + std::to_string(rc));
    }

    py::tuple get_kv(int layer, int start, int len) {
        py::array_t<uint16_t> k({len, cfg_.num_kv_heads, cfg_.head_dim});
        py::array_t<uint16_t> v({len, cfg_.num_kv_heads, cfg_.head_dim});
        int rc = matmul_decoder_get_kv(ctx_, layer, start, len, k.mutable_data(), v.mutable_data());
        if (rc != 0) throw std::runtime_error("get_kv failed with error code " + std::to_string(rc));
        return py::make_tuple(k, v);
    }

    py::array_t<float> hidden() {
        py::array_t<float> h(cfg_.hidden_dim);
        if (matmul_decoder_get_hidden(ctx_, h.mutable_data()) != 0) throw std::runtime_error("get_hidden failed");
        return h;
    }

    std::vector<int> generate(const std::vector<int>& prompt_tokens, int max_new_tokens, int top_k, float top_p,
                              float temperature, float repeat_penalty, py::object callback) {
        if (prompt_tokens.empty()) throw std::invalid_argument("generate: empty prompt");
        std::vector<int> out;
        std::vector<int> history(prompt_tokens);
        SamplingParams p = sampling_params_greedy();
        p.top_k = top_k;
        p.top_p = top_p;
        p.temperature = temperature;
        p.repeat_penalty = repeat_penalty;
        for (size_t i = 0; i + 1 < prompt_tokens.size(); i++) {
            int rc = matmul_decoder_step(ctx_, prompt_tokens[i], nullptr, nullptr);
            if (rc < 0) throw std::runtime_error("generate: prompt step failed " + std::to_string(rc));
        }
        int tok = prompt_tokens.back();
        for (int i = 0; i < max_new_tokens; i++) {
            // the token is drawn on the device (greedy: the argmax), with the
            // prompt and the tokens so far as the repeat-penalty list; no
            // logits are copied to the host
            p.repeat_tokens = history.data();
            p.n_repeat_tokens = (int)history.size();
            int next;
            {
                py::gil_scoped_release nogil;
                next = matmul_decoder_step_sample(ctx_, tok, nullptr, &p);
            }
            if (next < 0) throw std::runtime_error("generate: step failed " + std::to_string(next));
            out.push_back(next);
            history.push_back(next);
            if (!callback.is_none()) callback(next);
            tok = next;
        }
        return out;
    }

   private:
    MatmulDecoderContext* ctx_ = nullptr;
    MatmulDecoderConfig cfg_{};
};

class PyBatchDecoder {
   public:
    PyBatchDecoder(const std::string& model_dir, int n_seqs, int max_seq_len, const std::string& quant_type) {
        MatmulDecoderConfig cfg;
        if (matmul_decoder_load_config((model_dir + "/config.json").c_str(), &cfg) != 0)
            throw std::runtime_error("Failed to load config.json from " + model_dir);
        cfg.max_seq_len = max_seq_len;
        {
            py::gil_scoped_release nogil;
            b_ = matmul_decoder_batch_create(model_dir.c_str(), &cfg, parse_quant(quant_type), max_seq_len, n_seqs);
        }
        if (!b_) throw std::runtime_error("Failed to create BatchDecoder from " + model_dir);
        n_ = n_seqs;
        cfg_ = cfg;
    }
    ~PyBatchDecoder() {
        if (b_) matmul_decoder_batch_destroy(b_);
    }
    void set_kv(int seq, int layer, int start, harr k, harr v) {
        const py::ssize_t per = (py::ssize_t)cfg_.num_kv_heads * cfg_.head_dim;
        if (k.size() != v.size() || k.size() % per != 0) throw std::invalid_argument("set_kv: shape mismatch");
        int rc = matmul_decoder_batch_set_kv(b_, seq, layer, start, (int)(k.size() / per), k.data(), v.data());
        if (rc != 0) throw std::runtime_error("batch set_kv failed " + std::to_string(rc));
    }
    void set_seq_len(int seq, int n) {
        if (matmul_decoder_batch_set_seq_len(b_, seq, n) != 0) throw std::invalid_argument("set_seq_len");
    }
    int get_seq_len(int seq) const { return matmul_decoder_batch_get_seq_len(b_, seq); }
    py::array_t<int> step(py::array_t<int, py::array::c_style | py::array::forcecast> tokens, bool want_logits) {
        if (tokens.size() != n_) throw std::invalid_argument("step: need one token per sequence");
        py::array_t<int> out(n_);
        py::array_t<float> logits;
        float* lp = nullptr;
        if (want_logits) {
            logits = py::array_t<float>({(py::ssize_t)n_, (py::ssize_t)cfg_.vocab_size});
            lp = logits.mutable_data();
        }
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = matmul_decoder_batch_step(b_, tokens.data(), out.mutable_data(), lp);
        }
        if (rc != 0) throw std::runtime_error("batch step failed " + std::to_string(rc));
        if (want_logits) last_logits_ = logits;
        return out;
    }
    py::object last_logits() const { return last_logits_; }
    py::dict stats() const {
        MatmulDecoderStats s{};
        matmul_decoder_batch_get_stats(b_, &s);
        return stats_dict(s);
    }

   private:
    MatmulDecoderBatch* b_ = nullptr;
    int n_ = 0;
    MatmulDecoderConfig cfg_{};
    py::object last_logits_ = py::none();
};

PYBIND11_MODULE(matmul_decoder, m) {
    m.doc() = "Decoder runtime for NVIDIA B200 (sm_100a) behind the matmul_decoder API";
    py::class_<PyMatmulDecoder>(m, "MatmulDecoder")
        .def(py::init<const std::string&, int, const std::string&, const std::string&, bool>(),
             py::arg("model_dir"), py::arg("max_seq_len") = 4096, py::arg("quant_type") = "int4",
             py::arg("exec_mode") = "dual_core", py::arg("disable_npu_lm_head") = false)
        .def("step", &PyMatmulDecoder::step, py::arg("token_id"), py::arg("embedding") = py::none(),
             "Run one decoding step, return logits")
        .def("prefill", &PyMatmulDecoder::prefill, py::arg("token_id"), py::arg("embedding") = py::none(),
             "Run one prefill step (fills KV cache, skips lm_head); a 2-D embedding routes to batch prefill")
        .def("prefill_batch", &PyMatmulDecoder::prefill_batch, py::arg("embeddings"),
             "Batch prefill M tokens; embeddings must be 2D [M, hidden_dim]")
        .def("step_get_token", &PyMatmulDecoder::step_get_token, py::arg("token_id"),
             py::arg("embedding") = py::none(), "Run one decoding step, return the greedy token")
        .def("step_head", &PyMatmulDecoder::step_head, py::arg("token_id"), py::arg("embedding") = py::none(),
             py::arg("lm_head_idx") = 0, "Decoding step with lm_head number lm_head_idx (multi-head models)")
        .def("clear_kv_cache", &PyMatmulDecoder::clear_kv_cache, "Clear KV cache for new sequence")
        .def("generate", &PyMatmulDecoder::generate, py::arg("prompt_tokens"), py::arg("max_new_tokens") = 128,
             py::arg("top_k") = 1, py::arg("top_p") = 1.0f, py::arg("temperature") = 1.0f,
             py::arg("repeat_penalty") = 1.0f, py::arg("callback") = py::none(), "Generate tokens autoregressively")
        .def("set_kv", &PyMatmulDecoder::set_kv, py::arg("layer"), py::arg("start"), py::arg("k"), py::arg("v"))
        .def("get_kv", &PyMatmulDecoder::get_kv, py::arg("layer"), py::arg("start"), py::arg("length"))
        .def("set_seq_len", &PyMatmulDecoder::set_seq_len, py::arg("n"))
        .def_property_readonly("hidden", &PyMatmulDecoder::hidden)
        .def_property_readonly("seq_len", &PyMatmulDecoder::seq_len, "Current sequence length")
        .def_property_readonly("config", &PyMatmulDecoder::config, "Model configuration")
        .def_property_readonly("stats", &PyMatmulDecoder::stats, "Performance statistics")
        .def("__repr__", [](const PyMatmulDecoder&) { return "<MatmulDecoder>"; });

    py::class_<PyBatchDecoder>(m, "BatchDecoder")
        .def(py::init<const std::string&, int, int, const std::string&>(), py::arg("model_dir"),
             py::arg("n_seqs"), py::arg("max_seq_len") = 4096, py::arg("quant_type") = "int4")
        .def("set_kv", &PyBatchDecoder::set_kv)
        .def("set_seq_len", &PyBatchDecoder::set_seq_len)
        .def("get_seq_len", &PyBatchDecoder::get_seq_len)
        .def("step", &PyBatchDecoder::step, py::arg("tokens"), py::arg("want_logits") = false)
        .def_property_readonly("last_logits", &PyBatchDecoder::last_logits)
        .def_property_readonly("stats", &PyBatchDecoder::stats);

    m.def("config_qwen3_0_6b", []() {
        MatmulDecoderConfig c = matmul_decoder_config_qwen3_0_6b();
        return config_dict(c);
    }, "Default config for Qwen3-0.6B (dual-core)");
    m.def("config_qwen3_0_6b_single_core", []() {
        MatmulDecoderConfig c = matmul_decoder_config_qwen3_0_6b_single_core();
        return config_dict(c);
    }, "Default config for Qwen3-0.6B (single-core)");
    m.attr("__version__") = "1.0.0";
}
