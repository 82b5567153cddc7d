// Test infrastructure only: extern "C" entry points over the reference's own CPU
// code so that Python tests and the CPU baseline can call it through ctypes.
//
// This file is compiled together with the reference sources where they lie
// (oracle/Makefile, target `ref`); no reference source is copied here.  It only
// wraps the reference API:
//   dequantize / quantize          src/gguf/quantization.cpp:250-267, 354-360
//   matvec (FP32 / INT16)          src/models/transformer.cpp:100-119
//   load_model_weights (+ INT16)   src/models/transformer.cpp:135-310
//   Model::forward / generate      src/models/model.cpp:244-399
//   the output head's matvec       src/models/model.cpp:308-318 (timed alone)
// The handle mirrors what src/main.cpp:117-190 builds: a GGUFParser, the loaded
// ModelWeights moved into a Model, and a KVCache sized (layers, ctx, heads, hd).
#include "core/tensor.hpp"
#include "gguf/gguf_parser.hpp"
#include "gguf/quantization.hpp"
#include "models/model.hpp"
#include "models/transformer.hpp"

#include <chrono>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

using namespace inference;

namespace {

thread_local std::string g_err;

struct RefModel {
    std::unique_ptr<Model> model;
    std::unique_ptr<KVCache> cache;
};

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
    } catch (...) {
        g_err = "unknown exception";
    }
    return 1;
}

const HostWeight* pick_weight(const ModelWeights& w, const std::string& name, int layer) {
    if (name == "tok_embeddings") return &w.tok_embeddings;
    if (name == "output_norm") return &w.output_norm;
    if (name == "output") return w.output_tied ? &w.tok_embeddings : &w.output;
    if (layer < 0 || layer >= static_cast<int>(w.layers.size())) return nullptr;
    const auto& L = w.layers[static_cast<size_t>(layer)];
    if (name == "wq") return &L.wq;
    if (name == "wk") return &L.wk;
    if (name == "wv") return &L.wv;
    if (name == "wo") return &L.wo;
    if (name == "w1") return &L.w1;
    if (name == "w2") return &L.w2;
    if (name == "w3") return &L.w3;
    if (name == "attn_norm") return &L.attn_norm;
    if (name == "ffn_norm") return &L.ffn_norm;
    return nullptr;
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_dequantize(uint32_t dtype, const void* src, float* dst, int64_t n) {
    return guarded([&] { dequantize(static_cast<DataType>(dtype), src, dst, n); });
}

int ref_quantize(uint32_t dtype, const float* src, void* dst, int64_t n) {
    return guarded([&] { quantize(static_cast<DataType>(dtype), src, dst, n); });
}

int ref_matvec_f32(const float* W, const float* x, float* y, int64_t rows, int64_t cols) {
    return guarded([&] {
        HostWeight hw;
        hw.rows = rows;
        hw.cols = cols;
        hw.int16 = false;
        hw.data = Tensor(DataType::F32, {rows, cols});
        std::memcpy(hw.data.data(), W, static_cast<size_t>(rows * cols) * sizeof(float));
        matvec(hw, x, y, rows, cols);
    });
}

int ref_matvec_i16(const int16_t* q, const float* scale, const float* x, float* y,
                   int64_t rows, int64_t cols) {
    return guarded([&] {
        HostWeight hw;
        hw.rows = rows;
        hw.cols = cols;
        hw.int16 = true;
        hw.data = Tensor(DataType::I16, {rows, cols});
        hw.scale = Tensor(DataType::F32, {rows});
        std::memcpy(hw.data.data(), q, static_cast<size_t>(rows * cols) * sizeof(int16_t));
        std::memcpy(hw.scale.data(), scale, static_cast<size_t>(rows) * sizeof(float));
        matvec(hw, x, y, rows, cols);
    });
}

void* ref_model_load(const char* gguf_path, int host_int16) {
    RefModel* out = nullptr;
    guarded([&] {
        GGUFParser parser(gguf_path);
        auto weights = load_model_weights(parser, Device::cpu(), host_int16 != 0);
        auto h = std::make_unique<RefModel>();
        h->model = std::make_unique<Model>(std::move(weights), Device::cpu());
        h->cache = std::make_unique<KVCache>(h->model->n_layers(), h->model->max_seq_len(),
                                             h->model->n_heads(), h->model->head_dim());
        out = h.release();
    });
    return out;
}

void ref_model_free(void* h) { delete static_cast<RefModel*>(h); }

// cfg = {n_layers, embed_dim, n_heads, n_kv_heads, head_dim, vocab, max_seq, ffn, tied}
int ref_model_config(void* h, int64_t* cfg, float* rope_theta, float* rms_eps) {
    return guarded([&] {
        const ModelWeights& w = static_cast<RefModel*>(h)->model->weights();
        cfg[0] = w.n_layers;
        cfg[1] = w.embed_dim;
        cfg[2] = w.n_heads;
        cfg[3] = w.n_kv_heads;
        cfg[4] = w.head_dim;
        cfg[5] = w.vocab_size;
        cfg[6] = w.max_seq_len;
        cfg[7] = w.layers.empty() ? 0 : w.layers[0].w1.rows;
        cfg[8] = w.output_tied ? 1 : 0;
        *rope_theta = w.rope_theta;
        *rms_eps = w.rms_eps;
    });
}

// Shape and storage of one loaded weight: rows, cols, int16 flag.
int ref_model_weight_info(void* h, const char* name, int layer, int64_t* rows, int64_t* cols,
                          int* is_int16) {
    return guarded([&] {
        const HostWeight* hw = pick_weight(static_cast<RefModel*>(h)->model->weights(), name, layer);
        if (!hw) throw std::runtime_error(std::string("no weight ") + name);
        *rows = hw->rows;
        *cols = hw->cols;
        *is_int16 = hw->int16 ? 1 : 0;
    });
}

// Copies the loaded weight (F32 values, or INT16 values + per-row scales).
int ref_model_weight_copy(void* h, const char* name, int layer, void* data, float* scale) {
    return guarded([&] {
        const HostWeight* hw = pick_weight(static_cast<RefModel*>(h)->model->weights(), name, layer);
        if (!hw) throw std::runtime_error(std::string("no weight ") + name);
        std::memcpy(data, hw->data.data(), hw->data.byte_size());
        if (hw->int16 && scale) std::memcpy(scale, hw->scale.data(), hw->scale.byte_size());
    });
}

// Model::forward over T ids starting at start_pos (KV cache kept in the handle);
// writes the logits of all T rows ([T, vocab]).
int ref_model_forward(void* h, const int32_t* ids, int T, int start_pos, float* logits) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        if (start_pos == 0) m->cache->clear();
        Tensor input(DataType::I32, {1, T});
        std::memcpy(input.data(), ids, static_cast<size_t>(T) * sizeof(int32_t));
        Tensor lg = m->model->forward(input, m->cache.get(), start_pos);
        std::memcpy(logits, lg.data(), lg.byte_size());
    });
}

// Times the reference's output projection alone: matvec(output, x, logits) as
// Model::forward applies it (src/models/model.cpp:308-318), reps times on a fixed
// normalised input; *seconds = mean time per call.  Lets a caller separate the head
// from the per-layer cost of a forward pass.
int ref_model_time_head(void* h, int reps, double* seconds) {
    return guarded([&] {
        const ModelWeights& w = static_cast<RefModel*>(h)->model->weights();
        const HostWeight& out_w = w.output_tied ? w.tok_embeddings : w.output;
        std::vector<float> x(static_cast<size_t>(w.embed_dim), 0.01f);
        std::vector<float> y(static_cast<size_t>(w.vocab_size));
        if (reps < 1) reps = 1;
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < reps; ++i) matvec(out_w, x.data(), y.data(), w.vocab_size, w.embed_dim);
        const auto t1 = std::chrono::steady_clock::now();
        *seconds = std::chrono::duration<double>(t1 - t0).count() / reps;
    });
}

// Model::generate with temperature 0 and repetition penalty 1.0 (greedy):
// out receives prompt + max_tokens ids; *n_out the count written.
int ref_model_generate(void* h, const int32_t* prompt, int n_prompt, int max_tokens,
                       int32_t* out, int* n_out) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        InferenceConfig cfg;
        cfg.max_tokens = max_tokens;
        cfg.temperature = 0.0f;
        cfg.repetition_penalty = 1.0f;
        cfg.seed = -1;
        cfg.eos_token_id = -1;
        std::vector<int> p(prompt, prompt + n_prompt);
        std::vector<int> g = m->model->generate(p, cfg, *m->cache);
        for (size_t i = 0; i < g.size(); ++i) out[i] = g[i];
        *n_out = static_cast<int>(g.size());
    });
}

}  // extern "C"
