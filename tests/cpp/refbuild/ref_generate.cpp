// Test driver over the reference's own model code, built by tests/cpp/refbuild/Makefile
// from the reference's sources with WITH_CUDA, so that its generate_cuda
// (src/models/model_cuda.cpp:442-495) runs on this library's inference::cuda mirror.
//
//   ref_generate <model.gguf> <cpu|cuda> <host_int16 0|1> <gpu_int16 0|1> <n_new> <id>...
//
// Loads the GGUF as the reference's main does (GGUFParser, load_model_weights, Model),
// decodes greedily (temperature 0, repetition penalty 1) and prints "ids:" followed by
// the prompt and the generated ids.
#include "core/tensor.hpp"
#include "gguf/gguf_parser.hpp"
#include "models/cuda_model.hpp"
#include "models/model.hpp"
#include "models/transformer.hpp"

#include <cstdio>
#include <cstdlib>
#include <exception>
#include <string>
#include <vector>

int main(int argc, char** argv) {
    if (argc < 7) {
        std::fprintf(stderr, "usage: %s model.gguf cpu|cuda host_int16 gpu_int16 n_new id...\n", argv[0]);
        return 2;
    }
    try {
        const std::string path = argv[1], device = argv[2];
        const bool host_int16 = std::atoi(argv[3]) != 0, gpu_int16 = std::atoi(argv[4]) != 0;
        const int n_new = std::atoi(argv[5]);
        std::vector<int> prompt;
        for (int i = 6; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
        inference::GGUFParser parser(path);
        auto weights = inference::load_model_weights(parser, inference::Device::cpu(), host_int16);
        inference::Model model(std::move(weights), inference::Device::cpu());
        inference::InferenceConfig cfg;
        cfg.max_tokens = n_new;
        cfg.temperature = 0.0f;
        cfg.repetition_penalty = 1.0f;
        cfg.seed = -1;
        cfg.eos_token_id = -1;
        cfg.gpu_int16 = gpu_int16;
        std::vector<int> out;
        if (device == "cuda") {
            if (!inference::cuda_model_available()) {
                std::fprintf(stderr, "CUDA backend unavailable\n");
                return 3;
            }
            inference::GenerationStats st;
            out = inference::generate_cuda(model, prompt, cfg, &st);
        } else {
            inference::KVCache kv(model.n_layers(), model.max_seq_len(), model.n_heads(),
                                  model.head_dim());
            out = model.generate(prompt, cfg, kv);
        }
        std::printf("ids:");
        for (int t : out) std::printf(" %d", t);
        std::printf("\n");
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
