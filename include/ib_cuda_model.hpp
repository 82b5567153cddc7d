// inference::CudaModel: the native Llama runner (ib_model_* in ib_cuda.h) for C++
// callers.  The weights of a GGUF file stay in their block formats on the GPU
// (precision "native"), or are converted on the GPU to the reference's INT16 / FP32
// forms ("int16", "fp32": the values of the reference's --gpu-precision).  It takes
// the place of the reference's GpuState cache and generate_cuda loop
// (src/models/model_cuda.cpp:25-259, 442-495) for callers that hold the GGUF path.
// Failures throw std::runtime_error with the library's message.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace inference {

// Timing of one generate() call, the fields of the reference's GenerationStats
// (include/models/cuda_model.hpp:12-17), in milliseconds.
struct CudaModelStats {
    double init_ms = 0;
    double prefill_ms = 0;
    double decode_ms = 0;
    int generated = 0;
};

class CudaModel {
public:
    CudaModel(const std::string& gguf_path, const std::string& precision = "native",
              int device = 0, int max_seq = 0);
    ~CudaModel();
    CudaModel(const CudaModel&) = delete;
    CudaModel& operator=(const CudaModel&) = delete;

    // Greedy generation (temperature 0): prompt followed by up to max_tokens ids,
    // stopping at eos_token_id (>= 0) or the end of the context, with the batched
    // prefill and the decode loop of generate_cuda; the argmax runs on the device.
    std::vector<int> generate(const std::vector<int>& prompt, int max_tokens,
                              int eos_token_id = -1, CudaModelStats* stats = nullptr);
    // The steps one at a time, for callers that sample on the host: batched prefill of
    // ids at positions 0..n-1, then one decode step of `token` at `pos`; each writes the
    // step's logits (vocab() floats) and returns the greedy next id.
    int prefill(const std::vector<int>& ids, float* logits);
    int decode(int token, int pos, float* logits);
    int vocab() const;
    int max_seq() const;
    size_t weight_bytes() const;
    void* handle() const { return h_; }

private:
    void* h_ = nullptr;
    int vocab_ = 0, max_seq_ = 0;
};

}  // namespace inference
