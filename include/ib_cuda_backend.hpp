// C++ mirror of the reference's CUDA backend interface on top of the C ABI
// (include/ib_cuda.h).  Same namespace, names, Buffer handle and argument meaning
// as the reference's include/ops/cuda_backend.hpp:7-66, so src/models and tests
// written against that header compile unchanged; failures throw
// std::runtime_error with the library's message, as the reference's check()
// does (src/ops/cuda_backend.cpp:76-85).  The quantized entry points after the
// reference's set are additions for weights kept in GGUF block form.  The model
// runner on packed weights is in ib_cuda_model.hpp (kept apart so that this header
// can stand in for ops/cuda_backend.hpp next to the reference's models/cuda_model.hpp).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace inference::cuda {

struct Buffer {
    uint64_t ptr = 0;
    size_t bytes = 0;
    bool valid() const { return ptr != 0; }
};

// lifecycle / info
bool available();
std::string device_name();
size_t total_memory();
size_t free_memory();
void sync();
void shutdown();

// memory
Buffer alloc(size_t bytes);
void release(Buffer& b);
void upload(const Buffer& dst, const void* src, size_t bytes);
void download(void* dst, const Buffer& src, size_t bytes);

// ops (FP32 row-major, the reference's set)
void gemv(const Buffer& W, const Buffer& x, const Buffer& y, int M, int N);
void gemv_i16(const Buffer& W, const Buffer& row_scale, const Buffer& x, const Buffer& y, int M,
              int N);
void gemm(const Buffer& W, const Buffer& X, const Buffer& Y, int T, int M, int K);
void gemm_i16(const Buffer& W, const Buffer& row_scale, const Buffer& X, const Buffer& Y, int T,
              int M, int K);
void rmsnorm(const Buffer& x, const Buffer& w, const Buffer& out, int rows, int dim, float eps);
void silu(const Buffer& x, int n);
void mul(const Buffer& a, const Buffer& b, int n);
void add(const Buffer& a, const Buffer& b, int n);
void embedding(const Buffer& table, int id, const Buffer& out, int dim);
void embedding_i16(const Buffer& table, const Buffer& row_scale, int id, const Buffer& out,
                   int dim);
void embedding_batch(const Buffer& table, const Buffer& ids, const Buffer& out, int T, int dim);
void embedding_batch_i16(const Buffer& table, const Buffer& row_scale, const Buffer& ids,
                         const Buffer& out, int T, int dim);
void kv_write(const Buffer& kc, const Buffer& vc, const Buffer& k, const Buffer& v, int n_heads,
              int head_dim, int max_seq, int pos);
void kv_write_batch(const Buffer& kc, const Buffer& vc, const Buffer& k, const Buffer& v,
                    int n_heads, int head_dim, int max_seq, int start, int T);
void rope(const Buffer& q, const Buffer& k, const Buffer& table, int n_heads, int n_kv_heads,
          int head_dim, int pos);
void rope_batch(const Buffer& q, const Buffer& k, const Buffer& table, int n_heads,
                int n_kv_heads, int head_dim, int start, int T);
void attention(const Buffer& q, const Buffer& kc, const Buffer& vc, const Buffer& out,
               int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos, float scale);
void attention_batch(const Buffer& q, const Buffer& kc, const Buffer& vc, const Buffer& out,
                     int n_heads, int n_kv_heads, int head_dim, int max_seq, int start, int T,
                     float scale);

// quantized weights kept in GGUF block form (type = GGUF type code)
void dequantize(int type, const Buffer& blocks, const Buffer& out, int64_t rows, int64_t cols);
void dequantize_i16(int type, const Buffer& blocks, const Buffer& q, const Buffer& row_scale,
                    int64_t rows, int64_t cols);
void gemv_q(int type, const Buffer& W, const Buffer& x, const Buffer& y, int64_t rows,
            int64_t cols);
void gemm_q(int type, const Buffer& W, const Buffer& X, const Buffer& Y, int64_t T, int64_t rows,
            int64_t cols);
void embedding_q(int type, const Buffer& table, const Buffer& ids, const Buffer& out, int T,
                 int64_t vocab, int64_t dim);

}  // namespace inference::cuda
