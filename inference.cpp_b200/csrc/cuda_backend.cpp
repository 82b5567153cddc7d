// inference::cuda (the reference's backend interface, include/ops/cuda_backend.hpp)
// implemented on the C ABI: each call forwards to ib_* on the legacy stream and
// throws std::runtime_error("CUDA: ...") on failure (src/ops/cuda_backend.cpp:76-85).
#include <stdexcept>
#include <vector>

#include "../../include/ib_cuda.h"
#include "../../include/ib_cuda_backend.hpp"
#include "../../include/ib_cuda_model.hpp"

namespace inference::cuda {

namespace {

void check(int st) {
    if (st != IB_OK) throw std::runtime_error(ib_last_error());
}

void* P(const Buffer& b) { return reinterpret_cast<void*>(b.ptr); }
template <typename T>
T* Pt(const Buffer& b) { return reinterpret_cast<T*>(b.ptr); }

bool g_init = false;
void ensure() {
    if (!g_init) {
        check(ib_init(0));
        g_init = true;
    }
}

}  // namespace

bool available() {
    try {
        ensure();
        return ib_available() == 1;
    } catch (...) {
        return false;
    }
}

std::string device_name() {
    ensure();
    char buf[256];
    check(ib_device_name(buf, sizeof(buf)));
    return buf;
}

size_t total_memory() {
    ensure();
    size_t f = 0, t = 0;
    check(ib_memory_info(&f, &t));
    return t;
}

size_t free_memory() {
    ensure();
    size_t f = 0, t = 0;
    check(ib_memory_info(&f, &t));
    return f;
}

void sync() { check(ib_sync()); }
void shutdown() { check(ib_shutdown()); }

Buffer alloc(size_t bytes) {
    ensure();
    void* p = nullptr;
    check(ib_alloc(&p, bytes));
    Buffer b;
    b.ptr = reinterpret_cast<uint64_t>(p);
    b.bytes = bytes;
    return b;
}

void release(Buffer& b) {
    if (!b.ptr) return;
    check(ib_free(P(b)));
    b.ptr = 0;
    b.bytes = 0;
}

void upload(const Buffer& dst, const void* src, size_t bytes) { check(ib_upload(P(dst), src, bytes, nullptr)); }
void download(void* dst, const Buffer& src, size_t bytes) { check(ib_download(dst, P(src), bytes, nullptr)); }

void gemv(const Buffer& W, const Buffer& x, const Buffer& y, int M, int N) {
    check(ib_gemv(Pt<float>(W), Pt<float>(x), Pt<float>(y), M, N, nullptr));
}
void gemv_i16(const Buffer& W, const Buffer& row_scale, const Buffer& x, const Buffer& y, int M, int N) {
    check(ib_gemv_i16(Pt<int16_t>(W), Pt<float>(row_scale), Pt<float>(x), Pt<float>(y), M, N, nullptr));
}
void gemm(const Buffer& W, const Buffer& X, const Buffer& Y, int T, int M, int K) {
    check(ib_gemm(Pt<float>(W), Pt<float>(X), Pt<float>(Y), T, M, K, nullptr));
}
void gemm_i16(const Buffer& W, const Buffer& row_scale, const Buffer& X, const Buffer& Y, int T, int M, int K) {
    check(ib_gemm_i16(Pt<int16_t>(W), Pt<float>(row_scale), Pt<float>(X), Pt<float>(Y), T, M, K, nullptr));
}
void rmsnorm(const Buffer& x, const Buffer& w, const Buffer& out, int rows, int dim, float eps) {
    check(ib_rmsnorm(Pt<float>(x), Pt<float>(w), Pt<float>(out), rows, dim, eps, nullptr));
}
void silu(const Buffer& x, int n) { check(ib_silu(Pt<float>(x), n, nullptr)); }
void mul(const Buffer& a, const Buffer& b, int n) { check(ib_mul(Pt<float>(a), Pt<float>(b), n, nullptr)); }
void add(const Buffer& a, const Buffer& b, int n) { check(ib_add(Pt<float>(a), Pt<float>(b), n, nullptr)); }
void embedding(const Buffer& table, int id, const Buffer& out, int dim) {
    check(ib_embedding(Pt<float>(table), id, Pt<float>(out), dim, nullptr));
}
void embedding_i16(const Buffer& table, const Buffer& row_scale, int id, const Buffer& out, int dim) {
    check(ib_embedding_i16(Pt<int16_t>(table), Pt<float>(row_scale), id, Pt<float>(out), dim, nullptr));
}
void embedding_batch(const Buffer& table, const Buffer& ids, const Buffer& out, int T, int dim) {
    check(ib_embedding_batch(Pt<float>(table), Pt<int32_t>(ids), Pt<float>(out), T, dim, nullptr));
}
void embedding_batch_i16(const Buffer& table, const Buffer& row_scale, const Buffer& ids,
                         const Buffer& out, int T, int dim) {
    check(ib_embedding_batch_i16(Pt<int16_t>(table), Pt<float>(row_scale), Pt<int32_t>(ids),
                                 Pt<float>(out), T, dim, nullptr));
}
void kv_write(const Buffer& kc, const Buffer& vc, const Buffer& k, const Buffer& v, int n_heads,
              int head_dim, int max_seq, int pos) {
    check(ib_kv_write(Pt<float>(kc), Pt<float>(vc), Pt<float>(k), Pt<float>(v), n_heads, head_dim,
                      max_seq, pos, nullptr));
}
void kv_write_batch(const Buffer& kc, const Buffer& vc, const Buffer& k, const Buffer& v,
                    int n_heads, int head_dim, int max_seq, int start, int T) {
    check(ib_kv_write_batch(Pt<float>(kc), Pt<float>(vc), Pt<float>(k), Pt<float>(v), n_heads,
                            head_dim, max_seq, start, T, nullptr));
}
void rope(const Buffer& q, const Buffer& k, const Buffer& table, int n_heads, int n_kv_heads,
          int head_dim, int pos) {
    check(ib_rope(Pt<float>(q), Pt<float>(k), Pt<float>(table), n_heads, n_kv_heads, head_dim, pos,
                  nullptr));
}
void rope_batch(const Buffer& q, const Buffer& k, const Buffer& table, int n_heads,
                int n_kv_heads, int head_dim, int start, int T) {
    check(ib_rope_batch(Pt<float>(q), Pt<float>(k), Pt<float>(table), n_heads, n_kv_heads,
                        head_dim, start, T, nullptr));
}
void attention(const Buffer& q, const Buffer& kc, const Buffer& vc, const Buffer& out,
               int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos, float scale) {
    check(ib_attention(Pt<float>(q), Pt<float>(kc), Pt<float>(vc), Pt<float>(out), n_heads,
                       n_kv_heads, head_dim, max_seq, pos, scale, nullptr));
}
void attention_batch(const Buffer& q, const Buffer& kc, const Buffer& vc, const Buffer& out,
                     int n_heads, int n_kv_heads, int head_dim, int max_seq, int start, int T,
                     float scale) {
    check(ib_attention_batch(Pt<float>(q), Pt<float>(kc), Pt<float>(vc), Pt<float>(out), n_heads,
                             n_kv_heads, head_dim, max_seq, start, T, scale, nullptr));
}

void dequantize(int type, const Buffer& blocks, const Buffer& out, int64_t rows, int64_t cols) {
    check(ib_dequant_f32(type, P(blocks), Pt<float>(out), rows, cols, nullptr));
}
void dequantize_i16(int type, const Buffer& blocks, const Buffer& q, const Buffer& row_scale,
                    int64_t rows, int64_t cols) {
    check(ib_dequant_i16(type, P(blocks), Pt<int16_t>(q), Pt<float>(row_scale), rows, cols, nullptr));
}
void gemv_q(int type, const Buffer& W, const Buffer& x, const Buffer& y, int64_t rows, int64_t cols) {
    check(ib_gemv_q(type, P(W), Pt<float>(x), Pt<float>(y), rows, cols, nullptr));
}
void gemm_q(int type, const Buffer& W, const Buffer& X, const Buffer& Y, int64_t T, int64_t rows,
            int64_t cols) {
    check(ib_gemm_q(type, P(W), Pt<float>(X), Pt<float>(Y), T, rows, cols, nullptr));
}
void embedding_q(int type, const Buffer& table, const Buffer& ids, const Buffer& out, int T,
                 int64_t vocab, int64_t dim) {
    check(ib_embedding_q(type, P(table), Pt<int32_t>(ids), Pt<float>(out), T, vocab, dim, nullptr));
}

}  // namespace inference::cuda

namespace inference {

static int precision_code(const std::string& p) {
    if (p == "native") return IB_PRECISION_NATIVE;
    if (p == "int16") return IB_PRECISION_INT16;
    if (p == "fp32") return IB_PRECISION_FP32;
    throw std::runtime_error("--gpu-precision expects native, int16 or fp32");
}

CudaModel::CudaModel(const std::string& path, const std::string& precision, int device,
                     int max_seq) {
    if (ib_model_load_gguf(path.c_str(), precision_code(precision), device, max_seq, &h_) != IB_OK)
        throw std::runtime_error(ib_last_error());
    ib_model_config cfg{};
    if (ib_model_get_config(h_, &cfg) != IB_OK) throw std::runtime_error(ib_last_error());
    vocab_ = cfg.vocab;
    max_seq_ = cfg.max_seq;
}

CudaModel::~CudaModel() {
    if (h_) ib_model_free(h_);
}

std::vector<int> CudaModel::generate(const std::vector<int>& prompt, int max_tokens,
                                     int eos_token_id, CudaModelStats* stats) {
    std::vector<int32_t> in(prompt.begin(), prompt.end());
    std::vector<int32_t> out(prompt.size() + (size_t)(max_tokens > 0 ? max_tokens : 0));
    int n = 0;
    ib_generation_stats st{};
    if (ib_model_generate(h_, in.data(), (int)in.size(), max_tokens, eos_token_id, out.data(), &n,
                          &st) != IB_OK)
        throw std::runtime_error(ib_last_error());
    if (stats) {
        stats->init_ms = st.init_ms;
        stats->prefill_ms = st.prefill_ms;
        stats->decode_ms = st.decode_ms;
        stats->generated = st.generated;
    }
    return std::vector<int>(out.begin(), out.begin() + n);
}

int CudaModel::prefill(const std::vector<int>& ids, float* logits) {
    std::vector<int32_t> in(ids.begin(), ids.end());
    int32_t next = 0;
    if (ib_model_prefill(h_, in.data(), (int)in.size(), 0, logits, &next) != IB_OK)
        throw std::runtime_error(ib_last_error());
    return next;
}

int CudaModel::decode(int token, int pos, float* logits) {
    int32_t next = 0;
    if (ib_model_decode(h_, token, pos, logits, &next) != IB_OK)
        throw std::runtime_error(ib_last_error());
    return next;
}

int CudaModel::vocab() const { return vocab_; }
int CudaModel::max_seq() const { return max_seq_; }

size_t CudaModel::weight_bytes() const {
    size_t n = 0;
    if (ib_model_weight_bytes(h_, &n) != IB_OK) throw std::runtime_error(ib_last_error());
    return n;
}

}  // namespace inference
