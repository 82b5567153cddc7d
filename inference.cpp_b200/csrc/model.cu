// Native Llama runner over the quantized-weight kernels -- the B200 counterpart
// of the reference's GPU model driver (src/models/model_cuda.cpp):
//   upload_weights (:138-212)  -> ib_model_set_tensor / ib_model_finalize: GGUF
//                                 blocks are copied to HBM unchanged ("native"),
//                                 or converted on the GPU to INT16 + row scale
//                                 ("int16", bit-exact with make_weight) or FP32;
//   prefill (:293-368)         -> ib_model_prefill: batched GEMM per linear;
//   forward_token (:372-407)   -> ib_model_decode: one token, every kernel reads
//                                 the position from device memory so the step is
//                                 captured once as a CUDA graph and replayed;
//   pick_token / generate_cuda -> greedy argmax on the device, ib_model_generate.
// Layouts follow the reference: activations FP32, KV cache FP32
// [layer][Hkv][max_seq][head_dim], RoPE from a host-built cos/sin table
// (model_cuda.cpp:175-187).
#include <math.h>

#include <chrono>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "comm.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "gguf_reader.h"
#include "model.h"
#include "ops.cuh"
#include "quant.cuh"

namespace ib {

__global__ void silu_mul_kernel(float* __restrict__ g, const float* __restrict__ u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float a = g[i];
        g[i] = a * (1.0f / (1.0f + expf(-a))) * u[i];
    }
}

// Greedy feedback at the end of a captured step: token <- next, pos <- pos + 1,
// and the token is recorded at out_tokens[pos] (when given).
__global__ void feedback_kernel(int32_t* dev_i32, int32_t* out_tokens, int max_seq) {
    const int next = dev_i32[2], pos = dev_i32[1];
    if (out_tokens && pos >= 0 && pos < max_seq) out_tokens[pos] = next;
    dev_i32[0] = next;
    dev_i32[1] = pos + 1;
}

// Fused-path feedback: the head's argmax key gives the next token; the key is reset
// for the next step.
__global__ void feedback_best_kernel(unsigned long long* best, int32_t* dev_i32,
                                     int32_t* out_tokens, int max_seq, int* work, int n_work) {
    // the step's GEMV work counters for the next step (the GEMVs do not count out)
    for (int i = threadIdx.x; i < n_work; i += blockDim.x) work[i] = 0;
    if (threadIdx.x) return;
    const int next = argmax_key_row(*best);
    *best = 0ull;
    const int pos = dev_i32[1];
    dev_i32[2] = next;
    if (out_tokens && pos >= 0 && pos < max_seq) out_tokens[pos] = next;
    dev_i32[0] = next;
    dev_i32[1] = pos + 1;
}

__global__ void add_vec_kernel(float* __restrict__ a, const float* __restrict__ b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        a[i] += b[i];
}

// The output head as this rank sees it: its vocabulary rows (the tied embedding's rows
// through a non-owning view under tensor parallelism).
static const Linear& head_linear(const Model* m) {
    if (m->has_output) return m->out;
    return m->tp_size > 1 ? m->head_view : m->tok;
}

// Residual update after a row-split projection: rank 0 adds its partial to x, the other
// ranks store theirs, and the allreduce then leaves x + sum of partials on every rank.
static int tp_residual(Model* m, float* x, const float* part, size_t n, cudaStream_t st) {
    if (m->tp_rank == 0) {
        const int g = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
        add_vec_kernel<<<g, 256, 0, st>>>(x, part, (int)n);
        IB_LAUNCH_CHECK("add_vec_kernel");
    } else {
        IB_CUDA_CHECK(cudaMemcpyAsync(x, part, n * 4, cudaMemcpyDeviceToDevice, st));
    }
    return comm_allreduce_sum_f32(m->comm, x, n, st);
}

// logits (vocab) <- every rank's head rows; a copy without tensor parallelism.
static int gather_logits(Model* m, cudaStream_t st) {
    if (m->tp_size == 1) return IB_OK;
    return comm_allgather_f32(m->comm, m->logits_local, m->logits, (size_t)m->vocab_local, st);
}

static double now_ms() {
    return std::chrono::duration<double, std::milli>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

int Linear::forward(const float* x, float* y, cudaStream_t st) const {
    switch (repr) {
        case REPR_PACKED: return ib_gemv_q(type, w, x, y, rows, cols, st);
        case REPR_I16: return ib_gemv_i16(q, s, x, y, (int)rows, (int)cols, st);
        case REPR_F32: return ib_gemv(f, x, y, (int)rows, (int)cols, st);
    }
    return IB_ERR_INVALID;
}

int Linear::forward_batch(const float* X, float* Y, int T, cudaStream_t st) const {
    switch (repr) {
        case REPR_PACKED:
            // prepared planes: the automatic path's kernel for prompts of 128 tokens and more
            if (planes && T >= 128) return gemm_on_planes(planes, X, Y, T, (int)rows, (int)cols, st);
            return ib_gemm_q(type, w, X, Y, T, rows, cols, st);
        case REPR_I16: return ib_gemm_i16(q, s, X, Y, T, (int)rows, (int)cols, st);
        case REPR_F32: return ib_gemm(f, X, Y, T, (int)rows, (int)cols, st);
    }
    return IB_ERR_INVALID;
}

void Linear::release() {
    if (planes) cudaFree(planes);
    planes = nullptr;
    if (w) cudaFree(w);
    if (q) cudaFree(q);
    if (s) cudaFree(s);
    if (f) cudaFree(f);
    w = nullptr;
    q = nullptr;
    s = nullptr;
    f = nullptr;
}

Model::~Model() {
    if (graph_exec) cudaGraphExecDestroy(graph_exec);
    if (stream) cudaStreamDestroy(stream);
    tok.release();
    out.release();
    for (auto& L : layers) {
        for (Linear* l : {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3}) l->release();
        cudaFree(L.attn_norm);
        cudaFree(L.ffn_norm);
    }
    for (void* p : allocations) cudaFree(p);
    if (host_pinned) cudaFreeHost(host_pinned);
    if (tp_local) comm_peer_free(tp_size, tp_local, tp_peers);
}

}  // namespace ib

using namespace ib;

// Uploads this rank's shard of a [rows, cols] tensor: axis -1 whole, 0 = the rank's
// rows/tp_size rows, 1 = the rank's cols/tp_size columns of every row (whole blocks).
static int set_linear(Model* m, Linear& L, int type, int64_t rows, int64_t cols,
                      const void* data, int on_device, int axis = -1) {
    if (!is_quant(type) && type != IB_TYPE_F32 && type != IB_TYPE_F16) {
        set_error(std::string("model: unsupported tensor type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    const int N = m->tp_size, rk = m->tp_rank;
    const int64_t be = is_quant(type) ? block_elems(type) : 1;
    const int64_t eb = is_quant(type) ? block_bytes(type) : (type == IB_TYPE_F32 ? 4 : 2);
    const int64_t row_bytes = cols / be * eb;
    int64_t lrows = rows, lcols = cols, off = 0;
    if (N > 1 && axis == 0) {
        if (rows % N) {
            set_error("model: tensor rows not divisible by the tensor-parallel size");
            return IB_ERR_INVALID;
        }
        lrows = rows / N;
        off = lrows * rk * row_bytes;
    } else if (N > 1 && axis == 1) {
        if ((cols / be) % N) {
            set_error("model: tensor blocks per row not divisible by the tensor-parallel size");
            return IB_ERR_INVALID;
        }
        lcols = cols / N;
        off = lcols / be * eb * rk;
    }
    const int64_t lrow_bytes = lcols / be * eb;
    L.release();
    L.type = type;
    L.rows = lrows;
    L.cols = lcols;
    rows = lrows;
    cols = lcols;
    const int64_t nbytes = lrows * lrow_bytes;
    void* dev = nullptr;
    // +16 so 16-byte vector loads of the last block never leave the allocation
    IB_CUDA_CHECK(cudaMalloc(&dev, (size_t)nbytes + 16));
    IB_CUDA_CHECK(cudaMemcpy2DAsync(dev, (size_t)lrow_bytes, (const uint8_t*)data + off,
                                    (size_t)row_bytes, (size_t)lrow_bytes, (size_t)lrows,
                                    on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                    m->stream));
    const bool packed_ok = is_quant(type) && m->cfg.precision == IB_PRECISION_NATIVE;
    if (packed_ok) {
        L.repr = REPR_PACKED;
        L.w = dev;
        return IB_OK;
    }
    // INT16 (reference gpu_int16) or FP32 copies, produced on the GPU
    int st = IB_OK;
    if (m->cfg.precision == IB_PRECISION_INT16) {
        IB_CUDA_CHECK(cudaMalloc(&L.q, (size_t)(rows * cols) * 2 + 16));
        IB_CUDA_CHECK(cudaMalloc(&L.s, (size_t)rows * 4));
        float* tmp = nullptr;
        if (type == IB_TYPE_F16) {
            IB_CUDA_CHECK(cudaMalloc(&tmp, (size_t)(rows * cols) * 4));
            st = ib_dequant_f32(type, dev, tmp, rows, cols, m->stream);
            if (st == IB_OK) st = ib_dequant_i16(IB_TYPE_F32, tmp, L.q, L.s, rows, cols, m->stream);
        } else {
            st = ib_dequant_i16(type, dev, L.q, L.s, rows, cols, m->stream);
        }
        IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
        if (tmp) cudaFree(tmp);
        L.repr = REPR_I16;
    } else {
        IB_CUDA_CHECK(cudaMalloc(&L.f, (size_t)(rows * cols) * 4 + 16));
        st = ib_dequant_f32(type, dev, L.f, rows, cols, m->stream);
        IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
        L.repr = REPR_F32;
    }
    cudaFree(dev);
    return st;
}

static int set_vector(Model* m, float** dst, int type, int64_t n, const void* data, int on_device) {
    if (*dst) cudaFree(*dst);
    IB_CUDA_CHECK(cudaMalloc(dst, (size_t)n * 4));
    if (type == IB_TYPE_F32) {
        IB_CUDA_CHECK(cudaMemcpyAsync(*dst, data, (size_t)n * 4,
                                      on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                      m->stream));
        return IB_OK;
    }
    if (type == IB_TYPE_F16) {
        void* tmp = nullptr;
        IB_CUDA_CHECK(cudaMalloc(&tmp, (size_t)n * 2));
        IB_CUDA_CHECK(cudaMemcpyAsync(tmp, data, (size_t)n * 2,
                                      on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                      m->stream));
        int st = ib_dequant_f32(IB_TYPE_F16, tmp, *dst, 1, n, m->stream);
        IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
        cudaFree(tmp);
        return st;
    }
    set_error("model: norm weights must be F32 or F16");
    return IB_ERR_UNSUPPORTED;
}

static int model_create(const ib_model_config* cfg, int device, Comm* comm, void** out) {
    IB_REQUIRE(cfg && out, "null pointer argument");
    *out = nullptr;
    IB_REQUIRE(cfg->n_layers >= 0 && cfg->dim > 0 && cfg->n_heads > 0 && cfg->n_kv_heads > 0 &&
                   cfg->n_heads % cfg->n_kv_heads == 0 && cfg->dim % cfg->n_heads == 0 &&
                   cfg->ffn > 0 && cfg->vocab > 0 && cfg->max_seq > 0,
               "model: invalid configuration");
    IB_REQUIRE(cfg->precision >= 0 && cfg->precision <= 2, "model: precision must be 0, 1 or 2");
    IB_REQUIRE((cfg->dim / cfg->n_heads) % 2 == 0, "model: head_dim must be even");
    const int N = comm_world(comm);
    IB_REQUIRE(cfg->n_kv_heads % N == 0 && cfg->ffn % N == 0 && cfg->vocab % N == 0,
               "model: n_kv_heads, ffn and vocab must be divisible by the tensor-parallel size");
    int st = ib_init(device);
    if (st != IB_OK) return st;
    auto m = std::make_unique<Model>();
    m->full = *cfg;
    m->cfg = *cfg;
    m->cfg.n_heads = cfg->n_heads / N;
    m->cfg.n_kv_heads = cfg->n_kv_heads / N;
    m->cfg.ffn = cfg->ffn / N;
    m->comm = comm;
    m->tp_size = N;
    m->tp_rank = comm_rank(comm);
    m->vocab_local = cfg->vocab / N;
    m->vocab_base = m->vocab_local * m->tp_rank;
    m->device = device;
    m->HD = cfg->dim / cfg->n_heads;
    IB_CUDA_CHECK(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    m->layers.resize(cfg->n_layers);
    *out = m.release();
    return IB_OK;
}

extern "C" int ib_model_create(const ib_model_config* cfg, int device, void** out) {
    return model_create(cfg, device, nullptr, out);
}

extern "C" int ib_model_create_tp(const ib_model_config* cfg, int device, void* comm, void** out) {
    IB_REQUIRE(comm, "null communicator");
    return model_create(cfg, device, (Comm*)comm, out);
}

extern "C" int ib_model_free(void* h) {
    if (!h) return IB_OK;
    Model* m = (Model*)h;
    cudaSetDevice(m->device);
    delete m;
    return IB_OK;
}

// Tensor names as the reference loader reads them (src/models/transformer.cpp:267-306).
extern "C" int ib_model_set_tensor(void* h, const char* name, int type, int64_t rows,
                                   int64_t cols, const void* data, int on_device) {
    IB_REQUIRE(h && name && data, "null pointer argument");
    Model* m = (Model*)h;
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    IB_REQUIRE(!m->finalized, "model: tensors cannot change after finalize");
    const std::string n(name);
    const auto& c = m->full;  // shapes are checked against the whole model
    const int D = c.dim, HD = m->HD;
    auto expect = [&](int64_t r, int64_t cc) -> int {
        if (rows != r || cols != cc) {
            set_error("model: tensor " + n + " has shape [" + std::to_string(rows) + ", " +
                      std::to_string(cols) + "], expected [" + std::to_string(r) + ", " +
                      std::to_string(cc) + "]");
            return IB_ERR_INVALID;
        }
        return IB_OK;
    };
    int st;
    if (n == "token_embd.weight") {
        if ((st = expect(c.vocab, D))) return st;
        return set_linear(m, m->tok, type, rows, cols, data, on_device);
    }
    if (n == "output.weight") {
        if ((st = expect(c.vocab, D))) return st;
        m->has_output = true;
        return set_linear(m, m->out, type, rows, cols, data, on_device, 0);
    }
    if (n == "output_norm.weight") {
        if ((st = expect(1, D))) return st;
        return set_vector(m, &m->out_norm, type, D, data, on_device);
    }
    int l = -1;
    char kind[64] = {0};
    if (sscanf(name, "blk.%d.%63[a-z_].weight", &l, kind) != 2 || l < 0 || l >= c.n_layers) {
        set_error("model: unknown tensor " + n);
        return IB_ERR_INVALID;
    }
    Layer& L = m->layers[l];
    const std::string k(kind);
    if (k == "attn_q") { if ((st = expect((int64_t)c.n_heads * HD, D))) return st; return set_linear(m, L.wq, type, rows, cols, data, on_device, 0); }
    if (k == "attn_k") { if ((st = expect((int64_t)c.n_kv_heads * HD, D))) return st; return set_linear(m, L.wk, type, rows, cols, data, on_device, 0); }
    if (k == "attn_v") { if ((st = expect((int64_t)c.n_kv_heads * HD, D))) return st; return set_linear(m, L.wv, type, rows, cols, data, on_device, 0); }
    if (k == "attn_output") { if ((st = expect(D, (int64_t)c.n_heads * HD))) return st; return set_linear(m, L.wo, type, rows, cols, data, on_device, 1); }
    if (k == "ffn_gate") { if ((st = expect(c.ffn, D))) return st; return set_linear(m, L.w1, type, rows, cols, data, on_device, 0); }
    if (k == "ffn_down") { if ((st = expect(D, c.ffn))) return st; return set_linear(m, L.w2, type, rows, cols, data, on_device, 1); }
    if (k == "ffn_up") { if ((st = expect(c.ffn, D))) return st; return set_linear(m, L.w3, type, rows, cols, data, on_device, 0); }
    if (k == "attn_norm") { if ((st = expect(1, D))) return st; return set_vector(m, &L.attn_norm, type, D, data, on_device); }
    if (k == "ffn_norm") { if ((st = expect(1, D))) return st; return set_vector(m, &L.ffn_norm, type, D, data, on_device); }
    set_error("model: unknown tensor " + n);
    return IB_ERR_INVALID;
}

static int alloc_f(Model* m, float** p, size_t n) {
    IB_CUDA_CHECK(cudaMalloc(p, n * sizeof(float) + 16));
    m->allocations.push_back(*p);
    return IB_OK;
}

// (Re)allocates every layer's K and V cache, zeroed, in the element type kv_f16 selects.
static int alloc_kv(Model* m) {
    const auto& c = m->cfg;
    const size_t n = (size_t)c.n_kv_heads * c.max_seq * m->HD, eb = m->kv_f16 ? 2 : 4;
    for (auto& L : m->layers) {
        for (float** p : {&L.kc, &L.vc}) {
            if (*p) {
                for (auto& a : m->allocations)
                    if (a == *p) a = nullptr;
                IB_CUDA_CHECK(cudaFree(*p));
                *p = nullptr;
            }
            IB_CUDA_CHECK(cudaMalloc(p, n * eb + 16));
            m->allocations.push_back(*p);
            IB_CUDA_CHECK(cudaMemsetAsync(*p, 0, n * eb, m->stream));
        }
    }
    return IB_OK;
}

// The model's device buffers (everything but the tensor-parallel peer memory).
static int finalize_buffers(Model* m) {
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    const auto& c = m->cfg;
    auto missing = [&](const std::string& what) {
        set_error("model: tensor not set: " + what);
        return IB_ERR_INVALID;
    };
    if (m->tok.repr == REPR_NONE) return missing("token_embd.weight");
    if (!m->out_norm) return missing("output_norm.weight");
    for (int l = 0; l < c.n_layers; ++l) {
        Layer& L = m->layers[l];
        const std::string p = "blk." + std::to_string(l) + ".";
        if (L.wq.repr == REPR_NONE) return missing(p + "attn_q.weight");
        if (L.wk.repr == REPR_NONE) return missing(p + "attn_k.weight");
        if (L.wv.repr == REPR_NONE) return missing(p + "attn_v.weight");
        if (L.wo.repr == REPR_NONE) return missing(p + "attn_output.weight");
        if (L.w1.repr == REPR_NONE) return missing(p + "ffn_gate.weight");
        if (L.w2.repr == REPR_NONE) return missing(p + "ffn_down.weight");
        if (L.w3.repr == REPR_NONE) return missing(p + "ffn_up.weight");
        if (!L.attn_norm) return missing(p + "attn_norm.weight");
        if (!L.ffn_norm) return missing(p + "ffn_norm.weight");
    }
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn, V = c.vocab;
    const int S = c.max_seq;
    // VRAM preflight as the reference does before upload (model_cuda.cpp:243-252)
    const size_t kv_bytes = (size_t)c.n_layers * 2 * Hkv * (size_t)S * HD * (m->kv_f16 ? 2 : 4);
    size_t free_b = 0, total_b = 0;
    IB_CUDA_CHECK(cudaMemGetInfo(&free_b, &total_b));
    if (kv_bytes + (64ull << 20) > free_b) {
        set_error("CUDA: model needs ~" + std::to_string(kv_bytes >> 20) +
                  " MB VRAM for the KV cache but only " + std::to_string(free_b >> 20) +
                  " MB is free. Reduce the context length.");
        return IB_ERR_OOM;
    }
    {
        int st;
        if ((st = alloc_kv(m))) return st;
    }
    // RoPE table, computed on the host exactly as model_cuda.cpp:175-187 does
    const int half = HD / 2;
    std::vector<float> table((size_t)S * half * 2);
    for (int pos = 0; pos < S; ++pos)
        for (int j = 0; j < half; ++j) {
            const float freq = 1.0f / powf(c.rope_theta, (float)(2 * j) / (float)HD);
            const float angle = (float)pos * freq;
            table[((size_t)pos * half + j) * 2] = cosf(angle);
            table[((size_t)pos * half + j) * 2 + 1] = sinf(angle);
        }
    int st;
    if ((st = alloc_f(m, &m->rope_table, table.size()))) return st;
    IB_CUDA_CHECK(cudaMemcpyAsync(m->rope_table, table.data(), table.size() * 4,
                                  cudaMemcpyHostToDevice, m->stream));
    // decode activations
    float** bufs[] = {&m->x, &m->xn, &m->q, &m->k, &m->v, &m->att, &m->proj, &m->gate, &m->up,
                      &m->logits};
    const size_t sizes[] = {(size_t)D, (size_t)D, (size_t)H * HD, (size_t)Hkv * HD,
                            (size_t)Hkv * HD, (size_t)H * HD, (size_t)D, (size_t)F, (size_t)F,
                            (size_t)V};
    for (int i = 0; i < 10; ++i)
        if ((st = alloc_f(m, bufs[i], sizes[i]))) return st;
    if ((st = alloc_f(m, &m->att_part, attention_partial_bytes(H, HD, S - 1) / 4 + 1))) return st;
    IB_CUDA_CHECK(cudaMalloc(&m->dev_i32, 64));
    m->allocations.push_back(m->dev_i32);
    IB_CUDA_CHECK(cudaMalloc(&m->dev_tokens, (size_t)S * 4 + 16));
    m->allocations.push_back(m->dev_tokens);
    IB_CUDA_CHECK(cudaMalloc(&m->best, 16));
    m->allocations.push_back(m->best);
    IB_CUDA_CHECK(cudaMemsetAsync(m->best, 0, 16, m->stream));
    m->slab_kq = slab_kquant(m->layers.empty() ? m->tok.type : m->layers[0].wq.type);
    {
        uint8_t** slabs[] = {&m->slab_x, &m->slab_att, &m->slab_h};
        const int lens[] = {D, H * HD, F};
        for (int i = 0; i < 3; ++i) {
            IB_CUDA_CHECK(cudaMalloc(slabs[i], slab_total_bytes(lens[i], m->slab_kq) + 16));
            m->allocations.push_back(*slabs[i]);
        }
        if ((st = alloc_f(m, &m->ssq, (size_t)D / 32 + 1))) return st;
        if (m->tp_size == 1) {  // the down projection's K split (row groups of 16 rows)
            const size_t n_rg = ((size_t)D + 15) / 16;
            if ((st = alloc_f(m, &m->kpart, n_rg * 32))) return st;
            IB_CUDA_CHECK(cudaMalloc(&m->kcnt, n_rg * 4));
            m->allocations.push_back(m->kcnt);
            IB_CUDA_CHECK(cudaMemsetAsync(m->kcnt, 0, n_rg * 4, m->stream));
        }
        const size_t nwork = (size_t)(4 * c.n_layers + 1) * 2;
        IB_CUDA_CHECK(cudaMalloc(&m->gemv_work, nwork * 4));
        m->allocations.push_back(m->gemv_work);
        IB_CUDA_CHECK(cudaMemsetAsync(m->gemv_work, 0, nwork * 4, m->stream));
        if (attention_fused_ok(H, Hkv, HD)) {
            if ((st = alloc_f(m, &m->att_fpart, attention_fused_part_bytes(H, HD) / 4 + 1))) return st;
            IB_CUDA_CHECK(cudaMalloc(&m->att_counters, (size_t)Hkv * 4 + 16));
            m->allocations.push_back(m->att_counters);
            IB_CUDA_CHECK(cudaMemsetAsync(m->att_counters, 0, (size_t)Hkv * 4 + 16, m->stream));
        }
    }
    // the head rows of this rank: logits_local; the full logits are gathered on demand
    if (m->tp_size > 1) {
        if ((st = alloc_f(m, &m->logits_local, (size_t)m->vocab_local))) return st;
        if (!m->has_output) {  // tied embedding: a view of this rank's rows of the table
            Linear& hv = m->head_view;
            const Linear& t = m->tok;
            hv = Linear();
            hv.repr = t.repr;
            hv.type = t.type;
            hv.rows = m->vocab_local;
            hv.cols = t.cols;
            const int64_t vb = m->vocab_base;
            if (t.w) hv.w = (uint8_t*)t.w + vb * packed_bytes(t.type, 1, t.cols);
            if (t.q) hv.q = t.q + vb * t.cols;
            if (t.s) hv.s = t.s + vb;
            if (t.f) hv.f = t.f + vb * t.cols;
        }
    } else {
        m->logits_local = m->logits;
    }
    if (m->tp_size > 1) {
        uint32_t* seq = nullptr;
        IB_CUDA_CHECK(cudaMalloc(&seq, 16));
        m->allocations.push_back(seq);
        IB_CUDA_CHECK(cudaMemset(seq, 0, 16));
        m->tpx.seq = seq;
    }
    return IB_OK;
}

// Tensor parallelism: the peer memory of the fused step's exchange (its row-split GEMVs
// store their rows into every rank's region).  Collective: every rank joins with the
// status of its own set-up so far, and every rank fails if one did.
static int finalize_peers(Model* m, int local_status) {
    const int W = m->tp_size;
    int st = local_status;
    if (st == IB_OK && W > kMaxRanks) {
        set_error("model: at most 8 tensor-parallel ranks");
        st = IB_ERR_UNSUPPORTED;
    }
    void* local = nullptr;
    if ((st = comm_peer_alloc(m->comm, tp_region_bytes(W, m->cfg.dim), st, &local, m->tp_peers)))
        return st;
    m->tp_local = (uint8_t*)local;
    TpExchange& x = m->tpx;
    for (int q = 0; q < W; ++q) x.region[q] = (uint8_t*)m->tp_peers[q];
    x.rank = m->tp_rank;
    x.world = W;
    x.stride = m->cfg.dim;
    return IB_OK;
}

extern "C" int ib_model_finalize(void* h) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    if (m->finalized) return IB_OK;
    int st = finalize_buffers(m);
    if (m->tp_size > 1) st = finalize_peers(m, st);
    if (st) return st;
    m->fused_ok = fused_supported(m);
    if ((st = build_step_plan(m))) return st;
    IB_CUDA_CHECK(cudaMallocHost(&m->host_pinned, 256));
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    m->finalized = true;
    return IB_OK;
}

namespace ib {

// ---- fused decode path: five launches per layer ------------------------------------
//   QKV    RMSNorm(x) -> q, k, v in one GEMV over [wq; wk; wv]; RoPE; k, v into the cache
//   attn   split-K partial + combine (attention.cu)
//   wo     x += wo . att
//   ffn    RMSNorm(x) -> silu(w1 . xn) * (w3 . xn), gate and up rows paired per tile
//   down   x += w2 . h
// then the head (RMSNorm, logits, argmax) and the token feedback.
static FusedGemv fg_common(const Model* m) {
    FusedGemv p = {};
    p.eps = m->cfg.rms_eps;
    p.work_ext = 1;  // the step's feedback kernel zeroes the work counters
    return p;
}

static void fg_seg(FusedGemv& p, int i, const Linear& l) {
    p.W[i] = (const uint8_t*)l.w;
    p.type[i] = l.type;
    p.rows[i] = (int)l.rows;
    p.n_seg = i + 1;
}

static FusedGemv fg_qkv(const Model* m, const Layer& L) {
    FusedGemv p = fg_common(m);
    fg_seg(p, 0, L.wq);
    fg_seg(p, 1, L.wk);
    fg_seg(p, 2, L.wv);
    p.K = m->cfg.dim;
    p.slab = m->slab_x;
    p.ssq = m->ssq;
    p.q = m->q;
    p.kc = L.kc;
    p.vc = L.vc;
    p.kv_half = m->kv_f16 ? 1 : 0;
    p.rope = m->rope_table;
    p.pos = m->dev_i32 + 1;
    p.head_dim = m->HD;
    p.max_seq = m->cfg.max_seq;
    return p;
}

static FusedGemv fg_wo(const Model* m, const Layer& L) {
    FusedGemv p = fg_common(m);
    fg_seg(p, 0, L.wo);
    p.K = (int)L.wo.cols;
    p.slab = m->slab_att;
    p.y = m->x;
    p.tp = m->tpx;
    return p;
}

static FusedGemv fg_ffn_in(const Model* m, const Layer& L) {
    FusedGemv p = fg_common(m);
    fg_seg(p, 0, L.w1);
    fg_seg(p, 1, L.w3);
    p.paired = 1;
    p.K = m->cfg.dim;
    p.slab = m->slab_x;
    p.ssq = m->ssq;
    p.y = m->gate;
    return p;
}

static FusedGemv fg_ffn_out(const Model* m, const Layer& L) {
    FusedGemv p = fg_common(m);
    fg_seg(p, 0, L.w2);
    p.K = (int)L.w2.cols;
    p.slab = m->slab_h;
    p.y = m->x;
    p.tp = m->tpx;
    p.kpart = m->kpart;  // long rows split over K (null under TP)
    p.kcnt = m->kcnt;
    return p;
}

static FusedGemv fg_head(const Model* m) {
    FusedGemv p = fg_common(m);
    fg_seg(p, 0, head_linear(m));
    p.K = m->cfg.dim;
    p.slab = m->slab_x;
    p.ssq = m->ssq;
    p.y = m->logits_local;
    p.row_base = m->vocab_base;
    p.best = m->best;
    p.tp = m->tpx;
    return p;
}

static FusedGemv with_work(FusedGemv p, int* work) {
    p.work = work;
    return p;
}

bool fused_supported(const Model* m) {
    const auto& c = m->cfg;
    const Linear& O = head_linear(m);
    const int GS = m->slab_kq ? 256 : 32;
    if (c.dim % GS || c.ffn % GS || (c.n_heads * m->HD) % GS) return false;
    // the call sites get their work counters at launch (checked here with a stand-in)
    int* work = m->gemv_work;
    const int res_epi = m->tp_size > 1 ? EPI_ALLRED : EPI_RESID;
    FusedGemv head = fg_head(m);
    head.work = work;
    if (O.repr != REPR_PACKED || slab_kquant(O.type) != m->slab_kq ||
        !fused_gemv_supported(head, EPI_ARGMAX))
        return false;
    for (const Layer& L : m->layers) {
        for (const Linear* l : {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3})
            if (l->repr != REPR_PACKED || slab_kquant(l->type) != m->slab_kq) return false;
        if (!fused_gemv_supported(fg_qkv(m, L), EPI_QKV) ||
            !fused_gemv_supported(with_work(fg_wo(m, L), work), res_epi) ||
            !fused_gemv_supported(fg_ffn_in(m, L), EPI_SWIGLU) ||
            !fused_gemv_supported(with_work(fg_ffn_out(m, L), work), res_epi))
            return false;
    }
    return true;
}

// The second format of each fused pair (Q6_K, Q8_0, Q5_1): its rows use ring slot B.
static bool pair_member_b(int type) {
    return type == IB_TYPE_Q6_K || type == IB_TYPE_Q8_0 || type == IB_TYPE_Q5_1;
}

// ---- persistent decode step: the task plan ------------------------------------------
// Slab instances (inputs of the step's GEMVs, each with its readiness counters):
//   0               embedding -> layer 0's QKV
//   1 + 4l + 0      attention of layer l -> wo
//   1 + 4l + 1      x after wo -> gate+up (ffn_norm)
//   1 + 4l + 2      SwiGLU product -> down
//   1 + 4l + 3      x after down -> layer l+1's QKV (attn_norm) or the head (output_norm)
int build_step_plan(Model* m) {
    m->persistent_ok = false;
    const auto& c = m->cfg;
    if (m->tp_size > 1 || !m->fused_ok || m->kv_f16 || c.n_layers < 1 ||
        m->tok.repr != REPR_PACKED)
        return IB_OK;
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn;
    const bool kq = m->slab_kq;
    const int GS = kq ? 256 : 32, SE = kq ? 2048 : 1024, BE = kq ? 256 : 32;
    const int G = H / Hkv;
    if ((HD != 32 && HD != 64 && HD != 128) || G > 8 || G * HD > 1024 || (G * HD) % GS ||
        D % GS || F % GS || (H * HD) % GS || D % block_elems(m->tok.type))
        return IB_OK;
    const int kmax = std::max(std::max(D, F), H * HD);
    const int max_slices = (kmax + SE - 1) / SE, max_groups = kmax / GS;
    const int n_inst = 1 + 4 * c.n_layers;
    const int type_a = m->layers[0].wq.type;
    bool pad[2] = {false, false};
    std::vector<StepPhase> ph;
    int t = 0;
    auto add = [&](StepPhase p) {
        p.first = t;
        t += p.n;
        ph.push_back(p);
    };
    auto gemv = [&](const FusedGemv& g, int pro, int epi, int in_inst) {
        StepPhase p{};
        p.kind = TK_GEMV;
        p.g = g;
        p.g.work = nullptr;
        p.pro = pro;
        p.epi = epi;
        p.nb = g.K / BE;
        p.spg = (g.K + SE - 1) / SE;
        p.in_inst = in_inst;
        p.out_inst = -1;
        p.n = g.paired ? g.rows[0] / 8 : (g.rows[0] + g.rows[1] + g.rows[2] + 15) / 16;
        for (int sgm = 0; sgm < g.n_seg; ++sgm) {
            const int64_t rb = packed_bytes(g.type[sgm], 1, g.K);
            if (((uintptr_t)g.W[sgm] & 15) || rb % 16) pad[pair_member_b(g.type[sgm]) ? 1 : 0] = true;
        }
        return p;
    };
    {
        StepPhase e{};
        e.kind = TK_EMBED;
        e.n = D / GS;
        e.x = m->x;
        e.norm = m->layers[0].attn_norm;
        e.ssq = m->ssq;
        e.out_slab = m->slab_x;
        e.out_inst = 0;
        add(e);
    }
    int in_x = 0;  // instance of the next QKV's input
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = m->layers[l];
        const int base = 1 + 4 * l;
        StepPhase q = gemv(fg_qkv(m, L), PRO_NORM, EPI_QKV, in_x);
        q.layer = l;
        add(q);
        StepPhase a{};
        a.kind = TK_ATTN;
        a.n = Hkv * kStepAttMaxSplits;
        a.layer = l;
        a.q = m->q;
        a.kc = L.kc;
        a.vc = L.vc;
        a.out_slab = m->slab_att;
        a.out_inst = base;
        add(a);
        StepPhase wo = gemv(fg_wo(m, L), PRO_PLAIN, EPI_RESID, base);
        wo.out_inst = base + 1;
        wo.out_src = m->x;
        wo.out_norm = L.ffn_norm;
        wo.out_ssq = m->ssq;
        wo.out_slab = m->slab_x;
        wo.out_per_group = GS / 16;
        add(wo);
        StepPhase fi = gemv(fg_ffn_in(m, L), PRO_NORM, EPI_SWIGLU, base + 1);
        fi.out_inst = base + 2;
        fi.out_src = m->gate;
        fi.out_slab = m->slab_h;
        fi.out_per_group = GS / 8;
        add(fi);
        StepPhase dn = gemv(fg_ffn_out(m, L), PRO_PLAIN, EPI_RESID, base + 2);
        dn.out_inst = base + 3;
        dn.out_src = m->x;
        dn.out_norm = l + 1 < c.n_layers ? m->layers[l + 1].attn_norm : m->out_norm;
        dn.out_ssq = m->ssq;
        dn.out_slab = m->slab_x;
        dn.out_per_group = GS / 16;
        add(dn);
        in_x = base + 3;
    }
    add(gemv(fg_head(m), PRO_NORM, EPI_ARGMAX, in_x));
    StepParams& P = m->step;
    P = StepParams{};
    P.HD = HD;
    int grid = 0;
    int r = step_geometry(type_a, pad[0], pad[1], G, HD, P, &grid);
    if (r == IB_ERR_UNSUPPORTED) return IB_OK;  // the fused kernels stay in use
    if (r) return r;
    P.n_phases = (int)ph.size();
    P.n_tasks = t;
    P.max_slices = max_slices;
    P.max_groups = max_groups;
    P.max_kv = Hkv;
    P.ready_off = 2;
    P.grp_off = P.ready_off + n_inst * max_slices;
    P.att_ready_off = P.grp_off + n_inst * max_groups;
    P.att_done_off = P.att_ready_off + c.n_layers * Hkv;
    m->step_ctr_bytes = step_counter_bytes(n_inst, max_slices, max_groups, c.n_layers, Hkv);
    StepPhase* dph = nullptr;
    IB_CUDA_CHECK(cudaMalloc(&dph, ph.size() * sizeof(StepPhase)));
    m->allocations.push_back(dph);
    IB_CUDA_CHECK(cudaMemcpyAsync(dph, ph.data(), ph.size() * sizeof(StepPhase),
                                  cudaMemcpyHostToDevice, m->stream));
    P.phases = dph;
    IB_CUDA_CHECK(cudaMalloc(&P.ctr, m->step_ctr_bytes));
    m->allocations.push_back(P.ctr);
    IB_CUDA_CHECK(cudaMemsetAsync(P.ctr, 0, m->step_ctr_bytes, m->stream));
    IB_CUDA_CHECK(cudaMalloc(&P.att_acc, (size_t)H * kStepAttMaxSplits * HD * 4 + 16));
    m->allocations.push_back(P.att_acc);
    IB_CUDA_CHECK(cudaMalloc(&P.att_ml, (size_t)H * kStepAttMaxSplits * 8 + 16));
    m->allocations.push_back(P.att_ml);
    P.dev_i32 = m->dev_i32;
    P.tokens = m->dev_tokens;
    P.best = m->best;
    P.max_seq = c.max_seq;
    P.emb = (const uint8_t*)m->tok.w;
    P.emb_type = m->tok.type;
    P.vocab = c.vocab;
    P.dim = D;
    P.H = H;
    P.Hkv = Hkv;
    P.scale = 1.0f / sqrtf((float)HD);
    P.att_target = (G + 2) * HD / 16;
    m->step_grid = grid;
    m->step_type = type_a;
    m->persistent_ok = true;
    return IB_OK;
}

static int step_launches(Model* m) {
    IB_CUDA_CHECK(cudaMemsetAsync(m->step.ctr, 0, m->step_ctr_bytes, m->stream));
    return step_launch(m->step, m->step_type, m->step_grid, m->stream);
}

static bool persistent_active(const Model* m) {
    return m->use_persistent && m->persistent_ok && m->use_fused && m->fused_ok;
}

static int embed_launch(Model* m) {
    const auto& c = m->cfg;
    const int* tok = m->dev_i32;
    cudaStream_t st = m->stream;
    if (m->tok.repr == REPR_PACKED)
        return ib_embedding_q(m->tok.type, m->tok.w, tok, m->x, 1, c.vocab, c.dim, st);
    if (m->tok.repr == REPR_I16)
        return ib_embedding_batch_i16(m->tok.q, m->tok.s, tok, m->x, 1, c.dim, st);
    return ib_embedding_batch(m->tok.f, tok, m->x, 1, c.dim, st);
}

static int decode_launches_fused(Model* m) {
    const auto& c = m->cfg;
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn;
    const bool kq = m->slab_kq;
    cudaStream_t st = m->stream;
    const int* pos = m->dev_i32 + 1;
    const float scale = 1.0f / sqrtf((float)HD);
    const bool att_slab = m->att_counters && (H / Hkv * HD) % (kq ? 256 : 32) == 0;
    // row-split projections under TP: the GEMV adds every rank's rows (peer exchange)
    const int resid = m->tp_size > 1 ? EPI_ALLRED : EPI_RESID;
    // the slab kernel after such a GEMV completes x with the ranks' rows
    const TpExchange* tx = m->tp_size > 1 ? &m->tpx : nullptr;
    int r;
    if ((r = embed_launch(m))) return r;
    int* work = m->gemv_work;  // two counters per GEMV call site
    bool first = true;
    for (auto& L : m->layers) {
        FusedGemv qkv = fg_qkv(m, L), wo = fg_wo(m, L), fin = fg_ffn_in(m, L), fout = fg_ffn_out(m, L);
        qkv.work = work;
        wo.work = work + 2;
        fin.work = work + 4;
        fout.work = work + 6;
        work += 8;
        if ((r = xq_slab_launch(m->x, L.attn_norm, D, kq, m->slab_x, m->ssq, st, true,
                                first ? nullptr : tx)))
            return r;
        first = false;
        if ((r = fused_gemv_launch(qkv, PRO_NORM, EPI_QKV, st, true))) return r;
        if (att_slab) {  // attention writes the wo input's limb slab itself
            if ((r = attention_decode_fused(m->q, L.kc, L.vc, m->att, m->slab_att, kq, H, Hkv, HD,
                                            c.max_seq, scale, m->att_fpart, m->att_counters, st,
                                            pos, true, m->kv_f16)))
                return r;
        } else {
            if ((r = attention_decode(m->q, L.kc, L.vc, m->att, H, Hkv, HD, c.max_seq, 0, scale,
                                      m->att_part, st, pos, true, m->kv_f16)))
                return r;
            if ((r = xq_slab_launch(m->att, nullptr, H * HD, kq, m->slab_att, nullptr, st, true)))
                return r;
        }
        if ((r = fused_gemv_launch(wo, PRO_PLAIN, resid, st, true))) return r;
        if ((r = xq_slab_launch(m->x, L.ffn_norm, D, kq, m->slab_x, m->ssq, st, true, tx))) return r;
        if ((r = fused_gemv_launch(fin, PRO_NORM, EPI_SWIGLU, st, true))) return r;
        if ((r = xq_slab_launch(m->gate, nullptr, F, kq, m->slab_h, nullptr, st, true))) return r;
        if ((r = fused_gemv_launch(fout, PRO_PLAIN, resid, st, true))) return r;
    }
    if ((r = xq_slab_launch(m->x, m->out_norm, D, kq, m->slab_x, m->ssq, st, true,
                            m->layers.empty() ? nullptr : tx)))
        return r;
    FusedGemv head = fg_head(m);
    head.work = work;
    if ((r = fused_gemv_launch(head, PRO_NORM, EPI_ARGMAX, st, true))) return r;
    if (tx && (r = tp_key_max_launch(*tx, m->best, st))) return r;
    feedback_best_kernel<<<1, 256, 0, st>>>(m->best, m->dev_i32, m->dev_tokens, c.max_seq,
                                            m->gemv_work, (int)(work + 2 - m->gemv_work));
    IB_LAUNCH_CHECK("decode step");
    return IB_OK;
}

// One decode step for the token in dev_i32[0] at position dev_i32[1]; the greedy
// next token lands in dev_i32[2].  Every launch reads the position on the device.
static int decode_launches(Model* m) {
    if (persistent_active(m)) return step_launches(m);
    if (m->use_fused && m->fused_ok) return decode_launches_fused(m);
    const auto& c = m->cfg;
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn, V = c.vocab;
    cudaStream_t st = m->stream;
    const int* pos = m->dev_i32 + 1;
    const float scale = 1.0f / sqrtf((float)HD);
    int r;
    if ((r = embed_launch(m))) return r;
    const int g_ffn = (F + 255) / 256 < 1184 ? (F + 255) / 256 : 1184;
    for (auto& L : m->layers) {
        if ((r = rmsnorm_launch(m->x, L.attn_norm, m->xn, 1, D, c.rms_eps, st))) return r;
        if ((r = L.wq.forward(m->xn, m->q, st))) return r;
        if ((r = L.wk.forward(m->xn, m->k, st))) return r;
        if ((r = L.wv.forward(m->xn, m->v, st))) return r;
        if ((r = rope_launch(m->q, m->k, m->rope_table, H, Hkv, HD, 0, 1, st, pos))) return r;
        if ((r = kv_write_launch(L.kc, L.vc, m->k, m->v, Hkv, HD, c.max_seq, 0, 1, st, pos,
                                 m->kv_f16)))
            return r;
        if ((r = attention_decode(m->q, L.kc, L.vc, m->att, H, Hkv, HD, c.max_seq, 0, scale,
                                  m->att_part, st, pos, false, m->kv_f16)))
            return r;
        if ((r = L.wo.forward(m->att, m->proj, st))) return r;
        if ((r = tp_residual(m, m->x, m->proj, D, st))) return r;
        if ((r = rmsnorm_launch(m->x, L.ffn_norm, m->xn, 1, D, c.rms_eps, st))) return r;
        if ((r = L.w1.forward(m->xn, m->gate, st))) return r;
        if ((r = L.w3.forward(m->xn, m->up, st))) return r;
        silu_mul_kernel<<<g_ffn, 256, 0, st>>>(m->gate, m->up, F);
        if ((r = L.w2.forward(m->gate, m->proj, st))) return r;
        if ((r = tp_residual(m, m->x, m->proj, D, st))) return r;
    }
    if ((r = rmsnorm_launch(m->x, m->out_norm, m->xn, 1, D, c.rms_eps, st))) return r;
    if ((r = head_linear(m).forward(m->xn, m->logits_local, st))) return r;
    if ((r = gather_logits(m, st))) return r;
    if ((r = argmax_launch(m->logits, V, m->dev_i32 + 2, st))) return r;
    feedback_kernel<<<1, 1, 0, st>>>(m->dev_i32, m->dev_tokens, c.max_seq);
    IB_LAUNCH_CHECK("decode step");
    return IB_OK;
}

// A captured graph, destroyed on every return path (the executable graph instantiated
// from it keeps what it needs).
struct CapturedGraph {
    cudaGraph_t g = nullptr;
    ~CapturedGraph() {
        if (g) cudaGraphDestroy(g);
    }
};

static int ensure_graph(Model* m) {
    if (m->graph_exec || !m->use_graph) return IB_OK;
    CapturedGraph cg;
    IB_CUDA_CHECK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int r = decode_launches(m);
    cudaError_t e = cudaStreamEndCapture(m->stream, &cg.g);
    if (r != IB_OK) return r;
    IB_CUDA_CHECK(e);
    const cudaError_t ie = cudaGraphInstantiate(&m->graph_exec, cg.g, 0);
    if (ie != cudaSuccess) m->graph_exec = nullptr;
    IB_CUDA_CHECK(ie);
    return IB_OK;
}

int decode_step(Model* m, int token, int pos, float* host_logits, int* next) {
    IB_REQUIRE(pos >= 0 && pos < m->cfg.max_seq, "CUDA generate: position beyond the context");
    int* hp = (int*)m->host_pinned;
    hp[0] = token;
    hp[1] = pos;
    IB_CUDA_CHECK(cudaMemcpyAsync(m->dev_i32, hp, 8, cudaMemcpyHostToDevice, m->stream));
    int r = ensure_graph(m);
    if (r) return r;
    if (m->graph_exec) {
        IB_CUDA_CHECK(cudaGraphLaunch(m->graph_exec, m->stream));
    } else if ((r = decode_launches(m))) {
        return r;
    }
    IB_CUDA_CHECK(cudaMemcpyAsync(hp + 2, m->dev_i32 + 2, 4, cudaMemcpyDeviceToHost, m->stream));
    if (host_logits) {
        // the fused step keeps each rank's head rows local; gather them here (every rank
        // asks for logits on the same steps, so the collective matches)
        if (m->use_fused && m->fused_ok && (r = gather_logits(m, m->stream))) return r;
        IB_CUDA_CHECK(cudaMemcpyAsync(host_logits, m->logits, (size_t)m->cfg.vocab * 4,
                                      cudaMemcpyDeviceToHost, m->stream));
    }
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    if (next) *next = hp[2];
    return IB_OK;
}

static int ensure_prefill_scratch(Model* m, int T) {
    if (T <= m->pf_cap) return IB_OK;
    for (void* p : m->pf_bufs) cudaFree(p);
    m->pf_bufs.clear();
    const auto& c = m->cfg;
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn;
    float** bufs[] = {&m->pf_x, &m->pf_xn, &m->pf_q, &m->pf_k, &m->pf_v, &m->pf_att, &m->pf_proj,
                      &m->pf_gate, &m->pf_up};
    const size_t per[] = {(size_t)D, (size_t)D, (size_t)H * HD, (size_t)Hkv * HD, (size_t)Hkv * HD,
                          (size_t)H * HD, (size_t)D, (size_t)F, (size_t)F};
    size_t need = 0;
    for (size_t s : per) need += s * T * 4;
    size_t free_b = 0, total_b = 0;
    IB_CUDA_CHECK(cudaMemGetInfo(&free_b, &total_b));
    if (need + (32ull << 20) > free_b) {
        set_error("CUDA prefill: prompt needs ~" + std::to_string(need >> 20) +
                  " MB scratch but only " + std::to_string(free_b >> 20) +
                  " MB VRAM is free. Shorten the prompt or use the CPU backend.");
        return IB_ERR_OOM;
    }
    for (int i = 0; i < 9; ++i) {
        IB_CUDA_CHECK(cudaMalloc(bufs[i], per[i] * T * 4 + 16));
        m->pf_bufs.push_back(*bufs[i]);
    }
    IB_CUDA_CHECK(cudaMalloc(&m->pf_ids, (size_t)T * 4 + 16));
    m->pf_bufs.push_back(m->pf_ids);
    m->pf_cap = T;
    return IB_OK;
}

int prefill(Model* m, const int32_t* host_ids, int T, int start, float* host_logits, int* next) {
    const auto& c = m->cfg;
    IB_REQUIRE(T > 0 && start >= 0 && start + T <= c.max_seq, "CUDA generate: prompt longer than context");
    int r = ensure_prefill_scratch(m, T);
    if (r) return r;
    const int D = c.dim, H = c.n_heads, Hkv = c.n_kv_heads, HD = m->HD, F = c.ffn, V = c.vocab;
    cudaStream_t st = m->stream;
    IB_CUDA_CHECK(cudaMemcpyAsync(m->pf_ids, host_ids, (size_t)T * 4, cudaMemcpyHostToDevice, st));
    if (m->tok.repr == REPR_PACKED) r = ib_embedding_q(m->tok.type, m->tok.w, m->pf_ids, m->pf_x, T, V, D, st);
    else if (m->tok.repr == REPR_I16) r = ib_embedding_batch_i16(m->tok.q, m->tok.s, m->pf_ids, m->pf_x, T, D, st);
    else r = ib_embedding_batch(m->tok.f, m->pf_ids, m->pf_x, T, D, st);
    if (r) return r;
    const float scale = 1.0f / sqrtf((float)HD);
    for (auto& L : m->layers) {
        if ((r = rmsnorm_launch(m->pf_x, L.attn_norm, m->pf_xn, T, D, c.rms_eps, st))) return r;
        if ((r = L.wq.forward_batch(m->pf_xn, m->pf_q, T, st))) return r;
        if ((r = L.wk.forward_batch(m->pf_xn, m->pf_k, T, st))) return r;
        if ((r = L.wv.forward_batch(m->pf_xn, m->pf_v, T, st))) return r;
        if ((r = rope_launch(m->pf_q, m->pf_k, m->rope_table, H, Hkv, HD, start, T, st, nullptr))) return r;
        if ((r = kv_write_launch(L.kc, L.vc, m->pf_k, m->pf_v, Hkv, HD, c.max_seq, start, T, st,
                                 nullptr, m->kv_f16)))
            return r;
        if ((r = attention_batch_launch(m->pf_q, L.kc, L.vc, m->pf_att, H, Hkv, HD, c.max_seq, start,
                                        T, scale, st, m->kv_f16)))
            return r;
        if ((r = L.wo.forward_batch(m->pf_att, m->pf_proj, T, st))) return r;
        if ((r = tp_residual(m, m->pf_x, m->pf_proj, (size_t)T * D, st))) return r;
        if ((r = rmsnorm_launch(m->pf_x, L.ffn_norm, m->pf_xn, T, D, c.rms_eps, st))) return r;
        if ((r = L.w1.forward_batch(m->pf_xn, m->pf_gate, T, st))) return r;
        if ((r = L.w3.forward_batch(m->pf_xn, m->pf_up, T, st))) return r;
        silu_mul_kernel<<<1184, 256, 0, st>>>(m->pf_gate, m->pf_up, T * F);
        if ((r = L.w2.forward_batch(m->pf_gate, m->pf_proj, T, st))) return r;
        if ((r = tp_residual(m, m->pf_x, m->pf_proj, (size_t)T * D, st))) return r;
    }
    // logits of the last prompt position only (model_cuda.cpp:394-398)
    if ((r = rmsnorm_launch(m->pf_x + (size_t)(T - 1) * D, m->out_norm, m->xn, 1, D, c.rms_eps, st))) return r;
    if ((r = head_linear(m).forward(m->xn, m->logits_local, st))) return r;
    if ((r = gather_logits(m, st))) return r;
    if ((r = argmax_launch(m->logits, V, m->dev_i32 + 2, st))) return r;
    int* hp = (int*)m->host_pinned;
    IB_CUDA_CHECK(cudaMemcpyAsync(hp + 2, m->dev_i32 + 2, 4, cudaMemcpyDeviceToHost, st));
    if (host_logits)
        IB_CUDA_CHECK(cudaMemcpyAsync(host_logits, m->logits, (size_t)V * 4, cudaMemcpyDeviceToHost, st));
    IB_CUDA_CHECK(cudaStreamSynchronize(st));
    if (next) *next = hp[2];
    return IB_OK;
}

}  // namespace ib

extern "C" int ib_model_prefill(void* h, const int32_t* host_ids, int T, int start,
                                float* host_logits, int32_t* next) {
    IB_REQUIRE(h && host_ids, "null pointer argument");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized, "model: call ib_model_finalize first");
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    return prefill(m, host_ids, T, start, host_logits, next);
}

extern "C" int ib_model_decode(void* h, int32_t token, int pos, float* host_logits,
                               int32_t* next) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized, "model: call ib_model_finalize first");
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    return decode_step(m, token, pos, host_logits, next);
}

// n_steps greedy decode steps entirely on the device: token `token` at `pos`,
// each step's argmax fed back as the next input (no host round trip between
// steps).  The generated ids are copied to host_tokens[0..n_steps).
extern "C" int ib_model_decode_loop(void* h, int32_t token, int pos, int n_steps,
                                    int32_t* host_tokens) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized, "model: call ib_model_finalize first");
    IB_REQUIRE(n_steps >= 0 && pos >= 0 && pos + n_steps <= m->cfg.max_seq,
               "CUDA generate: position beyond the context");
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    int* hp = (int*)m->host_pinned;
    hp[0] = token;
    hp[1] = pos;
    IB_CUDA_CHECK(cudaMemcpyAsync(m->dev_i32, hp, 8, cudaMemcpyHostToDevice, m->stream));
    int r = ensure_graph(m);
    if (r) return r;
    for (int i = 0; i < n_steps; ++i) {
        if (m->graph_exec) IB_CUDA_CHECK(cudaGraphLaunch(m->graph_exec, m->stream));
        else if ((r = decode_launches(m))) return r;
    }
    if (host_tokens && n_steps > 0)
        IB_CUDA_CHECK(cudaMemcpyAsync(host_tokens, m->dev_tokens + pos, (size_t)n_steps * 4,
                                      cudaMemcpyDeviceToHost, m->stream));
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    return IB_OK;
}

// The stream the model launches on (cudaStream_t as void*), for event timing.
extern "C" int ib_model_stream(void* h, void** stream) {
    IB_REQUIRE(h && stream, "null pointer argument");
    *stream = ((Model*)h)->stream;
    return IB_OK;
}

// Kernels launched by one decode step (nodes of the captured graph).
extern "C" int ib_model_step_kernels(void* h, int* n) {
    IB_REQUIRE(h && n, "null pointer argument");
    Model* m = (Model*)h;
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    int r = ensure_graph(m);
    if (r) return r;
    CapturedGraph cg;
    IB_CUDA_CHECK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    r = decode_launches(m);
    cudaError_t e = cudaStreamEndCapture(m->stream, &cg.g);
    if (r) return r;
    IB_CUDA_CHECK(e);
    size_t count = 0;
    IB_CUDA_CHECK(cudaGraphGetNodes(cg.g, nullptr, &count));
    std::vector<cudaGraphNode_t> nodes(count);
    IB_CUDA_CHECK(cudaGraphGetNodes(cg.g, nodes.data(), &count));
    int k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        IB_CUDA_CHECK(cudaGraphNodeGetType(nd, &t));
        if (t == cudaGraphNodeTypeKernel) ++k;
    }
    *n = k;
    return IB_OK;
}

extern "C" int ib_model_set_fused(void* h, int enabled) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    m->use_fused = enabled != 0;
    if (m->graph_exec) {
        cudaGraphExecDestroy(m->graph_exec);
        m->graph_exec = nullptr;
    }
    return IB_OK;
}

extern "C" int ib_model_set_prefill_planes(void* h, int enabled) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized, "prefill planes: finalize the model first");
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    std::vector<Linear*> lins;
    for (auto& L : m->layers)
        for (Linear* l : {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3}) lins.push_back(l);
    if (!enabled) {
        for (Linear* l : lins)
            if (l->planes) {
                cudaFree(l->planes);
                l->planes = nullptr;
            }
        return IB_OK;
    }
    size_t need = 0;
    for (Linear* l : lins)
        if (l->repr == REPR_PACKED && !l->planes && gemm_planes_supported(l->type, 128, l->rows, l->cols))
            need += (size_t)l->rows * l->cols * 4 + 16;
    size_t free_b = 0, total_b = 0;
    IB_CUDA_CHECK(cudaMemGetInfo(&free_b, &total_b));
    if (need + (1ull << 30) > free_b) {
        set_error("prefill planes: need ~" + std::to_string(need >> 20) + " MB but only " +
                  std::to_string(free_b >> 20) + " MB is free");
        return IB_ERR_OOM;
    }
    for (Linear* l : lins) {
        if (l->repr != REPR_PACKED || l->planes ||
            !gemm_planes_supported(l->type, 128, l->rows, l->cols))
            continue;
        IB_CUDA_CHECK(cudaMalloc(&l->planes, (size_t)l->rows * l->cols * 4 + 16));
        int r = gemm_decode_planes(l->type, l->w, l->planes, l->rows, l->cols, m->stream);
        if (r) return r;
    }
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    return IB_OK;
}

extern "C" int ib_model_set_kv_type(void* h, int type) {
    IB_REQUIRE(h, "null model");
    IB_REQUIRE(type == IB_TYPE_F32 || type == IB_TYPE_F16, "KV cache type must be F32 or F16");
    Model* m = (Model*)h;
    const bool f16 = type == IB_TYPE_F16;
    if (f16 == m->kv_f16) return IB_OK;
    m->kv_f16 = f16;
    if (!m->finalized) return IB_OK;
    // a finalized model: new, empty caches (positions must be prefilled again)
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    if (m->graph_exec) {
        cudaGraphExecDestroy(m->graph_exec);
        m->graph_exec = nullptr;
    }
    int r = alloc_kv(m);
    if (r == IB_OK) r = build_step_plan(m);
    if (r == IB_OK) IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
    return r;
}

extern "C" int ib_model_kv_type(void* h, int* type) {
    IB_REQUIRE(h && type, "null pointer argument");
    *type = ((Model*)h)->kv_f16 ? IB_TYPE_F16 : IB_TYPE_F32;
    return IB_OK;
}

extern "C" int ib_model_set_persistent(void* h, int enabled) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    m->use_persistent = enabled != 0;
    if (m->graph_exec) {
        cudaGraphExecDestroy(m->graph_exec);
        m->graph_exec = nullptr;
    }
    return IB_OK;
}

extern "C" int ib_model_decode_path(void* h, int* path) {
    IB_REQUIRE(h && path, "null pointer argument");
    Model* m = (Model*)h;
    *path = persistent_active(m) ? IB_DECODE_PERSISTENT
            : (m->use_fused && m->fused_ok) ? IB_DECODE_FUSED : IB_DECODE_SEPARATE;
    return IB_OK;
}

extern "C" int ib_model_uses_fused(void* h, int* fused) {
    IB_REQUIRE(h && fused, "null pointer argument");
    Model* m = (Model*)h;
    *fused = (m->use_fused && m->fused_ok) ? 1 : 0;
    return IB_OK;
}

extern "C" int ib_model_set_graph(void* h, int enabled) {
    IB_REQUIRE(h, "null model");
    Model* m = (Model*)h;
    m->use_graph = enabled != 0;
    if (!m->use_graph && m->graph_exec) {
        cudaGraphExecDestroy(m->graph_exec);
        m->graph_exec = nullptr;
    }
    return IB_OK;
}

// Greedy generation with the reference's loop structure (generate_cuda,
// model_cuda.cpp:442-495): batched prefill, first token from the prefill
// logits, then one decode step per token until max_tokens, the context end, or
// eos_token_id (when >= 0).
extern "C" int ib_model_generate(void* h, const int32_t* prompt, int n_prompt, int max_tokens,
                                 int32_t eos_token_id, int32_t* out, int* n_out,
                                 ib_generation_stats* stats) {
    IB_REQUIRE(h && prompt && out && n_out, "null pointer argument");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized, "model: call ib_model_finalize first");
    if (n_prompt <= 0) {
        set_error("CUDA generate: empty prompt");
        return IB_ERR_INVALID;
    }
    if (n_prompt > m->cfg.max_seq) {
        set_error("CUDA generate: prompt longer than context");
        return IB_ERR_INVALID;
    }
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    const double t1 = now_ms();
    int n = 0;
    for (int i = 0; i < n_prompt; ++i) out[n++] = prompt[i];
    int next = 0;
    int r = prefill(m, prompt, n_prompt, 0, nullptr, &next);
    if (r) return r;
    const double t2 = now_ms();
    int pos = n_prompt;
    if (max_tokens > 0) out[n++] = next;
    for (int step = 1; step < max_tokens; ++step) {
        if (eos_token_id >= 0 && next == eos_token_id) break;
        if (pos >= m->cfg.max_seq) break;
        if ((r = decode_step(m, next, pos, nullptr, &next))) return r;
        ++pos;
        out[n++] = next;
    }
    const double t3 = now_ms();
    *n_out = n;
    if (stats) {
        stats->init_ms = 0;
        stats->prefill_ms = t2 - t1;
        stats->decode_ms = t3 - t2;
        stats->generated = n - n_prompt;
    }
    return IB_OK;
}

// Loads a GGUF file: metadata keys as load_model_weights reads them
// (src/models/transformer.cpp:139-154), tensors copied to HBM in their GGUF form.
static int load_gguf(const char* path, int precision, int device, int max_seq, Comm* comm,
                     void** out) {
    IB_REQUIRE(path && out, "null pointer argument");
    *out = nullptr;
    try {
        GGUFFile f;
        f.open(path);
        ib_model_config c{};
        c.n_layers = (int)f.get_int("llama.block_count", 0);
        c.dim = (int)f.get_int("llama.embedding_length", 0);
        c.n_heads = (int)f.get_int("llama.attention.head_count", 0);
        c.n_kv_heads = (int)f.get_int("llama.attention.head_count_kv", c.n_heads);
        c.max_seq = max_seq > 0 ? max_seq : (int)f.get_int("llama.context_length", 2048);
        c.rope_theta = f.get_float("llama.rope.freq_base", 10000.0f);
        c.rms_eps = f.get_float("llama.attention.layer_norm_rms_epsilon", 1e-6f);
        c.precision = precision;
        const auto* te = f.find("token_embd.weight");
        if (!te || te->dims.size() != 2) {
            set_error("Tensor not found: token_embd.weight");
            return IB_ERR_INVALID;
        }
        c.vocab = (int)te->dims[1];
        const auto* g = f.find("blk.0.ffn_gate.weight");
        c.ffn = g && g->dims.size() == 2 ? (int)g->dims[1] : (int)f.get_int("llama.feed_forward_length", 0);
        // Every tensor's shape, type and byte range are checked before any device work,
        // so a malformed file fails here with nothing to release.
        struct Planned {
            const GGUFFile::TensorInfo* t;
            int64_t rows, cols;
            const uint8_t* bytes;
        };
        std::vector<Planned> plan;
        for (const auto& t : f.tensors()) {
            if (t.dims.empty() || t.dims.size() > 4)
                throw std::runtime_error("GGUF: tensor " + t.name + " has " +
                                         std::to_string(t.dims.size()) + " dimensions");
            int64_t elems = 1;
            for (int64_t d : t.dims) {
                if (d <= 0 || d > INT32_MAX || elems > (int64_t(1) << 40) / d)
                    throw std::runtime_error("GGUF: tensor " + t.name + " has a dimension out of range");
                elems *= d;
            }
            const int64_t cols = t.dims[0], rows = elems / cols;
            const int64_t nb = t.type == IB_TYPE_F32 ? elems * 4
                               : t.type == IB_TYPE_F16 ? elems * 2
                                                       : packed_bytes(t.type, rows, cols);
            if (nb < 0) {
                set_error("model: unsupported tensor type in " + t.name);
                return IB_ERR_UNSUPPORTED;
            }
            plan.push_back({&t, rows, cols, f.data(t, (size_t)nb)});
        }
        void* h = nullptr;
        int st = model_create(&c, device, comm, &h);
        if (st) return st;
        for (const Planned& pl : plan) {
            const auto& t = *pl.t;
            st = ib_model_set_tensor(h, t.name.c_str(), t.type, pl.rows, pl.cols, pl.bytes, 0);
            if (st) {
                if (st == IB_ERR_INVALID && ib::last_error().rfind("model: unknown tensor", 0) == 0) continue;
                ib_model_free(h);
                return st;
            }
        }
        Model* m = (Model*)h;
        IB_CUDA_CHECK(cudaStreamSynchronize(m->stream));
        st = ib_model_finalize(h);
        if (st) {
            ib_model_free(h);
            return st;
        }
        *out = h;
        return IB_OK;
    } catch (const std::exception& e) {
        set_error(e.what());
        return IB_ERR_INVALID;
    }
}

extern "C" int ib_model_load_gguf(const char* path, int precision, int device, int max_seq,
                                  void** out) {
    return load_gguf(path, precision, device, max_seq, nullptr, out);
}

extern "C" int ib_model_load_gguf_tp(const char* path, int precision, int device, int max_seq,
                                     void* comm, void** out) {
    IB_REQUIRE(comm, "null communicator");
    return load_gguf(path, precision, device, max_seq, (Comm*)comm, out);
}

extern "C" int ib_model_tp_exchange_time(void* h, int rounds, float* us_per_round) {
    IB_REQUIRE(h && us_per_round && rounds > 0, "bad arguments");
    Model* m = (Model*)h;
    IB_REQUIRE(m->finalized && m->tp_size > 1 && m->tpx.world > 1,
               "exchange timing: not a finalized tensor-parallel model");
    IB_CUDA_CHECK(cudaSetDevice(m->device));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    IB_CUDA_CHECK(cudaEventCreate(&e0));
    IB_CUDA_CHECK(cudaEventCreate(&e1));
    int r = IB_OK;
    // one untimed round, then the timed ones (every rank runs the same rounds)
    for (int i = 0; i <= rounds && r == IB_OK; ++i) {
        if (i == 1 && cudaEventRecord(e0, m->stream) != cudaSuccess) r = IB_ERR_CUDA;
        if (r == IB_OK)
            r = tp_probe_launch(m->tpx, m->x, m->cfg.dim, m->slab_kq, m->slab_x, m->stream);
    }
    float ms = 0.f;
    if (r == IB_OK && (cudaEventRecord(e1, m->stream) != cudaSuccess ||
                       cudaEventSynchronize(e1) != cudaSuccess ||
                       cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess)) {
        set_error("exchange timing: event failure");
        r = IB_ERR_CUDA;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (r) return r;
    int fault = 0;
    if ((r = decode_fault_take(&fault))) return r;
    if (fault) {
        set_error("exchange timing: a peer's rows did not arrive (fault " + std::to_string(fault) + ")");
        return IB_ERR_TIMEOUT;
    }
    *us_per_round = ms * 1000.f / (float)rounds;
    return IB_OK;
}

extern "C" int ib_model_get_config(void* h, ib_model_config* cfg) {
    IB_REQUIRE(h && cfg, "null pointer argument");
    *cfg = ((Model*)h)->full;
    return IB_OK;
}

extern "C" int ib_model_weight_bytes(void* h, size_t* bytes) {
    IB_REQUIRE(h && bytes, "null pointer argument");
    Model* m = (Model*)h;
    size_t n = 0;
    auto add = [&](const Linear& L) {
        if (L.repr == REPR_PACKED) n += (size_t)packed_bytes(L.type, L.rows, L.cols);
        else if (L.repr == REPR_I16) n += (size_t)(L.rows * L.cols) * 2 + (size_t)L.rows * 4;
        else if (L.repr == REPR_F32) n += (size_t)(L.rows * L.cols) * 4;
    };
    add(m->tok);
    if (m->has_output) add(m->out);
    for (auto& L : m->layers)
        for (const Linear* l : {&L.wq, &L.wk, &L.wv, &L.wo, &L.w1, &L.w2, &L.w3}) add(*l);
    n += (size_t)m->cfg.dim * 4 * (1 + 2 * m->cfg.n_layers);
    *bytes = n;
    return IB_OK;
}
