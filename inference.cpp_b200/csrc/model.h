// Internal state of the native model runner (model.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/ib_cuda.h"
#include "decode.cuh"
#include "step.cuh"

namespace ib {

struct Comm;

enum Repr { REPR_NONE = 0, REPR_PACKED = 1, REPR_I16 = 2, REPR_F32 = 3 };

// One weight matrix [rows, cols]: GGUF blocks (packed), INT16 + row scale, or FP32.
struct Linear {
    int repr = REPR_NONE;
    int type = 0;
    int64_t rows = 0, cols = 0;
    void* w = nullptr;       // packed blocks
    int16_t* q = nullptr;    // INT16 values
    float* s = nullptr;      // INT16 row scales
    float* f = nullptr;      // FP32 values
    void* planes = nullptr;  // PACKED, optional: the weights as FP16 hi/lo planes (prefill)
    int forward(const float* x, float* y, cudaStream_t st) const;
    int forward_batch(const float* X, float* Y, int T, cudaStream_t st) const;
    void release();
};

struct Layer {
    Linear wq, wk, wv, wo, w1, w2, w3;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* kc = nullptr;  // [Hkv][max_seq][HD]: FP32, or __half when Model::kv_f16
    float* vc = nullptr;
};

struct Model {
    // With tensor parallelism cfg holds this rank's share (n_heads, n_kv_heads, ffn
    // divided by the TP size; dim and vocab whole) and `full` the model's configuration.
    ib_model_config cfg{};
    ib_model_config full{};
    Comm* comm = nullptr;  // not owned
    int tp_rank = 0, tp_size = 1;
    int vocab_local = 0, vocab_base = 0;  // output head rows of this rank
    Linear head_view;                     // tied embedding: this rank's head rows (not owned)
    float* logits_local = nullptr;        // == logits without TP
    // fused TP decode: the peer-memory exchange of the row-split GEMVs (decode.cuh)
    TpExchange tpx{};
    uint8_t* tp_local = nullptr;       // this rank's exchange region (owned)
    void* tp_peers[kMaxRanks] = {};    // every rank's region, mapped here
    int device = 0;
    int HD = 0;
    bool finalized = false;
    bool has_output = false;
    bool use_graph = true;
    bool use_fused = true;  // fused decode kernels when every weight supports them
    bool kv_f16 = false;    // the KV cache in FP16 (ib_model_set_kv_type)
    bool fused_ok = false;
    // K split of the down projection (one GPU): partial rows and arrival counters
    float* kpart = nullptr;
    int* kcnt = nullptr;
    // persistent decode step (step.cu): one kernel per token, single GPU
    bool use_persistent = false;
    bool persistent_ok = false;
    StepParams step{};
    int step_grid = 0, step_type = 0;
    size_t step_ctr_bytes = 0;
    Linear tok, out;
    float* out_norm = nullptr;
    std::vector<Layer> layers;
    float* rope_table = nullptr;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    // decode activations
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *proj = nullptr, *gate = nullptr, *up = nullptr, *logits = nullptr, *att_part = nullptr;
    int32_t* dev_i32 = nullptr;  // [0] token, [1] position, [2] next token
    unsigned long long* best = nullptr;  // fused head: (ordered logit << 32 | ~row) max
    // fused path: limb slabs of the GEMV inputs and RMSNorm sums of squares
    bool slab_kq = true;
    uint8_t *slab_x = nullptr, *slab_att = nullptr, *slab_h = nullptr;
    float* ssq = nullptr;
    int* gemv_work = nullptr;     // fused GEMV work counters, two per call site of a step
    float* att_fpart = nullptr;   // fused attention partials
    int* att_counters = nullptr;  // fused attention: per kv head, zero between steps
    int32_t* dev_tokens = nullptr;  // [max_seq] ids produced by decode steps, by position
    void* host_pinned = nullptr;
    // prefill scratch (grown on demand)
    int pf_cap = 0;
    float *pf_x = nullptr, *pf_xn = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr;
    float *pf_att = nullptr, *pf_proj = nullptr, *pf_gate = nullptr, *pf_up = nullptr;
    int32_t* pf_ids = nullptr;
    std::vector<void*> pf_bufs;
    std::vector<void*> allocations;
    ~Model();
};

int decode_step(Model* m, int token, int pos, float* host_logits, int* next);
// True when every decode GEMV of the model has a fused kernel (decode.cu).
bool fused_supported(const Model* m);
// Plans the persistent decode step when the model supports it (sets persistent_ok).
int build_step_plan(Model* m);
int prefill(Model* m, const int32_t* host_ids, int T, int start, float* host_logits, int* next);

}  // namespace ib
