// Internal launchers shared by the C-ABI wrappers and the model runner.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ib {

enum { WS_ATTENTION = 0, WS_GEMV = 1, WS_GEMM = 2, WS_GEMM_W = 3, WS_ATTN_PLANES = 4, WS_GEMM_PART = 5, WS_SLOTS = 6 };
int workspace_get(int slot, size_t bytes, void** out);
size_t attention_partial_bytes(int H, int HD, int pos);
// Decode attention in one launch (split flash-decode, last-CTA combine); also writes
// the output's limb slab when `slab` is set.  `counters` (n_kv_heads ints) must start
// at zero; they are left at zero.  part: attention_fused_part_bytes(H, HD).
bool attention_fused_ok(int H, int Hkv, int HD);
size_t attention_fused_part_bytes(int H, int HD);
// kv_half: the cache holds FP16 (kc, vc then point to __half), else FP32.
int attention_decode_fused(const float* q, const void* kc, const void* vc, float* out,
                           uint8_t* slab, bool slab_kq, int H, int Hkv, int HD, int max_seq,
                           float scale, float* part, int* counters, cudaStream_t st,
                           const int* pos_dev, bool pdl, bool kv_half = false);
int check_attention_args(int H, int Hkv, int HD, int max_seq, int pos);
// pos_dev != nullptr: the position is read on the device (graph-capturable) and the
// partial buffer must hold attention_partial_bytes(H, HD, max_seq - 1).
// kv_half: FP16 cache (the generic partial kernel).
int attention_decode(const float* q, const void* kc, const void* vc, float* out, int H,
                     int Hkv, int HD, int max_seq, int pos, float scale, float* part,
                     cudaStream_t st, const int* pos_dev, bool pdl = false, bool kv_half = false);
// Prefill attention as flash attention over K/V tiles on the tensor cores (attention.cu):
// head_dim 64 or 128, H a multiple of Hkv with H / Hkv dividing 128.
bool attention_prefill_ok(int H, int Hkv, int HD);
int attention_prefill(const float* q, const void* kc, const void* vc, float* out, int H, int Hkv,
                      int HD, int max_seq, int start, int T, float scale, cudaStream_t st,
                      bool kv_half = false);
int attention_batch_launch(const float* q, const void* kc, const void* vc, float* out, int H,
                           int Hkv, int HD, int max_seq, int start, int T, float scale,
                           cudaStream_t st, bool kv_half = false);
int rope_launch(float* q, float* k, const float* table, int H, int Hkv, int HD, int start,
                int T, cudaStream_t st, const int* start_dev);
int rmsnorm_launch(const float* x, const float* w, float* out, int rows, int dim, float eps,
                   cudaStream_t st);
int kv_write_launch(void* kc, void* vc, const float* k, const float* v, int Hkv, int HD,
                    int max_seq, int start, int T, cudaStream_t st, const int* start_dev,
                    bool kv_half = false);
int argmax_launch(const float* x, int n, int32_t* out, cudaStream_t st);
// op: 0 silu(a), 1 a *= b, 2 a += b
int elementwise_launch(int op, float* a, const float* b, int n, cudaStream_t st);
// Prefill GEMM on the tensor cores (gemm_tc.cu): packed weights, cols % 64 == 0.
bool gemm_tc_supported(int type, int64_t T, int64_t rows, int64_t cols);
// X (FP32, n values) -> FP16 hi/lo planes (gemm_tc.cu).
int gemm_split_x(const float* X, void* Xh, void* Xl, size_t n, cudaStream_t st);
// The tcgen05 GEMM on dequantised FP16 planes fed by TMA (gemm_tma.cu).
bool gemm_planes_supported(int type, int64_t T, int64_t rows, int64_t cols);
int gemm_q_planes(int type, const void* W, const float* X, float* Y, int T, int rows, int cols,
                  cudaStream_t st);
int gemm_planes_fault_take(int* code);
// The weights decoded once into FP16 hi/lo planes (4 bytes per weight: hi [rows][cols]
// then lo), and the GEMM on such planes.
int gemm_decode_planes(int type, const void* W, void* planes, int64_t rows, int64_t cols,
                       cudaStream_t st);
int gemm_on_planes(const void* planes, const float* X, float* Y, int T, int rows, int cols,
                   cudaStream_t st);
int gemm_q_tc(int type, const void* W, const float* X, float* Y, int T, int rows, int cols,
              cudaStream_t st);
int gemm_fault_take(int* code);
int gemm_q_simt(int type, const void* W, const float* X, float* Y, int T, int M, int K,
                cudaStream_t st);

}  // namespace ib
