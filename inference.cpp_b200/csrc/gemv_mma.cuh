// Int8-MMA fused dequant-GEMV (gemv_mma.cu): activation limbs and launchers.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ib {

// FP32 activation split into exact int8 limbs: limbs[K/32][4][32], one power-of-two
// scale per group (32 or 256 elements), FP32 sum per 32 elements.
struct XLimbs {
    int8_t* limbs = nullptr;
    float* scale = nullptr;
    float* sum32 = nullptr;
    float* sum16 = nullptr;
};

size_t xlimbs_bytes(int K);
void xlimbs_carve(void* base, int K, XLimbs& xb);
int xq_launch(const float* x, int K, int group, XLimbs& xb, cudaStream_t st);
int gemv_mma_group(int type);
bool gemv_mma_supported(int type);
int gemv_mma_align(int type);
int gemv_mma_launch(int type, const void* W, const XLimbs& xb, float* y, int64_t rows,
                    int64_t cols, cudaStream_t st);
// Launch set-up of every format's GEMV kernels on the current device (function
// attributes, shared-memory opt-in, occupancy, module loading), so later first calls of
// a format do none of it.  Idempotent and thread-safe.
int gemv_mma_prepare_device();
// Reads and clears the GEMV kernels' fault word (0 = no bounded wait expired).
int gemv_fault_take(int* code);

}  // namespace ib
