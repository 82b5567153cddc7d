// Shared plumbing for the C-ABI entry points: status codes, the thread-local
// last-error string, argument checks and stream conversion.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/ib_cuda.h"

namespace ib {

void set_error(const std::string& msg);
const std::string& last_error();

// GGUF type table (reference include/core/tensor.hpp:204-262).
inline int block_elems(int type) {
    switch (type) {
        case IB_TYPE_Q4_0: case IB_TYPE_Q5_0: case IB_TYPE_Q5_1: case IB_TYPE_Q8_0: return 32;
        case IB_TYPE_Q4_K: case IB_TYPE_Q6_K: return 256;
        case IB_TYPE_Q4_1: return 32;
        case IB_TYPE_Q2_K: case IB_TYPE_Q3_K: case IB_TYPE_Q5_K: return 256;
        case IB_TYPE_F32: case IB_TYPE_F16: case IB_TYPE_I16: return 1;
        default: return 0;
    }
}
inline int block_bytes(int type) {
    switch (type) {
        case IB_TYPE_F32: return 4;
        case IB_TYPE_F16: return 2;
        case IB_TYPE_I16: return 2;
        case IB_TYPE_Q4_0: return 18;
        case IB_TYPE_Q5_0: return 22;
        case IB_TYPE_Q5_1: return 24;
        case IB_TYPE_Q8_0: return 34;
        case IB_TYPE_Q4_K: return 144;
        case IB_TYPE_Q6_K: return 210;
        case IB_TYPE_Q4_1: return 20;
        case IB_TYPE_Q2_K: return 84;
        case IB_TYPE_Q3_K: return 110;
        case IB_TYPE_Q5_K: return 176;
        default: return 0;
    }
}
// The six formats the reference decodes (every kernel family takes them).
inline bool is_block_quant(int type) {
    return type == IB_TYPE_Q4_0 || type == IB_TYPE_Q5_0 || type == IB_TYPE_Q5_1 ||
           type == IB_TYPE_Q8_0 || type == IB_TYPE_Q4_K || type == IB_TYPE_Q6_K;
}
// Formats the reference sizes but does not decode (src/gguf/quantization.cpp:201-204
// throw), decoded here from the published GGUF layouts: dequantisation, embedding,
// a generic decode-as-you-go GEMV and the weight-planes GEMM take them.
inline bool is_extra_quant(int type) {
    return type == IB_TYPE_Q4_1 || type == IB_TYPE_Q2_K || type == IB_TYPE_Q3_K ||
           type == IB_TYPE_Q5_K;
}
inline bool is_quant(int type) { return is_block_quant(type) || is_extra_quant(type); }
inline const char* type_name(int type) {
    switch (type) {
        case IB_TYPE_F32: return "F32";
        case IB_TYPE_F16: return "F16";
        case IB_TYPE_Q4_0: return "Q4_0";
        case IB_TYPE_Q5_0: return "Q5_0";
        case IB_TYPE_Q5_1: return "Q5_1";
        case IB_TYPE_Q8_0: return "Q8_0";
        case IB_TYPE_Q4_K: return "Q4_K";
        case IB_TYPE_Q6_K: return "Q6_K";
        case IB_TYPE_Q4_1: return "Q4_1";
        case IB_TYPE_Q2_K: return "Q2_K";
        case IB_TYPE_Q3_K: return "Q3_K";
        case IB_TYPE_Q5_K: return "Q5_K";
        case IB_TYPE_I16: return "I16";
        default: return "?";
    }
}
// Packed bytes of a [rows, cols] tensor (reference type_nbytes, tensor.hpp:228-243).
inline int64_t packed_bytes(int type, int64_t rows, int64_t cols) {
    const int be = block_elems(type);
    if (be <= 0) return -1;
    return rows * (cols / be) * block_bytes(type);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace ib

// Returns from the enclosing C-ABI function with IB_ERR_CUDA on a CUDA error.
#define IB_CUDA_CHECK(expr)                                                           \
    do {                                                                              \
        cudaError_t e_ = (expr);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            ib::set_error(std::string("CUDA: ") + #expr + " failed: " +               \
                          cudaGetErrorString(e_));                                    \
            return IB_ERR_CUDA;                                                       \
        }                                                                             \
    } while (0)

// Checks the launch just issued (configuration errors surface here).
#define IB_LAUNCH_CHECK(what)                                                         \
    do {                                                                              \
        cudaError_t e_ = cudaGetLastError();                                          \
        if (e_ != cudaSuccess) {                                                      \
            ib::set_error(std::string("CUDA: ") + (what) + " failed: " +              \
                          cudaGetErrorString(e_));                                    \
            return IB_ERR_CUDA;                                                       \
        }                                                                             \
    } while (0)

#define IB_REQUIRE(cond, msg)                                                         \
    do {                                                                              \
        if (!(cond)) {                                                                \
            ib::set_error(std::string(msg));                                          \
            return IB_ERR_INVALID;                                                    \
        }                                                                             \
    } while (0)
