// Dequantisation kernels: packed GGUF blocks -> FP32 (bit-exact with the
// reference dequantize()), -> per-row symmetric INT16 (bit-exact with the
// reference make_weight / quantize_i16), and the dequantising embedding gather.
//
// Layout: one thread per 8 consecutive output elements; a warp covers 256
// contiguous outputs (one K-quant super-block, or 8 32-element blocks), so the
// FP32 stores are 2 x 16 B per thread, fully coalesced.  These kernels are
// HBM-bound on their output (4 B or 2 B per element vs <= 1.07 B read).
#include "common.cuh"
#include "quant.cuh"

namespace ib {

template <int TYPE>
__device__ __forceinline__ void deq_group(const uint8_t* W, int64_t gidx, float* y) {
    constexpr int BE = QFmt<TYPE>::BE, BB = QFmt<TYPE>::BB;
    constexpr int GPB = BE / 8;
    const int64_t b = gidx / GPB;
    deq8<TYPE>(W + b * BB, (int)(gidx % GPB), y);
}

template <int TYPE>
__global__ void __launch_bounds__(256) dequant_f32_kernel(const uint8_t* __restrict__ W,
                                                          float* __restrict__ out,
                                                          int64_t n_groups) {
    for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < n_groups;
         gi += (int64_t)gridDim.x * blockDim.x) {
        float y[8];
        deq_group<TYPE>(W, gi, y);
        float4* o = reinterpret_cast<float4*>(out + gi * 8);
        o[0] = make_float4(y[0], y[1], y[2], y[3]);
        o[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
}

__global__ void f16_to_f32_kernel(const uint16_t* __restrict__ in, float* __restrict__ out,
                                  int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = h2f(in[i]);
}

// One CTA per row: pass 1 finds max|w| (exact, order-free), pass 2 recomputes
// the dequantised values and rounds w * (1/scale) half away from zero.
template <int TYPE>
__global__ void __launch_bounds__(256) dequant_i16_kernel(const uint8_t* __restrict__ W,
                                                          int16_t* __restrict__ q,
                                                          float* __restrict__ row_scale,
                                                          int64_t cols) {
    const int64_t r = blockIdx.x;
    const int64_t gpr = cols / 8;  // groups per row
    const int64_t g0 = r * gpr;
    float amax = 0.0f;
    for (int64_t g = threadIdx.x; g < gpr; g += blockDim.x) {
        float y[8];
        deq_group<TYPE>(W, g0 + g, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = fabsf(y[i]);
            amax = a > amax ? a : amax;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = t > amax ? t : amax;
    }
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) amax = red[w] > amax ? red[w] : amax;
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 32767.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) row_scale[r] = scale;
    for (int64_t g = threadIdx.x; g < gpr; g += blockDim.x) {
        float y[8];
        deq_group<TYPE>(W, g0 + g, y);
        short v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float t = roundf(__fmul_rn(y[i], inv));  // half away from zero, as lround
            t = fminf(fmaxf(t, -32767.0f), 32767.0f);
            v[i] = (short)(int)t;
        }
        *reinterpret_cast<int4*>(q + (g0 + g) * 8) =
            make_int4((int)((uint32_t)(uint16_t)v[0] | ((uint32_t)(uint16_t)v[1] << 16)),
                      (int)((uint32_t)(uint16_t)v[2] | ((uint32_t)(uint16_t)v[3] << 16)),
                      (int)((uint32_t)(uint16_t)v[4] | ((uint32_t)(uint16_t)v[5] << 16)),
                      (int)((uint32_t)(uint16_t)v[6] | ((uint32_t)(uint16_t)v[7] << 16)));
    }
}

// The same requantisation with one warp per row (8 rows per CTA): the row maximum is a
// warp reduction (no block barrier), each lane decodes several groups per pass with its
// loads in flight together, and the second pass reads the row again from L1/L2.  Same
// arithmetic as dequant_i16_kernel, so the same bits.
template <int TYPE>
__global__ void __launch_bounds__(256) dequant_i16_warp_kernel(const uint8_t* __restrict__ W,
                                                               int16_t* __restrict__ q,
                                                               float* __restrict__ row_scale,
                                                               int64_t rows, int64_t cols) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int64_t gpr = cols / 8;
    const int64_t g0 = r * gpr;
    float amax = 0.0f;
#pragma unroll 4
    for (int64_t g = lane; g < gpr; g += 32) {
        float y[8];
        deq_group<TYPE>(W, g0 + g, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = fabsf(y[i]);
            amax = a > amax ? a : amax;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = t > amax ? t : amax;
    }
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 32767.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (lane == 0) row_scale[r] = scale;
#pragma unroll 4
    for (int64_t g = lane; g < gpr; g += 32) {
        float y[8];
        deq_group<TYPE>(W, g0 + g, y);
        short v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float t = roundf(__fmul_rn(y[i], inv));  // half away from zero, as lround
            t = fminf(fmaxf(t, -32767.0f), 32767.0f);
            v[i] = (short)(int)t;
        }
        *reinterpret_cast<int4*>(q + (g0 + g) * 8) =
            make_int4((int)((uint32_t)(uint16_t)v[0] | ((uint32_t)(uint16_t)v[1] << 16)),
                      (int)((uint32_t)(uint16_t)v[2] | ((uint32_t)(uint16_t)v[3] << 16)),
                      (int)((uint32_t)(uint16_t)v[4] | ((uint32_t)(uint16_t)v[5] << 16)),
                      (int)((uint32_t)(uint16_t)v[6] | ((uint32_t)(uint16_t)v[7] << 16)));
    }
}

// FP32 input rows for the INT16 requant (F32 tensors such as an FP32 output head).
__global__ void __launch_bounds__(256) requant_i16_f32_kernel(const float* __restrict__ W,
                                                             int16_t* __restrict__ q,
                                                             float* __restrict__ row_scale,
                                                             int64_t cols) {
    const int64_t r = blockIdx.x;
    const float* row = W + r * cols;
    float amax = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        const float a = fabsf(row[c]);
        amax = a > amax ? a : amax;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = t > amax ? t : amax;
    }
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) amax = red[w] > amax ? red[w] : amax;
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 32767.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) row_scale[r] = scale;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        float t = roundf(__fmul_rn(row[c], inv));
        t = fminf(fmaxf(t, -32767.0f), 32767.0f);
        q[r * cols + c] = (int16_t)(int)t;
    }
}

// out[t, :] = dequant(table[id_t, :]); one thread per 8 elements of one row.
template <int TYPE>
__global__ void __launch_bounds__(256) embedding_q_kernel(const uint8_t* __restrict__ table,
                                                          const int32_t* __restrict__ ids,
                                                          float* __restrict__ out, int T,
                                                          int64_t vocab, int64_t dim) {
    const int t = blockIdx.y;
    if (t >= T) return;
    int id = ids[t];
    if (id < 0 || id >= vocab) id = 0;
    const int64_t gpr = dim / 8;
    for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < gpr;
         g += (int64_t)gridDim.x * blockDim.x) {
        float y[8];
        deq_group<TYPE>(table, (int64_t)id * gpr + g, y);
        float4* o = reinterpret_cast<float4*>(out + (int64_t)t * dim + g * 8);
        o[0] = make_float4(y[0], y[1], y[2], y[3]);
        o[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
}

__global__ void embedding_f32_rows_kernel(const float* __restrict__ table,
                                          const int32_t* __restrict__ ids,
                                          float* __restrict__ out, int T, int64_t vocab,
                                          int64_t dim) {
    const int t = blockIdx.y;
    int id = ids[t];
    if (id < 0 || id >= vocab) id = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < dim;
         i += (int64_t)gridDim.x * blockDim.x)
        out[(int64_t)t * dim + i] = table[(int64_t)id * dim + i];
}

__global__ void embedding_f16_rows_kernel(const uint16_t* __restrict__ table,
                                          const int32_t* __restrict__ ids,
                                          float* __restrict__ out, int T, int64_t vocab,
                                          int64_t dim) {
    const int t = blockIdx.y;
    int id = ids[t];
    if (id < 0 || id >= vocab) id = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < dim;
         i += (int64_t)gridDim.x * blockDim.x)
        out[(int64_t)t * dim + i] = h2f(table[(int64_t)id * dim + i]);
}

static unsigned grid_for(int64_t n, int per_block = 256, int64_t cap = 148 * 32) {
    int64_t g = (n + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (unsigned)g;
}

#define IB_DISPATCH_QTYPE(type, KERNEL_CALL)                                          \
    switch (type) {                                                                   \
        case IB_TYPE_Q4_0: { constexpr int QT = IB_TYPE_Q4_0; KERNEL_CALL; break; }   \
        case IB_TYPE_Q5_0: { constexpr int QT = IB_TYPE_Q5_0; KERNEL_CALL; break; }   \
        case IB_TYPE_Q5_1: { constexpr int QT = IB_TYPE_Q5_1; KERNEL_CALL; break; }   \
        case IB_TYPE_Q8_0: { constexpr int QT = IB_TYPE_Q8_0; KERNEL_CALL; break; }   \
        case IB_TYPE_Q4_K: { constexpr int QT = IB_TYPE_Q4_K; KERNEL_CALL; break; }   \
        case IB_TYPE_Q6_K: { constexpr int QT = IB_TYPE_Q6_K; KERNEL_CALL; break; }   \
        case IB_TYPE_Q4_1: { constexpr int QT = IB_TYPE_Q4_1; KERNEL_CALL; break; }   \
        case IB_TYPE_Q2_K: { constexpr int QT = IB_TYPE_Q2_K; KERNEL_CALL; break; }   \
        case IB_TYPE_Q3_K: { constexpr int QT = IB_TYPE_Q3_K; KERNEL_CALL; break; }   \
        case IB_TYPE_Q5_K: { constexpr int QT = IB_TYPE_Q5_K; KERNEL_CALL; break; }   \
        default: break;                                                               \
    }

}  // namespace ib

using namespace ib;

static int check_shape(int type, const void* a, const void* b, int64_t rows, int64_t cols) {
    IB_REQUIRE(a != nullptr && b != nullptr, "null pointer argument");
    IB_REQUIRE(rows >= 0 && cols >= 0, "negative shape");
    const int be = block_elems(type);
    if (be == 0) {
        set_error(std::string("unsupported tensor type ") + std::to_string(type));
        return IB_ERR_UNSUPPORTED;
    }
    if (cols % (be > 8 ? be : 8) != 0 && be > 1) {
        set_error(std::string("cols must be a multiple of the ") + type_name(type) +
                  " block size");
        return IB_ERR_INVALID;
    }
    return IB_OK;
}

extern "C" int ib_dequant_f32(int type, const void* dev_blocks, float* dev_out, int64_t rows,
                              int64_t cols, void* stream) {
    if (rows == 0 || cols == 0) return IB_OK;
    if (type == IB_TYPE_F32 || type == IB_TYPE_F16) {
        IB_REQUIRE(dev_blocks && dev_out && rows > 0 && cols > 0, "bad arguments");
        const int64_t n = rows * cols;
        if (type == IB_TYPE_F32) {
            IB_CUDA_CHECK(cudaMemcpyAsync(dev_out, dev_blocks, (size_t)n * 4,
                                          cudaMemcpyDeviceToDevice, as_stream(stream)));
        } else {
            f16_to_f32_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(
                (const uint16_t*)dev_blocks, dev_out, n);
            IB_LAUNCH_CHECK("f16_to_f32_kernel");
        }
        return IB_OK;
    }
    int st = check_shape(type, dev_blocks, dev_out, rows, cols);
    if (st != IB_OK) return st;
    IB_REQUIRE(((uintptr_t)dev_out & 15) == 0, "FP32 output must be 16-byte aligned");
    IB_REQUIRE(((uintptr_t)dev_blocks & 1) == 0, "blocks must be 2-byte aligned");
    const int64_t n_groups = rows * cols / 8;
    const uint8_t* W = (const uint8_t*)dev_blocks;
    IB_DISPATCH_QTYPE(type, (dequant_f32_kernel<QT><<<grid_for(n_groups), 256, 0,
                                                     as_stream(stream)>>>(W, dev_out, n_groups)));
    IB_LAUNCH_CHECK("dequant_f32_kernel");
    return IB_OK;
}

extern "C" int ib_dequant_i16(int type, const void* dev_blocks, int16_t* dev_q,
                              float* dev_row_scale, int64_t rows, int64_t cols, void* stream) {
    if (rows == 0 || cols == 0) return IB_OK;
    IB_REQUIRE(dev_row_scale != nullptr, "null row_scale");
    IB_REQUIRE(rows <= 0x7FFFFFFF, "too many rows");
    if (type == IB_TYPE_F32) {
        IB_REQUIRE(dev_blocks && dev_q, "null pointer argument");
        requant_i16_f32_kernel<<<(unsigned)rows, 256, 0, as_stream(stream)>>>(
            (const float*)dev_blocks, dev_q, dev_row_scale, cols);
        IB_LAUNCH_CHECK("requant_i16_f32_kernel");
        return IB_OK;
    }
    int st = check_shape(type, dev_blocks, dev_q, rows, cols);
    if (st != IB_OK) return st;
    if (!is_quant(type)) {
        set_error("INT16 requantisation needs a block-quantised or F32 tensor");
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(((uintptr_t)dev_q & 15) == 0, "INT16 output must be 16-byte aligned");
    const uint8_t* W = (const uint8_t*)dev_blocks;
    // Many rows of moderate length: a warp per row (128256 x 4096 Q4_K: 1.36 -> 1.58 TB/s);
    // fewer or longer rows keep a CTA per row, which fills the GPU better (4096 x 4096 Q4_K:
    // 1.05 against 0.92 TB/s with a warp per row)
    if (rows >= 9472 && cols >= 2048 && cols <= 8192) {
        const unsigned grid = (unsigned)((rows + 7) / 8);
        IB_DISPATCH_QTYPE(type, (dequant_i16_warp_kernel<QT><<<grid, 256, 0, as_stream(stream)>>>(
                                    W, dev_q, dev_row_scale, rows, cols)));
        IB_LAUNCH_CHECK("dequant_i16_warp_kernel");
        return IB_OK;
    }
    IB_DISPATCH_QTYPE(type, (dequant_i16_kernel<QT><<<(unsigned)rows, 256, 0, as_stream(stream)>>>(
                                W, dev_q, dev_row_scale, cols)));
    IB_LAUNCH_CHECK("dequant_i16_kernel");
    return IB_OK;
}

extern "C" int ib_embedding_q(int type, const void* dev_table, const int32_t* dev_ids,
                              float* dev_out, int T, int64_t vocab, int64_t dim, void* stream) {
    if (T == 0 || dim == 0) return IB_OK;
    IB_REQUIRE(dev_table && dev_ids && dev_out, "null pointer argument");
    IB_REQUIRE(T > 0 && T <= 65535 && vocab > 0 && dim > 0, "bad embedding shape");
    dim3 grid(grid_for(dim / 8 > 0 ? dim / 8 : 1, 256, 64), (unsigned)T);
    if (type == IB_TYPE_F32) {
        embedding_f32_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(
            (const float*)dev_table, dev_ids, dev_out, T, vocab, dim);
        IB_LAUNCH_CHECK("embedding_f32_rows_kernel");
        return IB_OK;
    }
    if (type == IB_TYPE_F16) {
        embedding_f16_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(
            (const uint16_t*)dev_table, dev_ids, dev_out, T, vocab, dim);
        IB_LAUNCH_CHECK("embedding_f16_rows_kernel");
        return IB_OK;
    }
    int st = check_shape(type, dev_table, dev_out, vocab, dim);
    if (st != IB_OK) return st;
    IB_REQUIRE(((uintptr_t)dev_out & 15) == 0, "embedding output must be 16-byte aligned");
    IB_REQUIRE(((uintptr_t)dev_table & 1) == 0, "table must be 2-byte aligned");
    const uint8_t* W = (const uint8_t*)dev_table;
    IB_DISPATCH_QTYPE(type, (embedding_q_kernel<QT><<<grid, 256, 0, as_stream(stream)>>>(
                                W, dev_ids, dev_out, T, vocab, dim)));
    IB_LAUNCH_CHECK("embedding_q_kernel");
    return IB_OK;
}
