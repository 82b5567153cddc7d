// Non-GEMV operators of the Llama forward pass with the reference's argument
// meaning (include/ops/cuda_backend.hpp:39-64; kernels src/ops/cuda_kernels.cu),
// plus the CUDA-core batched GEMM on FP32, INT16 and packed weights.  Prefill on
// packed weights normally runs on the tensor cores (gemm_tc.cu) and its attention
// as flash attention (attention.cu, attention_prefill).
//
// Attention for one query position is a split-K "flash decode": CTA (kv head,
// position chunk) scores the whole GQA group against its chunk of the KV cache,
// keeps the running max / sum / weighted V (online softmax), and a combine kernel
// merges the chunks.  No shared-memory cap on the context length (the reference
// keeps (pos+1) scores in dynamic shared memory, cuda_backend.cpp:408).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "kv.cuh"
#include "ops.cuh"
#include "quant.cuh"

namespace ib {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x <= 1024; result valid in all threads.
__device__ float block_sum(float v, float* sh) {
    v = warp_sum_f(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = l < nw ? sh[l] : 0.f;
    return warp_sum_f(t);
}
__device__ float block_max(float v, float* sh) {
    v = warp_max_f(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = l < nw ? sh[l] : -INFINITY;
    return warp_max_f(t);
}

// ---- RMSNorm: out = x / sqrt(mean(x^2) + eps) * w (model.cpp:54-57) -------------
// One CTA per row; float4 path when dim % 4 == 0 and the row is 16-byte aligned
// (every thread's loads are issued before the reduction).
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w,
                                                       float* __restrict__ out, int dim,
                                                       float eps) {
    __shared__ float sh[32];
    const float* xr = x + (int64_t)blockIdx.x * dim;
    float* o = out + (int64_t)blockIdx.x * dim;
    const bool vec = (dim & 3) == 0 && ((((uintptr_t)xr) | ((uintptr_t)o) | ((uintptr_t)w)) & 15) == 0;
    float ss = 0.f;
    if (vec) {
        const int n4 = dim >> 2;
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = reinterpret_cast<const float4*>(xr)[i];
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        ss = block_sum(ss, sh);
        const float rms = sqrtf(ss / (float)dim + eps);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = reinterpret_cast<const float4*>(xr)[i];
            const float4 g = reinterpret_cast<const float4*>(w)[i];
            reinterpret_cast<float4*>(o)[i] =
                make_float4(v.x / rms * g.x, v.y / rms * g.y, v.z / rms * g.z, v.w / rms * g.w);
        }
        return;
    }
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, sh);
    const float rms = sqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) o[i] = xr[i] / rms * w[i];
}

__global__ void silu_kernel(float* x, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float g = x[i];
        x[i] = g * (1.0f / (1.0f + expf(-g)));
    }
}
__global__ void mul_kernel(float* a, const float* b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        a[i] *= b[i];
}
__global__ void add_kernel(float* a, const float* b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        a[i] += b[i];
}

__global__ void embedding_i16_kernel(const int16_t* table, const float* row_scale,
                                     const int32_t* ids, int id_const, float* out, int T,
                                     int dim) {
    const int t = blockIdx.x;
    const int id = ids ? ids[t] : id_const;
    const int16_t* row = table + (int64_t)id * dim;
    const float s = row_scale[id];
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[(int64_t)t * dim + i] = (float)row[i] * s;
}
__global__ void embedding_f32_kernel(const float* table, const int32_t* ids, int id_const,
                                     float* out, int T, int dim) {
    const int t = blockIdx.x;
    const int id = ids ? ids[t] : id_const;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        out[(int64_t)t * dim + i] = table[(int64_t)id * dim + i];
}

// ---- KV write: cache [n_heads][max_seq][head_dim] (cuda_kernels.cu:163-176,403-419)
template <typename KV>
__global__ void kv_write_kernel(KV* kc, KV* vc, const float* k, const float* v,
                                int n_heads, int head_dim, int max_seq, int start, int T,
                                const int* start_dev) {
    const int t = blockIdx.y;
    if (start_dev) start = *start_dev;
    if (start + t >= max_seq) return;
    const int total = n_heads * head_dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int h = i / head_dim, d = i - h * head_dim;
        const int64_t ci = ((int64_t)h * max_seq + start + t) * head_dim + d;
        kv_put(kc, ci, k[(int64_t)t * total + i]);
        kv_put(vc, ci, v[(int64_t)t * total + i]);
    }
}

// ---- RoPE from a cos/sin table: table[(pos*half + j)*2 + {0,1}] (cuda_kernels.cu:183-208)
__global__ void rope_kernel(float* q, float* k, const float* table, int n_heads,
                            int n_kv_heads, int head_dim, int start, const int* start_dev) {
    const int b = blockIdx.x, t = blockIdx.y, j = threadIdx.x, half = head_dim / 2;
    if (j >= half) return;
    if (start_dev) start = *start_dev;
    const int pos = start + t;
    const float c = table[((int64_t)pos * half + j) * 2];
    const float s = table[((int64_t)pos * half + j) * 2 + 1];
    float* vec = b < n_heads ? q + ((int64_t)t * n_heads + b) * head_dim
                             : k + ((int64_t)t * n_kv_heads + (b - n_heads)) * head_dim;
    const float x0 = vec[2 * j], x1 = vec[2 * j + 1];
    vec[2 * j] = x0 * c - x1 * s;
    vec[2 * j + 1] = x0 * s + x1 * c;
}

// ---- attention for a batch of query positions (prefill), causal ----------------
// q, out: [T][H][HD]; grid (H, T); dynamic shared (start+T) floats of scores.
template <typename KV>
__global__ void __launch_bounds__(128) attn_batch_kernel(const float* __restrict__ q,
                                                         const KV* __restrict__ kc,
                                                         const KV* __restrict__ vc,
                                                         float* __restrict__ out, int n_heads,
                                                         int n_kv_heads, int head_dim,
                                                         int max_seq, int start, int T,
                                                         float scale) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    __shared__ float qsh[256];
    const int h = blockIdx.x, t = blockIdx.y;
    const int hk = h / (n_heads / n_kv_heads);
    const int seq = start + t + 1;
    const float* qh = q + ((int64_t)t * n_heads + h) * head_dim;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) qsh[d] = qh[d];
    __syncthreads();
    const KV* kh = kc + (int64_t)hk * max_seq * head_dim;
    const KV* vh = vc + (int64_t)hk * max_seq * head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int s = warp; s < seq; s += 4) {
        float dot = 0.f;
        for (int d = lane; d < head_dim; d += 32)
            dot = fmaf(qsh[d], kv_at(kh, (size_t)s * head_dim + d), dot);
        dot = warp_sum_f(dot);
        if (lane == 0) sc[s] = dot * scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int s = threadIdx.x; s < seq; s += blockDim.x) m = fmaxf(m, sc[s]);
    m = block_max(m, red);
    float l = 0.f;
    for (int s = threadIdx.x; s < seq; s += blockDim.x) {
        const float e = expf(sc[s] - m);
        sc[s] = e;
        l += e;
    }
    l = block_sum(l, red);
    const float inv = 1.0f / l;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc = 0.f;
        for (int s = 0; s < seq; ++s) acc = fmaf(sc[s], kv_at(vh, (size_t)s * head_dim + d), acc);
        out[((int64_t)t * n_heads + h) * head_dim + d] = acc * inv;
    }
}

// ---- argmax (first maximum, as sample_argmax) -----------------------------------
__global__ void argmax_kernel(const float* __restrict__ x, int n, int32_t* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    // four independent float4 loads per thread and step (first maximum kept per lane)
    const bool vec = ((uintptr_t)x & 15) == 0;
    int i0 = 0;
    if (vec) {
        const int n4 = n >> 2, step = blockDim.x * 4;
        for (int b = threadIdx.x; b < n4; b += step) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                v[u] = b + u * blockDim.x < n4 ? reinterpret_cast<const float4*>(x)[b + u * blockDim.x]
                                              : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int base = 4 * (b + u * blockDim.x);
                const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (e[k] > bv || (e[k] == bv && base + k < bi)) { bv = e[k]; bi = base + k; }
            }
        }
        i0 = n4 * 4;
    }
    for (int i = i0 + threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        bv = l < nw ? sv[l] : -INFINITY;
        bi = l < nw ? si[l] : 0x7FFFFFFF;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (l == 0) *out = (bi == 0x7FFFFFFF) ? 0 : bi;
    }
}

// ---- batched GEMM on the CUDA cores: Y[T, M] = X[T, K] @ W[M, K]^T ---------------
// Tile 64 (W rows) x 64 (tokens) x 32 (K); 256 threads, 4x4 outputs each.
// The W tile is produced by a loader: FP32 copy, INT16 (scaled in the epilogue),
// or exact dequantisation of GGUF blocks (deq8).  Serves ib_gemm and ib_gemm_i16,
// and ib_gemm_q for shapes the tensor-core kernel (gemm_tc.cu) does not take or
// when ib_gemm_set_path(1) asks for it.
constexpr int GB_M = 64, GB_N = 64, GB_K = 32;

template <int TYPE>
__device__ __forceinline__ void load_w8(const void* W, int64_t K, int64_t row, int64_t k0,
                                        float* y) {
    if constexpr (TYPE == IB_TYPE_F32) {
        const float* p = (const float*)W + row * K + k0;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = p[i];
    } else if constexpr (TYPE == IB_TYPE_I16) {
        const int16_t* p = (const int16_t*)W + row * K + k0;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = (float)p[i];
    } else {
        constexpr int BE = QFmt<TYPE>::BE, BB = QFmt<TYPE>::BB;
        const uint8_t* blk = (const uint8_t*)W + (row * (K / BE) + k0 / BE) * BB;
        deq8<TYPE>(blk, (int)((k0 % BE) / 8), y);
    }
}

template <int TYPE>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const void* __restrict__ W,
                                                        const float* __restrict__ row_scale,
                                                        const float* __restrict__ X,
                                                        float* __restrict__ Y, int T, int M,
                                                        int K) {
    __shared__ __align__(16) float Ws[GB_K][GB_M + 4];
    __shared__ __align__(16) float Xs[GB_K][GB_N + 4];
    const int m0 = blockIdx.x * GB_M, t0 = blockIdx.y * GB_N;
    const int tid = threadIdx.x;
    const int tm = (tid & 15) * 4, tt = (tid >> 4) * 4;
    float acc[4][4] = {};
    const bool kvec = (K % 8) == 0;
    for (int k0 = 0; k0 < K; k0 += GB_K) {
        {  // W tile: 64 rows x 4 groups of 8
            const int r = tid >> 2, g = tid & 3;
            const int64_t row = m0 + r;
            const int kk = k0 + 8 * g;
            float y[8];
            if (row < M && kk + 8 <= K && kvec) {
                load_w8<TYPE>(W, K, row, kk, y);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) y[i] = 0.f;
                if (row < M && (TYPE == IB_TYPE_F32 || TYPE == IB_TYPE_I16)) {
                    for (int i = 0; i < 8 && kk + i < K; ++i)
                        y[i] = TYPE == IB_TYPE_F32 ? ((const float*)W)[row * K + kk + i]
                                                   : (float)((const int16_t*)W)[row * K + kk + i];
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) Ws[8 * g + i][r] = y[i];
        }
        {  // X tile: 64 tokens x 32
            const int r = tid >> 2, g = tid & 3;
            const int t = t0 + r;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int kk = k0 + 8 * g + i;
                Xs[8 * g + i][r] = (t < T && kk < K) ? X[(int64_t)t * K + kk] : 0.f;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < GB_K; ++k) {
            const float4 wv = *reinterpret_cast<const float4*>(&Ws[k][tm]);
            const float4 xv = *reinterpret_cast<const float4*>(&Xs[k][tt]);
            const float wa[4] = {wv.x, wv.y, wv.z, wv.w}, xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + tt + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + tm + j;
            if (m >= M) continue;
            float v = acc[i][j];
            if (TYPE == IB_TYPE_I16) v *= row_scale[m];
            Y[(int64_t)t * M + m] = v;
        }
    }
}

// Scratch for the C-ABI operators (split-K attention partials, GEMV activation
// limbs), one buffer per (slot, device), grown on demand.  Calls that share a
// slot must be ordered on one stream (each operator uses its own slot).
struct Workspace {
    std::mutex mu;
    std::vector<void*> ptr;
    std::vector<size_t> bytes;
};
static Workspace g_ws[WS_SLOTS];

int workspace_get(int slot, size_t bytes, void** out) {
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    Workspace& ws = g_ws[slot];
    std::lock_guard<std::mutex> lock(ws.mu);
    if ((int)ws.ptr.size() <= dev) {
        ws.ptr.resize(dev + 1, nullptr);
        ws.bytes.resize(dev + 1, 0);
    }
    if (ws.bytes[dev] < bytes) {
        if (ws.ptr[dev]) {
            IB_CUDA_CHECK(cudaDeviceSynchronize());
            IB_CUDA_CHECK(cudaFree(ws.ptr[dev]));
            ws.ptr[dev] = nullptr;
            ws.bytes[dev] = 0;
        }
        size_t b = bytes < (1u << 20) ? (1u << 20) : bytes;
        IB_CUDA_CHECK(cudaMalloc(&ws.ptr[dev], b));
        ws.bytes[dev] = b;
    }
    *out = ws.ptr[dev];
    return IB_OK;
}

template <int TYPE>
static int launch_gemm(const void* W, const float* rs, const float* X, float* Y, int T, int M,
                       int K, cudaStream_t st) {
    dim3 grid((M + GB_M - 1) / GB_M, (T + GB_N - 1) / GB_N);
    IB_REQUIRE(grid.y <= 65535, "T too large");
    gemm_simt_kernel<TYPE><<<grid, 256, 0, st>>>(W, rs, X, Y, T, M, K);
    IB_LAUNCH_CHECK("gemm_kernel");
    return IB_OK;
}

int gemm_q_simt(int type, const void* W, const float* X, float* Y, int T, int M, int K,
                cudaStream_t st) {
    switch (type) {
        case IB_TYPE_Q4_0: return launch_gemm<IB_TYPE_Q4_0>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q5_0: return launch_gemm<IB_TYPE_Q5_0>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q5_1: return launch_gemm<IB_TYPE_Q5_1>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q8_0: return launch_gemm<IB_TYPE_Q8_0>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q4_K: return launch_gemm<IB_TYPE_Q4_K>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q6_K: return launch_gemm<IB_TYPE_Q6_K>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q4_1: return launch_gemm<IB_TYPE_Q4_1>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q2_K: return launch_gemm<IB_TYPE_Q2_K>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q3_K: return launch_gemm<IB_TYPE_Q3_K>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_Q5_K: return launch_gemm<IB_TYPE_Q5_K>(W, nullptr, X, Y, T, M, K, st);
        case IB_TYPE_F32: return launch_gemm<IB_TYPE_F32>(W, nullptr, X, Y, T, M, K, st);
    }
    set_error("gemm: unsupported weight type");
    return IB_ERR_UNSUPPORTED;
}

int rope_launch(float* q, float* k, const float* table, int H, int Hkv, int HD, int start,
                int T, cudaStream_t st, const int* start_dev) {
    rope_kernel<<<dim3(H + Hkv, T), HD / 2, 0, st>>>(q, k, table, H, Hkv, HD, start, start_dev);
    IB_LAUNCH_CHECK("rope_kernel");
    return IB_OK;
}

int rmsnorm_launch(const float* x, const float* w, float* out, int rows, int dim, float eps,
                   cudaStream_t st) {
    rmsnorm_kernel<<<rows, dim >= 2048 ? 1024 : 256, 0, st>>>(x, w, out, dim, eps);
    IB_LAUNCH_CHECK("rmsnorm_kernel");
    return IB_OK;
}

int kv_write_launch(void* kc, void* vc, const float* k, const float* v, int Hkv, int HD,
                    int max_seq, int start, int T, cudaStream_t st, const int* start_dev,
                    bool kv_half) {
    const int total = Hkv * HD;
    const dim3 grid((total + 255) / 256, T);
    if (kv_half)
        kv_write_kernel<<<grid, 256, 0, st>>>((__half*)kc, (__half*)vc, k, v, Hkv, HD, max_seq,
                                              start, T, start_dev);
    else
        kv_write_kernel<<<grid, 256, 0, st>>>((float*)kc, (float*)vc, k, v, Hkv, HD, max_seq,
                                              start, T, start_dev);
    IB_LAUNCH_CHECK("kv_write_kernel");
    return IB_OK;
}

int attention_batch_launch(const float* q, const void* kc, const void* vc, float* out, int H,
                           int Hkv, int HD, int max_seq, int start, int T, float scale,
                           cudaStream_t st, bool kv_half) {
    if (attention_prefill_ok(H, Hkv, HD) && T > 0)
        return attention_prefill(q, kc, vc, out, H, Hkv, HD, max_seq, start, T, scale, st, kv_half);
    const size_t smem = (size_t)(start + T) * sizeof(float);
    const void* kern = kv_half ? (const void*)attn_batch_kernel<__half> : (const void*)attn_batch_kernel<float>;
    if (smem > 48 * 1024) {
        IB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(smem < 200 * 1024 ? 200 * 1024 : smem)));
    }
    if (kv_half)
        attn_batch_kernel<<<dim3(H, T), 128, smem, st>>>(q, (const __half*)kc, (const __half*)vc,
                                                         out, H, Hkv, HD, max_seq, start, T, scale);
    else
        attn_batch_kernel<<<dim3(H, T), 128, smem, st>>>(q, (const float*)kc, (const float*)vc,
                                                         out, H, Hkv, HD, max_seq, start, T, scale);
    IB_LAUNCH_CHECK("attention_batch_kernel");
    return IB_OK;
}

int argmax_launch(const float* x, int n, int32_t* out, cudaStream_t st) {
    argmax_kernel<<<1, 1024, 0, st>>>(x, n, out);
    IB_LAUNCH_CHECK("argmax_kernel");
    return IB_OK;
}

int elementwise_launch(int op, float* a, const float* b, int n, cudaStream_t st) {
    const int grid = (n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8;
    if (op == 0) silu_kernel<<<grid, 256, 0, st>>>(a, n);
    else if (op == 1) mul_kernel<<<grid, 256, 0, st>>>(a, b, n);
    else add_kernel<<<grid, 256, 0, st>>>(a, b, n);
    IB_LAUNCH_CHECK(op == 0 ? "silu_kernel" : op == 1 ? "mul_kernel" : "add_kernel");
    return IB_OK;
}

}  // namespace ib

using namespace ib;

extern "C" int ib_rmsnorm(const float* x, const float* w, float* out, int rows, int dim,
                          float eps, void* stream) {
    if (rows == 0) return IB_OK;
    IB_REQUIRE(x && w && out && rows > 0 && dim > 0, "bad rmsnorm arguments");
    return rmsnorm_launch(x, w, out, rows, dim, eps, as_stream(stream));
}

extern "C" int ib_silu(float* x, int n, void* stream) {
    if (n == 0) return IB_OK;
    IB_REQUIRE(x && n > 0, "bad silu arguments");
    return elementwise_launch(0, x, nullptr, n, as_stream(stream));
}
extern "C" int ib_mul(float* a, const float* b, int n, void* stream) {
    if (n == 0) return IB_OK;
    IB_REQUIRE(a && b && n > 0, "bad mul arguments");
    return elementwise_launch(1, a, b, n, as_stream(stream));
}
extern "C" int ib_add(float* a, const float* b, int n, void* stream) {
    if (n == 0) return IB_OK;
    IB_REQUIRE(a && b && n > 0, "bad add arguments");
    return elementwise_launch(2, a, b, n, as_stream(stream));
}

extern "C" int ib_embedding(const float* table, int id, float* out, int dim, void* stream) {
    IB_REQUIRE(table && out && dim > 0 && id >= 0, "bad embedding arguments");
    embedding_f32_kernel<<<1, 256, 0, as_stream(stream)>>>(table, nullptr, id, out, 1, dim);
    IB_LAUNCH_CHECK("embedding_kernel");
    return IB_OK;
}
extern "C" int ib_embedding_i16(const int16_t* table, const float* row_scale, int id, float* out,
                                int dim, void* stream) {
    IB_REQUIRE(table && row_scale && out && dim > 0 && id >= 0, "bad embedding_i16 arguments");
    embedding_i16_kernel<<<1, 256, 0, as_stream(stream)>>>(table, row_scale, nullptr, id, out, 1,
                                                           dim);
    IB_LAUNCH_CHECK("embedding_i16_kernel");
    return IB_OK;
}
extern "C" int ib_embedding_batch(const float* table, const int32_t* ids, float* out, int T,
                                  int dim, void* stream) {
    if (T == 0) return IB_OK;
    IB_REQUIRE(table && ids && out && T > 0 && dim > 0, "bad embedding_batch arguments");
    embedding_f32_kernel<<<T, 256, 0, as_stream(stream)>>>(table, ids, 0, out, T, dim);
    IB_LAUNCH_CHECK("embedding_batch_kernel");
    return IB_OK;
}
extern "C" int ib_embedding_batch_i16(const int16_t* table, const float* row_scale,
                                      const int32_t* ids, float* out, int T, int dim,
                                      void* stream) {
    if (T == 0) return IB_OK;
    IB_REQUIRE(table && row_scale && ids && out && T > 0 && dim > 0,
               "bad embedding_batch_i16 arguments");
    embedding_i16_kernel<<<T, 256, 0, as_stream(stream)>>>(table, row_scale, ids, 0, out, T, dim);
    IB_LAUNCH_CHECK("embedding_batch_i16_kernel");
    return IB_OK;
}

extern "C" int ib_kv_write(float* kc, float* vc, const float* k, const float* v, int n_heads,
                           int head_dim, int max_seq, int pos, void* stream) {
    IB_REQUIRE(kc && vc && k && v && n_heads > 0 && head_dim > 0, "bad kv_write arguments");
    IB_REQUIRE(pos >= 0 && pos < max_seq, "pos outside the KV cache");
    return kv_write_launch(kc, vc, k, v, n_heads, head_dim, max_seq, pos, 1, as_stream(stream),
                           nullptr);
}
extern "C" int ib_kv_write_batch(float* kc, float* vc, const float* k, const float* v,
                                 int n_heads, int head_dim, int max_seq, int start, int T,
                                 void* stream) {
    if (T == 0) return IB_OK;
    IB_REQUIRE(kc && vc && k && v && n_heads > 0 && head_dim > 0 && T > 0,
               "bad kv_write_batch arguments");
    IB_REQUIRE(start >= 0 && start + T <= max_seq, "positions outside the KV cache");
    return kv_write_launch(kc, vc, k, v, n_heads, head_dim, max_seq, start, T, as_stream(stream),
                           nullptr);
}

extern "C" int ib_rope(float* q, float* k, const float* table, int n_heads, int n_kv_heads,
                       int head_dim, int pos, void* stream) {
    IB_REQUIRE(q && k && table && n_heads > 0 && n_kv_heads >= 0 && head_dim > 1 &&
                   head_dim <= 2048 && pos >= 0,
               "bad rope arguments");
    return rope_launch(q, k, table, n_heads, n_kv_heads, head_dim, pos, 1, as_stream(stream), nullptr);
}
extern "C" int ib_rope_batch(float* q, float* k, const float* table, int n_heads,
                             int n_kv_heads, int head_dim, int start, int T, void* stream) {
    if (T == 0) return IB_OK;
    IB_REQUIRE(q && k && table && n_heads > 0 && head_dim > 1 && head_dim <= 2048 && start >= 0 &&
                   T > 0 && T <= 65535,
               "bad rope_batch arguments");
    return rope_launch(q, k, table, n_heads, n_kv_heads, head_dim, start, T, as_stream(stream),
                       nullptr);
}

extern "C" int ib_attention(const float* q, const float* kc, const float* vc, float* out,
                            int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos,
                            float scale, void* stream) {
    IB_REQUIRE(q && kc && vc && out, "null pointer argument");
    int st = check_attention_args(n_heads, n_kv_heads, head_dim, max_seq, pos);
    if (st != IB_OK) return st;
    void* part = nullptr;
    st = workspace_get(WS_ATTENTION, attention_partial_bytes(n_heads, head_dim, pos), &part);
    if (st != IB_OK) return st;
    return attention_decode(q, kc, vc, out, n_heads, n_kv_heads, head_dim, max_seq, pos, scale,
                            (float*)part, as_stream(stream), nullptr);
}

extern "C" size_t ib_attention_split_part_bytes(int n_heads, int head_dim) {
    return n_heads > 0 && head_dim > 0 ? attention_fused_part_bytes(n_heads, head_dim) : 0;
}

extern "C" int ib_attention_split(const float* q, const float* kc, const float* vc, float* out,
                                  int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                  const int32_t* pos_dev, float scale, float* part,
                                  int32_t* counters, void* stream) {
    IB_REQUIRE(q && kc && vc && out && pos_dev && part && counters, "null pointer argument");
    IB_REQUIRE(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0 && max_seq > 0,
               "n_heads must be a multiple of n_kv_heads");
    IB_REQUIRE(attention_fused_ok(n_heads, n_kv_heads, head_dim),
               "split attention needs head_dim % 4 == 0, head_dim <= 128 and a group <= 8");
    return attention_decode_fused(q, kc, vc, out, nullptr, false, n_heads, n_kv_heads, head_dim,
                                  max_seq, scale, part, counters, as_stream(stream), pos_dev,
                                  false);
}

extern "C" int ib_attention_batch(const float* q, const float* kc, const float* vc, float* out,
                                  int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                  int start, int T, float scale, void* stream) {
    if (T == 0) return IB_OK;
    IB_REQUIRE(q && kc && vc && out, "null pointer argument");
    IB_REQUIRE(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0, "bad head counts");
    IB_REQUIRE(head_dim > 0 && head_dim <= 256, "head_dim must be in (0, 256]");
    IB_REQUIRE(start >= 0 && T > 0 && start + T <= max_seq && T <= 65535,
               "positions outside the KV cache");
    return attention_batch_launch(q, kc, vc, out, n_heads, n_kv_heads, head_dim, max_seq, start,
                                  T, scale, as_stream(stream));
}

extern "C" int ib_argmax(const float* x, int n, int32_t* dev_out, void* stream) {
    IB_REQUIRE(x && dev_out && n > 0, "bad argmax arguments");
    return argmax_launch(x, n, dev_out, as_stream(stream));
}

extern "C" int ib_gemm(const float* W, const float* X, float* Y, int T, int M, int K,
                       void* stream) {
    if (T == 0 || M == 0) return IB_OK;
    IB_REQUIRE(W && X && Y && T > 0 && M > 0 && K > 0, "bad gemm arguments");
    return launch_gemm<IB_TYPE_F32>(W, nullptr, X, Y, T, M, K, as_stream(stream));
}
extern "C" int ib_gemm_i16(const int16_t* W, const float* row_scale, const float* X, float* Y,
                           int T, int M, int K, void* stream) {
    if (T == 0 || M == 0) return IB_OK;
    IB_REQUIRE(W && row_scale && X && Y && T > 0 && M > 0 && K > 0, "bad gemm_i16 arguments");
    return launch_gemm<IB_TYPE_I16>(W, row_scale, X, Y, T, M, K, as_stream(stream));
}

// 0: tensor-core GEMM where the shape allows (default); 1: the CUDA-core tiles.
static int g_gemm_path = 0;

extern "C" int ib_gemm_set_path(int path) {
    IB_REQUIRE(path >= 0 && path <= 3,
               "gemm path must be 0 (tensor cores, automatic), 1 (CUDA cores), 2 (tensor cores, "
               "staged blocks) or 3 (tensor cores, dequantised planes)");
    g_gemm_path = path;
    return IB_OK;
}

extern "C" int ib_gemm_q(int type, const void* dev_W, const float* dev_X, float* dev_Y,
                         int64_t T, int64_t rows, int64_t cols, void* stream) {
    if (T == 0 || rows == 0) return IB_OK;
    IB_REQUIRE(dev_W && dev_X && dev_Y && T > 0 && rows > 0 && cols > 0, "bad gemm_q arguments");
    IB_REQUIRE(T <= 65535 * 64 && rows < (1ll << 31) && cols < (1ll << 31), "gemm_q too large");
    if (!is_quant(type)) {
        set_error(std::string("ib_gemm_q: unsupported type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(cols % block_elems(type) == 0, "cols must be a multiple of the block size");
    cudaStream_t st = as_stream(stream);
    const bool planes = gemm_planes_supported(type, T, rows, cols);
    const bool staged = gemm_tc_supported(type, T, rows, cols);
    // automatic: prompts of kPlanesMinT tokens and more decode the weights once into FP16
    // planes (their decode is then shared by every token tile); shorter ones decode each
    // tile in the kernel
    constexpr int64_t kPlanesMinT = 128;
    if (planes && (g_gemm_path == 3 || (g_gemm_path == 0 && (T >= kPlanesMinT || !staged))))
        return gemm_q_planes(type, dev_W, dev_X, dev_Y, (int)T, (int)rows, (int)cols, st);
    if (staged && (g_gemm_path == 0 || g_gemm_path == 2))
        return gemm_q_tc(type, dev_W, dev_X, dev_Y, (int)T, (int)rows, (int)cols, st);
    return gemm_q_simt(type, dev_W, dev_X, dev_Y, (int)T, (int)rows, (int)cols, st);
}
