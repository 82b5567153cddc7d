// Element access to a KV cache [n_kv_heads][max_seq][head_dim] held in FP32 (the
// reference's layout, src/models/model_cuda.cpp:204-211) or FP16 (the native runner's
// reduced-precision option: half the bytes per position, values rounded to nearest).
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace ib {

template <typename KV>
__device__ __forceinline__ float kv_at(const KV* p, size_t i) {
    if constexpr (sizeof(KV) == 4) return p[i];
    else return __half2float(p[i]);
}

// elements 4 i4 .. 4 i4 + 3 (16-byte / 8-byte aligned rows), read-only path
template <typename KV>
__device__ __forceinline__ float4 kv_at4(const KV* p, size_t i4) {
    if constexpr (sizeof(KV) == 4) {
        return __ldg(reinterpret_cast<const float4*>(p) + i4);
    } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + i4);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
}

template <typename KV>
__device__ __forceinline__ void kv_put(KV* p, size_t i, float v) {
    if constexpr (sizeof(KV) == 4) p[i] = v;
    else p[i] = __float2half_rn(v);
}

}  // namespace ib
