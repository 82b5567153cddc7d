// Device-side decoding of GGUF blocks (layouts: reference
// include/gguf/quantization.hpp:13-34 and src/gguf/quantization.cpp:28-245).
//
// Element-exact helpers (deq8_*) reproduce the reference's FP32 expressions for
// eight consecutive elements of a block; they are used by the dequantisation
// kernels and the embedding gather, where results must match bit for bit.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ib_cuda.h"

namespace ib {

// Exact fp16 -> fp32 (reference fp16_to_fp32, quantization.cpp:9-27): subnormal
// halves become mant * 2^-24 (exact), exp 31 keeps its payload.
__device__ __forceinline__ float h2f(uint32_t h) {
    const uint32_t e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    if (e == 0) {
        const float v = __fmul_rn(__uint2float_rn(mant), 5.9604644775390625e-08f);
        return (h & 0x8000u) ? -v : v;
    }
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t f = (e == 31) ? (sign | 0x7F800000u | (mant << 13))
                                 : (sign | ((e + 112u) << 23) | (mant << 13));
    return __uint_as_float(f);
}

// Byte sources for the block decoders: read-only global loads, or generic loads (a
// block staged in shared memory).
struct GlobalBytes {
    __device__ static __forceinline__ uint32_t u8(const uint8_t* p) { return __ldg(p); }
    // 2-byte alignment holds for every field read this way (block strides are even).
    __device__ static __forceinline__ uint32_t u16(const uint8_t* p) {
        return __ldg(reinterpret_cast<const unsigned short*>(p));
    }
};
struct GenericBytes {
    __device__ static __forceinline__ uint32_t u8(const uint8_t* p) { return *p; }
    __device__ static __forceinline__ uint32_t u16(const uint8_t* p) {
        return *reinterpret_cast<const unsigned short*>(p);
    }
};

__device__ __forceinline__ uint32_t ld_u8(const uint8_t* p) { return GlobalBytes::u8(p); }
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return GlobalBytes::u16(p); }

// get_scale_min_k4 (quantization.cpp:151-159)
template <class B = GlobalBytes>
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& d, int& m) {
    if (j < 4) {
        d = B::u8(q + j) & 63;
        m = B::u8(q + j + 4) & 63;
    } else {
        d = (B::u8(q + j + 4) & 0xF) | ((B::u8(q + j - 4) >> 6) << 4);
        m = (B::u8(q + j + 4) >> 4) | ((B::u8(q + j) >> 6) << 4);
    }
}

// Eight consecutive elements [8g, 8g+8) of one block -> y[0..8), bit-exact; bytes read
// through B.
template <int TYPE, class B = GlobalBytes>
__device__ __forceinline__ void deq8(const uint8_t* blk, int g, float* y) {
    if constexpr (TYPE == IB_TYPE_Q4_0) {
        const float d = h2f(B::u16(blk));
        const uint8_t* qs = blk + 2 + 8 * (g & 1);
        const int sh = (g >> 1) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __fmul_rn((float)((int)((B::u8(qs + i) >> sh) & 0xF) - 8), d);
    } else if constexpr (TYPE == IB_TYPE_Q8_0) {
        const float d = h2f(B::u16(blk));
        const uint8_t* qs = blk + 2 + 8 * g;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __fmul_rn((float)(int8_t)B::u8(qs + i), d);
    } else if constexpr (TYPE == IB_TYPE_Q5_0) {
        const float d = h2f(B::u16(blk));
        const uint32_t qh = B::u16(blk + 2) | (B::u16(blk + 4) << 16);
        const int j0 = 8 * (g & 1), hi = g >> 1;
        const uint8_t* qs = blk + 6 + j0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int j = j0 + i;
            const int x = ((B::u8(qs + i) >> (4 * hi)) & 0xF) | (((qh >> (j + 16 * hi)) & 1) << 4);
            y[i] = __fmul_rn((float)(x - 16), d);
        }
    } else if constexpr (TYPE == IB_TYPE_Q5_1) {
        const float d = h2f(B::u16(blk)), m = h2f(B::u16(blk + 2));
        const uint32_t qh = B::u16(blk + 4) | (B::u16(blk + 6) << 16);
        const int j0 = 8 * (g & 1), hi = g >> 1;
        const uint8_t* qs = blk + 8 + j0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int j = j0 + i;
            const int x = ((B::u8(qs + i) >> (4 * hi)) & 0xF) | (((qh >> (j + 16 * hi)) & 1) << 4);
            // x*d is exact (5-bit x, fp16 d), so this equals the reference's x*d + m
            y[i] = __fadd_rn(__fmul_rn((float)x, d), m);
        }
    } else if constexpr (TYPE == IB_TYPE_Q4_K) {
        // element e = 64p + 32h + l, byte q[32p + l], nibble h; group g covers p = g/8,
        // h = (g/4)&1, l0 = 8*(g&3)
        const float d = h2f(B::u16(blk)), dmin = h2f(B::u16(blk + 2));
        const int p = g >> 3, h = (g >> 2) & 1, l0 = 8 * (g & 3);
        int sc, m;
        scale_min_k4<B>(2 * p + h, blk + 4, sc, m);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        const uint8_t* q = blk + 16 + 32 * p + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = (B::u8(q + i) >> (4 * h)) & 0xF;
            y[i] = __fsub_rn(__fmul_rn(d1, (float)v), m1);  // product exact
        }
    } else {
        static_assert(TYPE == IB_TYPE_Q6_K, "deq8: unsupported type");
        // element e = 128c + 32gg + l; ql[64c + l + 32(gg&1)] nibble gg>>1, qh[32c + l]
        // bits 2gg..2gg+1, scale sc[8c + 2gg + l/16]; y = (d*sc)*q
        const float d = h2f(B::u16(blk + 208));
        const int e0 = 8 * g, c = e0 >> 7, r = e0 & 127, gg = r >> 5, l0 = r & 31;
        const uint8_t* ql = blk + 64 * c + l0 + 32 * (gg & 1);
        const uint8_t* qh = blk + 128 + 32 * c + l0;
        const int s = (int)(int8_t)B::u8(blk + 192 + 8 * c + 2 * gg + (l0 >> 4));
        const float ds = __fmul_rn(d, (float)s);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int lo = (B::u8(ql + i) >> (4 * (gg >> 1))) & 0xF;
            const int hi = (B::u8(qh + i) >> (2 * gg)) & 3;
            const int q = (int)(int8_t)(lo | (hi << 4)) - 32;
            y[i] = __fmul_rn(ds, (float)q);
        }
    }
}

}  // namespace ib
