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

// Elements and bytes per block of each format, at compile time.
template <int TYPE>
struct QFmt {
    static constexpr int BE = (TYPE == IB_TYPE_Q4_K || TYPE == IB_TYPE_Q6_K ||
                               TYPE == IB_TYPE_Q2_K || TYPE == IB_TYPE_Q3_K ||
                               TYPE == IB_TYPE_Q5_K) ? 256 : 32;
    static constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                              TYPE == IB_TYPE_Q5_1 ? 24 : TYPE == IB_TYPE_Q8_0 ? 34 :
                              TYPE == IB_TYPE_Q4_K ? 144 : TYPE == IB_TYPE_Q6_K ? 210 :
                              TYPE == IB_TYPE_Q4_1 ? 20 : TYPE == IB_TYPE_Q2_K ? 84 :
                              TYPE == IB_TYPE_Q3_K ? 110 : 176;
};

// Eight consecutive elements [8g, 8g+8) of one block -> y[0..8), bit-exact; bytes read
// through B.  Q4_1, Q2_K, Q3_K and Q5_K follow the published GGUF layouts (the
// reference sizes these formats but does not decode them): every value is one exact
// product of the fp16 scale and small integers, plus at most one rounding.
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
    } else if constexpr (TYPE == IB_TYPE_Q4_1) {
        // d, m, qs[16]: element j < 16 low nibble of qs[j], j >= 16 high nibble of qs[j-16]
        const float d = h2f(B::u16(blk)), m = h2f(B::u16(blk + 2));
        const uint8_t* qs = blk + 4 + 8 * (g & 1);
        const int sh = (g >> 1) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            y[i] = __fadd_rn(__fmul_rn((float)((B::u8(qs + i) >> sh) & 0xF), d), m);  // product exact
    } else if constexpr (TYPE == IB_TYPE_Q5_K) {
        // as Q4_K, qs at 48, the fifth bit of element 64p + 32h + l in qh[l] bit 2p + h
        const float d = h2f(B::u16(blk)), dmin = h2f(B::u16(blk + 2));
        const int p = g >> 3, h = (g >> 2) & 1, l0 = 8 * (g & 3);
        int sc, m;
        scale_min_k4<B>(2 * p + h, blk + 4, sc, m);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        const uint8_t* q = blk + 48 + 32 * p + l0;
        const uint8_t* qh = blk + 16 + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = ((B::u8(q + i) >> (4 * h)) & 0xF) | (((B::u8(qh + i) >> (2 * p + h)) & 1) << 4);
            y[i] = __fsub_rn(__fmul_rn(d1, (float)v), m1);  // product exact
        }
    } else if constexpr (TYPE == IB_TYPE_Q2_K) {
        // scales[16] (scale | min << 4), qs[64], d, dmin: element e = 128h + 32j + 16k + l,
        // 2 bits at 2j of qs[32h + 16k + l], sub-block 8h + 2j + k = e / 16
        const float d = h2f(B::u16(blk + 80)), dmin = h2f(B::u16(blk + 82));
        const int e0 = 8 * g, h = e0 >> 7, j = (e0 >> 5) & 3, k = (e0 >> 4) & 1, l0 = e0 & 15;
        const int scm = (int)B::u8(blk + (e0 >> 4));
        const float dl = __fmul_rn(d, (float)(scm & 0xF)), ml = __fmul_rn(dmin, (float)(scm >> 4));
        const uint8_t* q = blk + 16 + 32 * h + 16 * k + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            y[i] = __fsub_rn(__fmul_rn(dl, (float)((B::u8(q + i) >> (2 * j)) & 3)), ml);
    } else if constexpr (TYPE == IB_TYPE_Q3_K) {
        // hmask[32], qs[64], scales[12], d: element e = 128h + 32j + 16k + l, q = 2 bits at
        // 2j of qs[32h + 16k + l] minus 4 unless hmask[16k + l] bit 4h + j; scale e / 16 as
        // a 6-bit value - 32 (low nibble: byte i or the high nibble of byte i - 8; top two
        // bits: byte 8 + i % 4 at bit 2 (i / 4))
        const float d = h2f(B::u16(blk + 108));
        const int e0 = 8 * g, h = e0 >> 7, j = (e0 >> 5) & 3, k = (e0 >> 4) & 1, l0 = e0 & 15;
        const int si = e0 >> 4;
        const int lo = si < 8 ? (int)(B::u8(blk + 96 + si) & 0xF) : (int)(B::u8(blk + 96 + si - 8) >> 4);
        const int hi = (int)((B::u8(blk + 104 + (si & 3)) >> (2 * (si >> 2))) & 3);
        const float dl = __fmul_rn(d, (float)((lo | (hi << 4)) - 32));
        const uint8_t* q = blk + 32 + 32 * h + 16 * k + l0;
        const uint8_t* hm = blk + 16 * k + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = (int)((B::u8(q + i) >> (2 * j)) & 3) -
                          (((B::u8(hm + i) >> (4 * h + j)) & 1) ? 0 : 4);
            y[i] = __fmul_rn(dl, (float)v);  // exact
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
