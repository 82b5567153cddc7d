// Per-block math of the int8-MMA dequant-GEMV, shared by the standalone GEMV
// (gemv_mma.cu) and the fused decode kernels (decode.cu).  Template flags: SMEM =
// weight blocks read from shared memory (TMA ring) instead of global memory; XS =
// activation limbs and sums read from shared memory instead of global memory.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "gemv_mma.cuh"
#include "ib_cuda.h"

namespace ib {
// ---- primitives ------------------------------------------------------------------
__device__ __forceinline__ void mma_k32(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1, int& d0, int& d1, int& d2,
                                        int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_k16(uint32_t a0, uint32_t a1, uint32_t b0, int& d0, int& d1,
                                        int& d2, int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%7,%8,%9,%10};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Loads that work on global (read-only path) or shared pointers.
template <bool SMEM>
struct Ld {
    static __device__ __forceinline__ uint32_t u16(const uint8_t* p) {
        if (SMEM) return *reinterpret_cast<const unsigned short*>(p);
        return __ldg(reinterpret_cast<const unsigned short*>(p));
    }
    static __device__ __forceinline__ uint32_t u32(const uint8_t* p) {
        if (SMEM) return *reinterpret_cast<const uint32_t*>(p);
        return __ldg(reinterpret_cast<const uint32_t*>(p));
    }
    static __device__ __forceinline__ uint32_t u32a2(const uint8_t* p) {  // 2-byte aligned
        return u16(p) | (u16(p + 2) << 16);
    }
    static __device__ __forceinline__ uint2 u64(const uint8_t* p) {
        if (SMEM) return *reinterpret_cast<const uint2*>(p);
        return __ldg(reinterpret_cast<const uint2*>(p));
    }
    static __device__ __forceinline__ uint4 u128(const uint8_t* p) {
        if (SMEM) return *reinterpret_cast<const uint4*>(p);
        return __ldg(reinterpret_cast<const uint4*>(p));
    }
};

// Limb split of one value at scale 2^e (|v| <= 127 * 2^e): v = 2^e (L0 + L1/2^7 +
// L2/2^14 + L3/2^21) + r, |r| <= 2^(e-22); every step is exact in FP32.
__device__ __forceinline__ void limb_split(float v, int e, int8_t (&L)[4]) {
    float tt = ldexpf(v, -e);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float r = rintf(tt);
        L[i] = (int8_t)(int)r;
        tt = (tt - r) * 128.0f;
    }
}

// Exponent of the power-of-two limb scale for a group whose max |x| is m.
__device__ __forceinline__ int limb_exp(float m) {
    int e = 0;
    if (m > 0.f) frexpf(m / 127.0f, &e);  // m/127 = f * 2^e, f in [0.5, 1) -> m / 2^e < 127
    return e;
}

// Loads of the activation limbs / scales / sums from global (read-only path) or shared.
template <bool XS>
struct LdX {
    static __device__ __forceinline__ uint2 u64(const int8_t* p) {
        if (XS) return *reinterpret_cast<const uint2*>(p);
        return __ldg(reinterpret_cast<const uint2*>(p));
    }
    static __device__ __forceinline__ uint32_t u32(const int8_t* p) {
        if (XS) return *reinterpret_cast<const uint32_t*>(p);
        return __ldg(reinterpret_cast<const uint32_t*>(p));
    }
    static __device__ __forceinline__ float f(const float* p) {
        if (XS) return *p;
        return __ldg(p);
    }
};

__device__ __forceinline__ float byte_f(uint32_t w, int i) {  // unsigned byte i of w as float
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 + i)) - 8388608.0f;
}
__device__ __forceinline__ float h2f_fast(uint32_t h) {  // exact for finite halves
    return __half2float(__ushort_as_half((unsigned short)h));
}
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

__device__ __forceinline__ void mma_k32_acc(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1, int& d0, int& d1, int& d2,
                                            int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d0), "+r"(d1), "+r"(d2), "+r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// "Split columns": one k32 MMA carries two different sub-blocks, P in K slots
// [0,16) and Q in [16,32).  B columns 0-3 hold P's four limbs (zero for K >= 16),
// columns 4-7 hold Q's (zero for K < 16), so D[row][col] never mixes them and
// every lane of a quad ends up owning useful sums: t = 0/1 -> sub-block P, limb
// pairs (0,1)/(2,3); t = 2/3 -> sub-block Q.  Each lane loads one limb word per MMA
// (limb g & 3 of P if g < 4, of Q if g >= 4) and scales one sub-block per row.
struct LaneCtx {
    int g, t;
    int half;  // 0: this lane's D columns belong to sub-block P, 1: to Q
    int lim;   // limb index this lane loads for B (g & 3)
    bool upper;  // g >= 4: the lane's B word goes to the K >= 16 half
    float cw;  // limb-pair weight: 2^-7 for limbs (0,1), 2^-21 for (2,3)
    float tm;  // 1 on the lane that adds its sub-block's offset term, else 0
};

__device__ __forceinline__ LaneCtx lane_ctx() {
    LaneCtx c;
    const int lane = threadIdx.x & 31;
    c.g = lane >> 2;
    c.t = lane & 3;
    c.half = c.t >> 1;
    c.lim = c.g & 3;
    c.upper = c.g >= 4;
    c.cw = (c.t & 1) ? 4.76837158203125e-07f : 0.0078125f;
    c.tm = (c.t & 1) ? 0.0f : 1.0f;
    return c;
}

// ---- per-block math, rows a (= g) and b (= g + 8) ---------------------------------
// Q4_K block kb.  Pair p = sub-blocks (2p: low nibbles, 2p+1: high nibbles) of qs
// bytes [32p, 32p+32).  Lane t holds bytes [8t, 8t+8): MMA m (0, 1) uses bytes
// [8t + 4m, +4), i.e. elements 8t+4m+i of both sub-blocks (P = 2p low, Q = 2p+1 high).
template <bool SMEM, bool XS>
__device__ __forceinline__ void block_q4k(const uint8_t* ba, const uint8_t* bb, int kb,
                                          const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                          float& acc_b) {
    using L = Ld<SMEM>;
    const uint4 ha = L::u128(ba), hb = L::u128(bb);
    uint2 qa[4], qb[4], lx[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        qa[p] = L::u64(ba + 16 + 32 * p + 8 * c.t);
        qb[p] = L::u64(bb + 16 + 32 * p + 8 * c.t);
        lx[p] = LdX<XS>::u64(xb.limbs + ((size_t)kb * 8 + 2 * p + c.upper) * 128 + c.lim * 32 +
                             8 * c.t);
    }
    const float s = LdX<XS>::f(xb.scale + kb);
    // 6-bit scales / mins of sub-blocks 0..7 as bytes (get_scale_min_k4, quantization.cpp:151-159)
    const uint32_t sca_lo = ha.y & 0x3F3F3F3Fu, ma_lo = ha.z & 0x3F3F3F3Fu;
    const uint32_t sca_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t scb_lo = hb.y & 0x3F3F3F3Fu, mb_lo = hb.z & 0x3F3F3F3Fu;
    const uint32_t scb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    const uint32_t mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
    const float da = h2f_fast(ha.x & 0xFFFF) * s * c.cw, dma = -h2f_fast(ha.x >> 16) * c.tm;
    const float db = h2f_fast(hb.x & 0xFFFF) * s * c.cw, dmb = -h2f_fast(hb.x >> 16) * c.tm;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t M = 0x0F0F0F0Fu;
        int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
        mma_k32_acc(qa[p].x & M, qb[p].x & M, (qa[p].x >> 4) & M, (qb[p].x >> 4) & M,
                    c.upper ? 0u : lx[p].x, c.upper ? lx[p].x : 0u, d0, d1, d2, d3);
        mma_k32_acc(qa[p].y & M, qb[p].y & M, (qa[p].y >> 4) & M, (qb[p].y >> 4) & M,
                    c.upper ? 0u : lx[p].y, c.upper ? lx[p].y : 0u, d0, d1, d2, d3);
        const int sub = 2 * p + c.half, bi = sub & 3;
        const float sum = LdX<XS>::f(xb.sum32 + (size_t)kb * 8 + sub);
        const uint32_t swa = p < 2 ? sca_lo : sca_hi, mwa = p < 2 ? ma_lo : ma_hi;
        const uint32_t swb = p < 2 ? scb_lo : scb_hi, mwb = p < 2 ? mb_lo : mb_hi;
        acc_a = fmaf(da * byte_f(swa, bi), (float)(d0 * 128 + d1), acc_a);
        acc_a = fmaf(dma * byte_f(mwa, bi), sum, acc_a);
        acc_b = fmaf(db * byte_f(swb, bi), (float)(d2 * 128 + d3), acc_b);
        acc_b = fmaf(dmb * byte_f(mwb, bi), sum, acc_b);
    }
}

// Q5_K block kb: Q4_K's arithmetic with 5-bit quants.  The same d, dmin and 6-bit scale /
// min header, qs at byte 48 (Q4_K: 16), and the fifth bit of element 64p + 32h + l in
// qh[l] (byte 16 + l) at bit 2p + h.  Lane t's bytes [8t, 8t+8) of each 32-byte chunk
// pair with qh bytes [8t, 8t+8): the bits go in at bit 4 of each quant byte, so the
// MMA's unsigned-fitting s8 operands hold q in [0, 31] (GGUF block layout; the reference
// sizes this format but does not decode it).
template <bool SMEM, bool XS>
__device__ __forceinline__ void block_q5k(const uint8_t* ba, const uint8_t* bb, int kb,
                                          const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                          float& acc_b) {
    using L = Ld<SMEM>;
    const uint4 ha = L::u128(ba), hb = L::u128(bb);
    const uint2 qha = L::u64(ba + 16 + 8 * c.t), qhb = L::u64(bb + 16 + 8 * c.t);
    uint2 qa[4], qb[4], lx[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        qa[p] = L::u64(ba + 48 + 32 * p + 8 * c.t);
        qb[p] = L::u64(bb + 48 + 32 * p + 8 * c.t);
        lx[p] = LdX<XS>::u64(xb.limbs + ((size_t)kb * 8 + 2 * p + c.upper) * 128 + c.lim * 32 +
                             8 * c.t);
    }
    const float s = LdX<XS>::f(xb.scale + kb);
    const uint32_t sca_lo = ha.y & 0x3F3F3F3Fu, ma_lo = ha.z & 0x3F3F3F3Fu;
    const uint32_t sca_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t scb_lo = hb.y & 0x3F3F3F3Fu, mb_lo = hb.z & 0x3F3F3F3Fu;
    const uint32_t scb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    const uint32_t mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
    const float da = h2f_fast(ha.x & 0xFFFF) * s * c.cw, dma = -h2f_fast(ha.x >> 16) * c.tm;
    const float db = h2f_fast(hb.x & 0xFFFF) * s * c.cw, dmb = -h2f_fast(hb.x >> 16) * c.tm;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t M = 0x0F0F0F0Fu, H = 0x01010101u;
        // fifth bits of this chunk's low (2p) and high (2p + 1) sub-blocks, at bit 4
        const uint32_t la0 = ((qha.x >> (2 * p)) & H) << 4, ua0 = ((qha.x >> (2 * p + 1)) & H) << 4;
        const uint32_t la1 = ((qha.y >> (2 * p)) & H) << 4, ua1 = ((qha.y >> (2 * p + 1)) & H) << 4;
        const uint32_t lb0 = ((qhb.x >> (2 * p)) & H) << 4, ub0 = ((qhb.x >> (2 * p + 1)) & H) << 4;
        const uint32_t lb1 = ((qhb.y >> (2 * p)) & H) << 4, ub1 = ((qhb.y >> (2 * p + 1)) & H) << 4;
        int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
        mma_k32_acc((qa[p].x & M) | la0, (qb[p].x & M) | lb0, ((qa[p].x >> 4) & M) | ua0,
                    ((qb[p].x >> 4) & M) | ub0, c.upper ? 0u : lx[p].x, c.upper ? lx[p].x : 0u,
                    d0, d1, d2, d3);
        mma_k32_acc((qa[p].y & M) | la1, (qb[p].y & M) | lb1, ((qa[p].y >> 4) & M) | ua1,
                    ((qb[p].y >> 4) & M) | ub1, c.upper ? 0u : lx[p].y, c.upper ? lx[p].y : 0u,
                    d0, d1, d2, d3);
        const int sub = 2 * p + c.half, bi = sub & 3;
        const float sum = LdX<XS>::f(xb.sum32 + (size_t)kb * 8 + sub);
        const uint32_t swa = p < 2 ? sca_lo : sca_hi, mwa = p < 2 ? ma_lo : ma_hi;
        const uint32_t swb = p < 2 ? scb_lo : scb_hi, mwb = p < 2 ? mb_lo : mb_hi;
        acc_a = fmaf(da * byte_f(swa, bi), (float)(d0 * 128 + d1), acc_a);
        acc_a = fmaf(dma * byte_f(mwa, bi), sum, acc_a);
        acc_b = fmaf(db * byte_f(swb, bi), (float)(d2 * 128 + d3), acc_b);
        acc_b = fmaf(dmb * byte_f(mwb, bi), sum, acc_b);
    }
}

// Q6_K block kb.  Element e = 128c + 32gg + l, 16-element sub-block 8c + 2gg + l/16.
// For (c, h = l/16) lane t covers l = 16h + 4t + i: ql bytes at 64c + 16h + 4t (gg 0:
// low, gg 2: high nibbles) and 64c + 32 + 16h + 4t (gg 1, 3), qh at 128 + 32c + 16h +
// 4t (bits 2gg).  One MMA pairs P = (c, 2q, h) with Q = (c, 2q+1, h).  u = q + 32 in
// [0, 63] is fed unsigned; the -32 uses the per-16 activation sums.
template <bool SMEM, bool XS>
__device__ __forceinline__ void block_q6k(const uint8_t* ba, const uint8_t* bb, int kb,
                                          const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                          float& acc_b) {
    using L = Ld<SMEM>;
    uint32_t sa[4], sb[4];  // 16 int8 scales per row
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sa[i] = L::u32a2(ba + 192 + 4 * i);
        sb[i] = L::u32a2(bb + 192 + 4 * i);
    }
    const float s = LdX<XS>::f(xb.scale + kb);
    const float da = h2f_fast(L::u16(ba + 208)), db = h2f_fast(L::u16(bb + 208));
    const float fa = da * s * c.cw, fb = db * s * c.cw;
    const float oa = -32.0f * da * c.tm, ob = -32.0f * db * c.tm;
    const int8_t* xl = xb.limbs + (size_t)kb * 8 * 128 + c.lim * 32 + 4 * c.t;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int o = 16 * h + 4 * c.t;
            const uint32_t a0 = L::u32a2(ba + 64 * cc + o), a1 = L::u32a2(ba + 64 * cc + 32 + o);
            const uint32_t ah = L::u32a2(ba + 128 + 32 * cc + o);
            const uint32_t b0 = L::u32a2(bb + 64 * cc + o), b1 = L::u32a2(bb + 64 * cc + 32 + o);
            const uint32_t bh = L::u32a2(bb + 128 + 32 * cc + o);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint32_t M = 0x0F0F0F0Fu, H = 0x03030303u;
                const int sh = 4 * q;
                const uint32_t bx = LdX<XS>::u32(xl + (4 * cc + 2 * q + c.upper) * 128 + 16 * h);
                int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
                mma_k32_acc(((a0 >> sh) & M) | (((ah >> sh) & H) << 4),
                            ((b0 >> sh) & M) | (((bh >> sh) & H) << 4),
                            ((a1 >> sh) & M) | (((ah >> (sh + 2)) & H) << 4),
                            ((b1 >> sh) & M) | (((bh >> (sh + 2)) & H) << 4),
                            c.upper ? 0u : bx, c.upper ? bx : 0u, d0, d1, d2, d3);
                const int sub = 8 * cc + 2 * (2 * q + c.half) + h;
                const int shs = 8 * (sub & 3);  // int8 scale, sign-extended
                const float sca = (float)(int)(int8_t)(sa[sub >> 2] >> shs);
                const float scb = (float)(int)(int8_t)(sb[sub >> 2] >> shs);
                const float sum = LdX<XS>::f(xb.sum16 + (size_t)kb * 16 + sub);
                acc_a = fmaf(fa * sca, (float)(d0 * 128 + d1), acc_a);
                acc_a = fmaf(oa * sca, sum, acc_a);
                acc_b = fmaf(fb * scb, (float)(d2 * 128 + d3), acc_b);
                acc_b = fmaf(ob * scb, sum, acc_b);
            }
        }
}

// 32-element blocks (Q4_0, Q5_0, Q5_1, Q8_0), two blocks per call: P = block kb in
// K slots [0,16), Q = block kb+1 in [16,32).  Lane t holds qs bytes [4t, 4t+4):
// MMA 0 takes their low nibbles (elements 4t..4t+3), MMA 1 the high nibbles (elements
// 16+4t..); for Q8_0 the int8 bytes [4t..] and [16+4t..].  has_q = false when kb is
// the row's last, unpaired block (Q's lanes then add nothing).
template <int TYPE, bool SMEM>
__device__ __forceinline__ void q32_unpack(const uint8_t* blk, int t, uint32_t& lo, uint32_t& hi) {
    using L = Ld<SMEM>;
    if (TYPE == IB_TYPE_Q8_0) {
        lo = L::u32a2(blk + 2 + 4 * t);
        hi = L::u32a2(blk + 18 + 4 * t);
        return;
    }
    uint32_t q, qh = 0;
    if (TYPE == IB_TYPE_Q5_1) {  // 24-byte blocks are 8-byte aligned
        qh = L::u32(blk + 4);
        q = L::u32(blk + 8 + 4 * t);
    } else if (TYPE == IB_TYPE_Q5_0) {
        qh = L::u32a2(blk + 2);
        q = L::u32a2(blk + 6 + 4 * t);
    } else {  // Q4_0
        q = L::u32a2(blk + 2 + 4 * t);
    }
    lo = q & 0x0F0F0F0Fu;
    hi = (q >> 4) & 0x0F0F0F0Fu;
    if (TYPE != IB_TYPE_Q4_0) {  // fifth bit: qh bit j -> bit 4 of element j's byte
        const uint32_t bl = (qh >> (4 * t)) & 0xFu, bh = (qh >> (16 + 4 * t)) & 0xFu;
        lo |= ((bl * 0x00204081u) & 0x01010101u) << 4;
        hi |= ((bh * 0x00204081u) & 0x01010101u) << 4;
    }
}

template <int TYPE, bool SMEM>
__device__ __forceinline__ void q32_scales(const uint8_t* blk, float& d, float& m) {
    using L = Ld<SMEM>;
    if (TYPE == IB_TYPE_Q5_1) {
        const uint32_t dm = L::u32(blk);
        d = h2f_fast(dm & 0xFFFF);
        m = h2f_fast(dm >> 16);
    } else {
        d = h2f_fast(L::u16(blk));
        m = 0.f;
    }
}

template <int TYPE, bool SMEM, bool XS>
__device__ __forceinline__ void block_q32(const uint8_t* ba, const uint8_t* bb, int kb, bool has_q,
                                          const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                          float& acc_b) {
    constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                       TYPE == IB_TYPE_Q5_1 ? 24 : 34;
    const int qoff = has_q ? BB : 0;
    uint32_t paL, paH, pbL, pbH, qaL, qaH, qbL, qbH;
    q32_unpack<TYPE, SMEM>(ba, c.t, paL, paH);
    q32_unpack<TYPE, SMEM>(bb, c.t, pbL, pbH);
    q32_unpack<TYPE, SMEM>(ba + qoff, c.t, qaL, qaH);
    q32_unpack<TYPE, SMEM>(bb + qoff, c.t, qbL, qbH);
    const int mine = kb + (has_q ? c.half : 0);  // block whose sums this lane owns
    const int8_t* xl = xb.limbs + ((size_t)kb + (has_q ? c.upper : 0)) * 128 + c.lim * 32 + 4 * c.t;
    const uint32_t x0 = LdX<XS>::u32(xl);
    const uint32_t x1 = LdX<XS>::u32(xl + 16);
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
    mma_k32_acc(paL, pbL, qaL, qbL, c.upper ? 0u : x0, c.upper ? x0 : 0u, d0, d1, d2, d3);
    mma_k32_acc(paH, pbH, qaH, qbH, c.upper ? 0u : x1, c.upper ? x1 : 0u, d0, d1, d2, d3);
    float dA, mA, dB, mB;
    const int own = (has_q && c.half) ? BB : 0;
    q32_scales<TYPE, SMEM>(ba + own, dA, mA);
    q32_scales<TYPE, SMEM>(bb + own, dB, mB);
    const float live = (has_q || c.half == 0) ? 1.0f : 0.0f;
    const float f = LdX<XS>::f(xb.scale + mine) * c.cw * live;
    const float sm = LdX<XS>::f(xb.sum32 + mine) * c.tm * live;
    acc_a = fmaf(dA * f, (float)(d0 * 128 + d1), acc_a);
    acc_b = fmaf(dB * f, (float)(d2 * 128 + d3), acc_b);
    // offsets: Q4_0 -8*d*sum, Q5_0 -16*d*sum, Q5_1 +m*sum (applied once per row)
    if (TYPE == IB_TYPE_Q4_0) {
        acc_a = fmaf(-8.0f * dA, sm, acc_a);
        acc_b = fmaf(-8.0f * dB, sm, acc_b);
    } else if (TYPE == IB_TYPE_Q5_0) {
        acc_a = fmaf(-16.0f * dA, sm, acc_a);
        acc_b = fmaf(-16.0f * dB, sm, acc_b);
    } else if (TYPE == IB_TYPE_Q5_1) {
        acc_a = fmaf(mA, sm, acc_a);
        acc_b = fmaf(mB, sm, acc_b);
    }
}

// ---- lean tiles: weights and limbs both in shared memory (fused kernels) ----------
// Shared-memory loads by 32-bit shared address with immediate offsets, so the inner
// loop spends no instructions on 64-bit address arithmetic.
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ float ldsf(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(a), "n"(OFF));
    return v;
}
__device__ __forceinline__ uint32_t bfe6(uint32_t w, uint32_t pos) {
    uint32_t r;
    asm("bfe.u32 %0, %1, %2, 6;" : "=r"(r) : "r"(w), "r"(pos));
    return r;
}
// A operand unsigned (quants), B signed (limbs).
__device__ __forceinline__ void mma_u8s8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, int& d0, int& d1, int& d2,
                                         int& d3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d0), "+r"(d1), "+r"(d2), "+r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// a * b + c on the FMA pipe (IMAD): the tile math is otherwise bound by the ALU pipe.
__device__ __forceinline__ uint32_t imad(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// Lane constants of the lean tiles (computed once per kernel).
struct LeanLane {
    uint32_t bm0, bm1;  // 1 / 0: this lane's limb word goes to K [0,16) (bm0) or [16,32) (bm1)
    uint32_t limb_off;  // byte offset of this lane's limb word inside a 256-element block
    uint32_t sum_off;   // byte offset of this lane's sub-block sum inside a block's sum32 run
    uint32_t sh0, sh1;  // bit position of this lane's 6-bit scale for even / odd pairs
    float hw;           // 1/16 on lanes whose sub-block was fed as high nibbles in place
};

__device__ __forceinline__ LeanLane lean_lane(const LaneCtx& c) {
    LeanLane l;
    l.bm0 = c.upper ? 0u : 1u;
    l.bm1 = 1u - l.bm0;
    l.limb_off = (uint32_t)(c.upper * 128 + c.lim * 32 + 8 * c.t);
    l.sum_off = (uint32_t)(4 * c.half);
    l.sh0 = 8u * c.half;
    l.sh1 = 16u + 8u * c.half;
    l.hw = c.half ? 0.0625f : 1.0f;
    return l;
}

// Q4_K block kb for tile rows a (wa) and b (wb); limbs at xl = limbs + kb * 1024,
// sums at xsum = sum32 + kb * 32 (shared addresses).  Same arithmetic as block_q4k
// except: high nibbles enter the MMA in place (x16, unsigned operand, scaled back by
// 1/16), and the 6-bit sub-block scales are applied in int32 across the block's
// sub-blocks (|sum| < 2^28), so the FP32 conversion happens once per block.
__device__ __forceinline__ void q4k_tile_lean(uint32_t wa, uint32_t wb, uint32_t xl,
                                              uint32_t xsum, float s, const LaneCtx& c,
                                              const LeanLane& l, float& acc_a, float& acc_b) {
    const uint4 ha = lds128(wa), hb = lds128(wb);
    const uint32_t qa0 = wa + 16 + 8 * c.t, qb0 = wb + 16 + 8 * c.t, x0 = xl + l.limb_off;
    const uint32_t xs0 = xsum + l.sum_off;
    uint2 qa[4], qb[4], lx[4];
    float sm[4];
    qa[0] = lds64<0>(qa0); qa[1] = lds64<32>(qa0); qa[2] = lds64<64>(qa0); qa[3] = lds64<96>(qa0);
    qb[0] = lds64<0>(qb0); qb[1] = lds64<32>(qb0); qb[2] = lds64<64>(qb0); qb[3] = lds64<96>(qb0);
    lx[0] = lds64<0>(x0); lx[1] = lds64<256>(x0); lx[2] = lds64<512>(x0); lx[3] = lds64<768>(x0);
    sm[0] = ldsf<0>(xs0); sm[1] = ldsf<8>(xs0); sm[2] = ldsf<16>(xs0); sm[3] = ldsf<24>(xs0);
    // 6-bit scales / mins of sub-blocks 0-3 (low words) and 4-7 (high words)
    const uint32_t sa_lo = ha.y, ma_lo = ha.z, sb_lo = hb.y, mb_lo = hb.z;
    const uint32_t sa_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t sb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
    const uint32_t mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
    int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;
    float ma = 0.f, mb = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t M = 0x0F0F0F0Fu;
        int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
        // low nibbles by mask (ALU); high nibbles in place as q - low (IMAD, FMA pipe);
        // the split-column B words by a 0/1 multiplier (IMAD)
        const uint32_t ax = qa[p].x & M, bx = qb[p].x & M, ay = qa[p].y & M, by = qb[p].y & M;
        mma_u8s8(ax, bx, imad(ax, 0xFFFFFFFFu, qa[p].x), imad(bx, 0xFFFFFFFFu, qb[p].x),
                 imad(lx[p].x, l.bm0, 0u), imad(lx[p].x, l.bm1, 0u), d0, d1, d2, d3);
        mma_u8s8(ay, by, imad(ay, 0xFFFFFFFFu, qa[p].y), imad(by, 0xFFFFFFFFu, qb[p].y),
                 imad(lx[p].y, l.bm0, 0u), imad(lx[p].y, l.bm1, 0u), d0, d1, d2, d3);
        const uint32_t sh = (p & 1) ? l.sh1 : l.sh0;
        const int sca = (int)bfe6(p < 2 ? sa_lo : sa_hi, sh);
        const int scb = (int)bfe6(p < 2 ? sb_lo : sb_hi, sh);
        ia0 += sca * d0;
        ia1 += sca * d1;
        ib0 += scb * d2;
        ib1 += scb * d3;
        ma = fmaf((float)bfe6(p < 2 ? ma_lo : ma_hi, sh), sm[p], ma);
        mb = fmaf((float)bfe6(p < 2 ? mb_lo : mb_hi, sh), sm[p], mb);
    }
    const float fs = s * c.cw * l.hw;
    const float fa = h2f_fast(ha.x & 0xFFFF) * fs, fb = h2f_fast(hb.x & 0xFFFF) * fs;
    acc_a = fmaf(fa, fmaf((float)ia0, 128.0f, (float)ia1), acc_a);
    acc_b = fmaf(fb, fmaf((float)ib0, 128.0f, (float)ib1), acc_b);
    acc_a = fmaf(-h2f_fast(ha.x >> 16) * c.tm, ma, acc_a);
    acc_b = fmaf(-h2f_fast(hb.x >> 16) * c.tm, mb, acc_b);
}

template <int TYPE>
struct Fmt {
    static constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                              TYPE == IB_TYPE_Q5_1 ? 24 : TYPE == IB_TYPE_Q8_0 ? 34 :
                              TYPE == IB_TYPE_Q4_K ? 144 : TYPE == IB_TYPE_Q5_K ? 176 : 210;
    static constexpr bool K = TYPE == IB_TYPE_Q4_K || TYPE == IB_TYPE_Q6_K || TYPE == IB_TYPE_Q5_K;
    // blocks per TMA stage (per row): 1152 B (Q4_K), 1408 B (Q5_K), 1680 B (Q6_K), 32 blocks otherwise
    static constexpr int KB = K ? 8 : 32;
    static constexpr int CHUNK = KB * BB;
    static constexpr int UNIT = K ? 1 : 2;  // blocks handled per block_math call
};

template <int TYPE, bool SMEM, bool XS = false>
__device__ __forceinline__ void block_math(const uint8_t* ba, const uint8_t* bb, int kb, int nb,
                                           const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                           float& acc_b) {
    if constexpr (TYPE == IB_TYPE_Q4_K) block_q4k<SMEM, XS>(ba, bb, kb, xb, c, acc_a, acc_b);
    else if constexpr (TYPE == IB_TYPE_Q6_K) block_q6k<SMEM, XS>(ba, bb, kb, xb, c, acc_a, acc_b);
    else if constexpr (TYPE == IB_TYPE_Q5_K) block_q5k<SMEM, XS>(ba, bb, kb, xb, c, acc_a, acc_b);
    else block_q32<TYPE, SMEM, XS>(ba, bb, kb, kb + 1 < nb, xb, c, acc_a, acc_b);
}

}  // namespace ib
