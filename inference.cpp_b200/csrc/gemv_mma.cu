// Fused dequant + GEMV on GGUF blocks (batch-1 decode; HBM-bound), sm_100a.
//
// Data movement: a CTA owns 16 consecutive rows.  A producer warp streams the
// rows' packed bytes with 1-D TMA bulk copies (cp.async.bulk, no multicast) into
// a ring of S shared-memory stages, one 16-row x KB-block slice per stage,
// guarded by mbarriers (full: transaction bytes; empty: one arrival per consumer
// warp).  The bytes in flight are set by the ring, not by registers or occupancy.
// Shapes whose row slices are not 16-byte aligned use the same math with direct
// global loads.
//
// Math: a SIMT FP32 dot product costs ~3 issue slots per 4-bit weight (unpack,
// int->float, FMA).  Here the quants are widened to int8 with one LOP3 per four
// weights and fed to mma.sync.m16n8k32.s8 (m16n8k16 for Q6_K's 16-element
// sub-blocks) as the dot-product engine; the FP32 activation is split once per
// call into four exact int8 limbs
//     x = s * (L0 + L1/2^7 + L2/2^14 + L3/2^21) + r,   |r| <= s * 2^-22,
// s a power of two per group (32 or 256 elements), one limb per MMA column, so
// every MMA returns exact integer dot products.  Block scales (d, d*sc, dmin*m,
// the Q4_0/Q5_0/Q6_K offsets) are applied in FP32 afterwards with the reference's
// definitions (src/gguf/quantization.cpp:28-245).  The result differs from a
// sequential FP32 dot product only by FP32 rounding of per-sub-block partials.
//
// MMA fragment use (lane = 4g + t): lane (g, t) supplies rows g and g+8 of the
// 16-row tile at K slots 4t..4t+3 and 16+4t..16+4t+3, and limb g (g < 4) of the
// activation at the same slots; D[row][limb] lands in lanes t = 0 (limbs 0, 1)
// and t = 1 (limbs 2, 3), combined as (c0 * 128 + c1) * 2^-7 or * 2^-21.
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv_mma.cuh"
#include "pipeline.cuh"
#include "quant.cuh"

namespace ib {

static __device__ int g_gemv_fault;

// ---- activation limbs ----------------------------------------------------------
// One warp per 32-element sub-group; lane i = element i.  The scale is shared by
// `group` elements (32 or 256): s = 2^e with max|x| / s <= 127.
__global__ void xq_kernel(const float* __restrict__ x, int K, int group, int8_t* __restrict__ limbs,
                          float* __restrict__ scale, float* __restrict__ sum32,
                          float* __restrict__ sum16) {
    const int lane = threadIdx.x & 31;
    const int sg = (blockIdx.x * (blockDim.x >> 5)) + (threadIdx.x >> 5);  // 32-group
    if (sg * 32 >= K) return;
    const int per = group / 32;
    const int gbase = (sg / per) * per;  // first 32-group of this scale group
    float m = 0.f;
    for (int q = 0; q < per; ++q) m = fmaxf(m, fabsf(x[(gbase + q) * 32 + lane]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int e = 0;
    float s = 1.0f;
    if (m > 0.f) {
        frexpf(m / 127.0f, &e);  // m/127 = f * 2^e, f in [0.5, 1)  ->  m / 2^e <= 127
        s = ldexpf(1.0f, e);
    }
    const float v = x[sg * 32 + lane];
    float tt = ldexpf(v, -e);  // exact
    int8_t L[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float r = rintf(tt);
        L[i] = (int8_t)(int)r;
        tt = (tt - r) * 128.0f;  // exact
    }
    int8_t* o = limbs + (size_t)sg * 128;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i * 32 + lane] = L[i];
    float sm = v;
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o2);
    if ((lane & 15) == 0) sum16[sg * 2 + (lane >> 4)] = sm;
    sm += __shfl_xor_sync(0xffffffffu, sm, 16);
    if (lane == 0) {
        sum32[sg] = sm;
        if (sg == gbase) scale[sg / per] = s;
    }
}

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
template <bool SMEM>
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
        lx[p] = __ldg(reinterpret_cast<const uint2*>(
            xb.limbs + ((size_t)kb * 8 + 2 * p + c.upper) * 128 + c.lim * 32 + 8 * c.t));
    }
    const float s = __ldg(xb.scale + kb);
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
        const float sum = __ldg(xb.sum32 + (size_t)kb * 8 + sub);
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
template <bool SMEM>
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
    const float s = __ldg(xb.scale + kb);
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
                const uint32_t bx = __ldg(reinterpret_cast<const uint32_t*>(
                    xl + (4 * cc + 2 * q + c.upper) * 128 + 16 * h));
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
                const float sum = __ldg(xb.sum16 + (size_t)kb * 16 + sub);
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

template <int TYPE, bool SMEM>
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
    const uint32_t x0 = __ldg(reinterpret_cast<const uint32_t*>(xl));
    const uint32_t x1 = __ldg(reinterpret_cast<const uint32_t*>(xl + 16));
    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
    mma_k32_acc(paL, pbL, qaL, qbL, c.upper ? 0u : x0, c.upper ? x0 : 0u, d0, d1, d2, d3);
    mma_k32_acc(paH, pbH, qaH, qbH, c.upper ? 0u : x1, c.upper ? x1 : 0u, d0, d1, d2, d3);
    float dA, mA, dB, mB;
    const int own = (has_q && c.half) ? BB : 0;
    q32_scales<TYPE, SMEM>(ba + own, dA, mA);
    q32_scales<TYPE, SMEM>(bb + own, dB, mB);
    const float live = (has_q || c.half == 0) ? 1.0f : 0.0f;
    const float f = __ldg(xb.scale + mine) * c.cw * live;
    const float sm = __ldg(xb.sum32 + mine) * c.tm * live;
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

template <int TYPE>
struct Fmt {
    static constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                              TYPE == IB_TYPE_Q5_1 ? 24 : TYPE == IB_TYPE_Q8_0 ? 34 :
                              TYPE == IB_TYPE_Q4_K ? 144 : 210;
    static constexpr bool K = TYPE == IB_TYPE_Q4_K || TYPE == IB_TYPE_Q6_K;
    // blocks per TMA stage (per row): 1152 B (Q4_K), 1680 B (Q6_K), 32 blocks otherwise
    static constexpr int KB = TYPE == IB_TYPE_Q4_K ? 8 : TYPE == IB_TYPE_Q6_K ? 8 : 32;
    static constexpr int CHUNK = KB * BB;
    static constexpr int UNIT = K ? 1 : 2;  // blocks handled per block_math call
};

template <int TYPE, bool SMEM>
__device__ __forceinline__ void block_math(const uint8_t* ba, const uint8_t* bb, int kb, int nb,
                                           const XLimbs& xb, const LaneCtx& c, float& acc_a,
                                           float& acc_b) {
    if constexpr (TYPE == IB_TYPE_Q4_K) block_q4k<SMEM>(ba, bb, kb, xb, c, acc_a, acc_b);
    else if constexpr (TYPE == IB_TYPE_Q6_K) block_q6k<SMEM>(ba, bb, kb, xb, c, acc_a, acc_b);
    else block_q32<TYPE, SMEM>(ba, bb, kb, kb + 1 < nb, xb, c, acc_a, acc_b);
}

// Deterministic reduction of the per-warp partials of the CTA's 16 rows.
template <int NW>
__device__ __forceinline__ void finish_rows(float (*red)[16], int warp, const LaneCtx& c,
                                            float acc_a, float acc_b, float* y, int row_base,
                                            int rows) {
    acc_a = quad_sum(acc_a);
    acc_b = quad_sum(acc_b);
    if (c.t == 0 && warp < NW) {
        red[warp][c.g] = acc_a;
        red[warp][c.g + 8] = acc_b;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) v += red[w][threadIdx.x];
        const int r = row_base + threadIdx.x;
        if (r < rows) y[r] = v;
    }
}

// ---- TMA-staged persistent kernel: NWC consumer warps + 1 producer warp --------------
// CTA c owns row groups (16 rows) c, c + G, c + 2G, ... (G = gridDim.x, chosen so the
// groups divide evenly over the CTAs).  The producer streams every group's stages
// through one ring without pausing between groups; consumers reduce each group's
// partials behind a named barrier (double-buffered, so one barrier per group).
template <int TYPE, int NWC, int S>
__global__ void __launch_bounds__((NWC + 1) * 32) gemv_tma_kernel(const uint8_t* __restrict__ W,
                                                                 XLimbs xb, float* __restrict__ y,
                                                                 int rows, int nb) {
    using F = Fmt<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];  // [S][16][CHUNK]
    __shared__ __align__(8) uint64_t full[S], empty[S];
    __shared__ float red[2][NWC][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_rg = (rows + 15) / 16;
    const int my_rg = blockIdx.x < n_rg ? (n_rg - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int spg = nb / F::KB;  // stages per row group
    const int total = my_rg * spg;
    const size_t rbytes = (size_t)nb * F::BB;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NWC);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == NWC) {
        // producer: one bulk copy per row per stage, lanes 0..n-1
        int issued = 0;
        for (int it = 0; it < total; ++it) {
            const int s = it % S;
            const int rg = blockIdx.x + (it / spg) * gridDim.x, st = it % spg;
            const int row_base = rg * 16, n = min(16, rows - row_base);
            if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1, &g_gemv_fault, 1)) break;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(n * F::CHUNK));
            __syncwarp();
            if (lane < n)
                bulk_g2s(smem + ((size_t)s * 16 + lane) * F::CHUNK,
                         W + (size_t)(row_base + lane) * rbytes + (size_t)st * F::CHUNK, F::CHUNK,
                         &full[s]);
            issued = it + 1;
        }
        // make sure no copy is still landing when the CTA retires (normally a no-op)
        for (int it = issued > S ? issued - S : 0; it < issued; ++it)
            mbar_wait(&full[it % S], (it / S) & 1, &g_gemv_fault, 2);
        return;
    }
    const LaneCtx c = lane_ctx();
    float acc_a = 0.f, acc_b = 0.f;
    bool ok = true;
    for (int it = 0; it < total; ++it) {
        const int s = it % S;
        const int rgl = it / spg, st = it % spg;
        const int row_base = (blockIdx.x + rgl * gridDim.x) * 16, n = min(16, rows - row_base);
        if (ok && !mbar_wait(&full[s], (it / S) & 1, &g_gemv_fault, 3)) ok = false;
        if (ok) {
            const int ra = min(c.g, n - 1), rb = min(c.g + 8, n - 1);
            const uint8_t* sa = smem + ((size_t)s * 16 + ra) * F::CHUNK;
            const uint8_t* sb = smem + ((size_t)s * 16 + rb) * F::CHUNK;
#pragma unroll
            for (int kbl = warp * F::UNIT; kbl < F::KB; kbl += NWC * F::UNIT)
                block_math<TYPE, true>(sa + kbl * F::BB, sb + kbl * F::BB, st * F::KB + kbl, nb,
                                       xb, c, acc_a, acc_b);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (st == spg - 1) {  // row group done: reduce the warps' partials
            acc_a = quad_sum(acc_a);
            acc_b = quad_sum(acc_b);
            float(*r)[16] = red[rgl & 1];
            if (c.t == 0) {
                r[warp][c.g] = acc_a;
                r[warp][c.g + 8] = acc_b;
            }
            asm volatile("bar.sync 1, %0;" ::"r"(NWC * 32) : "memory");
            if (warp == 0 && lane < n) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < NWC; ++w) v += r[w][lane];
                y[row_base + lane] = v;
            }
            acc_a = 0.f;
            acc_b = 0.f;
        }
    }
}

// ---- direct-load kernel (any alignment the format allows) -------------------------
template <int TYPE, int NW>
__global__ void __launch_bounds__(NW * 32) gemv_direct_kernel(const uint8_t* __restrict__ W,
                                                             XLimbs xb, float* __restrict__ y,
                                                             int rows, int nb) {
    using F = Fmt<TYPE>;
    __shared__ float red[NW][16];
    const int warp = threadIdx.x >> 5;
    const LaneCtx c = lane_ctx();
    const int row_base = blockIdx.x * 16;
    const int ra = min(row_base + c.g, rows - 1), rb = min(row_base + c.g + 8, rows - 1);
    const size_t rbytes = (size_t)nb * F::BB;
    const uint8_t* Wa = W + (size_t)ra * rbytes;
    const uint8_t* Wb = W + (size_t)rb * rbytes;
    float acc_a = 0.f, acc_b = 0.f;
    for (int kb = warp * F::UNIT; kb < nb; kb += NW * F::UNIT)
        block_math<TYPE, false>(Wa + (size_t)kb * F::BB, Wb + (size_t)kb * F::BB, kb, nb, xb, c,
                                acc_a, acc_b);
    finish_rows<NW>(red, warp, c, acc_a, acc_b, y, row_base, rows);
}

// ---- host side -------------------------------------------------------------------
int xq_launch(const float* x, int K, int group, XLimbs& xb, cudaStream_t st) {
    const int groups32 = K / 32;
    xq_kernel<<<(groups32 + 7) / 8, 256, 0, st>>>(x, K, group, xb.limbs, xb.scale, xb.sum32,
                                                   xb.sum16);
    IB_LAUNCH_CHECK("xq_kernel");
    return IB_OK;
}

size_t xlimbs_bytes(int K) {
    // limbs (128 B per 32) + scale per 32 (worst case) + sums per 32 and per 16,
    // each part 256-byte aligned
    const size_t g = (size_t)(K / 32);
    return ((g * 128 + 255) / 256 + (g * 4 + 255) / 256 * 2 + (g * 8 + 255) / 256) * 256;
}

void xlimbs_carve(void* base, int K, XLimbs& xb) {
    const size_t g = (size_t)(K / 32);
    char* p = (char*)base;
    xb.limbs = (int8_t*)p;
    p += (g * 128 + 255) / 256 * 256;
    xb.scale = (float*)p;
    p += (g * 4 + 255) / 256 * 256;
    xb.sum32 = (float*)p;
    p += (g * 4 + 255) / 256 * 256;
    xb.sum16 = (float*)p;
}

template <int TYPE>
static int launch_typed(const uint8_t* W, const XLimbs& xb, float* y, int64_t rows, int64_t cols,
                        cudaStream_t st) {
    using F = Fmt<TYPE>;
    constexpr int NWC = 8;
    constexpr int S = TYPE == IB_TYPE_Q6_K ? 2 : (TYPE == IB_TYPE_Q8_0 ? 3 : 4);
    const int nb = (int)(cols / (F::K ? 256 : 32));
    const int n_rg = (int)((rows + 15) / 16);
    const size_t rbytes = (size_t)nb * F::BB;
    const bool tma_ok = nb % F::KB == 0 && rbytes % 16 == 0 && ((uintptr_t)W & 15) == 0;
    if (tma_ok) {
        const size_t smem = (size_t)S * 16 * F::CHUNK;
        auto kern = gemv_tma_kernel<TYPE, NWC, S>;
        static int attr_dev_mask = 0;  // smem opt-in beyond 48 KB, once per device
        static int max_ctas[64] = {0};
        int dev = 0;
        IB_CUDA_CHECK(cudaGetDevice(&dev));
        if (!(attr_dev_mask & (1 << dev))) {
            if (smem + 2048 > 48 * 1024)
                IB_CUDA_CHECK(cudaFuncSetAttribute(
                    kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            int per_sm = 0, sms = 0;
            IB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern,
                                                                        (NWC + 1) * 32, smem));
            IB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
            max_ctas[dev & 63] = (per_sm > 0 ? per_sm : 1) * sms;
            attr_dev_mask |= 1 << dev;
        }
        // as many CTAs as fit, but dividing the row groups evenly
        const int cap = max_ctas[dev & 63];
        const int per = (n_rg + cap - 1) / cap;
        const int grid = (n_rg + per - 1) / per;
        kern<<<grid, (NWC + 1) * 32, smem, st>>>(W, xb, y, (int)rows, nb);
        IB_LAUNCH_CHECK("gemv_tma_kernel");
        return IB_OK;
    }
    gemv_direct_kernel<TYPE, 8><<<(unsigned)n_rg, 256, 0, st>>>(W, xb, y, (int)rows, nb);
    IB_LAUNCH_CHECK("gemv_direct_kernel");
    return IB_OK;
}

int gemv_mma_launch(int type, const void* W, const XLimbs& xb, float* y, int64_t rows,
                    int64_t cols, cudaStream_t st) {
    const uint8_t* w8 = (const uint8_t*)W;
    switch (type) {
        case IB_TYPE_Q4_K: return launch_typed<IB_TYPE_Q4_K>(w8, xb, y, rows, cols, st);
        case IB_TYPE_Q6_K: return launch_typed<IB_TYPE_Q6_K>(w8, xb, y, rows, cols, st);
        case IB_TYPE_Q4_0: return launch_typed<IB_TYPE_Q4_0>(w8, xb, y, rows, cols, st);
        case IB_TYPE_Q5_0: return launch_typed<IB_TYPE_Q5_0>(w8, xb, y, rows, cols, st);
        case IB_TYPE_Q5_1: return launch_typed<IB_TYPE_Q5_1>(w8, xb, y, rows, cols, st);
        case IB_TYPE_Q8_0: return launch_typed<IB_TYPE_Q8_0>(w8, xb, y, rows, cols, st);
    }
    set_error("gemv_mma: unsupported type");
    return IB_ERR_UNSUPPORTED;
}

int gemv_mma_group(int type) { return (type == IB_TYPE_Q4_K || type == IB_TYPE_Q6_K) ? 256 : 32; }

bool gemv_mma_supported(int type) {
    return type == IB_TYPE_Q4_K || type == IB_TYPE_Q6_K || type == IB_TYPE_Q4_0 ||
           type == IB_TYPE_Q5_0 || type == IB_TYPE_Q5_1 || type == IB_TYPE_Q8_0;
}

// Alignment each format's loads need from the weight base pointer.
int gemv_mma_align(int type) {
    switch (type) {
        case IB_TYPE_Q4_K: return 16;
        case IB_TYPE_Q5_1: return 8;
        default: return 2;
    }
}

int gemv_fault_take(int* code) {
    int v = 0, z = 0;
    IB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_gemv_fault, sizeof(int)));
    if (v) IB_CUDA_CHECK(cudaMemcpyToSymbol(g_gemv_fault, &z, sizeof(int)));
    *code = v;
    return IB_OK;
}

}  // namespace ib
