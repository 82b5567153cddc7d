// Fused dequant + GEMV on GGUF blocks (batch-1 decode):  y[r] = sum_c W[r,c] x[c].
//
// HBM-bound: each weight byte is read exactly once, the FP32 activation vector
// (<= 56 KB) is served from L1/L2.  A warp owns NR consecutive rows; its lanes
// split the row's blocks, load the packed bytes with the widest aligned loads the
// format allows (16 B for Q4_K whose 144-byte blocks are 16-byte aligned), unpack
// in registers and accumulate in FP32; the NR partial sums are reduced with warp
// shuffles.  Each lane's activation slice is loaded once and reused for its NR
// rows.  Per-block scales are factored out of the inner dot product:
//   sum_i (d*s*q_i - dmin*m) x_i = d*s*sum_i q_i x_i - dmin*m*sum_i x_i
// which is exact algebra and changes only the FP32 summation order (results are
// checked against the reference within a relative tolerance).
//
// Integer -> float conversion of small unsigned fields uses the exponent trick
// f = as_float(0x4B000000 | u) - 2^23, exact for u < 2^23.
#include "common.cuh"
#include "decode.cuh"
#include "gemv_mma.cuh"
#include "ops.cuh"
#include "quant.cuh"

namespace ib {

__device__ __forceinline__ float u2f(uint32_t u) {
    return __uint_as_float(0x4B000000u | u) - 8388608.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float4 ldx4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}

// ---------------------------------------------------------------------------
// Q4_K: 8 lanes per 144-byte super-block; lane s loads qs bytes [16s, 16s+16)
// (pair p = s/2 of sub-blocks 2p, 2p+1; elements l0..l0+15 of each, l0 = 16(s&1))
// plus the 16-byte header (d, dmin, scales) that its 8 lanes share.
// ---------------------------------------------------------------------------
template <int NR>
__device__ __forceinline__ void gemv_q4_k_rows(const uint8_t* __restrict__ W,
                                               const float* __restrict__ x, int64_t row0,
                                               int64_t rows, int64_t cols, float* acc) {
    const int lane = threadIdx.x & 31;
    const int s = lane & 7, slot = lane >> 3;
    const int p = s >> 1, l0 = 16 * (s & 1);
    const int64_t nb = cols / 256;
    const int64_t row_bytes = nb * 144;
    for (int64_t kb = slot; kb < nb; kb += 4) {
        const float* xb = x + kb * 256 + 64 * p + l0;
        float xl[16], xh[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 a = ldx4(xb + 4 * i), b = ldx4(xb + 32 + 4 * i);
            xl[4 * i] = a.x; xl[4 * i + 1] = a.y; xl[4 * i + 2] = a.z; xl[4 * i + 3] = a.w;
            xh[4 * i] = b.x; xh[4 * i + 1] = b.y; xh[4 * i + 2] = b.z; xh[4 * i + 3] = b.w;
        }
        float sxl = 0.f, sxh = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) { sxl += xl[i]; sxh += xh[i]; }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (row0 + r >= rows) break;
            const uint8_t* blk = W + (row0 + r) * row_bytes + kb * 144;
            const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * s));
            const float d = h2f(h.x & 0xFFFFu), dmin = h2f(h.x >> 16);
            // scales[12] = bytes of h.y, h.z, h.w; get_scale_min_k4 for j = 2p, 2p+1
            const uint32_t sb[3] = {h.y, h.z, h.w};
            auto byte_at = [&](int i) -> uint32_t { return (sb[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
            int sc0, m0, sc1, m1;
            {
                const int j = 2 * p;
                if (j < 4) { sc0 = byte_at(j) & 63; m0 = byte_at(j + 4) & 63; }
                else { sc0 = (byte_at(j + 4) & 0xF) | ((byte_at(j - 4) >> 6) << 4);
                       m0 = (byte_at(j + 4) >> 4) | ((byte_at(j) >> 6) << 4); }
            }
            {
                const int j = 2 * p + 1;
                if (j < 4) { sc1 = byte_at(j) & 63; m1 = byte_at(j + 4) & 63; }
                else { sc1 = (byte_at(j + 4) & 0xF) | ((byte_at(j - 4) >> 6) << 4);
                       m1 = (byte_at(j + 4) >> 4) | ((byte_at(j) >> 6) << 4); }
            }
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
            float dl = 0.f, dh = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint32_t byte = (qw[w] >> (8 * b)) & 0xFFu;
                    dl = fmaf(u2f(byte & 0xFu), xl[4 * w + b], dl);
                    dh = fmaf(u2f(byte >> 4), xh[4 * w + b], dh);
                }
            }
            acc[r] += d * ((float)sc0 * dl + (float)sc1 * dh) -
                      dmin * ((float)m0 * sxl + (float)m1 * sxh);
        }
    }
}

// ---------------------------------------------------------------------------
// Q6_K: 8 lanes per 210-byte super-block; lane s covers half-chunk c = s/4 and
// l in [l0, l0+8), l0 = 8(s&3), for the 4 quarter groups gg: elements
// 128c + 32gg + l.  Blocks are only 2-byte aligned, so fields load as u16.
// ---------------------------------------------------------------------------
template <int NR>
__device__ __forceinline__ void gemv_q6_k_rows(const uint8_t* __restrict__ W,
                                               const float* __restrict__ x, int64_t row0,
                                               int64_t rows, int64_t cols, float* acc) {
    const int lane = threadIdx.x & 31;
    const int s = lane & 7, slot = lane >> 3;
    const int c = s >> 2, l0 = 8 * (s & 3);
    const int64_t nb = cols / 256;
    const int64_t row_bytes = nb * 210;
    for (int64_t kb = slot; kb < nb; kb += 4) {
        float xv[4][8];
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
            const float* xp = x + kb * 256 + 128 * c + 32 * gg + l0;
            float4 a = ldx4(xp), b = ldx4(xp + 4);
            xv[gg][0] = a.x; xv[gg][1] = a.y; xv[gg][2] = a.z; xv[gg][3] = a.w;
            xv[gg][4] = b.x; xv[gg][5] = b.y; xv[gg][6] = b.z; xv[gg][7] = b.w;
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (row0 + r >= rows) break;
            const uint8_t* blk = W + (row0 + r) * row_bytes + kb * 210;
            const unsigned short* pa = reinterpret_cast<const unsigned short*>(blk + 64 * c + l0);
            const unsigned short* pb = reinterpret_cast<const unsigned short*>(blk + 64 * c + 32 + l0);
            const unsigned short* ph = reinterpret_cast<const unsigned short*>(blk + 128 + 32 * c + l0);
            uint32_t qa[4], qb[4], qh[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { qa[i] = __ldg(pa + i); qb[i] = __ldg(pb + i); qh[i] = __ldg(ph + i); }
            const uint8_t* scp = blk + 192 + 8 * c + (l0 >> 4);
            const float d = h2f(__ldg(reinterpret_cast<const unsigned short*>(blk + 208)));
            float part = 0.f;
#pragma unroll
            for (int gg = 0; gg < 4; ++gg) {
                float dot = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t src = (gg & 1) ? qb[i >> 1] : qa[i >> 1];
                    const uint32_t byte = (src >> (8 * (i & 1))) & 0xFFu;
                    const uint32_t lo = (byte >> (4 * (gg >> 1))) & 0xFu;
                    const uint32_t hi = ((qh[i >> 1] >> (8 * (i & 1))) >> (2 * gg)) & 3u;
                    // q - 32 with q = lo | hi << 4
                    const float qf = __uint_as_float(0x4B000000u | lo | (hi << 4)) - 8388640.0f;
                    dot = fmaf(qf, xv[gg][i], dot);
                }
                part = fmaf((float)(int8_t)__ldg(scp + 2 * gg), dot, part);
            }
            acc[r] = fmaf(d, part, acc[r]);
        }
    }
}

// ---------------------------------------------------------------------------
// 32-element formats: one lane per block, lanes stride over the row's blocks.
// ---------------------------------------------------------------------------
template <int TYPE, int NR>
__device__ __forceinline__ void gemv_q32_rows(const uint8_t* __restrict__ W,
                                              const float* __restrict__ x, int64_t row0,
                                              int64_t rows, int64_t cols, float* acc) {
    constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                       TYPE == IB_TYPE_Q5_1 ? 24 : 34;
    const int lane = threadIdx.x & 31;
    const int64_t nb = cols / 32;
    const int64_t row_bytes = nb * BB;
    for (int64_t kb = lane; kb < nb; kb += 32) {
        float xv[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 a = ldx4(x + kb * 32 + 4 * i);
            xv[4 * i] = a.x; xv[4 * i + 1] = a.y; xv[4 * i + 2] = a.z; xv[4 * i + 3] = a.w;
        }
        float sx = 0.f;
        if (TYPE != IB_TYPE_Q8_0) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sx += xv[i];
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (row0 + r >= rows) break;
            const uint8_t* blk = W + (row0 + r) * row_bytes + kb * BB;
            const unsigned short* p16 = reinterpret_cast<const unsigned short*>(blk);
            if (TYPE == IB_TYPE_Q8_0) {
                const float d = h2f(__ldg(p16));
                float dot = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t v = __ldg(p16 + 1 + i);
                    dot = fmaf((float)(int8_t)(v & 0xFF), xv[2 * i], dot);
                    dot = fmaf((float)(int8_t)(v >> 8), xv[2 * i + 1], dot);
                }
                acc[r] = fmaf(d, dot, acc[r]);
            } else {
                const int qs_off = TYPE == IB_TYPE_Q4_0 ? 1 : TYPE == IB_TYPE_Q5_0 ? 3 : 4;
                const float d = h2f(__ldg(p16));
                uint32_t qh = 0;
                if (TYPE == IB_TYPE_Q5_0) qh = __ldg(p16 + 1) | ((uint32_t)__ldg(p16 + 2) << 16);
                if (TYPE == IB_TYPE_Q5_1) qh = __ldg(p16 + 2) | ((uint32_t)__ldg(p16 + 3) << 16);
                float dot = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t v = __ldg(p16 + qs_off + i);
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        const int j = 2 * i + b;
                        const uint32_t byte = (v >> (8 * b)) & 0xFFu;
                        uint32_t lo = byte & 0xFu, hi = byte >> 4;
                        if (TYPE != IB_TYPE_Q4_0) {
                            lo |= ((qh >> j) & 1u) << 4;
                            hi |= ((qh >> (j + 16)) & 1u) << 4;
                        }
                        dot = fmaf(u2f(lo), xv[j], dot);
                        dot = fmaf(u2f(hi), xv[j + 16], dot);
                    }
                }
                if (TYPE == IB_TYPE_Q4_0) acc[r] = fmaf(d, dot - 8.0f * sx, acc[r]);
                else if (TYPE == IB_TYPE_Q5_0) acc[r] = fmaf(d, dot - 16.0f * sx, acc[r]);
                else {
                    const float m = h2f(__ldg(p16 + 1));
                    acc[r] = fmaf(d, dot, fmaf(m, sx, acc[r]));
                }
            }
        }
    }
}

template <int TYPE, int NR>
__global__ void __launch_bounds__(128) gemv_q_kernel(const uint8_t* __restrict__ W,
                                                     const float* __restrict__ x,
                                                     float* __restrict__ y, int64_t rows,
                                                     int64_t cols) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * NR;
    if (row0 >= rows) return;
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;
    if (TYPE == IB_TYPE_Q4_K) gemv_q4_k_rows<NR>(W, x, row0, rows, cols, acc);
    else if (TYPE == IB_TYPE_Q6_K) gemv_q6_k_rows<NR>(W, x, row0, rows, cols, acc);
    else gemv_q32_rows<TYPE, NR>(W, x, row0, rows, cols, acc);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == 0 && row0 + r < rows) y[row0 + r] = v;
    }
}

// ---------------------------------------------------------------------------
// FP32 / INT16 GEMV with the reference's semantics (cuda_kernels.cu:62-95):
// one warp per row, float4 / 4 x int16 loads, shuffle reduction.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemv_f32_kernel(const float* __restrict__ W,
                                                       const float* __restrict__ x,
                                                       float* __restrict__ y, int M, int N) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const float* w = W + (int64_t)row * N;
    float s = 0.f;
    if ((N & 3) == 0 && (((uintptr_t)w | (uintptr_t)x) & 15) == 0) {
        for (int k = lane * 4; k < N; k += 128) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w + k));
            const float4 b = __ldg(reinterpret_cast<const float4*>(x + k));
            s = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, s))));
        }
    } else {
        for (int k = lane; k < N; k += 32) s = fmaf(w[k], x[k], s);
    }
    s = warp_sum(s);
    if (lane == 0) y[row] = s;
}

__global__ void __launch_bounds__(256) gemv_i16_kernel(const int16_t* __restrict__ W,
                                                       const float* __restrict__ scale,
                                                       const float* __restrict__ x,
                                                       float* __restrict__ y, int M, int N) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= M) return;
    const int16_t* w = W + (int64_t)row * N;
    float s = 0.f;
    if ((N & 7) == 0 && (((uintptr_t)w & 15) | ((uintptr_t)x & 15)) == 0) {
        for (int k = lane * 8; k < N; k += 256) {
            const int4 a = __ldg(reinterpret_cast<const int4*>(w + k));
            const float4 b0 = __ldg(reinterpret_cast<const float4*>(x + k));
            const float4 b1 = __ldg(reinterpret_cast<const float4*>(x + k + 4));
            s = fmaf((float)(short)(a.x & 0xFFFF), b0.x, s);
            s = fmaf((float)(short)(a.x >> 16), b0.y, s);
            s = fmaf((float)(short)(a.y & 0xFFFF), b0.z, s);
            s = fmaf((float)(short)(a.y >> 16), b0.w, s);
            s = fmaf((float)(short)(a.z & 0xFFFF), b1.x, s);
            s = fmaf((float)(short)(a.z >> 16), b1.y, s);
            s = fmaf((float)(short)(a.w & 0xFFFF), b1.z, s);
            s = fmaf((float)(short)(a.w >> 16), b1.w, s);
        }
    } else {
        for (int k = lane; k < N; k += 32) s = fmaf((float)w[k], x[k], s);
    }
    s = warp_sum(s);
    if (lane == 0) y[row] = s * scale[row];
}

template <int TYPE, int NR>
static int launch_gemv_q(const uint8_t* W, const float* x, float* y, int64_t rows,
                         int64_t cols, cudaStream_t st) {
    constexpr int WARPS = 4;
    const int64_t rows_per_cta = (int64_t)WARPS * NR;
    const int64_t grid = (rows + rows_per_cta - 1) / rows_per_cta;
    gemv_q_kernel<TYPE, NR><<<(unsigned)grid, WARPS * 32, 0, st>>>(W, x, y, rows, cols);
    IB_LAUNCH_CHECK("gemv_q_kernel");
    return IB_OK;
}

// ---------------------------------------------------------------------------
// Q4_1, Q2_K, Q3_K, Q5_K: decode-as-you-go GEMV, lanes striding over the row's
// 8-element groups (deq8w: the bit-exact values of quant.cuh's deq8), NR rows per warp
// sharing each x load, FP32 accumulation and a shuffle reduction.
// ---------------------------------------------------------------------------
// deq8 of quant.cuh for the added formats with word loads instead of byte loads (the
// GEMV's blocks are aligned: Q5_K 16 bytes, Q4_1 and Q2_K 4, Q3_K 2); the same float
// operations in the same order, so the same values.
__device__ __forceinline__ uint32_t ldg32(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }
__device__ __forceinline__ uint32_t ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

template <int TYPE>
__device__ __forceinline__ void deq8w(const uint8_t* blk, int g, float* y) {
    if constexpr (TYPE == IB_TYPE_Q4_1) {
        const uint32_t hm = ldg32(blk);
        const float d = h2f(hm & 0xFFFF), m = h2f(hm >> 16);
        const uint8_t* qs = blk + 4 + 8 * (g & 1);
        const uint32_t w0 = ldg32(qs), w1 = ldg32(qs + 4);
        const int sh = (g >> 1) * 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t byte = byte_of(i < 4 ? w0 : w1, i & 3);
            y[i] = __fadd_rn(__fmul_rn((float)((byte >> sh) & 0xF), d), m);
        }
    } else if constexpr (TYPE == IB_TYPE_Q5_K) {
        const uint32_t hm = ldg32(blk);
        const float d = h2f(hm & 0xFFFF), dmin = h2f(hm >> 16);
        const int p = g >> 3, h = (g >> 2) & 1, l0 = 8 * (g & 3), j = 2 * p + h;
        const uint32_t s0 = ldg32(blk + 4), s1 = ldg32(blk + 8), s2 = ldg32(blk + 12);
        // get_scale_min_k4(j) on the 12 scale bytes
        auto sb = [&](int i) { return i < 4 ? byte_of(s0, i) : i < 8 ? byte_of(s1, i - 4) : byte_of(s2, i - 8); };
        int sc, m;
        if (j < 4) {
            sc = (int)(sb(j) & 63);
            m = (int)(sb(j + 4) & 63);
        } else {
            sc = (int)((sb(j + 4) & 0xF) | ((sb(j - 4) >> 6) << 4));
            m = (int)((sb(j + 4) >> 4) | ((sb(j) >> 6) << 4));
        }
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(blk + 48 + 32 * p + l0));
        const uint2 qh = __ldg(reinterpret_cast<const uint2*>(blk + 16 + l0));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t qb = byte_of(i < 4 ? q.x : q.y, i & 3);
            const uint32_t hb = byte_of(i < 4 ? qh.x : qh.y, i & 3);
            const int v = (int)(((qb >> (4 * h)) & 0xF) | (((hb >> j) & 1) << 4));
            y[i] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
        }
    } else if constexpr (TYPE == IB_TYPE_Q2_K) {
        const uint32_t dd = ldg32(blk + 80);
        const float d = h2f(dd & 0xFFFF), dmin = h2f(dd >> 16);
        const int e0 = 8 * g, h = e0 >> 7, j = (e0 >> 5) & 3, k = (e0 >> 4) & 1, l0 = e0 & 15;
        const int scm = (int)__ldg(blk + (e0 >> 4));
        const float dl = __fmul_rn(d, (float)(scm & 0xF)), ml = __fmul_rn(dmin, (float)(scm >> 4));
        const uint8_t* q = blk + 16 + 32 * h + 16 * k + l0;
        const uint32_t w0 = ldg32(q), w1 = ldg32(q + 4);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            y[i] = __fsub_rn(__fmul_rn(dl, (float)((byte_of(i < 4 ? w0 : w1, i & 3) >> (2 * j)) & 3)), ml);
    } else {
        static_assert(TYPE == IB_TYPE_Q3_K, "deq8w: unsupported type");
        const float d = h2f(ldg16(blk + 108));
        const int e0 = 8 * g, h = e0 >> 7, j = (e0 >> 5) & 3, k = (e0 >> 4) & 1, l0 = e0 & 15;
        const int si = e0 >> 4;
        const int lo = si < 8 ? (int)(__ldg(blk + 96 + si) & 0xF) : (int)(__ldg(blk + 96 + si - 8) >> 4);
        const int hi = (int)((__ldg(blk + 104 + (si & 3)) >> (2 * (si >> 2))) & 3);
        const float dl = __fmul_rn(d, (float)((lo | (hi << 4)) - 32));
        const uint8_t* q = blk + 32 + 32 * h + 16 * k + l0;
        const uint8_t* hm = blk + 16 * k + l0;
        uint32_t qw[4], hw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qw[i] = ldg16(q + 2 * i);
            hw[i] = ldg16(hm + 2 * i);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t qb = (qw[i >> 1] >> (8 * (i & 1))) & 0xFFu;
            const uint32_t hb = (hw[i >> 1] >> (8 * (i & 1))) & 0xFFu;
            const int v = (int)((qb >> (2 * j)) & 3) - (((hb >> (4 * h + j)) & 1) ? 0 : 4);
            y[i] = __fmul_rn(dl, (float)v);
        }
    }
}

template <int TYPE, int NR>
__global__ void __launch_bounds__(128) gemv_deq_kernel(const uint8_t* __restrict__ W,
                                                       const float* __restrict__ x,
                                                       float* __restrict__ y, int64_t rows,
                                                       int64_t cols) {
    // the CTA's 4 warps split the NR rows' groups (short dependent chains per warp); the
    // loop is unrolled so each lane has several groups' loads in flight
    constexpr int BE = QFmt<TYPE>::BE, BB = QFmt<TYPE>::BB, GPB = BE / 8;
    __shared__ float red[4][NR];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.x * NR;
    const int64_t gpr = cols / 8, row_bytes = cols / BE * BB;
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;
#pragma unroll 2
    for (int64_t g = threadIdx.x; g < gpr; g += 128) {
        const float4 a = ldx4(x + g * 8), b = ldx4(x + g * 8 + 4);
        const int64_t blk = g / GPB;
        const int sub = (int)(g - blk * GPB);
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (row0 + r >= rows) break;
            float v[8];
            deq8w<TYPE>(W + (row0 + r) * row_bytes + blk * BB, sub, v);
            float t = acc[r];
            t = fmaf(v[0], a.x, t);
            t = fmaf(v[1], a.y, t);
            t = fmaf(v[2], a.z, t);
            t = fmaf(v[3], a.w, t);
            t = fmaf(v[4], b.x, t);
            t = fmaf(v[5], b.y, t);
            t = fmaf(v[6], b.z, t);
            t = fmaf(v[7], b.w, t);
            acc[r] = t;
        }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) red[warp][r] = v;
    }
    __syncthreads();
    if (threadIdx.x < NR && row0 + threadIdx.x < rows)
        y[row0 + threadIdx.x] = (red[0][threadIdx.x] + red[1][threadIdx.x]) +
                                (red[2][threadIdx.x] + red[3][threadIdx.x]);
}

template <int TYPE>
static int launch_gemv_deq(const uint8_t* W, const float* x, float* y, int64_t rows,
                           int64_t cols, cudaStream_t st) {
    constexpr int NR = 2;
    const int64_t grid = (rows + NR - 1) / NR;
    IB_REQUIRE(grid <= 0x7FFFFFFF, "gemv: too many rows");
    gemv_deq_kernel<TYPE, NR><<<(unsigned)grid, 128, 0, st>>>(W, x, y, rows, cols);
    IB_LAUNCH_CHECK("gemv_deq_kernel");
    return IB_OK;
}

}  // namespace ib

using namespace ib;

extern "C" int ib_gemv_q(int type, const void* dev_W, const float* dev_x, float* dev_y,
                         int64_t rows, int64_t cols, void* stream) {
    if (rows == 0) return IB_OK;
    IB_REQUIRE(dev_W && dev_x && dev_y, "null pointer argument");
    IB_REQUIRE(rows > 0 && cols > 0, "bad GEMV shape");
    IB_REQUIRE(((uintptr_t)dev_x & 15) == 0, "x must be 16-byte aligned");
    const int be = block_elems(type);
    if (!is_quant(type)) {
        set_error(std::string("ib_gemv_q: unsupported type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(cols % be == 0, "cols must be a multiple of the block size");
    cudaStream_t st = as_stream(stream);
    const uint8_t* W = (const uint8_t*)dev_W;
    if (cols <= (1 << 30) && rows < (1ll << 31) && slab_supported(type)) {
        // limb slab of x, then the TMA-staged GEMV (decode.cu)
        const bool kq = slab_kquant(type);
        FusedGemv f = {};
        f.W[0] = W;
        f.type[0] = type;
        f.rows[0] = (int)rows;
        f.n_seg = 1;
        f.K = (int)cols;
        f.y = dev_y;
        f.slab = (const uint8_t*)16;  // placeholder for the shape check
        if (fused_gemv_supported(f, EPI_STORE)) {
            void* ws = nullptr;
            int r = workspace_get(WS_GEMV, slab_total_bytes((int)cols, kq), &ws);
            if (r != IB_OK) return r;
            if ((r = xq_slab_launch(dev_x, nullptr, (int)cols, kq, (uint8_t*)ws, nullptr, st, false)))
                return r;
            f.slab = (const uint8_t*)ws;
            return fused_gemv_launch(f, PRO_PLAIN, EPI_STORE, st, false);
        }
    }
    if (is_extra_quant(type)) {  // the decode-as-you-go GEMV (Q5_K: bases off 16 bytes)
        const uintptr_t align = type == IB_TYPE_Q5_K ? 16 : type == IB_TYPE_Q3_K ? 2 : 4;
        IB_REQUIRE(((uintptr_t)W & (align - 1)) == 0,
                   "weights must be aligned to " + std::to_string(align) + " bytes");
        switch (type) {
            case IB_TYPE_Q4_1: return launch_gemv_deq<IB_TYPE_Q4_1>(W, dev_x, dev_y, rows, cols, st);
            case IB_TYPE_Q2_K: return launch_gemv_deq<IB_TYPE_Q2_K>(W, dev_x, dev_y, rows, cols, st);
            case IB_TYPE_Q3_K: return launch_gemv_deq<IB_TYPE_Q3_K>(W, dev_x, dev_y, rows, cols, st);
            default: return launch_gemv_deq<IB_TYPE_Q5_K>(W, dev_x, dev_y, rows, cols, st);
        }
    }
    if (gemv_mma_supported(type) && ((uintptr_t)W % gemv_mma_align(type)) == 0 &&
        cols <= (1 << 30) && rows < (1ll << 31)) {
        void* ws = nullptr;
        int r = workspace_get(WS_GEMV, xlimbs_bytes((int)cols), &ws);
        if (r != IB_OK) return r;
        XLimbs xb;
        xlimbs_carve(ws, (int)cols, xb);
        if ((r = xq_launch(dev_x, (int)cols, gemv_mma_group(type), xb, st)) != IB_OK) return r;
        return gemv_mma_launch(type, W, xb, dev_y, rows, cols, st);
    }
    switch (type) {
        case IB_TYPE_Q4_K:
            IB_REQUIRE(((uintptr_t)W & 15) == 0, "Q4_K weights must be 16-byte aligned");
            return launch_gemv_q<IB_TYPE_Q4_K, 2>(W, dev_x, dev_y, rows, cols, st);
        case IB_TYPE_Q6_K:
            IB_REQUIRE(((uintptr_t)W & 1) == 0, "weights must be 2-byte aligned");
            return launch_gemv_q<IB_TYPE_Q6_K, 2>(W, dev_x, dev_y, rows, cols, st);
        case IB_TYPE_Q4_0:
            IB_REQUIRE(((uintptr_t)W & 1) == 0, "weights must be 2-byte aligned");
            return launch_gemv_q<IB_TYPE_Q4_0, 2>(W, dev_x, dev_y, rows, cols, st);
        case IB_TYPE_Q5_0:
            IB_REQUIRE(((uintptr_t)W & 1) == 0, "weights must be 2-byte aligned");
            return launch_gemv_q<IB_TYPE_Q5_0, 2>(W, dev_x, dev_y, rows, cols, st);
        case IB_TYPE_Q5_1:
            IB_REQUIRE(((uintptr_t)W & 1) == 0, "weights must be 2-byte aligned");
            return launch_gemv_q<IB_TYPE_Q5_1, 2>(W, dev_x, dev_y, rows, cols, st);
        case IB_TYPE_Q8_0:
            IB_REQUIRE(((uintptr_t)W & 1) == 0, "weights must be 2-byte aligned");
            return launch_gemv_q<IB_TYPE_Q8_0, 2>(W, dev_x, dev_y, rows, cols, st);
    }
    return IB_ERR_UNSUPPORTED;
}

extern "C" int ib_slab_bytes(int type, int64_t cols, size_t* bytes) {
    IB_REQUIRE(bytes && cols > 0 && cols <= (1 << 30), "bad arguments");
    if (!slab_supported(type)) {
        set_error(std::string("ib_slab_bytes: unsupported type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    *bytes = slab_total_bytes((int)cols, slab_kquant(type));
    return IB_OK;
}

extern "C" int ib_limb_slab(int type, const float* dev_x, int64_t cols, void* dev_slab, void* stream) {
    IB_REQUIRE(dev_x && dev_slab && cols > 0 && cols <= (1 << 30), "bad arguments");
    IB_REQUIRE(((uintptr_t)dev_slab & 15) == 0, "slab must be 16-byte aligned");
    if (!slab_supported(type)) {
        set_error(std::string("ib_limb_slab: unsupported type ") + type_name(type));
        return IB_ERR_UNSUPPORTED;
    }
    IB_REQUIRE(cols % block_elems(type) == 0, "cols must be a multiple of the block size");
    return xq_slab_launch(dev_x, nullptr, (int)cols, slab_kquant(type), (uint8_t*)dev_slab,
                          nullptr, as_stream(stream), false);
}

static int gemv_q_slab(int type, const void* dev_W, const void* dev_slab, float* dev_y,
                       int64_t rows, int64_t cols, void* stream, bool chained) {
    if (rows == 0) return IB_OK;
    IB_REQUIRE(dev_W && dev_slab && dev_y && rows > 0 && cols > 0, "bad arguments");
    IB_REQUIRE(cols <= (1 << 30) && rows < (1ll << 31), "bad GEMV shape");
    FusedGemv f = {};
    f.W[0] = (const uint8_t*)dev_W;
    f.type[0] = type;
    f.rows[0] = (int)rows;
    f.n_seg = 1;
    f.K = (int)cols;
    f.y = dev_y;
    f.slab = (const uint8_t*)dev_slab;
    if (!fused_gemv_supported(f, EPI_STORE)) {
        set_error("ib_gemv_q_slab: type, shape or alignment (16 bytes for W and the slab) "
                  "not supported");
        return IB_ERR_UNSUPPORTED;
    }
    return fused_gemv_launch(f, PRO_PLAIN, EPI_STORE, as_stream(stream), chained);
}

extern "C" int ib_gemv_q_slab(int type, const void* dev_W, const void* dev_slab, float* dev_y,
                              int64_t rows, int64_t cols, void* stream) {
    return gemv_q_slab(type, dev_W, dev_slab, dev_y, rows, cols, stream, false);
}

extern "C" int ib_gemv_q_slab_chained(int type, const void* dev_W, const void* dev_slab,
                                      float* dev_y, int64_t rows, int64_t cols, void* stream) {
    return gemv_q_slab(type, dev_W, dev_slab, dev_y, rows, cols, stream, true);
}

extern "C" int ib_gemv(const float* W, const float* x, float* y, int M, int N, void* stream) {
    if (M == 0) return IB_OK;
    IB_REQUIRE(W && x && y && M > 0 && N > 0, "bad gemv arguments");
    gemv_f32_kernel<<<(unsigned)((M + 7) / 8), 256, 0, as_stream(stream)>>>(W, x, y, M, N);
    IB_LAUNCH_CHECK("gemv_kernel");
    return IB_OK;
}

extern "C" int ib_gemv_i16(const int16_t* W, const float* row_scale, const float* x, float* y,
                           int M, int N, void* stream) {
    if (M == 0) return IB_OK;
    IB_REQUIRE(W && row_scale && x && y && M > 0 && N > 0, "bad gemv_i16 arguments");
    gemv_i16_kernel<<<(unsigned)((M + 7) / 8), 256, 0, as_stream(stream)>>>(W, row_scale, x, y,
                                                                          M, N);
    IB_LAUNCH_CHECK("gemv_i16_kernel");
    return IB_OK;
}
