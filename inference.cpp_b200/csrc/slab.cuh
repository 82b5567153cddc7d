// Device side of the limb slab (layout in decode.cuh): one warp writes the limbs,
// the limb scale and the sub-sums of one scale group of GS elements.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib {

// Slab geometry per weight family (must match slab_geom in decode.cuh).
template <bool KQ>
struct SlabG {
    static constexpr int SE = KQ ? 2048 : 1024;  // elements per slice
    static constexpr int GS = KQ ? 256 : 32;     // elements per limb scale
    static constexpr int SLICE = ((SE * 4 + (SE / GS + SE / 32 + SE / 16) * 4) + 15) / 16 * 16;
};

__device__ __forceinline__ float exp2i(int e) {  // 2^e for e in [-126, 127]
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

// Smallest e >= -126 with m <= 127 * 2^e, from the exponent bits (m >= 0).
__device__ __forceinline__ int limb_exp_bits(float m) {
    if (!(m > 0.f)) return 0;
    int e = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 133;  // floor(log2 m) - 6
    if (e < -126) e = -126;
    if (m > 127.0f * exp2i(e)) ++e;
    return e;
}

// Element of scale group gi that a lane holds as its j-th value: K-quant groups (256
// elements) give each lane 8 consecutive elements, 32-element groups one per lane.
template <bool KQ>
__device__ __forceinline__ int slab_elem(int gi, int j, int lane) {
    return KQ ? gi * 256 + 8 * lane + j : gi * 32 + 32 * j + lane;
}

// v[j] <- src[slab_elem<KQ>(gi, j, lane) - off] (float4 loads when aligned; CG: through
// L2 only, for data another CTA of the same launch wrote).
template <bool KQ, bool CG = false>
__device__ __forceinline__ void slab_load(const float* src, int gi, int lane,
                                          float (&v)[SlabG<KQ>::GS / 32]) {
    constexpr int PER = SlabG<KQ>::GS / 32;
    if constexpr (KQ) {
        const float* p = src + slab_elem<KQ>(gi, 0, lane);
        if (((uintptr_t)p & 15) == 0) {
            const float4* p4 = reinterpret_cast<const float4*>(p);
            const float4 a = CG ? __ldcg(p4) : p4[0], b = CG ? __ldcg(p4 + 1) : p4[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            return;
        }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const float* q = src + slab_elem<KQ>(gi, j, lane);
        v[j] = CG ? __ldcg(q) : *q;
    }
}

// Scale group gi, lane holding v[j] = element slab_elem<KQ>(gi, j, lane): writes the
// four exact int8 limbs of every element, the power-of-two scale and the 32/16-element
// sums.  With e the group's limb exponent, the limbs are the balanced base-128 digits
// (L0, L1, L2, L3), L1..L3 in [-64, 63], of X = round-to-nearest-even(v * 2^(21 - e)),
// |X| <= 127 * 2^21 (so |L0| <= 127): v = 2^(e-21) X + r, |r| <= 2^(e-22).
template <bool KQ>
__device__ __forceinline__ void slab_write_group(const float (&v)[SlabG<KQ>::GS / 32], int gi,
                                                 uint8_t* slab, int lane) {
    using G = SlabG<KQ>;
    constexpr int PER = G::GS / 32;
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int e = limb_exp_bits(m);
    const float inv_s = exp2i(-e);
    const int slice = (gi * G::GS) / G::SE, gl = (gi * G::GS - slice * G::SE) / G::GS;
    uint8_t* base = slab + (size_t)slice * G::SLICE;
    int8_t* limbs = reinterpret_cast<int8_t*>(base);
    float* scale = reinterpret_cast<float*>(base + G::SE * 4);
    float* sum32 = scale + G::SE / G::GS;
    float* sum16 = sum32 + G::SE / 32;
    // digits of X: the three low ones biased by 64 become 7-bit fields of X + B
    constexpr int B = 64 * (1 + 128 + 16384);
    uint32_t dg[4][PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int X = __float2int_rn((v[j] * inv_s) * 2097152.0f);  // both products exact
        const int u = X + B;
        dg[0][j] = (uint32_t)(u >> 21);
        dg[1][j] = (((uint32_t)u >> 14) & 127u) - 64u;
        dg[2][j] = (((uint32_t)u >> 7) & 127u) - 64u;
        dg[3][j] = ((uint32_t)u & 127u) - 64u;
    }
    if constexpr (KQ) {
        // lane: elements 8 * (lane & 3) .. + 7 of 32-group sg; limb i's 8 bytes in one store
        const int sg = gl * PER + (lane >> 2);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint2 w;
            w.x = __byte_perm(__byte_perm(dg[i][0], dg[i][1], 0x0040),
                              __byte_perm(dg[i][2], dg[i][3], 0x0040), 0x5410);
            w.y = __byte_perm(__byte_perm(dg[i][4], dg[i][5], 0x0040),
                              __byte_perm(dg[i][6], dg[i][7], 0x0040), 0x5410);
            *reinterpret_cast<uint2*>(limbs + (size_t)sg * 128 + i * 32 + 8 * (lane & 3)) = w;
        }
        float sm = v[0];
#pragma unroll
        for (int j = 1; j < PER; ++j) sm += v[j];
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);  // 16 elements
        if ((lane & 1) == 0) sum16[sg * 2 + ((lane >> 1) & 1)] = sm;
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);  // 32 elements
        if ((lane & 3) == 0) sum32[sg] = sm;
    } else {
        const int sg = gl;  // one 32-group; lane = element
#pragma unroll
        for (int i = 0; i < 4; ++i) limbs[(size_t)sg * 128 + i * 32 + lane] = (int8_t)dg[i][0];
        float sm = v[0];
#pragma unroll
        for (int o2 = 8; o2 > 0; o2 >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o2);
        if ((lane & 15) == 0) sum16[sg * 2 + (lane >> 4)] = sm;
        sm += __shfl_xor_sync(0xffffffffu, sm, 16);
        if (lane == 0) sum32[sg] = sm;
    }
    if (lane == 0) scale[gl] = exp2i(e);
}

}  // namespace ib
