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

// Scale group gi: lane holds v[j] = element (gi * GS + 32 j + lane).  Writes the four
// exact int8 limbs of every element, the power-of-two scale and the 32/16-element sums.
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
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int sg = gl * PER + j;  // 32-group within the slice
        float tt = v[j] * inv_s;      // exact: |tt| <= 127
        int8_t* o = limbs + (size_t)sg * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float r = rintf(tt);
            o[i * 32 + lane] = (int8_t)(int)r;
            tt = (tt - r) * 128.0f;
        }
        float sm = v[j];
#pragma unroll
        for (int o2 = 8; o2 > 0; o2 >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o2);
        if ((lane & 15) == 0) sum16[sg * 2 + (lane >> 4)] = sm;
        sm += __shfl_xor_sync(0xffffffffu, sm, 16);
        if (lane == 0) sum32[sg] = sm;
    }
    if (lane == 0) scale[gl] = exp2i(e);
}

}  // namespace ib
