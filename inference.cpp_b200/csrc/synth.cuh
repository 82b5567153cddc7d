// Seeded synthetic weights in GGUF block formats, identical on host and device.
//
// Values: w_i = std * z_i, where z_i is an Irwin-Hall sum of 12 uniforms minus 6
// (mean 0, variance 1) drawn from a counter-based splitmix64 stream keyed by
// (seed, i).  Only integer arithmetic, one int->float conversion and exactly
// rounded IEEE float operations are used, so the host build (compiled with
// -ffp-contract=off) and the device build (explicit __f*_rn intrinsics) produce
// the same bytes.  This is the data source for the configurations' "N(0, std)
// then quantised" weights; it is not part of any timed path.
//
// Encoders: Q4_0 and Q8_0 follow the reference quantiser (amax/7 or amax/127,
// truncating fp16 scale, round-half-away of x * (1/d):
// src/gguf/quantization.cpp:270-352).  Q5_0, Q5_1, Q4_K and Q6_K have no encoder
// in the reference; the ones below are this project's own simple min/max
// encoders, and produce any valid block of the layouts decoded at
// src/gguf/quantization.cpp:83-245.  Q4_1, Q2_K, Q3_K and Q5_K (sized by the
// reference, not decoded by it) get encoders of the same kind for the published GGUF
// layouts.
#pragma once
#include <stdint.h>
#include <math.h>

#ifdef __CUDACC__
#define SY_HD __host__ __device__ __forceinline__
#else
#define SY_HD inline
#endif

namespace ib_synth {

SY_HD float fmul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
SY_HD float fadd(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}
SY_HD float fsub(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}
SY_HD float fdiv(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fdiv_rn(a, b);
#else
    return a / b;
#endif
}
SY_HD float fbits(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    union { uint32_t u; float f; } c;
    c.u = u;
    return c.f;
#endif
}
SY_HD uint32_t ubits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    union { uint32_t u; float f; } c;
    c.f = f;
    return c.u;
#endif
}
SY_HD float fabs_(float a) { return fbits(ubits(a) & 0x7FFFFFFFu); }
SY_HD float fmax_(float a, float b) { return a > b ? a : b; }
SY_HD float fmin_(float a, float b) { return a < b ? a : b; }
// round half away from zero; exact for |v| < 2^23 (t and v - t are exact)
SY_HD float round_away(float v) {
    float t = truncf(v);
    float r = fsub(v, t);
    if (fabs_(r) >= 0.5f) t = fadd(t, v < 0.0f ? -1.0f : 1.0f);
    return t;
}
SY_HD int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

SY_HD uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// z ~ approx N(0,1): 12 uniforms of 24 bits; integer sum, one rounding on conversion.
SY_HD float normal(uint64_t seed, uint64_t i) {
    uint64_t key = splitmix64(seed) ^ (i * 0xD1342543DE82EF95ull);
    int64_t acc = 0;
    for (int k = 0; k < 6; ++k) {
        uint64_t r = splitmix64(key + (uint64_t)k * 0x9E3779B97F4A7C15ull);
        acc += (int64_t)(r & 0xFFFFFFull) + (int64_t)((r >> 24) & 0xFFFFFFull);
    }
    acc -= 6ll * (1ll << 24);
    return fmul((float)acc, 5.9604644775390625e-08f);  // * 2^-24, exact
}

SY_HD float value(uint64_t seed, uint64_t i, float stdv) { return fmul(normal(seed, i), stdv); }

// fp16 bits -> float (exact, subnormals included)
SY_HD float h2f(uint16_t h) {
    uint32_t e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    float v;
    if (e == 0) v = fmul((float)mant, 5.9604644775390625e-08f);
    else if (e == 31) v = fbits(0x7F800000u | (mant << 13));
    else v = fbits(((e + 112u) << 23) | (mant << 13));
    return (h & 0x8000u) ? -v : v;
}

// float -> fp16, truncating (the reference's fp32_to_fp16, quantization.cpp:270-283)
SY_HD uint16_t f2h_trunc(float f) {
    uint32_t x = ubits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    uint32_t mant = x & 0x7FFFFFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant = (mant | 0x800000u) >> (1 - e);
        return (uint16_t)(sign | (mant >> 13));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | (mant >> 13));
}

// float -> fp16, round to nearest even (non-negative finite inputs are all we need,
// but the sign is kept).  Subnormal results are produced for tiny scales.
SY_HD uint16_t f2h_rne(float f) {
    uint32_t x = ubits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    if (ax < 0x33000001u) return (uint16_t)sign;               // < 2^-25 (+) -> 0
    uint32_t e = ax >> 23, mant = (ax & 0x7FFFFFu) | 0x800000u;
    int shift;
    uint32_t base;
    if (e < 113) {  // subnormal half
        shift = (int)(126 - e);  // 14 + (113 - e) ... mant >> shift gives half mantissa
        base = 0;
    } else {
        shift = 13;
        base = (e - 112) << 10;
        mant &= 0x7FFFFFu;
    }
    uint32_t q = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q += 1;
    return (uint16_t)(sign | (base + q));
}

// ---- encoders: one block from `x` (32 or 256 floats) into `out` --------------------

// Q4_0 (18 B): reference quantize_q4_0 for a full block.
SY_HD void enc_q4_0(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmax_(amax, fabs_(x[j]));
    const float d = fdiv(amax, 7.0f);
    const float inv = (d != 0.0f) ? fdiv(1.0f, d) : 0.0f;
    uint16_t db = f2h_trunc(d);
    out[0] = (uint8_t)(db & 0xFF);
    out[1] = (uint8_t)(db >> 8);
    for (int j = 0; j < 16; ++j) {
        int lo = clampi((int)round_away(fmul(x[j], inv)), -8, 7);
        int hi = clampi((int)round_away(fmul(x[j + 16], inv)), -8, 7);
        out[2 + j] = (uint8_t)(((lo + 8) & 0x0F) | (((hi + 8) & 0x0F) << 4));
    }
}

// Q8_0 (34 B): reference quantize_q8_0 for a full block.
SY_HD void enc_q8_0(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmax_(amax, fabs_(x[j]));
    const float d = fdiv(amax, 127.0f);
    const float inv = (d != 0.0f) ? fdiv(1.0f, d) : 0.0f;
    uint16_t db = f2h_trunc(d);
    out[0] = (uint8_t)(db & 0xFF);
    out[1] = (uint8_t)(db >> 8);
    for (int j = 0; j < 32; ++j) {
        int q = clampi((int)round_away(fmul(x[j], inv)), -128, 127);
        out[2 + j] = (uint8_t)(int8_t)q;
    }
}

// Q5_0 (22 B): d = amax/15, q = round(x/d) + 16 in [0,31].
SY_HD void enc_q5_0(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmax_(amax, fabs_(x[j]));
    uint16_t dh = f2h_rne(fdiv(amax, 15.0f));
    float df = h2f(dh);
    out[0] = (uint8_t)(dh & 0xFF);
    out[1] = (uint8_t)(dh >> 8);
    uint32_t qh = 0;
    int q[32];
    for (int j = 0; j < 32; ++j) {
        int v = df > 0.0f ? (int)round_away(fdiv(x[j], df)) : 0;
        q[j] = clampi(v + 16, 0, 31);
        qh |= (uint32_t)((q[j] >> 4) & 1) << j;
    }
    for (int b = 0; b < 4; ++b) out[2 + b] = (uint8_t)(qh >> (8 * b));
    for (int j = 0; j < 16; ++j) out[6 + j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
}

// Q5_1 (24 B): d = (max-min)/31, m = min, q = round((x-m)/d) in [0,31].
SY_HD void enc_q5_1(const float* x, uint8_t* out) {
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; ++j) { mn = fmin_(mn, x[j]); mx = fmax_(mx, x[j]); }
    uint16_t dh = f2h_rne(fdiv(fsub(mx, mn), 31.0f));
    uint16_t mh = f2h_rne(mn);
    float df = h2f(dh), mf = h2f(mh);
    out[0] = (uint8_t)(dh & 0xFF);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xFF);
    out[3] = (uint8_t)(mh >> 8);
    uint32_t qh = 0;
    int q[32];
    for (int j = 0; j < 32; ++j) {
        int v = df > 0.0f ? (int)round_away(fdiv(fsub(x[j], mf), df)) : 0;
        q[j] = clampi(v, 0, 31);
        qh |= (uint32_t)((q[j] >> 4) & 1) << j;
    }
    for (int b = 0; b < 4; ++b) out[4 + b] = (uint8_t)(qh >> (8 * b));
    for (int j = 0; j < 16; ++j) out[8 + j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
}

// Q4_K (144 B): 8 sub-blocks of 32 with 6-bit scale and min.
SY_HD void enc_q4_k(const float* x, uint8_t* out) {
    float scale[8], minv[8];
    float msc = 0.0f, mmn = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = 0.0f, mx = x[32 * j];
        for (int l = 0; l < 32; ++l) { mn = fmin_(mn, x[32 * j + l]); mx = fmax_(mx, x[32 * j + l]); }
        scale[j] = fdiv(fsub(mx, mn), 15.0f);
        minv[j] = -mn;
        msc = fmax_(msc, scale[j]);
        mmn = fmax_(mmn, minv[j]);
    }
    uint16_t dh = f2h_rne(fdiv(msc, 63.0f)), mh = f2h_rne(fdiv(mmn, 63.0f));
    float df = h2f(dh), mf = h2f(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = df > 0.0f ? clampi((int)round_away(fdiv(scale[j], df)), 0, 63) : 0;
        m[j] = mf > 0.0f ? clampi((int)round_away(fdiv(minv[j], mf)), 0, 63) : 0;
    }
    out[0] = (uint8_t)(dh & 0xFF);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xFF);
    out[3] = (uint8_t)(mh >> 8);
    uint8_t* s = out + 4;
    for (int k = 0; k < 4; ++k) {
        s[k] = (uint8_t)((sc[k] & 63) | ((sc[k + 4] >> 4) << 6));
        s[k + 4] = (uint8_t)((m[k] & 63) | ((m[k + 4] >> 4) << 6));
        s[k + 8] = (uint8_t)((sc[k + 4] & 0xF) | ((m[k + 4] & 0xF) << 4));
    }
    uint8_t* qs = out + 16;
    for (int p = 0; p < 4; ++p) {
        int q[64];
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * p + h;
            const float a = fmul(mf, (float)m[j]);
            const float b = fmul(df, (float)sc[j]);
            for (int l = 0; l < 32; ++l) {
                int v = b > 0.0f ? (int)round_away(fdiv(fadd(x[32 * j + l], a), b)) : 0;
                q[32 * h + l] = clampi(v, 0, 15);
            }
        }
        for (int l = 0; l < 32; ++l) qs[32 * p + l] = (uint8_t)(q[l] | (q[32 + l] << 4));
    }
}

// Q6_K (210 B): 16 sub-blocks of 16 with int8 scales, q in [-32,31].
SY_HD void enc_q6_k(const float* x, uint8_t* out) {
    float scale[16], msc = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int l = 0; l < 16; ++l) amax = fmax_(amax, fabs_(x[16 * j + l]));
        scale[j] = fdiv(amax, 31.0f);
        msc = fmax_(msc, scale[j]);
    }
    uint16_t dh = f2h_rne(fdiv(msc, 127.0f));
    float df = h2f(dh);
    int sc[16];
    for (int j = 0; j < 16; ++j)
        sc[j] = df > 0.0f ? clampi((int)round_away(fdiv(scale[j], df)), 0, 127) : 0;
    uint8_t* ql = out;
    uint8_t* qh = out + 128;
    int8_t* s8 = (int8_t*)(out + 192);
    for (int i = 0; i < 64; ++i) qh[i] = 0;
    for (int j = 0; j < 16; ++j) s8[j] = (int8_t)sc[j];
    out[208] = (uint8_t)(dh & 0xFF);
    out[209] = (uint8_t)(dh >> 8);
    for (int e = 0; e < 256; ++e) {
        const float b = fmul(df, (float)sc[e / 16]);
        int v = b > 0.0f ? (int)round_away(fdiv(x[e], b)) : 0;
        int u = clampi(v, -32, 31) + 32;
        const int c = e / 128, r = e % 128, g = r / 32, l = r % 32;
        uint8_t* qlp = ql + 64 * c + l + 32 * (g & 1);
        if (g < 2) *qlp = (uint8_t)((*qlp & 0xF0) | (u & 0xF));
        else *qlp = (uint8_t)((*qlp & 0x0F) | ((u & 0xF) << 4));
        qh[32 * c + l] |= (uint8_t)(((u >> 4) & 3) << (2 * g));
    }
}

// Q4_1 (20 B): d = (max-min)/15, m = min, q = round((x-m)/d) in [0,15].
SY_HD void enc_q4_1(const float* x, uint8_t* out) {
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; ++j) { mn = fmin_(mn, x[j]); mx = fmax_(mx, x[j]); }
    uint16_t dh = f2h_rne(fdiv(fsub(mx, mn), 15.0f));
    uint16_t mh = f2h_rne(mn);
    float df = h2f(dh), mf = h2f(mh);
    out[0] = (uint8_t)(dh & 0xFF);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xFF);
    out[3] = (uint8_t)(mh >> 8);
    int q[32];
    for (int j = 0; j < 32; ++j) {
        int v = df > 0.0f ? (int)round_away(fdiv(fsub(x[j], mf), df)) : 0;
        q[j] = clampi(v, 0, 15);
    }
    for (int j = 0; j < 16; ++j) out[4 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

// Q5_K (176 B): as Q4_K with 5-bit quants (sub-block scale (max-min)/31).
SY_HD void enc_q5_k(const float* x, uint8_t* out) {
    float scale[8], minv[8];
    float msc = 0.0f, mmn = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = 0.0f, mx = x[32 * j];
        for (int l = 0; l < 32; ++l) { mn = fmin_(mn, x[32 * j + l]); mx = fmax_(mx, x[32 * j + l]); }
        scale[j] = fdiv(fsub(mx, mn), 31.0f);
        minv[j] = -mn;
        msc = fmax_(msc, scale[j]);
        mmn = fmax_(mmn, minv[j]);
    }
    uint16_t dh = f2h_rne(fdiv(msc, 63.0f)), mh = f2h_rne(fdiv(mmn, 63.0f));
    float df = h2f(dh), mf = h2f(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = df > 0.0f ? clampi((int)round_away(fdiv(scale[j], df)), 0, 63) : 0;
        m[j] = mf > 0.0f ? clampi((int)round_away(fdiv(minv[j], mf)), 0, 63) : 0;
    }
    out[0] = (uint8_t)(dh & 0xFF);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xFF);
    out[3] = (uint8_t)(mh >> 8);
    uint8_t* s = out + 4;
    for (int k = 0; k < 4; ++k) {
        s[k] = (uint8_t)((sc[k] & 63) | ((sc[k + 4] >> 4) << 6));
        s[k + 4] = (uint8_t)((m[k] & 63) | ((m[k + 4] >> 4) << 6));
        s[k + 8] = (uint8_t)((sc[k + 4] & 0xF) | ((m[k + 4] & 0xF) << 4));
    }
    uint8_t* qh = out + 16;
    uint8_t* qs = out + 48;
    for (int l = 0; l < 32; ++l) qh[l] = 0;
    for (int p = 0; p < 4; ++p) {
        int q[64];
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * p + h;
            const float a = fmul(mf, (float)m[j]);
            const float b = fmul(df, (float)sc[j]);
            for (int l = 0; l < 32; ++l) {
                int v = b > 0.0f ? (int)round_away(fdiv(fadd(x[32 * j + l], a), b)) : 0;
                q[32 * h + l] = clampi(v, 0, 31);
                qh[l] |= (uint8_t)(((q[32 * h + l] >> 4) & 1) << j);
            }
        }
        for (int l = 0; l < 32; ++l) qs[32 * p + l] = (uint8_t)((q[l] & 0xF) | ((q[32 + l] & 0xF) << 4));
    }
}

// Q2_K (84 B): 16 sub-blocks of 16, 4-bit scale and min, 2-bit quants.  Sub-block
// b = 8h + 2j + k holds elements 16b.. at bits 2j of qs[32h + 16k + l].
SY_HD void enc_q2_k(const float* x, uint8_t* out) {
    float scale[16], minv[16], msc = 0.0f, mmn = 0.0f;
    for (int b = 0; b < 16; ++b) {
        float mn = 0.0f, mx = x[16 * b];
        for (int l = 0; l < 16; ++l) { mn = fmin_(mn, x[16 * b + l]); mx = fmax_(mx, x[16 * b + l]); }
        scale[b] = fdiv(fsub(mx, mn), 3.0f);
        minv[b] = -mn;
        msc = fmax_(msc, scale[b]);
        mmn = fmax_(mmn, minv[b]);
    }
    uint16_t dh = f2h_rne(fdiv(msc, 15.0f)), mh = f2h_rne(fdiv(mmn, 15.0f));
    float df = h2f(dh), mf = h2f(mh);
    for (int i = 16; i < 80; ++i) out[i] = 0;
    for (int b = 0; b < 16; ++b) {
        int sc = df > 0.0f ? clampi((int)round_away(fdiv(scale[b], df)), 0, 15) : 0;
        int m = mf > 0.0f ? clampi((int)round_away(fdiv(minv[b], mf)), 0, 15) : 0;
        out[b] = (uint8_t)(sc | (m << 4));
        const float a = fmul(mf, (float)m), dd = fmul(df, (float)sc);
        const int h = b >> 3, j = (b >> 1) & 3, k = b & 1;
        for (int l = 0; l < 16; ++l) {
            int v = dd > 0.0f ? (int)round_away(fdiv(fadd(x[16 * b + l], a), dd)) : 0;
            out[16 + 32 * h + 16 * k + l] |= (uint8_t)(clampi(v, 0, 3) << (2 * j));
        }
    }
    out[80] = (uint8_t)(dh & 0xFF);
    out[81] = (uint8_t)(dh >> 8);
    out[82] = (uint8_t)(mh & 0xFF);
    out[83] = (uint8_t)(mh >> 8);
}

// Q3_K (110 B): 16 sub-blocks of 16 with 6-bit scales (stored + 32), 3-bit signed
// quants in [-4, 3]: the low 2 bits in qs, the sign-side bit in hmask (set: q >= 0).
SY_HD void enc_q3_k(const float* x, uint8_t* out) {
    float scale[16], msc = 0.0f;
    for (int b = 0; b < 16; ++b) {
        float amax = 0.0f;
        for (int l = 0; l < 16; ++l) amax = fmax_(amax, fabs_(x[16 * b + l]));
        scale[b] = fdiv(amax, 4.0f);
        msc = fmax_(msc, scale[b]);
    }
    uint16_t dh = f2h_rne(fdiv(msc, 31.0f));
    float df = h2f(dh);
    for (int i = 0; i < 108; ++i) out[i] = 0;
    uint8_t* hm = out;
    uint8_t* qs = out + 32;
    uint8_t* sc = out + 96;
    for (int b = 0; b < 16; ++b) {
        int s = df > 0.0f ? clampi((int)round_away(fdiv(scale[b], df)), 0, 31) : 0;
        const int u = s + 32;
        if (b < 8) sc[b] |= (uint8_t)(u & 0xF);
        else sc[b - 8] |= (uint8_t)((u & 0xF) << 4);
        sc[8 + (b & 3)] |= (uint8_t)((u >> 4) << (2 * (b >> 2)));
        const float dd = fmul(df, (float)s);
        const int h = b >> 3, j = (b >> 1) & 3, k = b & 1;
        for (int l = 0; l < 16; ++l) {
            int v = dd > 0.0f ? (int)round_away(fdiv(x[16 * b + l], dd)) : 0;
            v = clampi(v, -4, 3);
            const int q2 = v < 0 ? v + 4 : v;
            qs[32 * h + 16 * k + l] |= (uint8_t)(q2 << (2 * j));
            if (v >= 0) hm[16 * k + l] |= (uint8_t)(1 << (4 * h + j));
        }
    }
    out[108] = (uint8_t)(dh & 0xFF);
    out[109] = (uint8_t)(dh >> 8);
}

SY_HD int block_elems(int type) {
    return (type == 10 || type == 11 || type == 12 || type == 13 || type == 14) ? 256 : 32;
}
SY_HD int block_bytes(int type) {
    switch (type) {
        case 2: return 18;
        case 3: return 20;
        case 10: return 84;
        case 11: return 110;
        case 13: return 176;
        case 6: return 22;
        case 7: return 24;
        case 8: return 34;
        case 12: return 144;
        case 14: return 210;
        default: return 0;
    }
}

// Encode block `b` of a row-major [rows, cols] tensor whose element (r, c) has
// counter r*cols + c.  Returns false for an unsupported type.
SY_HD bool encode_block(int type, uint64_t seed, float stdv, int64_t cols, int64_t b,
                        uint8_t* out) {
    const int be = block_elems(type);
    const int64_t bpr = cols / be;
    const int64_t r = b / bpr, c0 = (b % bpr) * be;
    float x[256];
    for (int i = 0; i < be; ++i) x[i] = value(seed, (uint64_t)(r * cols + c0 + i), stdv);
    switch (type) {
        case 2: enc_q4_0(x, out); return true;
        case 3: enc_q4_1(x, out); return true;
        case 10: enc_q2_k(x, out); return true;
        case 11: enc_q3_k(x, out); return true;
        case 13: enc_q5_k(x, out); return true;
        case 6: enc_q5_0(x, out); return true;
        case 7: enc_q5_1(x, out); return true;
        case 8: enc_q8_0(x, out); return true;
        case 12: enc_q4_k(x, out); return true;
        case 14: enc_q6_k(x, out); return true;
        default: return false;
    }
}

}  // namespace ib_synth
