/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the quantized-weight path.
 *
 * A plain-C restatement of the reference's CPU algorithms (0xiamsanj/inference.cpp),
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg to check
 * and time results.  Nothing in the product links or calls this file.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the
 * reference compiled from its own sources (oracle/_ref, built by oracle/Makefile)
 * and against the committed golden fixtures in tests/golden/.
 *
 * Rounding notes.  The reference is built with -O3 -mavx2 -mfma.  g++ vectorises
 * the contiguous dot products (matvec, sum of squares, q.k) as 8-wide multiplies
 * followed by in-order scalar adds, i.e. every product is rounded before it is
 * added; only scalar remainder iterations (n % 4 != 0, or n < 8) and loops it
 * cannot vectorise (the strided p.V sum) are contracted to fused multiply-adds.
 * dot() below reproduces that order.  In dequantisation every product (fp16
 * scale x 6-bit sub-scale x <=6-bit quant) is exact in FP32, so contraction
 * cannot change those results.  This file is compiled with -ffp-contract=off.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* GGUF type codes (include/core/tensor.hpp:16-37) */
enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
       T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_I16 = 17 };

/* Elements per block: include/core/tensor.hpp:246-262 */
int orc_block_size(int t) {
    switch (t) {
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return 32;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
        default: return 1;
    }
}

/* Bytes per block: include/core/tensor.hpp:204-223 */
int orc_block_bytes(int t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: return 2;
        case T_Q4_0: return 18;
        case T_Q4_1: return 20;
        case T_Q2_K: return 84;
        case T_Q3_K: return 110;
        case T_Q5_K: return 176;
        case T_Q5_0: return 22;
        case T_Q5_1: return 24;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

/* fp16 -> fp32 incl. subnormals: src/gguf/quantization.cpp:9-27 */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    if (e == 0) {
        float v = ldexpf((float)mant, -24);
        return (h & 0x8000u) ? -v : v;
    }
    uint32_t f = (e == 31) ? (sign | 0x7F800000u | (mant << 13))
                           : (sign | ((e + 112u) << 23) | (mant << 13));
    float out;
    memcpy(&out, &f, 4);
    return out;
}

static uint16_t rd16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }
static uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }

/* Q4_0: src/gguf/quantization.cpp:33-54 */
static void dq_q4_0(const uint8_t* b, float* y, int64_t n) {
    for (int64_t i = 0; i < (n + 31) / 32; ++i) {
        const uint8_t* blk = b + i * 18;
        float d = orc_fp16_to_fp32(rd16(blk));
        int64_t rem = n - i * 32;
        for (int j = 0; j < 16; ++j) {
            int x0 = (blk[2 + j] & 0x0F) - 8, x1 = (blk[2 + j] >> 4) - 8;
            if (j < rem) y[i * 32 + j] = x0 * d;
            if (j + 16 < rem) y[i * 32 + j + 16] = x1 * d;
        }
    }
}

/* Q8_0: src/gguf/quantization.cpp:59-77 */
static void dq_q8_0(const uint8_t* b, float* y, int64_t n) {
    for (int64_t i = 0; i < (n + 31) / 32; ++i) {
        const uint8_t* blk = b + i * 34;
        float d = orc_fp16_to_fp32(rd16(blk));
        int64_t rem = n - i * 32;
        for (int j = 0; j < 32 && j < rem; ++j) y[i * 32 + j] = (int8_t)blk[2 + j] * d;
    }
}

/* Q5_0: src/gguf/quantization.cpp:83-106 */
static void dq_q5_0(const uint8_t* b, float* y, int64_t n) {
    for (int64_t i = 0; i < (n + 31) / 32; ++i) {
        const uint8_t* blk = b + i * 22;
        float d = orc_fp16_to_fp32(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        const uint8_t* qs = blk + 6;
        int64_t rem = n - i * 32;
        for (int j = 0; j < 16; ++j) {
            int x0 = (qs[j] & 0x0F) | (((qh >> j) & 1) << 4);
            int x1 = (qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
            if (j < rem) y[i * 32 + j] = (x0 - 16) * d;
            if (j + 16 < rem) y[i * 32 + j + 16] = (x1 - 16) * d;
        }
    }
}

/* Q5_1: src/gguf/quantization.cpp:112-137 (x*d + m; the product is exact) */
static void dq_q5_1(const uint8_t* b, float* y, int64_t n) {
    for (int64_t i = 0; i < (n + 31) / 32; ++i) {
        const uint8_t* blk = b + i * 24;
        float d = orc_fp16_to_fp32(rd16(blk)), m = orc_fp16_to_fp32(rd16(blk + 2));
        uint32_t qh = rd32(blk + 4);
        const uint8_t* qs = blk + 8;
        int64_t rem = n - i * 32;
        for (int j = 0; j < 16; ++j) {
            int x0 = (qs[j] & 0x0F) | (((qh >> j) & 1) << 4);
            int x1 = (qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
            if (j < rem) y[i * 32 + j] = x0 * d + m;
            if (j + 16 < rem) y[i * 32 + j + 16] = x1 * d + m;
        }
    }
}

/* get_scale_min_k4: src/gguf/quantization.cpp:151-159 */
static void scale_min_k4(int j, const uint8_t* q, int* d, int* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Q4_K: src/gguf/quantization.cpp:161-198 */
static void dq_q4_k(const uint8_t* b, float* y, int64_t n) {
    for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = b + sb * 144;
        float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* q = blk + 16;
        float* o = y + sb * 256;
        for (int p = 0; p < 4; ++p) {
            int s0, m0, s1, m1;
            scale_min_k4(2 * p, sc, &s0, &m0);
            scale_min_k4(2 * p + 1, sc, &s1, &m1);
            float d1 = d * s0, mm1 = dmin * m0, d2 = d * s1, mm2 = dmin * m1;
            for (int l = 0; l < 32; ++l) *o++ = d1 * (q[l] & 0x0F) - mm1;
            for (int l = 0; l < 32; ++l) *o++ = d2 * (q[l] >> 4) - mm2;
            q += 32;
        }
    }
}

/* Q6_K: src/gguf/quantization.cpp:211-245 ((d*sc)*q left to right) */
static void dq_q6_k(const uint8_t* b, float* y, int64_t n) {
    for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = b + sb * 210;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        float d = orc_fp16_to_fp32(rd16(blk + 208));
        float* o = y + sb * 256;
        for (int c = 0; c < 2; ++c) {
            for (int l = 0; l < 32; ++l) {
                int is = l / 16;
                int q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                o[l] = d * sc[is] * q1;
                o[l + 32] = d * sc[is + 2] * q2;
                o[l + 64] = d * sc[is + 4] * q3;
                o[l + 96] = d * sc[is + 6] * q4;
            }
            o += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* ---- formats the reference sizes (include/core/tensor.hpp:204-223) but does not
 * decode (src/gguf/quantization.cpp:201-204 throw): restated from the published GGUF
 * block layouts (the `gguf` Python package, 0.19.0, decodes them the same way; the CPU
 * tests pin these functions to it).  Every value is one exact product (fp16 scale x
 * small integers) plus at most one rounding, so evaluation order cannot change it. */

/* Q4_1 (20 B): d, m (fp16), qs[16]; element j = qs[j] low nibble, j + 16 high nibble;
 * y = d * q + m */
static void dq_q4_1(const uint8_t* b, float* y, int64_t n) {
    for (int64_t i = 0; i < n / 32; ++i) {
        const uint8_t* blk = b + i * 20;
        float d = orc_fp16_to_fp32(rd16(blk)), m = orc_fp16_to_fp32(rd16(blk + 2));
        for (int j = 0; j < 16; ++j) {
            y[i * 32 + j] = (float)(blk[4 + j] & 0x0F) * d + m;
            y[i * 32 + j + 16] = (float)(blk[4 + j] >> 4) * d + m;
        }
    }
}

/* Q5_K (176 B): d, dmin (fp16), scales[12] (6-bit scale/min pairs as Q4_K), qh[32],
 * qs[128].  Chunk p of 64: sub-blocks 2p (low nibbles of qs[32p..], high bit qh bit 2p)
 * and 2p + 1 (high nibbles, qh bit 2p + 1); y = (d*sc) * q5 - dmin*m */
static void dq_q5_k(const uint8_t* b, float* y, int64_t n) {
    for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = b + sb * 176;
        float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* q = blk + 48;
        float* o = y + sb * 256;
        for (int p = 0; p < 4; ++p) {
            int s0, m0, s1, m1;
            scale_min_k4(2 * p, sc, &s0, &m0);
            scale_min_k4(2 * p + 1, sc, &s1, &m1);
            float d1 = d * s0, mm1 = dmin * m0, d2 = d * s1, mm2 = dmin * m1;
            for (int l = 0; l < 32; ++l)
                *o++ = d1 * ((q[l] & 0x0F) + (((qh[l] >> (2 * p)) & 1) << 4)) - mm1;
            for (int l = 0; l < 32; ++l)
                *o++ = d2 * ((q[l] >> 4) + (((qh[l] >> (2 * p + 1)) & 1) << 4)) - mm2;
            q += 32;
        }
    }
}

/* Q2_K (84 B): scales[16] (low nibble scale, high nibble min), qs[64], d, dmin (fp16).
 * Element e = 128h + 32j + 16k + l: 2-bit q = qs[32h + 16k + l] >> 2j, sub-block
 * 8h + 2j + k; y = (d*sc) * q - dmin*m */
static void dq_q2_k(const uint8_t* b, float* y, int64_t n) {
    for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = b + sb * 84;
        float d = orc_fp16_to_fp32(rd16(blk + 80)), dmin = orc_fp16_to_fp32(rd16(blk + 82));
        float* o = y + sb * 256;
        for (int e = 0; e < 256; ++e) {
            int h = e >> 7, j = (e >> 5) & 3, k = (e >> 4) & 1, l = e & 15;
            int scm = blk[8 * h + 2 * j + k];
            int q = (blk[16 + 32 * h + 16 * k + l] >> (2 * j)) & 3;
            float dl = d * (scm & 0xF), ml = dmin * (scm >> 4);
            o[e] = dl * q - ml;
        }
    }
}

/* Q3_K (110 B): hmask[32], qs[64], scales[12] (16 signed 6-bit scales: low nibbles in
 * bytes 0-7, scale i >= 8 in the high nibble of byte i - 8, the top 2 bits of scale i
 * in byte 8 + i%4 at bit 2(i/4); value - 32), d (fp16).  Element e = 128h + 32j + 16k +
 * l: q = (qs[32h + 16k + l] >> 2j & 3) - (hmask[16k + l] bit 4h + j ? 0 : 4), sub-block
 * 8h + 2j + k; y = (d*s) * q */
static int q3k_scale(const uint8_t* sc, int i) {
    int lo = i < 8 ? (sc[i] & 0xF) : (sc[i - 8] >> 4);
    int hi = (sc[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

static void dq_q3_k(const uint8_t* b, float* y, int64_t n) {
    for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = b + sb * 110;
        const uint8_t* hm = blk;
        const uint8_t* qs = blk + 32;
        const uint8_t* sc = blk + 96;
        float d = orc_fp16_to_fp32(rd16(blk + 108));
        float* o = y + sb * 256;
        for (int e = 0; e < 256; ++e) {
            int h = e >> 7, j = (e >> 5) & 3, k = (e >> 4) & 1, l = e & 15;
            int q = ((qs[32 * h + 16 * k + l] >> (2 * j)) & 3) -
                    (((hm[16 * k + l] >> (4 * h + j)) & 1) ? 0 : 4);
            float dl = d * q3k_scale(sc, 8 * h + 2 * j + k);
            o[e] = dl * q;
        }
    }
}

/* dequantize dispatch: src/gguf/quantization.cpp:250-267 (+ F32/F16 from
 * src/models/transformer.cpp:176-199).  Returns 0, or -1 for an unsupported type. */
int orc_dequantize(int t, const void* src, float* dst, int64_t n) {
    const uint8_t* b = (const uint8_t*)src;
    switch (t) {
        case T_F32: memcpy(dst, src, (size_t)n * 4); return 0;
        case T_F16:
            for (int64_t i = 0; i < n; ++i) dst[i] = orc_fp16_to_fp32(rd16(b + 2 * i));
            return 0;
        case T_Q4_0: dq_q4_0(b, dst, n); return 0;
        case T_Q5_0: dq_q5_0(b, dst, n); return 0;
        case T_Q5_1: dq_q5_1(b, dst, n); return 0;
        case T_Q8_0: dq_q8_0(b, dst, n); return 0;
        case T_Q4_K: dq_q4_k(b, dst, n); return 0;
        case T_Q4_1: dq_q4_1(b, dst, n); return 0;
        case T_Q5_K: dq_q5_k(b, dst, n); return 0;
        case T_Q2_K: dq_q2_k(b, dst, n); return 0;
        case T_Q3_K: dq_q3_k(b, dst, n); return 0;
        case T_Q6_K: dq_q6_k(b, dst, n); return 0;
        default: return -1;
    }
}

/* fp32_to_fp16 (truncating): src/gguf/quantization.cpp:270-283 */
static uint16_t f32_to_f16_trunc(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
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

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* quantize_q4_0 / quantize_q8_0: src/gguf/quantization.cpp:285-352 */
int orc_quantize(int t, const float* src, void* dst, int64_t n) {
    uint8_t* base = (uint8_t*)dst;
    if (t != T_Q4_0 && t != T_Q8_0) return -1;
    const int q8 = (t == T_Q8_0);
    const int bb = q8 ? 34 : 18;
    for (int64_t i = 0; i < (n + 31) / 32; ++i) {
        uint8_t* blk = base + i * bb;
        float amax = 0;
        for (int j = 0; j < 32; ++j) {
            int64_t idx = i * 32 + j;
            if (idx < n) amax = fmaxf(amax, fabsf(src[idx]));
        }
        const float d = amax / (q8 ? 127.0f : 7.0f);
        const float inv = (d != 0) ? 1.0f / d : 0;
        uint16_t db = f32_to_f16_trunc(d);
        memcpy(blk, &db, 2);
        if (q8) {
            for (int j = 0; j < 32; ++j) {
                int64_t idx = i * 32 + j;
                blk[2 + j] = (uint8_t)(int8_t)(idx < n ? clampi((int)roundf(src[idx] * inv), -128, 127) : 0);
            }
        } else {
            for (int j = 0; j < 16; ++j) {
                int lo = 0, hi = 0;
                int64_t i0 = i * 32 + j, i1 = i0 + 16;
                if (i0 < n) lo = clampi((int)roundf(src[i0] * inv), -8, 7);
                if (i1 < n) hi = clampi((int)roundf(src[i1] * inv), -8, 7);
                blk[2 + j] = (uint8_t)(((lo + 8) & 0x0F) | (((hi + 8) & 0x0F) << 4));
            }
        }
    }
    return 0;
}

/* Symmetric per-row INT16 requant: make_weight, src/models/transformer.cpp:208-251
 * (identical to quantize_i16, src/models/model_cuda.cpp:62-99). */
void orc_requant_i16(const float* w, int64_t rows, int64_t cols, int16_t* q, float* scale) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* row = w + r * cols;
        float amax = 0.0f;
        for (int64_t c = 0; c < cols; ++c) {
            float a = fabsf(row[c]);
            if (a > amax) amax = a;
        }
        const float s = amax > 0.0f ? amax / 32767.0f : 1.0f;
        const float inv = 1.0f / s;
        scale[r] = s;
        for (int64_t c = 0; c < cols; ++c) {
            long v = lroundf(row[c] * inv);
            if (v > 32767) v = 32767;
            if (v < -32767) v = -32767;
            q[r * cols + c] = (int16_t)v;
        }
    }
}

/* Sequential sum of a[i]*b[i] in the reference build's rounding: products rounded
 * then added in order, except the scalar remainder (all of it when n < 8, else
 * the n % 4 tail), which is fused. */
static float dot(const float* a, const float* b, int64_t n, float s) {
    int64_t i = 0;
    if (n >= 8) {
        int64_t m = n & ~(int64_t)7;
        if (n - m >= 4) m += 4;
        for (; i < m; ++i) s += a[i] * b[i];
    }
    for (; i < n; ++i) s = fmaf(a[i], b[i], s);
    return s;
}

static float dot_i16(const int16_t* a, const float* b, int64_t n, float s) {
    int64_t i = 0;
    if (n >= 8) {
        int64_t m = n & ~(int64_t)7;
        if (n - m >= 4) m += 4;
        for (; i < m; ++i) s += (float)a[i] * b[i];
    }
    for (; i < n; ++i) s = fmaf((float)a[i], b[i], s);
    return s;
}

/* Threads of the row loops below (1 = sequential).  Rows are independent and each row's
 * sum keeps the sequential order above, so the result does not depend on the count. */
static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n > 0 ? n : 1; }

/* dot() of four rows against one x, interleaved so the four sums proceed side by side;
 * each sum sees exactly the operations dot() would apply to its row. */
static void dot4(const float* a0, const float* a1, const float* a2, const float* a3,
                 const float* b, int64_t n, float* out) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int64_t i = 0;
    if (n >= 8) {
        int64_t m = n & ~(int64_t)7;
        if (n - m >= 4) m += 4;
        for (; i < m; ++i) {
            const float x = b[i];
            s0 += a0[i] * x; s1 += a1[i] * x; s2 += a2[i] * x; s3 += a3[i] * x;
        }
    }
    for (; i < n; ++i) {
        s0 = fmaf(a0[i], b[i], s0); s1 = fmaf(a1[i], b[i], s1);
        s2 = fmaf(a2[i], b[i], s2); s3 = fmaf(a3[i], b[i], s3);
    }
    out[0] = s0; out[1] = s1; out[2] = s2; out[3] = s3;
}

/* matvec: src/models/transformer.cpp:100-119 */
void orc_matvec_f32(const float* W, const float* x, float* y, int64_t rows, int64_t cols) {
    const int64_t r4 = rows & ~(int64_t)3;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && rows >= 256)
    for (int64_t r = 0; r < r4; r += 4)
        dot4(W + r * cols, W + (r + 1) * cols, W + (r + 2) * cols, W + (r + 3) * cols, x, cols,
             y + r);
    for (int64_t r = r4; r < rows; ++r) y[r] = dot(W + r * cols, x, cols, 0.0f);
}

void orc_matvec_i16(const int16_t* q, const float* scale, const float* x, float* y,
                    int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && rows >= 256)
    for (int64_t r = 0; r < rows; ++r) y[r] = dot_i16(q + r * cols, x, cols, 0.0f) * scale[r];
}

/* ---------------------------------------------------------------------------
 * Llama forward, token by token: Model::forward / attention_forward /
 * ffn_forward / transformer_block, src/models/model.cpp:23-321, and greedy
 * Model::generate (:323-399) with temperature 0 and repetition penalty 1.
 * Weights are held as FP32 (host_int16 = false) or INT16 + row scale.
 * ------------------------------------------------------------------------- */
typedef struct {
    int64_t rows, cols;
    int int16;
    float* f;
    int16_t* q;
    float* s;
} OWeight;

typedef struct {
    int n_layers, D, H, Hkv, HD, V, FFN, max_seq;
    float theta, eps;
    OWeight tok, out_norm, out;
    int tied;
    OWeight* L; /* per layer: wq wk wv wo w1 w2 w3 attn_norm ffn_norm */
    float* kc;  /* [layers][Hkv][max_seq][HD] */
    float* vc;
} OModel;

enum { W_Q, W_K, W_V, W_O, W_1, W_2, W_3, W_AN, W_FN, W_PER_LAYER };

void* orc_model_create(int n_layers, int D, int H, int Hkv, int V, int FFN, int max_seq,
                       float theta, float eps) {
    OModel* m = (OModel*)calloc(1, sizeof(OModel));
    m->n_layers = n_layers; m->D = D; m->H = H; m->Hkv = Hkv; m->HD = D / H;
    m->V = V; m->FFN = FFN; m->max_seq = max_seq; m->theta = theta; m->eps = eps;
    m->tied = 1;
    m->L = (OWeight*)calloc((size_t)n_layers * W_PER_LAYER, sizeof(OWeight));
    size_t kv = (size_t)n_layers * Hkv * max_seq * m->HD;
    m->kc = (float*)calloc(kv, 4);
    m->vc = (float*)calloc(kv, 4);
    return m;
}

static void free_w(OWeight* w) { free(w->f); free(w->q); free(w->s); }

void orc_model_free(void* h) {
    OModel* m = (OModel*)h;
    if (!m) return;
    free_w(&m->tok); free_w(&m->out_norm); free_w(&m->out);
    for (int i = 0; i < m->n_layers * W_PER_LAYER; ++i) free_w(&m->L[i]);
    free(m->L); free(m->kc); free(m->vc); free(m);
}

/* which: 0 tok_embeddings, 1 output_norm, 2 output, 10+k layer weight k.
 * Packed GGUF bytes are dequantised to FP32 (load_tensor) and 2-D weights other than
 * norms are requantised to INT16 when int16 != 0 (make_weight). */
int orc_model_set(void* h, int which, int layer, int type, const void* data,
                  int64_t rows, int64_t cols, int int16) {
    OModel* m = (OModel*)h;
    OWeight* w;
    int quantize = 1;
    if (which == 0) w = &m->tok;
    else if (which == 1) { w = &m->out_norm; quantize = 0; }
    else if (which == 2) { w = &m->out; m->tied = 0; }
    else {
        int k = which - 10;
        if (k < 0 || k >= W_PER_LAYER || layer < 0 || layer >= m->n_layers) return -1;
        w = &m->L[layer * W_PER_LAYER + k];
        if (k == W_AN || k == W_FN) quantize = 0;
    }
    free_w(w);
    memset(w, 0, sizeof(*w));
    w->rows = rows; w->cols = cols;
    float* f = (float*)malloc((size_t)(rows * cols) * 4);
    if (orc_dequantize(type, data, f, rows * cols) != 0) { free(f); return -1; }
    if (quantize && int16) {
        w->int16 = 1;
        w->q = (int16_t*)malloc((size_t)(rows * cols) * 2);
        w->s = (float*)malloc((size_t)rows * 4);
        orc_requant_i16(f, rows, cols, w->q, w->s);
        free(f);
    } else {
        w->f = f;
    }
    return 0;
}

static void mv(const OWeight* w, const float* x, float* y, int64_t rows, int64_t cols) {
    if (w->int16) orc_matvec_i16(w->q, w->s, x, y, rows, cols);
    else orc_matvec_f32(w->f, x, y, rows, cols);
}

/* mv() for T inputs X[T][cols] -> Y[T][rows]: each output is the same sequential sum
 * as mv() gives it.  FP32 weights: the inputs are transposed to XT[cols][16] and one
 * weight row is multiplied against 16 inputs at once, one vector lane per input, each
 * lane doing dot()'s products and additions in dot()'s order (no contraction: this file
 * is compiled with -ffp-contract=off); the scalar tail is fused as in dot(). */
typedef float v8f __attribute__((vector_size(32)));

static void mv_batch(const OWeight* w, const float* X, float* Y, int T, int64_t rows,
                     int64_t cols) {
    if (T == 1) { mv(w, X, Y, rows, cols); return; }
    int64_t m = 0;  /* dot()'s unfused part */
    if (cols >= 8) {
        m = cols & ~(int64_t)7;
        if (cols - m >= 4) m += 4;
    }
    for (int t0 = 0; t0 < T; t0 += 16) {
        const int nt = T - t0 < 16 ? T - t0 : 16;
        float* XT = (float*)aligned_alloc(32, (size_t)cols * 16 * 4);
        for (int64_t j = 0; j < cols; ++j)
            for (int t = 0; t < 16; ++t) XT[j * 16 + t] = t < nt ? X[(size_t)(t0 + t) * cols + j] : 0.0f;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && rows >= 64)
        for (int64_t r = 0; r < rows; ++r) {
            float o[16];
            if (w->int16) {
                for (int t = 0; t < nt; ++t)
                    o[t] = dot_i16(w->q + r * cols, X + (size_t)(t0 + t) * cols, cols, 0.0f) * w->s[r];
            } else {
                const float* wr = w->f + r * cols;
                v8f a0 = {0}, a1 = {0};
                for (int64_t j = 0; j < m; ++j) {
                    const float wj = wr[j];
                    const v8f wv = {wj, wj, wj, wj, wj, wj, wj, wj};
                    const v8f x0 = *(const v8f*)(XT + j * 16), x1 = *(const v8f*)(XT + j * 16 + 8);
                    a0 = a0 + wv * x0;
                    a1 = a1 + wv * x1;
                }
                for (int t = 0; t < 8; ++t) { o[t] = a0[t]; o[t + 8] = a1[t]; }
                for (int64_t j = m; j < cols; ++j)
                    for (int t = 0; t < 16; ++t) o[t] = fmaf(wr[j], XT[j * 16 + t], o[t]);
            }
            for (int t = 0; t < nt; ++t) Y[(size_t)(t0 + t) * rows + r] = o[t];
        }
        free(XT);
    }
}

static void emb_row(const OWeight* w, int tok, float* out, int64_t dim) {
    if (!w->int16) memcpy(out, w->f + (int64_t)tok * dim, (size_t)dim * 4);
    else for (int64_t i = 0; i < dim; ++i) out[i] = (float)w->q[(int64_t)tok * dim + i] * w->s[tok];
}

static float sumsq(const float* x, int n) { return dot(x, x, n, 0.0f); }

/* T tokens at absolute positions pos0..pos0+T-1, layer by layer.  Every token goes
 * through exactly the arithmetic of a token-by-token forward: the block's k/v rows
 * enter the cache before any of its attention runs, and token t attends to positions
 * <= pos0 + t only.  logits (may be NULL: the head is then skipped) receives the V
 * logits of the last token. */
static void forward_block(OModel* m, const int* toks, int T, int pos0, float* logits) {
    const int D = m->D, H = m->H, Hkv = m->Hkv, HD = m->HD, F = m->FFN;
    const int last = pos0 + T - 1;
    float* x = (float*)malloc((size_t)T * D * 4);
    float* xn = (float*)malloc((size_t)T * D * 4);
    float* q = (float*)malloc((size_t)T * H * HD * 4);
    float* k = (float*)malloc((size_t)T * Hkv * HD * 4);
    float* v = (float*)malloc((size_t)T * Hkv * HD * 4);
    float* att = (float*)malloc((size_t)T * H * HD * 4);
    float* scores = (float*)malloc((size_t)T * H * (last + 1) * 4);
    float* o = (float*)malloc((size_t)T * D * 4);
    float* g = (float*)malloc((size_t)T * F * 4);
    float* u = (float*)malloc((size_t)T * F * 4);
    for (int t = 0; t < T; ++t) {
        int tok = toks[t];
        if (tok < 0 || tok >= m->V) tok = 0;
        emb_row(&m->tok, tok, x + (size_t)t * D, D);
    }
    for (int l = 0; l < m->n_layers; ++l) {
        OWeight* L = &m->L[l * W_PER_LAYER];
        for (int t = 0; t < T; ++t) {
            const float* xt = x + (size_t)t * D;
            float rms = sqrtf(sumsq(xt, D) / D + m->eps);
            for (int d = 0; d < D; ++d) xn[(size_t)t * D + d] = xt[d] / rms * L[W_AN].f[d];
        }
        mv_batch(&L[W_Q], xn, q, T, H * HD, D);
        mv_batch(&L[W_K], xn, k, T, Hkv * HD, D);
        mv_batch(&L[W_V], xn, v, T, Hkv * HD, D);
        float* kc = m->kc + (size_t)l * Hkv * m->max_seq * HD;
        float* vc = m->vc + (size_t)l * Hkv * m->max_seq * HD;
        for (int t = 0; t < T; ++t) {
            const int pos = pos0 + t;
            float* qt = q + (size_t)t * H * HD;
            float* kt = k + (size_t)t * Hkv * HD;
            for (int hh = 0; hh < H + Hkv; ++hh) {
                float* vec = hh < H ? qt + hh * HD : kt + (hh - H) * HD;
                for (int d = 0; d < HD; d += 2) {
                    float freq = 1.0f / powf(m->theta, (float)d / HD);
                    float ang = pos * freq;
                    float c = cosf(ang), s = sinf(ang);
                    float a = vec[d], b = vec[d + 1];
                    vec[d] = a * c - b * s;
                    vec[d + 1] = a * s + b * c;
                }
            }
            for (int hk = 0; hk < Hkv; ++hk)
                for (int d = 0; d < HD; ++d) {
                    kc[((size_t)hk * m->max_seq + pos) * HD + d] = kt[hk * HD + d];
                    vc[((size_t)hk * m->max_seq + pos) * HD + d] = v[(size_t)t * Hkv * HD + hk * HD + d];
                }
        }
        const int grp = H / Hkv;
#pragma omp parallel for schedule(dynamic) num_threads(g_threads) if (g_threads > 1 && T * H > 1)
        for (int th = 0; th < T * H; ++th) {
            const int t = th / H, hq = th % H, pos = pos0 + t;
            const float* qh = q + (size_t)t * H * HD + (size_t)hq * HD;
            float* sc = scores + (size_t)th * (last + 1);
            const float* kh = kc + (size_t)(hq / grp) * m->max_seq * HD;
            const float* vh = vc + (size_t)(hq / grp) * m->max_seq * HD;
            float mx = -INFINITY;
            for (int s = 0; s <= pos; ++s) {
                float sco = 0.0f;
                for (int d = 0; d < HD; ++d) sco = fmaf(qh[d], kh[(size_t)s * HD + d], sco);
                sco /= sqrtf((float)HD);
                sc[s] = sco;
                mx = fmaxf(mx, sco);
            }
            float se = 0;
            for (int s = 0; s <= pos; ++s) { sc[s] = expf(sc[s] - mx); se += sc[s]; }
            for (int s = 0; s <= pos; ++s) sc[s] /= se;
            for (int d = 0; d < HD; ++d) {
                float acc = 0;
                for (int s = 0; s <= pos; ++s) acc = fmaf(sc[s], vh[(size_t)s * HD + d], acc);
                att[(size_t)t * H * HD + hq * HD + d] = acc;
            }
        }
        mv_batch(&L[W_O], att, o, T, D, H * HD);
        for (size_t i = 0; i < (size_t)T * D; ++i) x[i] += o[i];
        for (int t = 0; t < T; ++t) {
            const float* xt = x + (size_t)t * D;
            float rms = sqrtf(sumsq(xt, D) / D + m->eps);
            for (int d = 0; d < D; ++d) xn[(size_t)t * D + d] = xt[d] / rms * L[W_FN].f[d];
        }
        mv_batch(&L[W_1], xn, g, T, F, D);
        for (size_t i = 0; i < (size_t)T * F; ++i) g[i] *= 1.0f / (1.0f + expf(-g[i]));
        mv_batch(&L[W_3], xn, u, T, F, D);
        for (size_t i = 0; i < (size_t)T * F; ++i) g[i] *= u[i];
        mv_batch(&L[W_2], g, o, T, D, F);
        for (size_t i = 0; i < (size_t)T * D; ++i) x[i] += o[i];
    }
    if (logits) {
        const float* xt = x + (size_t)(T - 1) * D;
        float rms = sqrtf(sumsq(xt, D) / D + m->eps);
        for (int d = 0; d < D; ++d) xn[d] = xt[d] / rms * m->out_norm.f[d];
        mv(m->tied ? &m->tok : &m->out, xn, logits, m->V, D);
    }
    free(x); free(xn); free(q); free(k); free(v); free(att); free(scores); free(o); free(g); free(u);
}

/* One token at absolute position pos; writes V logits (logits may be NULL: the output
 * head is then skipped, as nothing reads it). */
static void forward_one(OModel* m, int tok, int pos, float* logits) {
    forward_block(m, &tok, 1, pos, logits);
}

/* sample_argmax: src/ops/ops.cpp:424-438 (first maximum wins) */
int orc_argmax(const float* p, int n) {
    int best = 0;
    float bv = p[0];
    for (int i = 1; i < n; ++i)
        if (p[i] > bv) { bv = p[i]; best = i; }
    return best;
}

/* Logits of T tokens fed at positions start..start+T-1 ([T, V]). */
int orc_model_forward(void* h, const int32_t* ids, int T, int start, float* logits) {
    OModel* m = (OModel*)h;
    for (int t = 0; t < T; ++t) {
        if (start + t >= m->max_seq) return -1;
        forward_one(m, ids[t], start + t, logits + (size_t)t * m->V);
    }
    return 0;
}

/* Greedy generate: out = prompt followed by max_tokens new ids.  If last_logits
 * is non-NULL it receives the logits that picked each new token ([max_tokens, V]). */
int orc_model_generate(void* h, const int32_t* prompt, int n_prompt, int max_tokens,
                       int32_t* out, float* all_logits) {
    OModel* m = (OModel*)h;
    float* lg = (float*)malloc((size_t)m->V * 4);
    int n = 0;
    for (int i = 0; i < n_prompt; ++i) out[n++] = prompt[i];
    int pos = 0;
    if (n_prompt > m->max_seq) { free(lg); return -1; }
    /* the prompt in blocks of up to 16 tokens; only the last position's logits pick a
     * token */
    for (int i = 0; i < n_prompt; i += 16) {
        const int T = n_prompt - i < 16 ? n_prompt - i : 16;
        forward_block(m, (const int*)prompt + i, T, pos, i + T == n_prompt ? lg : NULL);
        pos += T;
    }
    for (int step = 0; step < max_tokens; ++step) {
        if (all_logits) memcpy(all_logits + (size_t)step * m->V, lg, (size_t)m->V * 4);
        int next = orc_argmax(lg, m->V);
        out[n++] = next;
        if (step + 1 == max_tokens) break;
        if (pos >= m->max_seq) break;
        forward_one(m, next, pos++, lg);
    }
    free(lg);
    return n;
}
