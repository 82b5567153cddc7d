// Causal GQA attention for one query position over the FP32 KV cache
// [n_kv_heads][max_seq][head_dim] -- the reference's attention_kernel
// (src/ops/cuda_kernels.cu:216-267; CPU: src/models/model.cpp:111-151) computed
// as a split-K "flash decode":
//   partial: CTA (kv head, chunk of positions) scores its chunk for the whole GQA
//            group, keeps the chunk max m, the exp-sum l and the unnormalised
//            weighted V sum;
//   combine: out = sum_c e^(m_c - M) acc_c / sum_c e^(m_c - M) l_c.
// The fast partial (head_dim <= 128, group <= 8) uses 64-position chunks: a warp
// owns 16 positions, lanes split head_dim in float4s, every K and V row load of
// the warp is issued before any of its arithmetic.  Other shapes use a generic
// partial with 128-position chunks.  With `pos_dev` the position is read on the
// device (the grid then spans the whole cache and chunks past the position exit),
// so a decode step can be captured once in a CUDA graph.
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "kv.cuh"
#include "ops.cuh"
#include "pdl.cuh"
#include "slab.cuh"

namespace ib {

constexpr int ATT_CH_FAST = 64;
constexpr int ATT_CH_GENERIC = 128;
constexpr int ATT_MAX_GROUP = 16;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// A coherent (L2) load of a word another kernel writes, never merged with another load.
__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- fast partial ----------------------------------------------------------------
template <int GMAX>
__global__ void __launch_bounds__(128) attn_partial_fast_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ part, int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos,
    float scale, int n_chunks, const int* __restrict__ pos_dev) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int CH = ATT_CH_FAST, PW = CH / 4;  // 4 warps x 16 positions
    __shared__ float4 qs[GMAX][32];
    __shared__ float sc[GMAX][CH];
    __shared__ float4 accs[4][GMAX][32];
    __shared__ float ms[GMAX], ls[GMAX];
    if (pos_dev) pos = *pos_dev;
    const int G = n_heads / n_kv_heads;
    const int hk = blockIdx.x, chunk = blockIdx.y;
    const int s0 = chunk * CH;
    if (s0 > pos || pos >= max_seq) return;  // beyond the live context
    const int n = min(CH, pos + 1 - s0);
    const int nv = head_dim >> 2;  // float4 per row
    int lpp = 1;
    while (lpp < nv) lpp <<= 1;   // lanes per position
    const int ppp = 32 / lpp;     // positions per warp pass
    const int passes = (PW + ppp - 1) / ppp;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pp = lane / lpp, li = lane % lpp;
    const float4* q4 = reinterpret_cast<const float4*>(q) + (size_t)(hk * G) * nv;
    for (int i = tid; i < G * nv; i += 128) qs[i / nv][i % nv] = q4[i];
    __syncthreads();
    const float4* k4 = reinterpret_cast<const float4*>(kc) + ((size_t)hk * max_seq + s0) * nv;
    const float4* v4 = reinterpret_cast<const float4*>(vc) + ((size_t)hk * max_seq + s0) * nv;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 kv[PW];
#pragma unroll
    for (int p = 0; p < PW; ++p) {
        const int s = warp * PW + p * ppp + pp;
        const bool ok = p < passes && p * ppp + pp < PW && s < n && li < nv;
        kv[p] = ok ? __ldg(k4 + (size_t)s * nv + li) : z4;
    }
#pragma unroll
    for (int p = 0; p < PW; ++p) {
        if (p >= passes) break;
        const int s = warp * PW + p * ppp + pp;
        float d[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            const float4 a = li < nv && g < G ? qs[g][li] : z4;
            d[g] = a.x * kv[p].x + a.y * kv[p].y + a.z * kv[p].z + a.w * kv[p].w;
        }
        for (int o = 1; o < lpp; o <<= 1)
#pragma unroll
            for (int g = 0; g < GMAX; ++g) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
        if (li == 0 && p * ppp + pp < PW && s < n)
#pragma unroll
            for (int g = 0; g < GMAX; ++g)
                if (g < G) sc[g][s] = d[g] * scale;
    }
    __syncthreads();
    for (int g = warp; g < G; g += 4) {
        const float a = lane < n ? sc[g][lane] : -INFINITY;
        const float b = lane + 32 < n ? sc[g][lane + 32] : -INFINITY;
        const float m = wmax(fmaxf(a, b));
        const float ea = lane < n ? expf(a - m) : 0.f, eb = lane + 32 < n ? expf(b - m) : 0.f;
        const float l = wsum(ea + eb);
        sc[g][lane] = ea;
        sc[g][lane + 32] = eb;
        if (lane == 0) {
            ms[g] = m;
            ls[g] = l;
        }
    }
    __syncthreads();
    float4 acc[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) acc[g] = z4;
#pragma unroll
    for (int p = 0; p < PW; ++p) {
        const int s = warp * PW + p * ppp + pp;
        const bool ok = p < passes && p * ppp + pp < PW && s < n && li < nv;
        kv[p] = ok ? __ldg(v4 + (size_t)s * nv + li) : z4;
    }
#pragma unroll
    for (int p = 0; p < PW; ++p) {
        if (p >= passes) break;
        const int s = warp * PW + p * ppp + pp;
        if (p * ppp + pp < PW && s < n) {
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                const float w = g < G ? sc[g][s] : 0.f;
                acc[g].x = fmaf(w, kv[p].x, acc[g].x);
                acc[g].y = fmaf(w, kv[p].y, acc[g].y);
                acc[g].z = fmaf(w, kv[p].z, acc[g].z);
                acc[g].w = fmaf(w, kv[p].w, acc[g].w);
            }
        }
    }
    for (int o = lpp; o < 32; o <<= 1)
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            acc[g].x += __shfl_xor_sync(0xffffffffu, acc[g].x, o);
            acc[g].y += __shfl_xor_sync(0xffffffffu, acc[g].y, o);
            acc[g].z += __shfl_xor_sync(0xffffffffu, acc[g].z, o);
            acc[g].w += __shfl_xor_sync(0xffffffffu, acc[g].w, o);
        }
    if (pp == 0 && li < nv)
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            if (g < G) accs[warp][g][li] = acc[g];
    __syncthreads();
    for (int i = tid; i < G * nv; i += 128) {
        const int g = i / nv, l4 = i % nv;
        float4 a = accs[0][g][l4];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            const float4 b = accs[w][g][l4];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        float* out = part + ((size_t)(hk * G + g) * n_chunks + chunk) * (head_dim + 2);
        if (l4 == 0) {
            out[0] = ms[g];
            out[1] = ls[g];
        }
        out[2 + 4 * l4] = a.x;
        out[3 + 4 * l4] = a.y;
        out[4 + 4 * l4] = a.z;
        out[5 + 4 * l4] = a.w;
    }
}

// ---- generic partial (any head_dim <= 256, group <= 16; FP32 or FP16 cache) ---------
template <typename KV>
__global__ void __launch_bounds__(128) attn_partial_generic_kernel(
    const float* __restrict__ q, const KV* __restrict__ kc, const KV* __restrict__ vc,
    float* __restrict__ part, int n_heads, int n_kv_heads, int head_dim, int max_seq, int pos,
    float scale, int n_chunks, const int* __restrict__ pos_dev) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int CH = ATT_CH_GENERIC;
    extern __shared__ float smem[];
    __shared__ float red[32];
    if (pos_dev) pos = *pos_dev;
    const int G = n_heads / n_kv_heads;
    const int hk = blockIdx.x, chunk = blockIdx.y;
    if (chunk * CH > pos || pos >= max_seq) return;
    const int s0 = chunk * CH, n = min(s0 + CH, pos + 1) - s0;
    float* qs = smem;               // [G][HD]
    float* sc = smem + G * head_dim;  // [G][CH]
    for (int i = threadIdx.x; i < G * head_dim; i += blockDim.x)
        qs[i] = q[(size_t)(hk * G) * head_dim + i];
    __syncthreads();
    const KV* kh = kc + (size_t)hk * max_seq * head_dim;
    const KV* vh = vc + (size_t)hk * max_seq * head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int s = warp; s < n; s += 4) {
        const KV* kr = kh + (size_t)(s0 + s) * head_dim;
        float dots[ATT_MAX_GROUP];
#pragma unroll
        for (int g = 0; g < ATT_MAX_GROUP; ++g) dots[g] = 0.f;
        for (int d = lane; d < head_dim; d += 32) {
            const float kv = kv_at(kr, (size_t)d);
#pragma unroll
            for (int g = 0; g < ATT_MAX_GROUP; ++g)
                if (g < G) dots[g] = fmaf(qs[g * head_dim + d], kv, dots[g]);
        }
#pragma unroll
        for (int g = 0; g < ATT_MAX_GROUP; ++g)
            if (g < G) {
                const float v = wsum(dots[g]);
                if (lane == 0) sc[g * CH + s] = v * scale;
            }
    }
    __syncthreads();
    for (int g = 0; g < G; ++g) {
        float m = -INFINITY;
        for (int s = threadIdx.x; s < n; s += blockDim.x) m = fmaxf(m, sc[g * CH + s]);
        m = wmax(m);
        __syncthreads();
        if (lane == 0) red[warp] = m;
        __syncthreads();
        m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        float l = 0.f;
        for (int s = threadIdx.x; s < n; s += blockDim.x) {
            const float e = expf(sc[g * CH + s] - m);
            sc[g * CH + s] = e;
            l += e;
        }
        l = wsum(l);
        __syncthreads();
        if (lane == 0) red[warp] = l;
        __syncthreads();
        l = red[0] + red[1] + red[2] + red[3];
        float* pp = part + ((size_t)(hk * G + g) * n_chunks + chunk) * (head_dim + 2);
        if (threadIdx.x == 0) {
            pp[0] = m;
            pp[1] = l;
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc[ATT_MAX_GROUP];
#pragma unroll
        for (int g = 0; g < ATT_MAX_GROUP; ++g) acc[g] = 0.f;
        for (int s = 0; s < n; ++s) {
            const float vv = kv_at(vh, (size_t)(s0 + s) * head_dim + d);
#pragma unroll
            for (int g = 0; g < ATT_MAX_GROUP; ++g)
                if (g < G) acc[g] = fmaf(sc[g * CH + s], vv, acc[g]);
        }
        for (int g = 0; g < G; ++g)
            part[((size_t)(hk * G + g) * n_chunks + chunk) * (head_dim + 2) + 2 + d] = acc[g];
    }
}

// grid n_heads: out[h, :] = sum_c e^(m_c - M) acc_c / sum_c e^(m_c - M) l_c
__global__ void attn_combine_kernel(const float* __restrict__ part, float* __restrict__ out,
                                    int head_dim, int n_chunks, int ch, int n_live,
                                    const int* __restrict__ pos_dev) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x;
    const float* p = part + (size_t)h * n_chunks * (head_dim + 2);
    const int live = pos_dev ? *pos_dev / ch + 1 : n_live;
    float M = -INFINITY;
    for (int c = 0; c < live; ++c) M = fmaxf(M, p[(size_t)c * (head_dim + 2)]);
    float L = 0.f;
    for (int c = 0; c < live; ++c) {
        const float* pc = p + (size_t)c * (head_dim + 2);
        L += expf(pc[0] - M) * pc[1];
    }
    const float inv = 1.0f / L;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc = 0.f;
        for (int c = 0; c < live; ++c) {
            const float* pc = p + (size_t)c * (head_dim + 2);
            acc = fmaf(expf(pc[0] - M), pc[2 + d], acc);
        }
        out[(size_t)h * head_dim + d] = acc * inv;
    }
}

static bool fast_ok(int H, int Hkv, int HD) {
    return HD % 4 == 0 && HD <= 128 && H / Hkv <= 8;
}

int attention_decode(const float* q, const void* kc, const void* vc, float* out, int H,
                     int Hkv, int HD, int max_seq, int pos, float scale, float* part,
                     cudaStream_t st, const int* pos_dev, bool pdl, bool kv_half) {
    const int G = H / Hkv;
    const bool fast = !kv_half && fast_ok(H, Hkv, HD) && ((uintptr_t)q % 16 == 0) &&
                      ((uintptr_t)kc % 16 == 0) && ((uintptr_t)vc % 16 == 0);
    const int ch = fast ? ATT_CH_FAST : ATT_CH_GENERIC;
    // with pos_dev the grid covers the whole cache and chunks past *pos_dev exit
    const int n_chunks = pos_dev ? (max_seq + ch - 1) / ch : pos / ch + 1;
    const dim3 grid(Hkv, n_chunks);
    if (fast) {
        auto kern = G <= 1 ? attn_partial_fast_kernel<1> : G <= 2 ? attn_partial_fast_kernel<2> :
                    G <= 4 ? attn_partial_fast_kernel<4> : attn_partial_fast_kernel<8>;
        IB_CUDA_CHECK(launch_pdl(kern, grid, dim3(128), 0, st, pdl, q, (const float*)kc,
                                 (const float*)vc, part, H, Hkv, HD, max_seq, pos, scale, n_chunks,
                                 pos_dev));
    } else if (kv_half) {
        const size_t smem = (size_t)(G * HD + G * ATT_CH_GENERIC) * sizeof(float);
        IB_CUDA_CHECK(launch_pdl(attn_partial_generic_kernel<__half>, grid, dim3(128), smem, st,
                                 pdl, q, (const __half*)kc, (const __half*)vc, part, H, Hkv, HD,
                                 max_seq, pos, scale, n_chunks, pos_dev));
    } else {
        const size_t smem = (size_t)(G * HD + G * ATT_CH_GENERIC) * sizeof(float);
        IB_CUDA_CHECK(launch_pdl(attn_partial_generic_kernel<float>, grid, dim3(128), smem, st,
                                 pdl, q, (const float*)kc, (const float*)vc, part, H, Hkv, HD,
                                 max_seq, pos, scale, n_chunks, pos_dev));
    }
    IB_LAUNCH_CHECK("attention_partial_kernel");
    IB_CUDA_CHECK(launch_pdl(attn_combine_kernel, dim3(H), dim3(128), 0, st, pdl, part, out, HD,
                             n_chunks, ch, pos / ch + 1, pos_dev));
    IB_LAUNCH_CHECK("attention_combine_kernel");
    return IB_OK;
}

// ---- fused decode attention ---------------------------------------------------------
// Grid (kv head, split), 256 threads.  Split sp owns positions [sp * per, (sp + 1) * per)
// with per = ceil((pos + 1) / ATT_SPLITS) rounded up to whole 64-position tiles, and runs
// an online softmax over its tiles.  In a tile each warp takes 8 positions, 2 at a time:
// 16 lanes per position, each lane 1 or 2 float4 of the head dimension (K and V rows of
// the warp's positions are all loaded before any arithmetic).  Partials (running max,
// exp-sum, unnormalised P.V) go to `part`; the last CTA of each kv head (atomic
// counter, reset after use) combines them and writes the head outputs and, when `slab`
// is set, their limb slab for the next GEMV.
constexpr int ATT_TILE = 64;
constexpr int ATT_SPLITS = 64;
constexpr int ATT_WARPS = 8;

template <int GMAX, typename KV>
__global__ void __launch_bounds__(ATT_WARPS * 32, 2) attn_fused_kernel(
    const float* __restrict__ q, const KV* __restrict__ kc, const KV* __restrict__ vc,
    float* __restrict__ part_acc, float2* __restrict__ part_ml, int* __restrict__ counters,
    float* __restrict__ out, uint8_t* __restrict__ slab, int slab_kq, int n_heads, int n_kv_heads,
    int head_dim, int max_seq, float scale, const int* __restrict__ pos_dev) {
    pdl_launch_dependents();
    constexpr int LPP = 16, PPP = 32 / LPP;  // lanes per position, positions per pass
    constexpr int PW = ATT_TILE / ATT_WARPS;  // positions per warp per tile
    constexpr int PASSES = PW / PPP;
    constexpr int NVL = 2;                    // float4 per lane (head_dim <= 128)
    static_assert(GMAX * 32 <= ATT_WARPS * 32, "one query float4 per thread");
    __shared__ float4 qs[GMAX][32];
    __shared__ float sc[GMAX][ATT_TILE];
    __shared__ float alpha[GMAX], mrun[GMAX], lrun[GMAX];
    __shared__ float4 accs[ATT_WARPS][GMAX][32];
    __shared__ float wsp[GMAX][ATT_SPLITS];
    __shared__ float linv[GMAX];
    __shared__ __align__(16) float ovals[GMAX * 128];
    __shared__ int is_last;
    const int G = n_heads / n_kv_heads;
    const int hk = blockIdx.x, sp = blockIdx.y;
    const int nv = head_dim >> 2;  // float4 per row
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pp = lane / LPP, li = lane % LPP;
    const KV* kb = kc + (size_t)hk * max_seq * head_dim;  // element rows; float4 units below
    const KV* vb = vc + (size_t)hk * max_seq * head_dim;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 kr[PASSES][NVL], vr[PASSES][NVL];
#pragma unroll
    for (int p = 0; p < PASSES; ++p)
#pragma unroll
        for (int k = 0; k < NVL; ++k) kr[p][k] = vr[p][k] = z4;
    // rows t0 + s, s < n, with lo <= t0 + s < hi of the tile at t0; the others keep
    // their registers
    auto load_tile = [&](int t0, int n, int lo, int hi) {
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const int s = warp * PW + p * PPP + pp;
#pragma unroll
            for (int k = 0; k < NVL; ++k) {
                const int c = li + LPP * k;
                if (s < n && c < nv && t0 + s >= lo && t0 + s < hi) {
                    kr[p][k] = kv_at4(kb, (size_t)(t0 + s) * nv + c);
                    vr[p][k] = kv_at4(vb, (size_t)(t0 + s) * nv + c);
                }
            }
        }
    };
    // every row of the tile at t0 (zeros past n): no register outlives its tile
    auto load_full = [&](int t0, int n) {
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const int s = warp * PW + p * PPP + pp;
#pragma unroll
            for (int k = 0; k < NVL; ++k) {
                const int c = li + LPP * k;
                const bool ok = s < n && c < nv;
                kr[p][k] = ok ? kv_at4(kb, (size_t)(t0 + s) * nv + c) : z4;
                vr[p][k] = ok ? kv_at4(vb, (size_t)(t0 + s) * nv + c) : z4;
            }
        }
    };
    // this split's positions [p0, p1) for the token at `at`; live = splits in use
    int live = 0, p0 = 0, p1 = 0;
    auto span = [&](int at) {
        const int n_pos = at + 1;
        int per = (n_pos + ATT_SPLITS - 1) / ATT_SPLITS;
        per = (per + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
        live = (n_pos + per - 1) / per;
        p0 = sp * per;
        p1 = min(n_pos, p0 + per);
    };
    // K and V rows below the step's position were written by earlier steps and do not
    // change during this one (the previous kernel, the QKV projection, writes row `pos`
    // only), so for groups of up to 4 the first tile's other rows are loaded before the
    // wait on that kernel, while the CTAs that reach it early overlap its tail.  The
    // position word changes only between steps (a kernel launched without the PDL
    // attribute ends each step); it is read again after the wait, and a different value
    // reloads the whole tile.  Measured on the decode step at position 2050: Llama-3-8B
    // (group 4) 2.26 against 2.38 ms; Llama-3-70B (group 8, whose registers already
    // spill) 12.11 against 11.92 ms, so the group-8 kernel loads every tile after the
    // wait and after the query, in the loop below.
    constexpr bool kPrefetch = GMAX <= 4;
    int pos_pre = -1;
    if (kPrefetch) pos_pre = ld_relaxed_gpu(pos_dev);
    const bool pre = kPrefetch && pos_pre >= 0 && pos_pre < max_seq;
    if (pre) {
        span(pos_pre);
        if (sp < live) load_tile(p0, min(ATT_TILE, p1 - p0), 0, pos_pre);
    }
    pdl_wait();
    // the query (G * nv <= 256 float4, one per thread) and the position word in one
    // round trip: neither depends on the other
    const float4* q4 = reinterpret_cast<const float4*>(q) + (size_t)(hk * G) * nv;
    const float4 qv = tid < G * nv ? q4[tid] : z4;
    const int pos = ld_relaxed_gpu(pos_dev);
    if (pos < 0 || pos >= max_seq) return;
    span(pos);
    if (sp >= live) return;
    if (pre && pos == pos_pre)
        load_tile(p0, min(ATT_TILE, p1 - p0), pos, pos + 1);
    else if (kPrefetch)
        load_full(p0, min(ATT_TILE, p1 - p0));
    if (tid < G * nv) qs[tid / nv][tid % nv] = qv;
    if (tid < G) {
        mrun[tid] = -INFINITY;
        lrun[tid] = 0.f;
    }
    __syncthreads();
    float4 acc[GMAX][NVL];
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
#pragma unroll
        for (int k = 0; k < NVL; ++k) acc[g][k] = z4;
    for (int t0 = p0; t0 < p1; t0 += ATT_TILE) {
        const int n = min(ATT_TILE, p1 - t0);
        // without the prefetch every tile, the first included, loads here, after the
        // query is in shared memory
        if (!kPrefetch || t0 != p0) load_full(t0, n);
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const int s = warp * PW + p * PPP + pp;
            float d[GMAX];
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                float t = 0.f;
#pragma unroll
                for (int k = 0; k < NVL; ++k) {
                    const int c = li + LPP * k;
                    const float4 a = c < nv && g < G ? qs[g][c] : z4;
                    t += a.x * kr[p][k].x + a.y * kr[p][k].y + a.z * kr[p][k].z + a.w * kr[p][k].w;
                }
                d[g] = t;
            }
#pragma unroll
            for (int o = 1; o < LPP; o <<= 1)
#pragma unroll
                for (int g = 0; g < GMAX; ++g) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
            if (li == 0 && s < n)
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    if (g < G) sc[g][s] = d[g] * scale;
        }
        __syncthreads();
        for (int g = warp; g < G; g += ATT_WARPS) {  // online softmax over the tile
            const float a = lane < n ? sc[g][lane] : -INFINITY;
            const float b = lane + 32 < n ? sc[g][lane + 32] : -INFINITY;
            const float mt = wmax(fmaxf(a, b));
            const float mo = mrun[g], mn = fmaxf(mo, mt);
            const float ea = lane < n ? expf(a - mn) : 0.f;
            const float eb = lane + 32 < n ? expf(b - mn) : 0.f;
            const float lt = wsum(ea + eb);
            sc[g][lane] = ea;
            sc[g][lane + 32] = eb;
            if (lane == 0) {
                const float al = mo == -INFINITY ? 0.f : expf(mo - mn);
                alpha[g] = al;
                lrun[g] = lrun[g] * al + lt;
                mrun[g] = mn;
            }
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            const float al = g < G ? alpha[g] : 0.f;
#pragma unroll
            for (int k = 0; k < NVL; ++k) {
                acc[g][k].x *= al;
                acc[g][k].y *= al;
                acc[g][k].z *= al;
                acc[g][k].w *= al;
            }
        }
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const int s = warp * PW + p * PPP + pp;
            if (s < n) {
#pragma unroll
                for (int g = 0; g < GMAX; ++g) {
                    const float w = g < G ? sc[g][s] : 0.f;
#pragma unroll
                    for (int k = 0; k < NVL; ++k) {
                        acc[g][k].x = fmaf(w, vr[p][k].x, acc[g][k].x);
                        acc[g][k].y = fmaf(w, vr[p][k].y, acc[g][k].y);
                        acc[g][k].z = fmaf(w, vr[p][k].z, acc[g][k].z);
                        acc[g][k].w = fmaf(w, vr[p][k].w, acc[g][k].w);
                    }
                }
            }
        }
        __syncthreads();
    }
    // lanes li and li + 16 hold the two position streams of the same dims
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
#pragma unroll
        for (int k = 0; k < NVL; ++k) {
            acc[g][k].x += __shfl_xor_sync(0xffffffffu, acc[g][k].x, 16);
            acc[g][k].y += __shfl_xor_sync(0xffffffffu, acc[g][k].y, 16);
            acc[g][k].z += __shfl_xor_sync(0xffffffffu, acc[g][k].z, 16);
            acc[g][k].w += __shfl_xor_sync(0xffffffffu, acc[g][k].w, 16);
        }
    if (pp == 0)
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
#pragma unroll
            for (int k = 0; k < NVL; ++k) {
                const int c = li + LPP * k;
                if (g < G && c < nv) accs[warp][g][c] = acc[g][k];
            }
    __syncthreads();
    for (int i = tid; i < G * nv; i += ATT_WARPS * 32) {
        const int g = i / nv, l4 = i % nv;
        float4 a = accs[0][g][l4];
#pragma unroll
        for (int w = 1; w < ATT_WARPS; ++w) {
            const float4 b = accs[w][g][l4];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        const size_t row = (size_t)(hk * G + g) * ATT_SPLITS + sp;
        reinterpret_cast<float4*>(part_acc + row * head_dim)[l4] = a;
        if (l4 == 0) part_ml[row] = make_float2(mrun[g], lrun[g]);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&counters[hk], 1) == live - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // combine the live splits of this kv head
    for (int g = warp; g < G; g += ATT_WARPS) {
        const size_t r0 = (size_t)(hk * G + g) * ATT_SPLITS;
        const float2 a = lane < live ? __ldcg(part_ml + r0 + lane) : make_float2(-INFINITY, 0.f);
        const float2 b = lane + 32 < live ? __ldcg(part_ml + r0 + lane + 32)
                                          : make_float2(-INFINITY, 0.f);
        const float M = wmax(fmaxf(a.x, b.x));
        const float wa = lane < live ? expf(a.x - M) : 0.f;
        const float wb = lane + 32 < live ? expf(b.x - M) : 0.f;
        const float L = wsum(wa * a.y + wb * b.y);
        wsp[g][lane] = wa;
        wsp[g][lane + 32] = wb;
        if (lane == 0) linv[g] = 1.0f / L;
    }
    __syncthreads();
    // two threads per output float4, each over half of the splits; the loop runs on
    // whole warps (every lane reaches the pair shuffle), lanes past the end idle
    for (int i0 = warp * 32; i0 < 2 * G * nv; i0 += ATT_WARPS * 32) {
        const int i = i0 + lane;
        const bool act = i < 2 * G * nv;
        const int pair = act ? i >> 1 : 0, half = i & 1;
        const int g = pair / nv, l4 = pair % nv;
        const float4* src = reinterpret_cast<const float4*>(part_acc) +
                            ((size_t)(hk * G + g) * ATT_SPLITS) * nv + l4;
        float4 a = z4;
        for (int c0 = half; act && c0 < live; c0 += 16) {
            float4 b[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + 2 * u;
                b[u] = c < live ? __ldcg(src + (size_t)c * nv) : z4;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + 2 * u;
                const float w = c < live ? wsp[g][c] : 0.f;
                a.x = fmaf(w, b[u].x, a.x);
                a.y = fmaf(w, b[u].y, a.y);
                a.z = fmaf(w, b[u].z, a.z);
                a.w = fmaf(w, b[u].w, a.w);
            }
        }
        a.x += __shfl_xor_sync(0xffffffffu, a.x, 1);
        a.y += __shfl_xor_sync(0xffffffffu, a.y, 1);
        a.z += __shfl_xor_sync(0xffffffffu, a.z, 1);
        a.w += __shfl_xor_sync(0xffffffffu, a.w, 1);
        if (act && half == 0) {
            const float inv = linv[g];
            a.x *= inv;
            a.y *= inv;
            a.z *= inv;
            a.w *= inv;
            reinterpret_cast<float4*>(out + (size_t)(hk * G + g) * head_dim)[l4] = a;
            reinterpret_cast<float4*>(ovals + g * head_dim)[l4] = a;
        }
    }
    if (tid == 0) counters[hk] = 0;
    if (!slab) return;
    __syncthreads();
    const int n_el = G * head_dim;
    const int base_el = hk * n_el;
    if (slab_kq) {
        constexpr int GS = SlabG<true>::GS;
        for (int gl = warp; gl < n_el / GS; gl += ATT_WARPS) {
            float v[GS / 32];
            slab_load<true>(ovals, gl, lane, v);
            slab_write_group<true>(v, (base_el + gl * GS) / GS, slab, lane);
        }
    } else {
        constexpr int GS = SlabG<false>::GS;
        for (int gl = warp; gl < n_el / GS; gl += ATT_WARPS) {
            float v[GS / 32];
            slab_load<false>(ovals, gl, lane, v);
            slab_write_group<false>(v, (base_el + gl * GS) / GS, slab, lane);
        }
    }
}

bool attention_fused_ok(int H, int Hkv, int HD) { return fast_ok(H, Hkv, HD); }

size_t attention_fused_part_bytes(int H, int HD) {
    return (size_t)H * ATT_SPLITS * ((size_t)HD * 4 + 8) + 256;
}

int attention_decode_fused(const float* q, const void* kc, const void* vc, float* out,
                           uint8_t* slab, bool slab_kq, int H, int Hkv, int HD, int max_seq,
                           float scale, float* part, int* counters, cudaStream_t st,
                           const int* pos_dev, bool pdl, bool kv_half) {
    IB_REQUIRE(fast_ok(H, Hkv, HD) && pos_dev && counters && part, "fused attention: bad arguments");
    IB_REQUIRE(((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc | (uintptr_t)out | (uintptr_t)part) % 16 == 0,
               "fused attention: pointers must be 16-byte aligned");
    const int G = H / Hkv;
    if (slab) {
        const int GS = slab_kq ? SlabG<true>::GS : SlabG<false>::GS;
        IB_REQUIRE((G * HD) % GS == 0, "fused attention: head group not a whole limb group");
    }
    float* part_acc = part;
    float2* part_ml = reinterpret_cast<float2*>(part + (size_t)H * ATT_SPLITS * HD);
    const dim3 grid(Hkv, ATT_SPLITS);
    if (kv_half) {
        auto kern = G <= 1 ? attn_fused_kernel<1, __half> : G <= 2 ? attn_fused_kernel<2, __half> :
                    G <= 4 ? attn_fused_kernel<4, __half> : attn_fused_kernel<8, __half>;
        IB_CUDA_CHECK(launch_pdl(kern, grid, dim3(ATT_WARPS * 32), 0, st, pdl, q,
                                 (const __half*)kc, (const __half*)vc, part_acc, part_ml, counters,
                                 out, slab, slab_kq ? 1 : 0, H, Hkv, HD, max_seq, scale, pos_dev));
        return IB_OK;
    }
    auto kern = G <= 1 ? attn_fused_kernel<1, float> : G <= 2 ? attn_fused_kernel<2, float> :
                G <= 4 ? attn_fused_kernel<4, float> : attn_fused_kernel<8, float>;
    IB_CUDA_CHECK(launch_pdl(kern, grid, dim3(ATT_WARPS * 32), 0, st, pdl, q, (const float*)kc,
                             (const float*)vc, part_acc, part_ml, counters, out, slab,
                             slab_kq ? 1 : 0, H, Hkv, HD, max_seq, scale, pos_dev));
    return IB_OK;
}

size_t attention_partial_bytes(int H, int HD, int pos) {
    const int n_chunks = pos / ATT_CH_FAST + 1;  // the smaller chunk size bounds both paths
    return (size_t)H * n_chunks * (HD + 2) * sizeof(float);
}

int check_attention_args(int H, int Hkv, int HD, int max_seq, int pos) {
    IB_REQUIRE(H > 0 && Hkv > 0 && H % Hkv == 0, "n_heads must be a multiple of n_kv_heads");
    IB_REQUIRE(H / Hkv <= ATT_MAX_GROUP, "GQA group larger than 16 is not supported");
    IB_REQUIRE(HD > 0 && HD <= 256, "head_dim must be in (0, 256]");
    IB_REQUIRE(pos >= 0 && pos < max_seq, "pos outside the KV cache");
    const size_t smem = (size_t)((H / Hkv) * HD + (H / Hkv) * ATT_CH_GENERIC) * sizeof(float);
    IB_REQUIRE(fast_ok(H, Hkv, HD) || smem <= 48 * 1024,
               "attention group too large for shared memory");
    return IB_OK;
}

// ---- prefill attention: causal, GQA, on the tensor cores ------------------------------
// Scores and the P.V product run as mma.sync.m16n8k16 (FP16 operands, FP32 accumulate)
// with every FP32 operand split into two FP16 parts, x = hi + lo (hi = fp16(x), lo =
// fp16(x - hi)), and the three products hi.hi + hi.lo + lo.hi accumulated in FP32:
// about 22 bits per operand instead of FP32's 24, the dropped lo.lo term below 2^-22
// of the product.  K and V of the positions in range are split once per call by
// kv_planes_kernel into FP16 planes [kv head][position][head_dim] (hi and lo); the
// query rows are scaled by `scale` (the reference's dot * scale,
// src/ops/cuda_kernels.cu attention_batch_kernel) and split while they are staged.
//
// One CTA of 8 warps per (kv head, block of 128 query rows); rows r = g * QT + tq are
// (query head g of the group, query q0 + tq), QT = 128 / G, so the group's heads share
// every K/V tile.  Warp w owns rows 16w..16w+15: their query fragments stay in
// registers, the scores of a 64-position tile are an 16 x 64 accumulator whose layout
// is the A-operand layout of the P.V product (no shuffle), the online-softmax state
// (max, sum) of the lane's two rows is reduced over the 4 lanes of a quad, and O is a
// 16 x head_dim accumulator.  K/V tiles (4 planes of 64 positions) arrive by cp.async,
// double-buffered; the first stage's buffer stages the query rows before the loop.
// Shared-memory rows are padded by 16 bytes, so the 8 rows of an ldmatrix hit distinct
// banks.
constexpr int AP_ROWS = 128, AP_BK = 64, AP_WARPS = 8;

template <int HD>
__host__ __device__ constexpr int ap_ld() { return HD + 8; }  // padded row, halves

template <int HD>
constexpr size_t attn_prefill_smem() {
    return (size_t)2 * 4 * AP_BK * ap_ld<HD>() * 2;  // 2 stages x 4 planes
}

__device__ __forceinline__ void ap_cp16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x0, x1) -> packed FP16 hi parts and lo parts
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// K and V rows [0, n_pos) of every kv head into FP16 hi/lo planes
// [n_kv_heads][n_pos][head_dim] (planes: K hi, K lo, V hi, V lo).
template <typename KV>
__global__ void kv_planes_kernel(const KV* __restrict__ kc, const KV* __restrict__ vc,
                                 __half* __restrict__ planes, int Hkv, int max_seq, int HD,
                                 int n_pos) {
    const size_t per = (size_t)Hkv * n_pos * HD;  // elements per plane
    const size_t n4 = per / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t e = i * 4;
        const int d = (int)(e % HD);
        const size_t hp = e / HD;  // kv head * n_pos + position
        const int pos = (int)(hp % n_pos), hk = (int)(hp / n_pos);
        const size_t src = ((size_t)hk * max_seq + pos) * HD + d;
        const float4 k = kv_at4(kc, src / 4);
        const float4 v = kv_at4(vc, src / 4);
        uint32_t h0, l0, h1, l1;
        split2(k.x, k.y, h0, l0);
        split2(k.z, k.w, h1, l1);
        *reinterpret_cast<uint2*>(planes + e) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(planes + per + e) = make_uint2(l0, l1);
        split2(v.x, v.y, h0, l0);
        split2(v.z, v.w, h1, l1);
        *reinterpret_cast<uint2*>(planes + 2 * per + e) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(planes + 3 * per + e) = make_uint2(l0, l1);
    }
}

template <int HD>
__global__ void __launch_bounds__(AP_WARPS * 32, 1)
    attn_prefill_kernel(const float* __restrict__ q, const __half* __restrict__ planes,
                        float* __restrict__ out, int H, int Hkv, int n_pos, int start, int T,
                        float scale) {
    constexpr int LD = ap_ld<HD>(), KS = HD / 16, NT = HD / 8;
    constexpr int PLANE = AP_BK * LD;  // halves per plane tile
    extern __shared__ __align__(128) __half apsm[];
    const int G = H / Hkv, QT = AP_ROWS / G;
    const int hk = blockIdx.y;
    const int q0 = (gridDim.x - 1 - blockIdx.x) * QT;  // the longest rows first
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, cq = lane & 3;
    const size_t per = (size_t)Hkv * n_pos * HD;
    const __half* kh = planes + (size_t)hk * n_pos * HD;
    const int kv_end = start + (q0 + QT < T ? q0 + QT : T);  // positions [0, kv_end)
    const int n_tiles = (kv_end + AP_BK - 1) / AP_BK;
    auto load_tile = [&](int tile, int buf) {
        __half* dst = apsm + (size_t)buf * 4 * PLANE;
        constexpr int CH = HD / 8;  // 16-byte chunks per row
        for (int i = tid; i < 4 * AP_BK * CH; i += AP_WARPS * 32) {
            const int pl = i / (AP_BK * CH), rem = i - pl * AP_BK * CH;
            const int rr = rem / CH, c8 = rem - rr * CH;
            const int pos = tile * AP_BK + rr;
            const bool valid = pos < kv_end;
            const __half* src = kh + pl * per + (size_t)(valid ? pos : 0) * HD + 8 * c8;
            ap_cp16(dst + pl * PLANE + rr * LD + 8 * c8, src, valid);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // stage the query rows (scaled, split) in stage 1's buffer: hi rows then lo rows
    {
        __half* qh = apsm + 4 * PLANE;
        __half* ql = qh + AP_ROWS * LD;
        for (int i = tid; i < AP_ROWS * HD / 2; i += AP_WARPS * 32) {
            const int r = i / (HD / 2), c2 = i - r * (HD / 2);
            const int t = q0 + r % QT;
            float2 v = make_float2(0.f, 0.f);
            if (t < T) v = *reinterpret_cast<const float2*>(q + ((size_t)t * H + hk * G + r / QT) * HD + 2 * c2);
            uint32_t h, l;
            split2(v.x * scale, v.y * scale, h, l);
            *reinterpret_cast<uint32_t*>(qh + r * LD + 2 * c2) = h;
            *reinterpret_cast<uint32_t*>(ql + r * LD + 2 * c2) = l;
        }
    }
    load_tile(0, 0);
    __syncthreads();
    uint32_t qa[KS][4], qb[KS][4];  // this warp's query fragments, hi and lo
    {
        const int mat = lane >> 3, rr = lane & 7;
        const int row = warp * 16 + (mat & 1) * 8 + rr;
        const uint32_t base = (uint32_t)__cvta_generic_to_shared(apsm + 4 * PLANE);
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const uint32_t off = (uint32_t)((row * LD + kk * 16 + (mat >> 1) * 8) * 2);
            ldsm_x4(base + off, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
            ldsm_x4(base + AP_ROWS * LD * 2 + off, qb[kk][0], qb[kk][1], qb[kk][2], qb[kk][3]);
        }
    }
    __syncthreads();  // stage 1's buffer is free for K/V
    // the lane's two rows: r0 = 16 warp + gq, r1 = r0 + 8
    int qp[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) qp[h] = start + q0 + (warp * 16 + gq + 8 * h) % QT;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    const int row_min = start + q0;  // the smallest query position of the CTA
    for (int tile = 0; tile < n_tiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < n_tiles) {
            load_tile(tile + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint32_t sb = (uint32_t)__cvta_generic_to_shared(apsm + (size_t)buf * 4 * PLANE);
        const int mat = lane >> 3, rr = lane & 7;
        // S = Q K^T over the tile's 64 positions (8 n-tiles)
        float sc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                const int pos = 16 * jp + (mat >> 1) * 8 + rr;
                const uint32_t off = (uint32_t)((pos * LD + kk * 16 + (mat & 1) * 8) * 2);
                uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
                ldsm_x4(sb + off, h0, h1, h2, h3);                  // K hi
                ldsm_x4(sb + PLANE * 2 + off, l0, l1, l2, l3);      // K lo
                mma16816(sc[2 * jp], qa[kk], h0, h1);
                mma16816(sc[2 * jp], qa[kk], l0, l1);
                mma16816(sc[2 * jp], qb[kk], h0, h1);
                mma16816(sc[2 * jp + 1], qa[kk], h2, h3);
                mma16816(sc[2 * jp + 1], qa[kk], l2, l3);
                mma16816(sc[2 * jp + 1], qb[kk], h2, h3);
            }
        }
        // causal mask on tiles that reach past the CTA's smallest query position
        const int t0 = tile * AP_BK;
        if (t0 + AP_BK - 1 > row_min) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int kp = t0 + 8 * j + 2 * cq + (e & 1);
                    if (kp > qp[e >> 1]) sc[j][e] = -INFINITY;
                }
        }
        // online softmax of the lane's two rows (quad reductions)
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fmaxf(sc[j][2 * h], sc[j][2 * h + 1]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(m[h], mx);  // finite: position 0 is in every row's range
            alpha[h] = expf(m[h] - mn);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                sc[j][2 * h] = expf(sc[j][2 * h] - mn);
                sc[j][2 * h + 1] = expf(sc[j][2 * h + 1] - mn);
                sum += sc[j][2 * h] + sc[j][2 * h + 1];
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            l[h] = l[h] * alpha[h] + sum;
            m[h] = mn;
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        // O += P V: the score accumulators are the A fragments of P (16 positions per step)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            uint32_t ph[4], pl[4];
            split2(sc[2 * ks][0], sc[2 * ks][1], ph[0], pl[0]);
            split2(sc[2 * ks][2], sc[2 * ks][3], ph[1], pl[1]);
            split2(sc[2 * ks + 1][0], sc[2 * ks + 1][1], ph[2], pl[2]);
            split2(sc[2 * ks + 1][2], sc[2 * ks + 1][3], ph[3], pl[3]);
            const int pos = 16 * ks + (mat & 1) * 8 + rr;
#pragma unroll
            for (int dp = 0; dp < NT / 2; ++dp) {
                const uint32_t off = (uint32_t)((pos * LD + dp * 16 + (mat >> 1) * 8) * 2);
                uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
                ldsm_x4_t(sb + PLANE * 4 + off, h0, h1, h2, h3);  // V hi
                ldsm_x4_t(sb + PLANE * 6 + off, l0, l1, l2, l3);  // V lo
                mma16816(o[2 * dp], ph, h0, h1);
                mma16816(o[2 * dp], ph, l0, l1);
                mma16816(o[2 * dp], pl, h0, h1);
                mma16816(o[2 * dp + 1], ph, h2, h3);
                mma16816(o[2 * dp + 1], ph, l2, l3);
                mma16816(o[2 * dp + 1], pl, h2, h3);
            }
        }
        __syncthreads();  // this buffer is refilled two tiles on
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int r = warp * 16 + gq + 8 * h, t = q0 + r % QT;
        if (t >= T) continue;
        const float inv = 1.0f / l[h];
        float* dst = out + ((size_t)t * H + hk * G + r / QT) * HD + 2 * cq;
#pragma unroll
        for (int n = 0; n < NT; ++n)
            *reinterpret_cast<float2*>(dst + 8 * n) = make_float2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
    }
}

bool attention_prefill_ok(int H, int Hkv, int HD) {
    if (Hkv <= 0 || H % Hkv) return false;
    const int G = H / Hkv;
    return (HD == 64 || HD == 128) && G >= 1 && G <= AP_ROWS && AP_ROWS % G == 0;
}

template <int HD>
static int launch_prefill(const float* q, const void* kc, const void* vc, float* out, int H,
                          int Hkv, int max_seq, int start, int T, float scale, cudaStream_t st,
                          bool kv_half) {
    static std::mutex mu;
    static bool attr[64] = {};
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !attr[dev]) {
            IB_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<HD>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)attn_prefill_smem<HD>()));
            attr[dev] = true;
        }
    }
    const int n_pos = start + T;
    const size_t per = (size_t)Hkv * n_pos * HD;
    void* ws = nullptr;
    int r;
    if ((r = workspace_get(WS_ATTN_PLANES, per * 4 * sizeof(__half), &ws))) return r;
    __half* planes = (__half*)ws;
    const size_t n4 = per / 4;
    const int g = (int)((n4 + 255) / 256 < 148 * 16 ? (n4 + 255) / 256 : 148 * 16);
    if (kv_half)  // the lo planes come out zero: FP16 values split exactly
        kv_planes_kernel<<<g, 256, 0, st>>>((const __half*)kc, (const __half*)vc, planes, Hkv,
                                            max_seq, HD, n_pos);
    else
        kv_planes_kernel<<<g, 256, 0, st>>>((const float*)kc, (const float*)vc, planes, Hkv,
                                            max_seq, HD, n_pos);
    IB_LAUNCH_CHECK("kv_planes_kernel");
    const int QT = AP_ROWS / (H / Hkv);
    const dim3 grid((T + QT - 1) / QT, Hkv);
    IB_REQUIRE(grid.x <= 0x7FFFFFFF && Hkv <= 65535, "attention: too many rows");
    attn_prefill_kernel<HD><<<grid, AP_WARPS * 32, attn_prefill_smem<HD>(), st>>>(
        q, planes, out, H, Hkv, n_pos, start, T, scale);
    IB_LAUNCH_CHECK("attn_prefill_kernel");
    return IB_OK;
}

int attention_prefill(const float* q, const void* kc, const void* vc, float* out, int H, int Hkv,
                      int HD, int max_seq, int start, int T, float scale, cudaStream_t st,
                      bool kv_half) {
    IB_REQUIRE(attention_prefill_ok(H, Hkv, HD), "attention: unsupported shape for the prefill kernel");
    IB_REQUIRE(T > 0 && start >= 0 && start + T <= max_seq, "attention: positions beyond the cache");
    IB_REQUIRE(((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc | (uintptr_t)out) % 16 == 0,
               "attention: pointers must be 16-byte aligned");
    if (HD == 128)
        return launch_prefill<128>(q, kc, vc, out, H, Hkv, max_seq, start, T, scale, st, kv_half);
    return launch_prefill<64>(q, kc, vc, out, H, Hkv, max_seq, start, T, scale, st, kv_half);
}

}  // namespace ib
