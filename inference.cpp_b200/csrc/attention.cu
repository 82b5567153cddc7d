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
#include "common.cuh"
#include "ops.cuh"
#include "pdl.cuh"

namespace ib {

constexpr int ATT_CH_FAST = 64;
constexpr int ATT_CH_GENERIC = 128;
constexpr int ATT_MAX_GROUP = 16;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
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

// ---- generic partial (any head_dim <= 256, group <= 16) ---------------------------
__global__ void __launch_bounds__(128) attn_partial_generic_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
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
    const float* kh = kc + (size_t)hk * max_seq * head_dim;
    const float* vh = vc + (size_t)hk * max_seq * head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int s = warp; s < n; s += 4) {
        const float* kr = kh + (size_t)(s0 + s) * head_dim;
        float dots[ATT_MAX_GROUP];
#pragma unroll
        for (int g = 0; g < ATT_MAX_GROUP; ++g) dots[g] = 0.f;
        for (int d = lane; d < head_dim; d += 32) {
            const float kv = kr[d];
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
            const float vv = vh[(size_t)(s0 + s) * head_dim + d];
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

int attention_decode(const float* q, const float* kc, const float* vc, float* out, int H,
                     int Hkv, int HD, int max_seq, int pos, float scale, float* part,
                     cudaStream_t st, const int* pos_dev, bool pdl) {
    const int G = H / Hkv;
    const bool fast = fast_ok(H, Hkv, HD) && ((uintptr_t)q % 16 == 0) &&
                      ((uintptr_t)kc % 16 == 0) && ((uintptr_t)vc % 16 == 0);
    const int ch = fast ? ATT_CH_FAST : ATT_CH_GENERIC;
    // with pos_dev the grid covers the whole cache and chunks past *pos_dev exit
    const int n_chunks = pos_dev ? (max_seq + ch - 1) / ch : pos / ch + 1;
    const dim3 grid(Hkv, n_chunks);
    if (fast) {
        auto kern = G <= 1 ? attn_partial_fast_kernel<1> : G <= 2 ? attn_partial_fast_kernel<2> :
                    G <= 4 ? attn_partial_fast_kernel<4> : attn_partial_fast_kernel<8>;
        IB_CUDA_CHECK(launch_pdl(kern, grid, dim3(128), 0, st, pdl, q, kc, vc, part, H, Hkv, HD,
                                 max_seq, pos, scale, n_chunks, pos_dev));
    } else {
        const size_t smem = (size_t)(G * HD + G * ATT_CH_GENERIC) * sizeof(float);
        IB_CUDA_CHECK(launch_pdl(attn_partial_generic_kernel, grid, dim3(128), smem, st, pdl, q,
                                 kc, vc, part, H, Hkv, HD, max_seq, pos, scale, n_chunks, pos_dev));
    }
    IB_LAUNCH_CHECK("attention_partial_kernel");
    IB_CUDA_CHECK(launch_pdl(attn_combine_kernel, dim3(H), dim3(128), 0, st, pdl, part, out, HD,
                             n_chunks, ch, pos / ch + 1, pos_dev));
    IB_LAUNCH_CHECK("attention_combine_kernel");
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

}  // namespace ib
