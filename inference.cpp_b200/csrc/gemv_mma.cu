// Fused dequant + GEMV on GGUF blocks (batch-1 decode; HBM-bound), sm_100a.
//
// Data movement: a CTA owns 16 consecutive rows.  A producer warp streams the
// rows' packed bytes with 1-D TMA bulk copies (cp.async.bulk, no multicast) into
// a ring of S shared-memory stages, one 16-row x KB-block slice per stage,
// guarded by mbarriers (full: transaction bytes; empty: one arrival per consumer
// warp).  The bytes in flight are set by the ring, not by registers or occupancy.
// Rows that do not start on a 16-byte boundary are copied from the boundary below
// (row slots 16 bytes longer, per-row offsets); the last stage of a row may hold
// fewer blocks.  Only a weight base that is not 16-byte aligned takes direct global
// loads.
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

#include <mutex>

#include "common.cuh"
#include "gemv_math.cuh"
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
// partials behind a named barrier (double-buffered, so one barrier per group).  `slot`
// is the row stride in a stage: CHUNK, or CHUNK + 16 when rows do not start on 16-byte
// boundaries (a row is then copied from the boundary below it, at the same offset in
// every stage, since CHUNK is a multiple of 16).  GEN: such rows, or rows whose length
// is not a whole number of stages; the instantiation without it keeps the aligned case
// free of the per-row offsets and lengths.
template <int TYPE, int NWC, int S, bool GEN>
__global__ void __launch_bounds__((NWC + 1) * 32) gemv_tma_kernel(const uint8_t* __restrict__ W,
                                                                 XLimbs xb, float* __restrict__ y,
                                                                 int rows, int nb, int slot) {
    using F = Fmt<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];  // [S][16][slot]
    __shared__ __align__(8) uint64_t full[S], empty[S];
    __shared__ float red[2][NWC][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_rg = (rows + 15) / 16;
    const int my_rg = blockIdx.x < n_rg ? (n_rg - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int spg = GEN ? (nb + F::KB - 1) / F::KB : nb / F::KB;  // stages per row group
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
            const uint8_t* src = W + (size_t)(row_base + min(lane, n - 1)) * rbytes;
            uint32_t off = 0, len = F::CHUNK, tot = (uint32_t)(n * F::CHUNK);
            if (GEN) {
                const int nbl = min(F::KB, nb - st * F::KB);
                off = (uint32_t)((uintptr_t)src & 15u);
                len = lane < n ? (off + (uint32_t)(nbl * F::BB) + 15u) & ~15u : 0u;
                tot = len;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
            }
            if (lane == 0) mbar_arrive_expect_tx(&full[s], tot);
            __syncwarp();
            if (lane < n)
                bulk_g2s(smem + ((size_t)s * 16 + lane) * (GEN ? slot : F::CHUNK),
                         src - off + (size_t)st * F::CHUNK, len, &full[s]);
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
            int oa = 0, ob = 0;
            if (GEN) {
                oa = (int)((uintptr_t)(W + (size_t)(row_base + ra) * rbytes) & 15u);
                ob = (int)((uintptr_t)(W + (size_t)(row_base + rb) * rbytes) & 15u);
            }
            const uint8_t* sa = smem + ((size_t)s * 16 + ra) * (GEN ? slot : F::CHUNK) + oa;
            const uint8_t* sb = smem + ((size_t)s * 16 + rb) * (GEN ? slot : F::CHUNK) + ob;
            const int nbl = nb - st * F::KB;
            if (!GEN || nbl >= F::KB) {
#pragma unroll
                for (int kbl = warp * F::UNIT; kbl < F::KB; kbl += NWC * F::UNIT)
                    block_math<TYPE, true>(sa + kbl * F::BB, sb + kbl * F::BB, st * F::KB + kbl,
                                           nb, xb, c, acc_a, acc_b);
            } else {
                for (int kbl = warp * F::UNIT; kbl < nbl; kbl += NWC * F::UNIT)
                    block_math<TYPE, true>(sa + kbl * F::BB, sb + kbl * F::BB, st * F::KB + kbl,
                                           nb, xb, c, acc_a, acc_b);
            }
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

// Per-device launch set-up of each format's kernels: the shared-memory opt-in and the
// occupancy of the TMA kernel, and the function attributes of the direct-load kernel
// (which also makes the runtime load a lazily loaded module).  Done once per (device,
// format) under a mutex, so concurrent first calls from several host threads are safe.
constexpr int kSetupDevices = 64;
static std::mutex g_setup_mu;
static uint64_t g_setup_done[kSetupDevices];  // bit fmt_slot(TYPE) per device
static int g_max_ctas[kSetupDevices][6][2];  // [.][.][general instantiation]

template <int TYPE>
constexpr int fmt_slot() {
    return TYPE == IB_TYPE_Q4_K ? 0 : TYPE == IB_TYPE_Q6_K ? 1 : TYPE == IB_TYPE_Q4_0 ? 2
         : TYPE == IB_TYPE_Q5_0 ? 3 : TYPE == IB_TYPE_Q5_1 ? 4 : 5;
}

template <int TYPE>
constexpr int ring_stages() {
    return TYPE == IB_TYPE_Q6_K ? 2 : (TYPE == IB_TYPE_Q8_0 ? 3 : 4);
}

template <int TYPE>
constexpr size_t ring_bytes(bool pad) {
    return (size_t)ring_stages<TYPE>() * 16 * (Fmt<TYPE>::CHUNK + (pad ? 16 : 0));
}

// With g_setup_mu held: the set-up of TYPE on device dev; cap[gen] = resident CTAs of
// the aligned / general TMA kernel.
template <int TYPE>
static int setup_typed_locked(int dev, int* cap) {
    constexpr int NWC = 8, S = ring_stages<TYPE>(), slot = fmt_slot<TYPE>();
    if (!(g_setup_done[dev] & (1ull << slot))) {
        int sms = 0;
        IB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        for (int gen = 0; gen < 2; ++gen) {
            auto kern = gen ? gemv_tma_kernel<TYPE, NWC, S, true> : gemv_tma_kernel<TYPE, NWC, S, false>;
            const size_t smem = ring_bytes<TYPE>(gen != 0);  // the general case: padded rows
            if (smem + 2048 > 48 * 1024)
                IB_CUDA_CHECK(cudaFuncSetAttribute(
                    kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            int per_sm = 0;
            IB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern,
                                                                        (NWC + 1) * 32, smem));
            g_max_ctas[dev][slot][gen] = (per_sm > 0 ? per_sm : 1) * sms;
        }
        cudaFuncAttributes fa;
        IB_CUDA_CHECK(cudaFuncGetAttributes(&fa, gemv_direct_kernel<TYPE, 8>));
        g_setup_done[dev] |= 1ull << slot;
    }
    cap[0] = g_max_ctas[dev][slot][0];
    cap[1] = g_max_ctas[dev][slot][1];
    return IB_OK;
}

static int current_device(int* dev) {
    IB_CUDA_CHECK(cudaGetDevice(dev));
    IB_REQUIRE(*dev >= 0 && *dev < kSetupDevices, "gemv: device ordinal out of range");
    return IB_OK;
}

template <int TYPE>
static int launch_typed(const uint8_t* W, const XLimbs& xb, float* y, int64_t rows, int64_t cols,
                        cudaStream_t st) {
    using F = Fmt<TYPE>;
    constexpr int NWC = 8;
    constexpr int S = ring_stages<TYPE>();
    const int nb = (int)(cols / (F::K ? 256 : 32));
    const int n_rg = (int)((rows + 15) / 16);
    const bool pad = (size_t)nb * F::BB % 16 != 0;
    const bool gen = pad || nb % F::KB != 0;
    if (((uintptr_t)W & 15) == 0) {
        const size_t smem = ring_bytes<TYPE>(pad);
        int dev = 0, cap[2] = {0, 0}, r;
        if ((r = current_device(&dev))) return r;
        {
            std::lock_guard<std::mutex> lock(g_setup_mu);
            if ((r = setup_typed_locked<TYPE>(dev, cap))) return r;
        }
        // as many CTAs as fit, but dividing the row groups evenly
        const int per = (n_rg + cap[gen] - 1) / cap[gen];
        const int grid = (n_rg + per - 1) / per;
        auto kern = gen ? gemv_tma_kernel<TYPE, NWC, S, true> : gemv_tma_kernel<TYPE, NWC, S, false>;
        kern<<<grid, (NWC + 1) * 32, smem, st>>>(W, xb, y, (int)rows, nb,
                                                 F::CHUNK + (pad ? 16 : 0));
        IB_LAUNCH_CHECK("gemv_tma_kernel");
        return IB_OK;
    }
    gemv_direct_kernel<TYPE, 8><<<(unsigned)n_rg, 256, 0, st>>>(W, xb, y, (int)rows, nb);
    IB_LAUNCH_CHECK("gemv_direct_kernel");
    return IB_OK;
}

int gemv_mma_prepare_device() {
    int dev = 0, cap[2] = {0, 0}, r;
    if ((r = current_device(&dev))) return r;
    cudaFuncAttributes fa;
    IB_CUDA_CHECK(cudaFuncGetAttributes(&fa, xq_kernel));
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if ((r = setup_typed_locked<IB_TYPE_Q4_K>(dev, cap))) return r;
    if ((r = setup_typed_locked<IB_TYPE_Q6_K>(dev, cap))) return r;
    if ((r = setup_typed_locked<IB_TYPE_Q4_0>(dev, cap))) return r;
    if ((r = setup_typed_locked<IB_TYPE_Q5_0>(dev, cap))) return r;
    if ((r = setup_typed_locked<IB_TYPE_Q5_1>(dev, cap))) return r;
    return setup_typed_locked<IB_TYPE_Q8_0>(dev, cap);
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
