// Prefill GEMM on dequantised planes: Y[T, rows] = X[T, cols] . W^T, for prompts long
// enough that re-dequantising a weight tile per token tile would dominate.
//
// gemm_tc.cu dequantises each 128-row weight tile again for every 128-token tile (16
// times at T = 2048).  Here the packed blocks are decoded once per call into two FP16
// planes W = Wh + Wl (hi = fp16(w), lo = fp16(w - hi); the bit-exact element
// expressions of quant.cuh), next to X's planes (split_x_kernel), and a pure tensor-core
// GEMM consumes them:
//   producer warp   one thread issues, per 32-column step, four 2-D TMA tile loads
//                   (cp.async.bulk.tensor, 64-byte swizzle, no multicast) into a
//                   four-stage ring: Wh, Wl (128 rows) and Xh, Xl (256 tokens),
//                   completing on the stage's
//                   mbarrier; rows and tokens past the edges are filled with zeros
//   MMA warp        one thread issues per 16-column slice tcgen05.mma kind::f16
//                   M 128 x N 256 for Wh.Xh + Wh.Xl + Wl.Xh into an FP32 accumulator of
//                   128 lanes x 256 columns in tensor memory, and tcgen05.commit frees
//                   the stage
//   epilogue warps  four warps read the accumulator (tcgen05.ld, warp w owns lanes
//                   32 (w % 4)..) and store Y with coalesced rows
// Accuracy is that of gemm_tc.cu: each product keeps about 2^-21 of its value (the
// dropped Wl.Xl term is below 2^-22).  Every mbarrier wait is bounded and records a
// fault code; the MMA thread always ends with the commit the epilogue waits for, so the
// accumulator is released only after the last MMA.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "ops.cuh"
#include "pipeline.cuh"
#include "quant.cuh"

namespace ib {

static __device__ int g_gemm_tma_fault;

constexpr int TM_M = 128;   // weight rows per tile (MMA M)
constexpr int TM_N = 256;   // tokens per tile (MMA N)
constexpr int TM_BK = 32;   // columns per stage: one 64-byte swizzle row of fp16
constexpr int TM_STAGES = 4;
constexpr int TM_A = TM_M * TM_BK * 2;  // 8 KB
constexpr int TM_B = TM_N * TM_BK * 2;  // 16 KB
constexpr int TM_STAGE = 2 * TM_A + 2 * TM_B;
constexpr int TM_THREADS = 6 * 32;      // producer, MMA, four epilogue warps
constexpr size_t TM_SMEM = (size_t)TM_STAGES * TM_STAGE + 1024;

// ---- weights -> FP16 hi/lo planes -----------------------------------------------------
template <int TYPE>
__global__ void __launch_bounds__(256) dequant_planes_kernel(const uint8_t* __restrict__ W,
                                                             __half* __restrict__ Wh,
                                                             __half* __restrict__ Wl,
                                                             int64_t n8, int64_t cols) {
    constexpr int BE = QFmt<TYPE>::BE, BB = QFmt<TYPE>::BB;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = i * 8, blk = e / BE;  // rows are whole blocks: e indexes the blocks
        float v[8];
        deq8<TYPE>(W + blk * BB, (int)((e % BE) >> 3), v);
        uint32_t h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half h0 = __float2half_rn(v[2 * k]), h1 = __float2half_rn(v[2 * k + 1]);
            const __half l0 = __float2half_rn(v[2 * k] - __half2float(h0));
            const __half l1 = __float2half_rn(v[2 * k + 1] - __half2float(h1));
            h[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            l[k] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        reinterpret_cast<uint4*>(Wh)[i] = make_uint4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<uint4*>(Wl)[i] = make_uint4(l[0], l[1], l[2], l[3]);
    }
    (void)cols;
}

// ---- tcgen05 / TMA building blocks ------------------------------------------------------
__device__ __forceinline__ void tm_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tm_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major tile, 64-byte swizzle (layout type 4), 8-row groups 512 bytes apart, sm_100
// descriptor (version 1).
__device__ __forceinline__ uint64_t tm_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// kind::f16: D FP32, A and B FP16, both K-major, M x N.
constexpr uint32_t tm_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tm_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

__device__ __forceinline__ void tm_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tm_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
          "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
          "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D tiled TMA load (no multicast) of the box at (x = column, y = row) into shared
// memory, completing on bar.  x is a multiple of 32 fp16 (64 bytes).
__device__ __forceinline__ void tma_load2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                           uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Work of CTA b (one-dimensional grid): b < n_full is the whole tile b (token tiles vary
// fastest); the rest are `split` parts along K of each tile of the last, partly filled
// wave, whose FP32 partial tiles go to `part` ([tail tile][part][token][row]) for
// gemm_tail_reduce_kernel.  Splitting the tail keeps every SM busy to the end: 896
// tiles on 148 SMs are six full waves and 8 tiles, which would hold one wave alone.
struct TmWork {
    int n_ntiles;  // token tiles per row tile
    int n_full;    // tiles computed whole
    int split;     // parts per tail tile (1: no tail split)
    int kps;       // k-steps per part
    float* part;
};

__global__ void __launch_bounds__(TM_THREADS, 1)
    gemm_planes_kernel(const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                       const __grid_constant__ CUtensorMap mXh, const __grid_constant__ CUtensorMap mXl,
                       float* __restrict__ Y, int T, int rows, int cols, const TmWork wk) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[TM_STAGES], empty[TM_STAGES], acc_full;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // token tiles vary fastest: the CTAs resident together share weight strips (each
    // strip's planes come from DRAM once and serve every token tile from L2), and the
    // X planes (2 x T x cols x 2 bytes) stay in L2
    const int b = (int)blockIdx.x;
    const bool is_part = b >= wk.n_full;
    const int tail = is_part ? (b - wk.n_full) / wk.split : 0;
    const int pi = is_part ? (b - wk.n_full) - tail * wk.split : 0;
    const int tile = is_part ? wk.n_full + tail : b;
    const int n0 = (tile % wk.n_ntiles) * TM_N, m0 = (tile / wk.n_ntiles) * TM_M;
    const int n_k_all = cols / TM_BK;
    const int k_begin = is_part ? pi * wk.kps : 0;
    const int k_end = is_part ? min(n_k_all, k_begin + wk.kps) : n_k_all;
    const int n_k = k_end - k_begin;  // >= 1: the host sizes the parts
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    if (threadIdx.x == 0) {
        for (int s = 0; s < TM_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) {  // accumulator: 128 lanes x 256 FP32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base)),
                     "r"(TM_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tm_fence_before();
    __syncthreads();
    tm_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mWh)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mXh)) : "memory");
            int issued = 0;
            for (int kt = 0; kt < n_k; ++kt) {
                const int s = kt % TM_STAGES, u = kt / TM_STAGES;
                if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1, &g_gemm_tma_fault, 41)) break;
                const uint32_t st = base + (uint32_t)(s * TM_STAGE);
                mbar_arrive_expect_tx(&full[s], (uint32_t)TM_STAGE);
                const int k0 = (k_begin + kt) * TM_BK;
                tma_load2d(st, &mWh, k0, m0, &full[s]);
                tma_load2d(st + TM_A, &mWl, k0, m0, &full[s]);
                tma_load2d(st + 2 * TM_A, &mXh, k0, n0, &full[s]);
                tma_load2d(st + 2 * TM_A + TM_B, &mXl, k0, n0, &full[s]);
                issued = kt + 1;
            }
            // every issued copy lands before the CTA can end
            for (int j = issued > TM_STAGES ? issued - TM_STAGES : 0; j < issued; ++j)
                mbar_wait(&full[j % TM_STAGES], (j / TM_STAGES) & 1, &g_gemm_tma_fault, 42);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tm_idesc(TM_M, TM_N);
            for (int kt = 0; kt < n_k; ++kt) {
                const int s = kt % TM_STAGES, u = kt / TM_STAGES;
                if (!mbar_wait(&full[s], u & 1, &g_gemm_tma_fault, 43)) break;
                tm_fence_after();
                const uint32_t st = base + (uint32_t)(s * TM_STAGE);
#pragma unroll
                for (int kk = 0; kk < TM_BK / 16; ++kk) {
                    const uint32_t off = (uint32_t)kk * 32;  // 16 fp16 columns
                    const uint64_t ah = tm_desc(st + off), al = tm_desc(st + TM_A + off);
                    const uint64_t bh = tm_desc(st + 2 * TM_A + off);
                    const uint64_t bl = tm_desc(st + 2 * TM_A + TM_B + off);
                    tm_mma(tmem, ah, bh, idesc, (kt | kk) != 0);  // kt counts from k_begin
                    tm_mma(tmem, ah, bl, idesc, 1u);
                    tm_mma(tmem, al, bh, idesc, 1u);
                }
                tm_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            tm_commit(&acc_full);  // completes after every MMA issued above
        }
        __syncwarp();
    } else {
        // epilogue: TMEM lanes 32 (warp % 4) .. are tile rows; 32 columns (tokens) per load
        const bool have = __all_sync(0xffffffffu, mbar_wait(&acc_full, 0, &g_gemm_tma_fault, 44));
        tm_fence_after();
        if (have) {
            const int q = warp & 3, orow = m0 + 32 * q + lane;
            float* pt = is_part ? wk.part + ((size_t)(tail * wk.split + pi) * TM_N) * TM_M : nullptr;
            for (int c0 = 0; c0 < TM_N; c0 += 32) {
                if (n0 + c0 >= T) break;  // warp-uniform
                uint32_t v[32];
                tm_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
                if (is_part) {  // the whole partial tile, rows contiguous
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        pt[(size_t)(c0 + jj) * TM_M + 32 * q + lane] = __uint_as_float(v[jj]);
                } else if (orow < rows) {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        const int t = n0 + c0 + jj;
                        if (t < T) Y[(size_t)t * rows + orow] = __uint_as_float(v[jj]);
                    }
                }
            }
        }
    }
    tm_fence_before();
    __syncthreads();
    if (warp == 1) {
        tm_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TM_N)
                     : "memory");
    }
}

// Y <- the sum of each tail tile's parts, in part order (deterministic).
__global__ void gemm_tail_reduce_kernel(const float* __restrict__ part, float* __restrict__ Y,
                                        int T, int rows, int n_ntiles, int n_full, int n_tail,
                                        int split) {
    const int64_t per = (int64_t)TM_N * TM_M;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)n_tail * per;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / per);
        const int rem = (int)(i - (int64_t)t * per), c = rem / TM_M, r = rem - c * TM_M;
        const int tile = n_full + t;
        const int tok = (tile % n_ntiles) * TM_N + c, row = (tile / n_ntiles) * TM_M + r;
        if (tok >= T || row >= rows) continue;
        const float* p = part + ((size_t)t * split * TM_N + c) * TM_M + r;
        float acc = 0.f;
        for (int k = 0; k < split; ++k) acc += p[(size_t)k * per];
        Y[(size_t)tok * rows + row] = acc;
    }
}

// ---- host side --------------------------------------------------------------------------
static int tensor_map_2d(CUtensorMap* map, const void* base, int64_t inner, int64_t outer,
                         int box_outer) {
    static PFN_cuTensorMapEncodeTiled encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = (PFN_cuTensorMapEncodeTiled)fn;
    });
    if (!encode) {
        set_error("gemm: cuTensorMapEncodeTiled is not available");
        return IB_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TM_BK, (cuuint32_t)box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("gemm: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
        return IB_ERR_CUDA;
    }
    return IB_OK;
}

template <int TYPE>
static int planes_for(const void* W, __half* Wh, __half* Wl, int64_t rows, int64_t cols,
                      cudaStream_t st) {
    const int64_t n8 = rows * cols / 8;
    const int g = (int)((n8 + 255) / 256 < 8192 ? (n8 + 255) / 256 : 8192);
    dequant_planes_kernel<TYPE><<<g, 256, 0, st>>>((const uint8_t*)W, Wh, Wl, n8, cols);
    IB_LAUNCH_CHECK("dequant_planes_kernel");
    return IB_OK;
}

bool gemm_planes_supported(int type, int64_t T, int64_t rows, int64_t cols) {
    return is_quant(type) && T >= 1 && rows >= 1 && cols % TM_BK == 0 &&
           T * cols < (1ll << 31) && rows * cols < (1ll << 34) &&
           (rows + TM_M - 1) / TM_M <= 65535;
}

int gemm_decode_planes(int type, const void* W, void* planes, int64_t rows, int64_t cols,
                       cudaStream_t st) {
    __half* Wh = (__half*)planes;
    __half* Wl = Wh + (size_t)rows * cols;
    switch (type) {
        case IB_TYPE_Q4_0: return planes_for<IB_TYPE_Q4_0>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q5_0: return planes_for<IB_TYPE_Q5_0>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q5_1: return planes_for<IB_TYPE_Q5_1>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q8_0: return planes_for<IB_TYPE_Q8_0>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q4_K: return planes_for<IB_TYPE_Q4_K>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q6_K: return planes_for<IB_TYPE_Q6_K>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q4_1: return planes_for<IB_TYPE_Q4_1>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q2_K: return planes_for<IB_TYPE_Q2_K>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q3_K: return planes_for<IB_TYPE_Q3_K>(W, Wh, Wl, rows, cols, st);
        case IB_TYPE_Q5_K: return planes_for<IB_TYPE_Q5_K>(W, Wh, Wl, rows, cols, st);
    }
    set_error("gemm: unsupported type");
    return IB_ERR_UNSUPPORTED;
}

int gemm_on_planes(const void* planes, const float* X, float* Y, int T, int rows, int cols,
                   cudaStream_t st) {
    IB_REQUIRE(planes && ((uintptr_t)planes & 15) == 0, "gemm: weight planes must be 16-byte aligned");
    IB_REQUIRE(T >= 1 && rows >= 1 && cols % TM_BK == 0 && (int64_t)T * cols < (1ll << 31) &&
                   (int64_t)rows * cols < (1ll << 34) && (rows + TM_M - 1) / TM_M <= 65535,
               "gemm: shape not supported by the planes kernel");
    const size_t nx = (size_t)T * cols, nw = (size_t)rows * cols;
    void* wsx = nullptr;
    int r = workspace_get(WS_GEMM, 2 * nx * sizeof(__half) + 256, &wsx);
    if (r) return r;
    __half* Xh = (__half*)wsx;
    __half* Xl = Xh + nx;
    const __half* Wh = (const __half*)planes;
    const __half* Wl = Wh + nw;
    if ((r = gemm_split_x(X, Xh, Xl, nx, st))) return r;
    CUtensorMap mWh, mWl, mXh, mXl;
    if ((r = tensor_map_2d(&mWh, Wh, cols, rows, TM_M))) return r;
    if ((r = tensor_map_2d(&mWl, Wl, cols, rows, TM_M))) return r;
    if ((r = tensor_map_2d(&mXh, Xh, cols, T, TM_N))) return r;
    if ((r = tensor_map_2d(&mXl, Xl, cols, T, TM_N))) return r;
    static std::mutex mu;
    static bool attr_set[64] = {};
    static int n_sm[64] = {};
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 0 || dev >= 64) {
            set_error("gemm: device ordinal out of range");
            return IB_ERR_INVALID;
        }
        if (!attr_set[dev]) {
            IB_CUDA_CHECK(cudaFuncSetAttribute(gemm_planes_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TM_SMEM));
            IB_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev));
            attr_set[dev] = true;
        }
    }
    // the last wave: when it is at most half full, its tiles are split along K so that
    // every SM has work to the end (one CTA per SM)
    const int n_ntiles = (T + TM_N - 1) / TM_N, n_mtiles = (rows + TM_M - 1) / TM_M;
    const int64_t n_tiles = (int64_t)n_ntiles * n_mtiles;
    const int n_k = cols / TM_BK, sms = n_sm[dev];
    const int tail = (int)(n_tiles % sms);
    TmWork wk{n_ntiles, (int)n_tiles, 1, n_k, nullptr};
    if (n_tiles > sms && tail > 0 && 2 * tail <= sms && n_k >= 8) {
        int split = sms / tail;
        if (split > n_k / 4) split = n_k / 4;  // parts of four k-steps at least
        const int kps = (n_k + split - 1) / split;
        split = (n_k + kps - 1) / kps;        // every part non-empty
        if (split >= 2) {
            void* wp = nullptr;
            if ((r = workspace_get(WS_GEMM_PART, (size_t)tail * split * TM_N * TM_M * 4, &wp)))
                return r;
            wk = TmWork{n_ntiles, (int)(n_tiles - tail), split, kps, (float*)wp};
        }
    }
    const int64_t grid = wk.split > 1 ? wk.n_full + (int64_t)tail * wk.split : n_tiles;
    IB_REQUIRE(grid <= 0x7FFFFFFF, "gemm: too many tiles");
    gemm_planes_kernel<<<(unsigned)grid, TM_THREADS, TM_SMEM, st>>>(mWh, mWl, mXh, mXl, Y, T, rows,
                                                                   cols, wk);
    IB_LAUNCH_CHECK("gemm_planes_kernel");
    if (wk.split > 1) {
        const int64_t n = (int64_t)tail * TM_N * TM_M;
        gemm_tail_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
            wk.part, Y, T, rows, n_ntiles, wk.n_full, tail, wk.split);
        IB_LAUNCH_CHECK("gemm_tail_reduce_kernel");
    }
    return IB_OK;
}

int gemm_q_planes(int type, const void* W, const float* X, float* Y, int T, int rows, int cols,
                  cudaStream_t st) {
    IB_REQUIRE(gemm_planes_supported(type, T, rows, cols), "gemm: shape not supported by the planes kernel");
    const size_t nw = (size_t)rows * cols;
    void* wsw = nullptr;
    int r = workspace_get(WS_GEMM_W, 2 * nw * sizeof(__half) + 256, &wsw);
    if (r) return r;
    if ((r = gemm_decode_planes(type, W, wsw, rows, cols, st))) return r;
    return gemm_on_planes(wsw, X, Y, T, rows, cols, st);
}

int gemm_planes_fault_take(int* code) {
    int v = 0, z = 0;
    IB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_gemm_tma_fault, sizeof(int)));
    if (v) IB_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_tma_fault, &z, sizeof(int)));
    *code = v;
    return IB_OK;
}

}  // namespace ib

using namespace ib;

extern "C" size_t ib_gemm_planes_bytes(int64_t rows, int64_t cols) {
    return rows > 0 && cols > 0 ? (size_t)rows * cols * 4 : 0;
}

extern "C" int ib_gemm_prepare_planes(int type, const void* dev_W, int64_t rows, int64_t cols,
                                      void* dev_planes, void* stream) {
    IB_REQUIRE(dev_W && dev_planes && rows > 0 && cols > 0, "bad arguments");
    IB_REQUIRE(gemm_planes_supported(type, 1, rows, cols), "gemm: shape not supported by the planes kernel");
    IB_REQUIRE(((uintptr_t)dev_planes & 15) == 0, "gemm: weight planes must be 16-byte aligned");
    return gemm_decode_planes(type, dev_W, dev_planes, rows, cols, as_stream(stream));
}

extern "C" int ib_gemm_planes(const void* dev_planes, const float* dev_X, float* dev_Y, int64_t T,
                              int64_t rows, int64_t cols, void* stream) {
    IB_REQUIRE(dev_planes && dev_X && dev_Y, "null pointer argument");
    if (T == 0 || rows == 0) return IB_OK;
    IB_REQUIRE(T > 0 && rows > 0 && cols > 0 && T < (1ll << 31) && rows < (1ll << 31) &&
                   cols < (1ll << 31),
               "bad shape");
    return gemm_on_planes(dev_planes, dev_X, dev_Y, (int)T, (int)rows, (int)cols,
                          as_stream(stream));
}
