// Prefill GEMM on the 5th-generation tensor cores: Y[T, rows] = X[T, cols] . W^T with W
// in its packed GGUF blocks -- the B200 counterpart of the reference's batched GPU
// matmul (src/ops/cuda_backend.cpp gemm kernels, called from prefill in
// src/models/model_cuda.cpp:293-368).
//
// Tile: 128 weight rows (MMA M) x 128 tokens (MMA N), K in steps of 64.  Sixteen
// producer warps stage, per 256 columns, the tile rows' packed blocks in shared memory
// with coalesced 16-byte loads; per 64-column step they dequantise them (the
// bit-exact element expressions of quant.cuh) and copy the 128 tokens x 64 columns of
// X, each value split into an FP16 pair v = hi + lo (hi = fp16(v), lo = fp16(v - hi)),
// into 128-byte-swizzled K-major tiles.  One thread issues, per 16-column slice,
// tcgen05.mma kind::f16 for hi.hi + hi.lo + lo.hi into an FP32 accumulator of 128
// lanes x 128 columns in tensor memory, and tcgen05.commit releases the stage to the
// producers.  The three products keep each term to about 2^-21 of its value, so the
// GEMM matches an FP32 matmul to rounding (the dropped lo.lo term is below 2^-22).
// The epilogue warps read the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32(w%4).. = tile rows, columns 32(w/4)..) and store Y.  Every mbarrier wait is
// bounded (fault word, as in the other pipelines) and the producers' named barriers
// are reached by every producer on every step whatever failed; the MMA thread always
// ends with a commit the epilogue waits for, so tensor memory is released only after
// the last MMA has finished.
#include <cuda_fp16.h>

#include <string>

#include "common.cuh"
#include "ops.cuh"
#include "pipeline.cuh"
#include "quant.cuh"

namespace ib {

static __device__ int g_gemm_fault;

constexpr int TC_M = 128;      // weight rows per tile (MMA M)
constexpr int TC_N = 128;      // tokens per tile (MMA N)
constexpr int TC_BK = 64;      // columns per stage (one 128-byte swizzle row of fp16)
constexpr int TC_SEGC = 256;   // columns per staged run of packed blocks
constexpr int TC_STAGES = 2;
constexpr int TC_TILE = TC_M * TC_BK * 2;  // bytes of one fp16 operand tile (16 KB)
constexpr int TC_STAGE = 4 * TC_TILE;      // A hi, A lo, B hi, B lo
constexpr int TC_PROD = 512;               // producer / epilogue threads (16 warps)
constexpr int TC_THREADS = TC_PROD + 32;   // + the MMA warp
static_assert(TC_PROD % 128 == 0 && 2048 % TC_PROD == 0, "producer mapping");

// Packed bytes of 256 columns of a row, and their row stride in shared memory (16 x an
// odd number, so 16-byte loads of 8 consecutive rows hit distinct bank groups; Q6_K's
// 210-byte runs start 2-byte aligned and are staged from the 16-byte boundary below).
template <int TYPE>
struct RawSeg {
    static constexpr int BE = (TYPE == IB_TYPE_Q4_K || TYPE == IB_TYPE_Q6_K) ? 256 : 32;
    static constexpr int BB = TYPE == IB_TYPE_Q4_0 ? 18 : TYPE == IB_TYPE_Q5_0 ? 22 :
                              TYPE == IB_TYPE_Q5_1 ? 24 : TYPE == IB_TYPE_Q8_0 ? 34 :
                              TYPE == IB_TYPE_Q4_K ? 144 : 210;
    static constexpr int SEG = TC_SEGC / BE * BB;
    static constexpr int NCH = (SEG + 15) / 16 + (SEG % 16 ? 1 : 0);  // chunks, worst case
    static constexpr int RS = ((NCH & 1) ? NCH : NCH + 1) * 16;
};

template <int TYPE>
constexpr size_t tc_smem_bytes() {  // fp16 stages, two staged runs, alignment slack
    return (size_t)TC_STAGES * TC_STAGE + 2 * (size_t)TC_M * RawSeg<TYPE>::RS + 1024;
}

// ---- tcgen05 building blocks (inline PTX) ----------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes
// apart (leading offset unused for this layout, 1 by convention), sm_100 version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D FP32, A and B FP16, both K-major, M x N.
constexpr uint32_t tc_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 consecutive FP32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
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

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Eight FP32 values -> their FP16 hi/lo pairs (two 16-byte chunks).
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half h0 = __float2half_rn(v[2 * i]), h1 = __float2half_rn(v[2 * i + 1]);
        const __half l0 = __float2half_rn(v[2 * i] - __half2float(h0));
        const __half l1 = __float2half_rn(v[2 * i + 1] - __half2float(h1));
        h[i] = pack_h2(h0, h1);
        l[i] = pack_h2(l0, l1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// 16-byte asynchronous copy global -> shared (zero-filled when !valid); completion is
// tracked through cp_async_arrive on an mbarrier.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}

// Arrives on bar once every cp.async this thread issued so far has landed (the arrival
// is counted in the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ---- 16-element decoders for blocks staged in shared memory --------------------------
// The element expressions are deq8's (bit-exact); the bytes come from 16-byte loads.

// Byte k of the 12 scale bytes held in three words.
__device__ __forceinline__ int scale_byte(uint32_t s0, uint32_t s1, uint32_t s2, int k) {
    const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
    return (int)((w >> (8 * (k & 3))) & 0xFFu);
}

// Q4_K elements e0..e0+15 (e0 % 16 == 0) of a 16-byte-aligned block.
__device__ __forceinline__ void deq16_q4k(const uint8_t* blk, int e0, float* y) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);  // d, dmin, scales[12]
    const int sb = e0 >> 5, p = sb >> 1, h = sb & 1, l0 = e0 & 31;
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * p + l0);
    const float d = h2f(hd.x & 0xFFFFu), dmin = h2f(hd.x >> 16);
    int sc, m;  // get_scale_min_k4(sb)
    if (sb < 4) {
        sc = scale_byte(hd.y, hd.z, hd.w, sb) & 63;
        m = scale_byte(hd.y, hd.z, hd.w, sb + 4) & 63;
    } else {
        sc = (scale_byte(hd.y, hd.z, hd.w, sb + 4) & 0xF) | ((scale_byte(hd.y, hd.z, hd.w, sb - 4) >> 6) << 4);
        m = (scale_byte(hd.y, hd.z, hd.w, sb + 4) >> 4) | ((scale_byte(hd.y, hd.z, hd.w, sb) >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int v = (int)((w[i >> 2] >> (8 * (i & 3) + 4 * h)) & 0xFu);
        y[i] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
    }
}

// 16 bytes at byte offset off (even) of a 16-byte-aligned staged row, as four words;
// the offset's position within 16 bytes is the same for every thread of the warp.
__device__ __forceinline__ void lds16_at(const uint8_t* row, int off, uint32_t (&o)[4]) {
    const int a = off & ~15, sh = off & 15;
    const uint4 x = *reinterpret_cast<const uint4*>(row + a);
    const uint4 z = *reinterpret_cast<const uint4*>(row + a + 16);
    const uint32_t w[8] = {x.x, x.y, x.z, x.w, z.x, z.y, z.z, z.w};
    const uint32_t bs = (uint32_t)(sh & 3) * 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t lo, hi;
        switch (sh >> 2) {  // warp-uniform
            case 0: lo = w[k]; hi = w[k + 1]; break;
            case 1: lo = w[k + 1]; hi = w[k + 2]; break;
            case 2: lo = w[k + 2]; hi = w[k + 3]; break;
            default: lo = w[k + 3]; hi = w[k + 4]; break;
        }
        o[k] = __funnelshift_r(lo, hi, bs);
    }
}

// Q6_K elements e0..e0+15 (e0 % 16 == 0) of the block at byte offset o (even, < 16)
// of a 16-byte-aligned staged row.
__device__ __forceinline__ void deq16_q6k(const uint8_t* row, int o, int e0, float* y) {
    const int c = e0 >> 7, r = e0 & 127, gg = r >> 5, l0 = r & 31;
    uint32_t ql[4], qh[4];
    lds16_at(row, o + 64 * c + 32 * (gg & 1) + l0, ql);
    lds16_at(row, o + 128 + 32 * c + l0, qh);
    const float d = h2f(*reinterpret_cast<const unsigned short*>(row + o + 208));
    const int sc = (int)(int8_t)row[o + 192 + 8 * c + 2 * gg + (l0 >> 4)];
    const float ds = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int lo = (int)((ql[i >> 2] >> (8 * (i & 3) + 4 * (gg >> 1))) & 0xFu);
        const int hi = (int)((qh[i >> 2] >> (8 * (i & 3) + 2 * gg)) & 3u);
        const int q = (int)(int8_t)(lo | (hi << 4)) - 32;
        y[i] = __fmul_rn(ds, (float)q);
    }
}

__device__ __forceinline__ void bar_producers() {
    asm volatile("bar.sync 1, %0;" ::"r"(TC_PROD) : "memory");
}

template <int TYPE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const uint8_t* __restrict__ W, const __half* __restrict__ Xh,
                   const __half* __restrict__ Xl, float* __restrict__ Y, int T, int rows, int cols,
                   int64_t row_bytes) {
    using R = RawSeg<TYPE>;
    constexpr int RUN = TC_SEGC / TC_BK;  // 64-column steps per staged run
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[TC_STAGES], empty[TC_STAGES], rawfull[2], acc_full;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, tid = threadIdx.x;
    const int m0 = blockIdx.x * TC_M, n0 = blockIdx.y * TC_N;
    const int n_k = cols / TC_BK, n_run = cols / TC_SEGC;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t raw_s = base + TC_STAGES * TC_STAGE;  // two runs of 128 x RS bytes
    uint8_t* const raw = smem_raw + (raw_s - smem_u32(smem_raw));
    if (tid == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&full[s], 2 * TC_PROD);  // dequant arrivals + B-copy arrivals
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) mbar_init(&rawfull[b], TC_PROD);
        mbar_init(&acc_full, 1);
        fence_mbar_init();
    }
    if (warp == TC_PROD / 32) {  // tensor-memory accumulator: 128 lanes x TC_N FP32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base)),
                     "r"(TC_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp < TC_PROD / 32) {
        // packed bytes of columns [256 j, 256 j + 256) of the tile rows -> run buffer j & 1
        auto stage_run = [&](int j) {
            const uint32_t dst = raw_s + (uint32_t)((j & 1) * TC_M * R::RS);
            for (int i = tid; i < TC_M * R::NCH; i += TC_PROD) {
                const int rr = i / R::NCH, c = i - rr * R::NCH;
                if (m0 + rr >= rows) continue;
                const int64_t start = (int64_t)(m0 + rr) * row_bytes + (int64_t)j * R::SEG;
                const int64_t a0 = start & ~(int64_t)15;
                if (a0 + 16 * c >= start + R::SEG) continue;  // beyond this run
                cp_async16(dst + (uint32_t)(rr * R::RS + 16 * c), W + a0 + 16 * c, true);
            }
            cp_async_arrive(&rawfull[j & 1]);
        };
        const int r = tid & 127, h = tid >> 7;  // dequant: tile row r, columns 16h..16h+15
        const int row = m0 + r;
        bool ok = true;
        stage_run(0);
        for (int kt = 0; kt < n_k; ++kt) {
            const int s = kt % TC_STAGES, u = kt / TC_STAGES, sub = kt % RUN, j = kt / RUN;
            const int k0 = kt * TC_BK;
            if (sub == 0) {
                bar_producers();  // everyone is done with run j - 1: its buffer takes run j + 1
                if (j + 1 < n_run) stage_run(j + 1);
                if (ok && !mbar_wait(&rawfull[j & 1], (j >> 1) & 1, &g_gemm_fault, 34)) ok = false;
            }
            if (u > 0 && ok && !mbar_wait(&empty[s], (u - 1) & 1, &g_gemm_fault, 31)) ok = false;
            const uint32_t st = base + (uint32_t)(s * TC_STAGE);
            if (ok) {
                // B: both planes of X, asynchronously; consecutive threads take consecutive
                // 16-byte chunks of a token row
#pragma unroll
                for (int i = 0; i < 2048 / TC_PROD; ++i) {
                    const int idx = tid + TC_PROD * i, plane = idx >> 10, rem = idx & 1023;
                    const int t = rem >> 3, c = rem & 7;
                    const __half* X = plane ? Xl : Xh;
                    const bool valid = n0 + t < T;
                    const __half* src = X + (size_t)(valid ? n0 + t : 0) * cols + k0 + 8 * c;
                    cp_async16(st + (2 + plane) * TC_TILE + sw128_off(t, c), src, valid);
                }
            }
            cp_async_arrive(&full[s]);
            if (ok) {
                // A: 16 columns of tile row r from the staged run
                constexpr int CPT = TC_BK / 8 / (TC_PROD / TC_M);  // 16-byte chunks per thread
                if (row < rows) {
                    const int64_t start = (int64_t)row * row_bytes + (int64_t)j * R::SEG;
                    const uint8_t* srow = raw + (j & 1) * TC_M * R::RS + r * R::RS;
                    const int o = (int)(start & 15);
                    if constexpr (TYPE == IB_TYPE_Q4_K || TYPE == IB_TYPE_Q6_K) {
                        static_assert(CPT == 2, "16 columns per thread");
                        float v[16];
                        if constexpr (TYPE == IB_TYPE_Q4_K) deq16_q4k(srow, sub * TC_BK + 16 * h, v);
                        else deq16_q6k(srow, o, sub * TC_BK + 16 * h, v);
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            uint4 hi, lo;
                            split8(v + 8 * i, hi, lo);
                            sts128(st + sw128_off(r, 2 * h + i), hi);
                            sts128(st + TC_TILE + sw128_off(r, 2 * h + i), lo);
                        }
                    } else {
                        const uint8_t* run = srow + o;
#pragma unroll
                        for (int i = 0; i < CPT; ++i) {
                            const int kc = sub * TC_BK + 8 * (CPT * h + i);  // column within the run
                            float v[8];
                            deq8<TYPE, GenericBytes>(run + (kc / R::BE) * R::BB, (kc % R::BE) >> 3, v);
                            uint4 hi, lo;
                            split8(v, hi, lo);
                            sts128(st + sw128_off(r, CPT * h + i), hi);
                            sts128(st + TC_TILE + sw128_off(r, CPT * h + i), lo);
                        }
                    }
                } else {
                    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int i = 0; i < CPT; ++i) {
                        sts128(st + sw128_off(r, CPT * h + i), z);
                        sts128(st + TC_TILE + sw128_off(r, CPT * h + i), z);
                    }
                }
            }
            // the tensor core reads these tiles through the async proxy
            fence_proxy_async_smem();
            mbar_arrive(&full[s]);
        }
        // ---- epilogue: TMEM lanes 32 (warp % 4) .. = tile rows, columns 32 (warp / 4) ..
        // tcgen05.ld is warp-collective: the whole warp takes the same branch
        const bool have = __all_sync(0xffffffffu, mbar_wait(&acc_full, 0, &g_gemm_fault, 33));
        tc_fence_after();
        if (have) {
            const int q = warp & 3, orow = m0 + 32 * q + (tid & 31);
            for (int c0 = 32 * (warp >> 2); c0 < TC_N; c0 += 32 * (TC_PROD / 128)) {
                uint32_t v[32];
                tc_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
                if (orow < rows) {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        const int t = n0 + c0 + jj;
                        if (t < T) Y[(size_t)t * rows + orow] = __uint_as_float(v[jj]);
                    }
                }
            }
        }
        // no copy of this thread may still be landing when the CTA ends
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (tid == TC_PROD) {
        // ---- MMA issuer
        constexpr uint32_t idesc = tc_idesc(TC_M, TC_N);
        bool ok = true;
        for (int kt = 0; kt < n_k && ok; ++kt) {
            const int s = kt % TC_STAGES, u = kt / TC_STAGES;
            if (!mbar_wait(&full[s], u & 1, &g_gemm_fault, 32)) {
                ok = false;
                break;
            }
            // the B tiles came through cp.async, the A tiles through stores: both reach the
            // tensor core's (async) proxy through this fence
            fence_proxy_async_smem();
            tc_fence_after();
            const uint32_t st = base + (uint32_t)(s * TC_STAGE);
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
                const uint32_t off = (uint32_t)kk * 32;  // 16 fp16 columns
                const uint64_t ah = sw128_desc(st + off), al = sw128_desc(st + TC_TILE + off);
                const uint64_t bh = sw128_desc(st + 2 * TC_TILE + off);
                const uint64_t bl = sw128_desc(st + 3 * TC_TILE + off);
                tc_mma(tmem, ah, bh, idesc, (kt | kk) != 0);
                tc_mma(tmem, ah, bl, idesc, 1u);
                tc_mma(tmem, al, bh, idesc, 1u);
            }
            tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        tc_commit(&acc_full);  // completes after every MMA issued above
    }
    // every thread's tensor-memory use is over before the allocation is returned
    tc_fence_before();
    __syncthreads();
    if (warp == TC_PROD / 32) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_N)
                     : "memory");
    }
}

// X (FP32) -> FP16 hi/lo planes.
__global__ void split_x_kernel(const float* __restrict__ X, __half* __restrict__ Xh,
                               __half* __restrict__ Xl, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = X[i];
        const __half h = __float2half_rn(v);
        Xh[i] = h;
        Xl[i] = __float2half_rn(v - __half2float(h));
    }
}

int gemm_split_x(const float* X, void* Xh, void* Xl, size_t n, cudaStream_t st) {
    const int g = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    split_x_kernel<<<g, 256, 0, st>>>(X, (__half*)Xh, (__half*)Xl, n);
    IB_LAUNCH_CHECK("split_x_kernel");
    return IB_OK;
}

template <int TYPE>
static int launch_tc(const void* W, const float* X, float* Y, int T, int rows, int cols,
                     cudaStream_t st) {
    const size_t n = (size_t)T * cols;
    void* ws = nullptr;
    int r = workspace_get(WS_GEMM, 2 * n * sizeof(__half) + 256, &ws);
    if (r) return r;
    __half* Xh = (__half*)ws;
    __half* Xl = Xh + n;
    if ((r = gemm_split_x(X, Xh, Xl, n, st))) return r;
    auto kern = gemm_tc_kernel<TYPE>;
    static bool attr_set[64] = {};
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 64 && !attr_set[dev]) {
        IB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)tc_smem_bytes<TYPE>()));
        attr_set[dev] = true;
    }
    const dim3 grid((rows + TC_M - 1) / TC_M, (T + TC_N - 1) / TC_N);
    IB_REQUIRE(grid.y <= 65535, "gemm: too many tokens");
    const int64_t row_bytes = packed_bytes(TYPE, 1, cols);
    kern<<<grid, TC_THREADS, tc_smem_bytes<TYPE>(), st>>>((const uint8_t*)W, Xh, Xl, Y, T, rows, cols,
                                                           row_bytes);
    IB_LAUNCH_CHECK("gemm_tc_kernel");
    return IB_OK;
}

// Runs of 256 columns; Q6_K rows must end on 16-byte boundaries (cols % 2048 == 0) so the
// 16-byte staging loads stay inside the weights.
bool gemm_tc_supported(int type, int64_t T, int64_t rows, int64_t cols) {
    return is_block_quant(type) && T >= 1 && rows >= 1 && cols % TC_SEGC == 0 &&
           (type != IB_TYPE_Q6_K || cols % 2048 == 0) && T * cols < (1ll << 31) &&
           rows < (1ll << 31);
}

int gemm_q_tc(int type, const void* W, const float* X, float* Y, int T, int rows, int cols,
              cudaStream_t st) {
    switch (type) {
        case IB_TYPE_Q4_0: return launch_tc<IB_TYPE_Q4_0>(W, X, Y, T, rows, cols, st);
        case IB_TYPE_Q5_0: return launch_tc<IB_TYPE_Q5_0>(W, X, Y, T, rows, cols, st);
        case IB_TYPE_Q5_1: return launch_tc<IB_TYPE_Q5_1>(W, X, Y, T, rows, cols, st);
        case IB_TYPE_Q8_0: return launch_tc<IB_TYPE_Q8_0>(W, X, Y, T, rows, cols, st);
        case IB_TYPE_Q4_K: return launch_tc<IB_TYPE_Q4_K>(W, X, Y, T, rows, cols, st);
        case IB_TYPE_Q6_K: return launch_tc<IB_TYPE_Q6_K>(W, X, Y, T, rows, cols, st);
    }
    set_error("gemm: unsupported type");
    return IB_ERR_UNSUPPORTED;
}

int gemm_fault_take(int* code) {
    int v = 0, z = 0;
    IB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_gemm_fault, sizeof(int)));
    if (v) IB_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_fault, &z, sizeof(int)));
    *code = v;
    return IB_OK;
}

}  // namespace ib
