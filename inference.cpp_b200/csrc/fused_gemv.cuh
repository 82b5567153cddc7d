// Device-side building blocks of the fused decode GEMV, shared by the per-operation
// kernels (decode.cu) and the persistent decode-step kernel (step.cu): block-format
// pairs, the tensor-parallel exchange's tagged stores and bounded waits, the row-group
// geometry of a FusedGemv, its epilogues, the bounded mbarrier reduction of a row
// group's partials and the per-stage block math.  Functions that can give up on a wait
// record a code in the caller's fault word.
#pragma once
#include <math.h>
#include <stdint.h>

#include "decode.cuh"
#include "gemv_math.cuh"
#include "kv.cuh"
#include "pipeline.cuh"
#include "slab.cuh"

namespace ib {

constexpr int kNWC = 8;        // consumer warps
constexpr int kMaxStages = 8;  // ring stages

template <int TA, int TB>
struct Pair {
    using FA = Fmt<TA>;
    using FB = Fmt<TB>;
    static_assert(FA::K == FB::K && FA::KB == FB::KB && FA::UNIT == FB::UNIT,
                  "the two formats of a fused kernel share block geometry");
    static constexpr bool KQ = FA::K;
    static constexpr int BE = KQ ? 256 : 32;  // elements per block
    static constexpr int KB = FA::KB;         // blocks per stage per row
    static constexpr int UNIT = FA::UNIT;
    static constexpr int SE = SlabG<KQ>::SE;  // elements per stage = slab slice
    static constexpr int GS = SlabG<KQ>::GS;  // elements per limb scale
    static constexpr int SLICE = SlabG<KQ>::SLICE;
    static_assert(SE == KB * BE, "a pipeline stage covers one slab slice");
};

// ---- tensor-parallel exchange ----------------------------------------------------------
// Every exchanged 32-bit word travels as one 64-bit store of (tag << 32 | word), tag =
// exchange number + 1: the receiver polls each word until its tag matches, so no fence,
// flag or counter orders the data (a 64-bit aligned store is single-copy atomic).  A
// rank that never sends (it died, or took another path) costs the waiting rank at most
// this long; the wait then records fault 21 and the step's results are invalid.
constexpr unsigned long long kExchangeTimeoutNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_tagged(uint64_t* a, uint32_t tag, uint32_t word) {
    const uint64_t v = ((uint64_t)tag << 32) | word;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* a) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

// Waits for the word at a to carry `tag`; false (fault 21) once the deadline passes.
__device__ __forceinline__ bool wait_tagged(const uint64_t* a, uint32_t tag, uint32_t& word,
                                            unsigned long long& t0, int* fault) {
    for (uint32_t i = 0;; ++i) {
        const uint64_t v = ld_relaxed_sys(a);
        if ((uint32_t)(v >> 32) == tag) {
            word = (uint32_t)v;
            return true;
        }
        if (i == 0 && t0 == 0ull) t0 = globaltimer_ns();
        if (i >= 32) {
            if (globaltimer_ns() - t0 > kExchangeTimeoutNs) {
                atomicCAS(fault, 0, 21);
                return false;
            }
            __nanosleep(64);
        }
    }
}

__device__ __forceinline__ uint8_t* tp_region(const TpExchange& x, int q) {
    uint8_t* r = x.region[0];
#pragma unroll
    for (int i = 1; i < kMaxRanks; ++i)
        if (q == i) r = x.region[i];
    return r;
}

// True when the kernel instance ends with an exchange.
template <int EPI>
__device__ __forceinline__ bool tp_exchanges(const FusedGemv& p) {
    return EPI == EPI_ALLRED || (EPI == EPI_ARGMAX && p.tp.world > 1);
}

// True when a launch splits its row groups over K (FusedGemv::kpart): residual-add
// GEMVs whose rows span more than 8 stages (K > 16384).  Measured on the decode step:
// the Llama-3-70B down projection (14 stages) 11.04 against 11.17 ms per step; the
// Llama-3-8B one (7 stages) 2.34 against 2.19 ms, where the per-unit fence and counter
// on warp 0 cost more than the shorter chains gain.
template <int EPI>
__host__ __device__ __forceinline__ bool k_split(const FusedGemv& p, int spg) {
    return EPI == EPI_RESID && p.kpart && p.kcnt && !p.paired && spg > 8;
}

// Run once by the last CTA out, after every CTA's rows are pushed: sends this rank's
// key (ARGMAX; the CTAs' atomicMax are fenced before their arrival) and advances the
// exchange counter the pushes and the receivers derive their tag from.
template <int EPI>
__device__ __forceinline__ void tp_finish(const FusedGemv& p) {
    const TpExchange& x = p.tp;
    const uint32_t e = __ldcg(x.seq);
    if (EPI == EPI_ARGMAX) {
        const unsigned long long key = atomicAdd(p.best, 0ull);
        const size_t at = ((size_t)(e & 1u) * x.world + x.rank) * 2;
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < x.world) {
                uint64_t* k = (uint64_t*)(x.region[q] + tp_keys_offset(x.world, x.stride)) + at;
                st_tagged(k, e + 1, (uint32_t)key);
                st_tagged(k + 1, e + 1, (uint32_t)(key >> 32));
            }
    }
    *x.seq = e + 1;
}

// ---- row geometry --------------------------------------------------------------------
__device__ __forceinline__ int total_rows(const FusedGemv& p) {
    return p.paired ? 2 * p.rows[0] : p.rows[0] + p.rows[1] + p.rows[2];
}

// Rows of row group rg that exist (16 except in the last group of a ragged last
// segment).
__device__ __forceinline__ int group_rows(const FusedGemv& p, int rg) {
    if (p.paired) return 16;
    const int left = total_rows(p) - rg * 16;
    return left < 16 ? left : 16;
}

// Tile row i (0..15) of row group rg -> (segment, row within the segment); rows past
// the end map to the last row.
__device__ __forceinline__ void tile_row(const FusedGemv& p, int rg, int i, int& seg, int& lr) {
    if (p.paired) {
        seg = i >> 3;
        lr = rg * 8 + (i & 7);
        return;
    }
    int R = rg * 16 + i;
    const int tot = total_rows(p);
    if (R >= tot) R = tot - 1;
    if (R < p.rows[0]) {
        seg = 0;
        lr = R;
    } else if (R < p.rows[0] + p.rows[1]) {
        seg = 1;
        lr = R - p.rows[0];
    } else {
        seg = 2;
        lr = R - p.rows[0] - p.rows[1];
    }
}

template <int TA, int TB>
__device__ __forceinline__ bool group_is_b(const FusedGemv& p, int rg) {
    if (TA == TB) return false;
    int seg, lr;
    tile_row(p, rg, 0, seg, lr);
    return p.type[seg] == TB;
}

// RMSNorm divisor sqrt(sum(x^2) / K + eps) from the per-group sums (warp-wide).
template <int GS>
__device__ __forceinline__ float rms_of(const FusedGemv& p, int lane) {
    float t = 0.f;
    for (int i = lane; i < p.K / GS; i += 32) t += p.ssq[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return sqrtf(t / (float)p.K + p.eps);
}

// ---- epilogue ------------------------------------------------------------------------
// What a row group's epilogue reads from global memory, loaded by warp 0 when the row
// group's first stage arrives so that the loads overlap the group's math: the residual
// rows (RESID) and the RoPE factors of the position (QKV).  Nothing in the launch writes
// them before the epilogue: the row group's own rows are written only there, and the
// rotary table and the position are fixed during a step.
struct EpiPre {
    float y, c, s;
    int ps;
};

template <int EPI>
__device__ __forceinline__ EpiPre epi_fetch(const FusedGemv& p, int rg, int lane, int ps) {
    EpiPre e{0.f, 1.f, 0.f, ps};
    if (EPI == EPI_RESID) {
        if (lane < group_rows(p, rg)) e.y = p.y[rg * 16 + lane];
    } else if (EPI == EPI_QKV) {
        int seg = 0, lr = 0;
        tile_row(p, rg, lane & 15, seg, lr);
        if (seg < 2) {
            const int HD = p.head_dim, j = (lr % HD) >> 1;
            e.c = p.rope[((size_t)ps * (HD / 2) + j) * 2];
            e.s = p.rope[((size_t)ps * (HD / 2) + j) * 2 + 1];
        }
    }
    return e;
}

// Row-group epilogue on warp 0: lanes 0..15 hold the finished rows (v); e holds what
// epi_fetch loaded for them.
template <int EPI>
__device__ __forceinline__ void epilogue(const FusedGemv& p, int rg, int lane, float v,
                                         const EpiPre& e) {
    const unsigned FULL = 0xffffffffu;
    int seg = 0, lr = 0;
    tile_row(p, rg, lane & 15, seg, lr);
    const bool live = lane < group_rows(p, rg);
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
        const int R = rg * 16 + lane;
        if (live) {
            if (EPI == EPI_STORE) p.y[R] = v;
            else p.y[R] = e.y + v;
        }
    } else if (EPI == EPI_QKV) {
        const int HD = p.head_dim;
        const int d = lr % HD;
        const int ps = e.ps;
        const float other = __shfl_xor_sync(FULL, v, 1);
        float out = v;
        if (seg < 2) {  // RoPE, rope_kernel's formula on the pair (2j, 2j+1)
            const float c = e.c, s = e.s;
            out = (d & 1) == 0 ? v * c - other * s : other * s + v * c;
        }
        if (live) {
            if (seg == 0) {
                p.q[lr] = out;
            } else {
                const size_t at = ((size_t)(lr / HD) * p.max_seq + ps) * HD + d;
                float* dst = seg == 1 ? p.kc : p.vc;
                if (p.kv_half) kv_put((__half*)dst, at, out);
                else dst[at] = out;
            }
        }
    } else if (EPI == EPI_SWIGLU) {
        const float u = __shfl_down_sync(FULL, v, 8);
        if (lane < 8) p.y[rg * 8 + lane] = v * (1.0f / (1.0f + expf(-v))) * u;
    } else if (EPI == EPI_ALLRED) {
        const int R = rg * 16 + lane;
        if (live) {  // this rank's row R into slot row [rank] of every rank's region
            const TpExchange& x = p.tp;
            const uint32_t e = __ldcg(x.seq);
            const size_t at = ((size_t)(e & 1u) * x.world + x.rank) * x.stride + R;
#pragma unroll
            for (int q = 0; q < kMaxRanks; ++q)
                if (q < x.world) st_tagged((uint64_t*)x.region[q] + at, e + 1, __float_as_uint(v));
        }
    } else if (EPI == EPI_ARGMAX) {
        const int R = rg * 16 + lane;
        unsigned long long key = 0ull;
        if (live) {
            p.y[R] = v;
            if (!(v != v)) {  // NaN never wins (the argmax kernel compares with >)
                const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
                const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
                key = ((unsigned long long)o << 32) |
                      (unsigned long long)(0xFFFFFFFFu - (uint32_t)(p.row_base + R));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(FULL, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key) atomicMax(p.best, key);
    }
}

// The epilogue with its reads made on the spot (the persistent step's epilogue warp).
template <int EPI>
__device__ __forceinline__ void epilogue(const FusedGemv& p, int rg, int lane, float v) {
    epilogue<EPI>(p, rg, lane, v, epi_fetch<EPI>(p, rg, lane, EPI == EPI_QKV ? *p.pos : 0));
}

// Sums the consumer warps' partials of the row group, applies the RMSNorm divisor and
// runs the epilogue, with bounded mbarrier handshakes (the TMA kernel's consumer warps
// leave their loop independently after a failed wait):
// every warp posts its partials to red[b] and arrives on rfull[b]; warp 0 waits, reduces,
// runs the epilogue and frees the buffer on rfree[b]; a warp reusing red[b] (two row
// groups later) first waits for that free.  Use u = rgl >> 1 of buffer b = rgl & 1.
// half >= 0: the unit is that half of a K-split row group (FusedGemv::kpart).
template <int EPI>
__device__ __forceinline__ bool finish_group_mbar(const FusedGemv& p, float (*red)[kNWC][16],
                                                  uint64_t* rfull, uint64_t* rfree, int rgl,
                                                  int rg, int warp, int lane, const LaneCtx& c,
                                                  float rms, float& acc_a, float& acc_b,
                                                  int* fault, const EpiPre& pre, int half = -1) {
    const int b = rgl & 1, u = rgl >> 1;
    acc_a = quad_sum(acc_a);
    acc_b = quad_sum(acc_b);
    if (warp != 0 && u > 0 && !mbar_wait(&rfree[b], (u - 1) & 1, fault, 15))
        return false;
    if (c.t == 0) {
        red[b][warp][c.g] = acc_a;
        red[b][warp][c.g + 8] = acc_b;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfull[b]);
    acc_a = 0.f;
    acc_b = 0.f;
    if (warp != 0) return true;
    if (!mbar_wait(&rfull[b], u & 1, fault, 16)) return false;
    float v = 0.f;
    if (lane < 16) {
#pragma unroll
        for (int w = 0; w < kNWC; ++w) v += red[b][w][lane];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfree[b]);
    if (half >= 0) {  // K split: the second half of the row group to finish adds both
        if (lane < 16) p.kpart[((size_t)rg * 2 + half) * 16 + lane] = v;
        __threadfence();
        __syncwarp();
        int second = 0;
        if (lane == 0) second = atomicAdd(p.kcnt + rg, 1);
        if (!__shfl_sync(0xffffffffu, second, 0)) return true;
        __threadfence();
        const float o = lane < 16 ? __ldcg(p.kpart + ((size_t)rg * 2 + (half ^ 1)) * 16 + lane) : 0.f;
        v = half == 0 ? v + o : o + v;
        if (lane == 0) p.kcnt[rg] = 0;
    }
    epilogue<EPI>(p, rg, lane, v / rms, pre);
    return true;
}

// One stage of the 16 tile rows (limb slice at `slab`) for this warp's share of the
// blocks: rows ra / rb start at byte offsets oa / ob of their row slots.  FULL: the
// stage holds KB blocks (loops unrolled); otherwise nbl < KB, the last stage of a row
// whose length is not a whole number of stages.
template <int TYPE, int KB, int SE, int GS, bool FULL>
__device__ __forceinline__ void stage_math(const uint8_t* base, const uint8_t* slab, int slot,
                                           int ra, int rb, int oa, int ob, int nbl,
                                           const LaneCtx& c, const LeanLane& ll, int warp,
                                           float& acc_a, float& acc_b) {
    using F = Fmt<TYPE>;
    if constexpr (TYPE == IB_TYPE_Q4_K) {
        const uint32_t b = smem_u32(base), x = smem_u32(slab);
        const uint32_t wa = b + (uint32_t)(ra * slot + oa), wb = b + (uint32_t)(rb * slot + ob);
        const uint32_t scale = x + SE * 4, sum32 = scale + (SE / GS) * 4;
        auto one = [&](int kbl) {
            q4k_tile_lean(wa + kbl * F::BB, wb + kbl * F::BB, x + kbl * 1024, sum32 + kbl * 32,
                          ldsf<0>(scale + kbl * 4), c, ll, acc_a, acc_b);
        };
        if constexpr (FULL) {
#pragma unroll
            for (int kbl = warp; kbl < KB; kbl += kNWC) one(kbl);
        } else {
            for (int kbl = warp; kbl < nbl; kbl += kNWC) one(kbl);
        }
    } else {
        XLimbs xs;
        xs.limbs = (int8_t*)slab;
        xs.scale = (float*)(slab + SE * 4);
        xs.sum32 = xs.scale + SE / GS;
        xs.sum16 = xs.sum32 + SE / 32;
        const uint8_t* sa = base + (size_t)ra * slot + oa;
        const uint8_t* sb = base + (size_t)rb * slot + ob;
        if constexpr (FULL) {
#pragma unroll
            for (int kbl = warp * F::UNIT; kbl < KB; kbl += kNWC * F::UNIT)
                block_math<TYPE, true, true>(sa + kbl * F::BB, sb + kbl * F::BB, kbl, KB, xs, c,
                                             acc_a, acc_b);
        } else {
            for (int kbl = warp * F::UNIT; kbl < nbl; kbl += kNWC * F::UNIT)
                block_math<TYPE, true, true>(sa + kbl * F::BB, sb + kbl * F::BB, kbl, nbl, xs, c,
                                             acc_a, acc_b);
        }
    }
}


}  // namespace ib
