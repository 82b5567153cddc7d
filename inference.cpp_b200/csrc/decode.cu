// Fused decode GEMV on GGUF blocks for the native Llama runner (sm_100a).
//
// Two kernels replace the chain  RMSNorm -> GEMV(s) -> elementwise  of the reference's
// forward_token (src/models/model_cuda.cpp:372-407):
//   xq_slab   splits the FP32 input (for a normed input: x * w, with per-group sums of
//             x^2 kept for the RMSNorm) once into exact int8 limbs, written as a slab of
//             per-stage slices (layout in decode.cuh);
//   GEMV      a producer warp streams, per pipeline stage, the packed bytes of 16 weight
//             rows plus the matching limb slice with 1-D TMA bulk copies (no multicast)
//             into a shared-memory ring; eight consumer warps run the int8-MMA block
//             math of gemv_math.cuh on it; the epilogue applies the RMSNorm divisor
//             sqrt(mean(x^2) + eps) (src/ops/cuda_kernels.cu:101-130) and one of
//             STORE, RESID (residual add), QKV (RoPE on q/k with the reference's table,
//             q to a buffer, k/v into the cache at the device position), SWIGLU
//             (silu(gate) * up, gate and up rows paired in one tile) or ARGMAX (logits
//             + a 64-bit atomic max of (ordered logit, ~row): the first maximum, as the
//             argmax kernel's tie rule).
// Weights are constant, so the producer issues the first ring fill before
// griddepcontrol.wait: under programmatic dependent launch the weight stream of a
// GEMV overlaps the tail of the previous kernel.
#include <math.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "decode.cuh"
#include "gemv_math.cuh"
#include "gemv_mma.cuh"
#include "pdl.cuh"
#include "pipeline.cuh"
#include "slab.cuh"
#include "fused_gemv.cuh"

namespace ib {

static __device__ int g_decode_fault;

bool slab_kquant(int type) {
    return type == IB_TYPE_Q4_K || type == IB_TYPE_Q6_K || type == IB_TYPE_Q5_K;
}

bool slab_supported(int type) { return gemv_mma_supported(type) || type == IB_TYPE_Q5_K; }

// After a head GEMV with an ARGMAX exchange: *best <- the maximum key over the ranks.
__global__ void tp_key_max_kernel(const TpExchange x, unsigned long long* best) {
    const uint32_t e1 = __ldcg(x.seq);
    const uint64_t* keys = (const uint64_t*)(tp_region(x, x.rank) + tp_keys_offset(x.world, x.stride)) +
                           (size_t)((e1 - 1u) & 1u) * x.world * 2;
    unsigned long long b = 0ull, t0 = 0ull;
    for (int src = 0; src < x.world; ++src) {
        uint32_t lo, hi;
        if (!wait_tagged(keys + 2 * src, e1, lo, t0, &g_decode_fault) ||
            !wait_tagged(keys + 2 * src + 1, e1, hi, t0, &g_decode_fault))
            return;
        const unsigned long long k = ((unsigned long long)hi << 32) | lo;
        b = k > b ? k : b;
    }
    *best = b;
}

// ---- limb slab ----------------------------------------------------------------------
// One warp per scale group of GS elements.  TP: x is first completed with the rows of
// the exchange that produced it, x[i] += sum over the ranks in rank order (the same
// values on every rank), and written back.
template <bool KQ, bool TP>
__global__ void __launch_bounds__(256) xq_slab_kernel(float* __restrict__ x,
                                                      const float* __restrict__ norm, int K,
                                                      uint8_t* __restrict__ slab,
                                                      float* __restrict__ ssq,
                                                      const TpExchange tp) {
    pdl_launch_dependents();
    constexpr int GS = SlabG<KQ>::GS, PER = GS / 32;
    // the norm weights are constant: loaded while the previous kernel finishes
    float w[PER];
    {
        const int g0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (norm && g0 * GS < K) slab_load<KQ>(norm, g0, threadIdx.x & 31, w);
    }
    pdl_wait();
    const uint64_t* parts = nullptr;
    uint32_t tag = 0;
    if constexpr (TP) {
        tag = __ldcg(tp.seq);  // the exchange that produced x's rows: number tag - 1
        parts = (const uint64_t*)tp_region(tp, tp.rank) + (size_t)((tag - 1u) & 1u) * tp.world * tp.stride;
    }
    const int lane = threadIdx.x & 31;
    const int gi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gi * GS >= K) return;
    float v[PER];
    slab_load<KQ>(x, gi, lane, v);
    if constexpr (TP) {
        // x += every rank's rows in rank order; a rank's PER words are loaded together
        // (one round trip when they have landed), then any stragglers are polled
        unsigned long long t0 = 0ull;
        bool ok = true;
        for (int q = 0; q < tp.world && ok; ++q) {
            const uint64_t* src = parts + (size_t)q * tp.stride;
            uint64_t wv[PER];
#pragma unroll
            for (int j = 0; j < PER; ++j) wv[j] = ld_relaxed_sys(src + slab_elem<KQ>(gi, j, lane));
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                uint32_t w = (uint32_t)wv[j];
                if ((uint32_t)(wv[j] >> 32) != tag && ok)
                    ok = wait_tagged(src + slab_elem<KQ>(gi, j, lane), tag, w, t0, &g_decode_fault);
                v[j] += __uint_as_float(w);
            }
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) x[slab_elem<KQ>(gi, j, lane)] = v[j];
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        float t = v[j];
        ss = fmaf(t, t, ss);
        if (norm) t *= w[j];
        v[j] = t;
    }
    if (ssq) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) ssq[gi] = ss;
    }
    slab_write_group<KQ>(v, gi, slab, lane);
}

int xq_slab_launch(const float* x, const float* norm, int K, bool kquant, uint8_t* slab,
                   float* ssq, cudaStream_t st, bool pdl, const TpExchange* tp) {
    IB_REQUIRE(x && slab && K > 0, "xq_slab: bad arguments");
    const int GS = kquant ? 256 : 32;
    IB_REQUIRE(K % GS == 0, "xq_slab: K must be a multiple of the limb group");
    const int groups = K / GS, grid = (groups + 7) / 8;
    float* xw = const_cast<float*>(x);  // written back only when completing an exchange
    const bool ex = tp && tp->world > 1;
    IB_REQUIRE(!ex || (tp->world <= kMaxRanks && K <= tp->stride && tp->seq),
               "xq_slab: bad exchange");
    const TpExchange none{};
    const TpExchange& t = ex ? *tp : none;
    if (kquant && ex)
        IB_CUDA_CHECK(launch_pdl(xq_slab_kernel<true, true>, dim3(grid), dim3(256), 0, st, pdl, xw,
                                 norm, K, slab, ssq, t));
    else if (kquant)
        IB_CUDA_CHECK(launch_pdl(xq_slab_kernel<true, false>, dim3(grid), dim3(256), 0, st, pdl, xw,
                                 norm, K, slab, ssq, t));
    else if (ex)
        IB_CUDA_CHECK(launch_pdl(xq_slab_kernel<false, true>, dim3(grid), dim3(256), 0, st, pdl, xw,
                                 norm, K, slab, ssq, t));
    else
        IB_CUDA_CHECK(launch_pdl(xq_slab_kernel<false, false>, dim3(grid), dim3(256), 0, st, pdl,
                                 xw, norm, K, slab, ssq, t));
    return IB_OK;
}

int tp_key_max_launch(const TpExchange& x, unsigned long long* best, cudaStream_t st) {
    IB_REQUIRE(best && x.world > 1 && x.world <= kMaxRanks && x.seq, "tp key max: bad arguments");
    tp_key_max_kernel<<<1, 1, 0, st>>>(x, best);
    IB_CUDA_CHECK(cudaGetLastError());
    return IB_OK;
}

// ---- TMA-staged persistent kernel: kNWC consumer warps + 1 producer warp ---------
// Stage layout: 16 weight rows at slot_a / slot_b bytes apart (padded so the
// consumers' loads of 8 rows spread over the shared-memory banks), then the limb
// slice at byte wbytes.  GEN: rows whose length is not a whole number of stages, or
// that do not start on 16-byte boundaries (the instantiation without it keeps the
// producer's and consumers' per-stage work to the aligned case).
template <int TA, int TB, int PRO, int EPI, bool GEN>
__global__ void __launch_bounds__((kNWC + 1) * 32)
    fused_tma_kernel(const FusedGemv p, int S, int slot_a, int slot_b, int wbytes) {
    using P = Pair<TA, TB>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], rfull[2], rfree[2];
    __shared__ int stage_rg[kMaxStages], stage_st[kMaxStages];
    __shared__ int warps_done;
    __shared__ float red[2][kNWC][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = p.K / P::BE;
    const int spg = GEN ? (nb + P::KB - 1) / P::KB : nb / P::KB;  // GEN: the last may be short
    const int stage_bytes = wbytes + P::SLICE;
    const int n_rg = p.paired ? p.rows[0] / 8 : (total_rows(p) + 15) / 16;
    // work units: row groups, or (K split) halves of row groups, unit u = 2 rg + half
    const bool ks = k_split<EPI>(p, spg);
    const int n_units = ks ? 2 * n_rg : n_rg, mid = (spg + 1) >> 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNWC);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&rfull[b], kNWC);
            mbar_init(&rfree[b], 1);
        }
        warps_done = 0;
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    if (warp == kNWC) {
        // producer: lanes 0..15 copy weight rows, lane 16 the limb slice.  Work units come
        // from the work counter (or the static stride); stage_rg[s] tells the consumers
        // which unit a stage holds, -1 ends their loop (stage_st[s]: its stage index).  Stage slot s and its phase
        // advance incrementally (no divisions in the loop).  A row that does not start on
        // a 16-byte boundary is copied from the boundary below it (the offset is the same
        // in every stage: a full stage is a multiple of 16 bytes) and its copy length
        // rounded up to 16 bytes; the row slots have room for the extra 16 bytes.
        auto limbs = [&](int slot_s, int st) {
            if (lane == 16)
                bulk_g2s(smem + (size_t)slot_s * stage_bytes + wbytes,
                         p.slab + (size_t)st * P::SLICE, (uint32_t)P::SLICE, &full[slot_s]);
        };
        int s = 0, ph = 0, it = 0, k = 0;
        bool waited = false, ok = true;
        for (;;) {
            int u = (int)blockIdx.x + k * (int)gridDim.x;
            if (p.work) {
                int r = 0;
                if (lane == 0) r = atomicAdd(p.work, 1);
                u = __shfl_sync(0xffffffffu, r, 0);
            }
            ++k;
            if (u >= n_units) break;
            const int rg = ks ? u >> 1 : u;
            const int st0 = ks && (u & 1) ? mid : 0, st1 = ks && !(u & 1) ? mid : spg;
            const bool isb = group_is_b<TA, TB>(p, rg);
            const int bb = isb ? Fmt<TB>::BB : Fmt<TA>::BB;
            const int chunk = P::KB * bb;
            const int n = group_rows(p, rg);
            const int slot = isb ? slot_b : slot_a;
            const uint8_t* src = p.W[0];
            uint32_t off = 0;
            if (lane < n) {
                int seg, lr;
                tile_row(p, rg, lane, seg, lr);
                src = p.W[seg] + (size_t)lr * nb * bb;
                if (GEN) {
                    off = (uint32_t)((uintptr_t)src & 15u);
                    src -= off;
                }
            }
            for (int st = st0; st < st1; ++st, ++it) {
                if (it >= S && !mbar_wait(&empty[s], ph ^ 1, &g_decode_fault, 11)) {
                    ok = false;
                    break;
                }
                uint32_t len = (uint32_t)chunk, tot = (uint32_t)(n * chunk);
                if (GEN) {
                    const int nbl = nb - st * P::KB < P::KB ? nb - st * P::KB : P::KB;
                    len = lane < n ? (off + (uint32_t)(nbl * bb) + 15u) & ~15u : 0u;
                    tot = len;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
                }
                if (lane == 0) {
                    stage_rg[s] = u;
                    stage_st[s] = st;
                    mbar_arrive_expect_tx(&full[s], tot + (uint32_t)P::SLICE);
                }
                __syncwarp();
                if (lane < n)
                    bulk_g2s(smem + (size_t)s * stage_bytes + (size_t)lane * slot,
                             src + (size_t)st * chunk, len, &full[s]);
                if (waited) {
                    limbs(s, st);
                } else if (it == S - 1) {
                    // weights (constant) of the first ring fill are in flight: now wait for
                    // the previous kernel before reading its limb slab
                    pdl_wait();
                    waited = true;
                    for (int j = 0; j < S; ++j) limbs(j, stage_st[j]);
                }
                if (++s == S) {
                    s = 0;
                    ph ^= 1;
                }
            }
            if (!ok) break;
        }
        if (!waited) {
            pdl_wait();
            for (int j = 0; j < it; ++j) limbs(j, stage_st[j]);
        }
        // every issued copy lands before the CTA can exit
        for (int j = it > S ? it - S : 0; j < it; ++j)
            mbar_wait(&full[j % S], (j / S) & 1, &g_decode_fault, 12);
        // end-of-work sentinel in the next slot (once the consumers have released it)
        if (ok && (it < S || mbar_wait(&empty[s], ph ^ 1, &g_decode_fault, 14)) && lane == 0) {
            stage_rg[s] = -1;
            mbar_arrive(&full[s]);
        }
        return;
    }
    pdl_wait();
    const int ps = (EPI == EPI_QKV && warp == 0) ? *p.pos : 0;  // fixed during a step
    // the RMSNorm divisor is applied by warp 0's epilogue only
    const float rms = (PRO == PRO_NORM && warp == 0) ? rms_of<P::GS>(p, lane) : 1.0f;
    const LaneCtx c = lane_ctx();
    const LeanLane ll = lean_lane(c);
    float acc_a = 0.f, acc_b = 0.f;
    int s = 0, ph = 0, rgl = 0;
    bool ok = true;
    while (ok) {
        if (!mbar_wait(&full[s], ph, &g_decode_fault, 13)) break;
        const int u = stage_rg[s];
        if (u < 0) break;
        const int rg = ks ? u >> 1 : u;
        const int st0 = ks && (u & 1) ? mid : 0, st1 = ks && !(u & 1) ? mid : spg;
        const bool isb = group_is_b<TA, TB>(p, rg);
        const int n = group_rows(p, rg);
        const int ra = c.g < n ? c.g : n - 1, rb = c.g + 8 < n ? c.g + 8 : n - 1;
        EpiPre pre{};
        if (warp == 0) pre = epi_fetch<EPI>(p, rg, lane, ps);
        const size_t rbytes = (size_t)nb * (isb ? Fmt<TB>::BB : Fmt<TA>::BB);
        int oa = 0, ob = 0;
        if (GEN) {
            int seg, lr;
            tile_row(p, rg, ra, seg, lr);
            oa = (int)((uintptr_t)(p.W[seg] + (size_t)lr * rbytes) & 15u);
            tile_row(p, rg, rb, seg, lr);
            ob = (int)((uintptr_t)(p.W[seg] + (size_t)lr * rbytes) & 15u);
        }
        for (int st = st0; st < st1; ++st) {
            if (st > st0 && !mbar_wait(&full[s], ph, &g_decode_fault, 13)) {
                ok = false;
                break;
            }
            const uint8_t* base = smem + (size_t)s * stage_bytes;
            const uint8_t* slab = base + wbytes;
            const int nbl = nb - st * P::KB;
            if (!GEN || nbl >= P::KB) {
                if (isb)
                    stage_math<TB, P::KB, P::SE, P::GS, true>(base, slab, slot_b, ra, rb, oa, ob,
                                                              P::KB, c, ll, warp, acc_a, acc_b);
                else
                    stage_math<TA, P::KB, P::SE, P::GS, true>(base, slab, slot_a, ra, rb, oa, ob,
                                                              P::KB, c, ll, warp, acc_a, acc_b);
            } else {
                if (isb)
                    stage_math<TB, P::KB, P::SE, P::GS, false>(base, slab, slot_b, ra, rb, oa, ob,
                                                               nbl, c, ll, warp, acc_a, acc_b);
                else
                    stage_math<TA, P::KB, P::SE, P::GS, false>(base, slab, slot_a, ra, rb, oa, ob,
                                                               nbl, c, ll, warp, acc_a, acc_b);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        if (!ok) break;
        if (!finish_group_mbar<EPI>(p, red, rfull, rfree, rgl, rg, warp, lane, c, rms, acc_a,
                                    acc_b, &g_decode_fault, pre, ks ? (u & 1) : -1))
            break;
        ++rgl;
    }
    // the last consumer warp of the last CTA out resets the work counters (and ends the
    // exchange: its key and the exchange counter)
    if (EPI == EPI_ARGMAX && tp_exchanges<EPI>(p) && warp == 0) __threadfence();
    if (p.work && (!p.work_ext || tp_exchanges<EPI>(p)) && lane == 0 &&
        atomicAdd(&warps_done, 1) == kNWC - 1 && atomicAdd(p.work + 1, 1) == (int)gridDim.x - 1) {
        if (tp_exchanges<EPI>(p)) tp_finish<EPI>(p);
        p.work[0] = 0;
        p.work[1] = 0;
    }
}

// ---- host side ----------------------------------------------------------------------
// Row stride in a stage: >= the chunk (+16 bytes when rows do not start on 16-byte
// boundaries), a multiple of 16, and congruent to 32 (Q4_K's 8-byte loads) or 16 (the
// 2/4-byte loads of the other formats) modulo 128.
static int ring_slot(int type, int chunk, bool pad) {
    const int want = (type == IB_TYPE_Q4_K || type == IB_TYPE_Q5_K) ? 32 : 16;
    int s = (chunk + (pad ? 16 : 0) + 15) / 16 * 16;
    while (s % 128 != want) s += 16;
    return s;
}

// Format pairs of the fused kernels: 0 Q4_K/Q6_K, 1 Q4_0/Q8_0, 2 Q5_0/Q5_1, 3 Q5_K/Q6_K
// (Q6_K serves both K-quant pairs).
static bool in_pair(int type, int pr) {
    switch (pr) {
        case 0: return type == IB_TYPE_Q4_K || type == IB_TYPE_Q6_K;
        case 1: return type == IB_TYPE_Q4_0 || type == IB_TYPE_Q8_0;
        case 2: return type == IB_TYPE_Q5_0 || type == IB_TYPE_Q5_1;
        case 3: return type == IB_TYPE_Q5_K || type == IB_TYPE_Q6_K;
    }
    return false;
}

// The pair of a GEMV's segments (-1: none): Q5_K anywhere selects pair 3.
static int pair_of(const FusedGemv& p) {
    int pr = -1;
    for (int s = 0; s < p.n_seg && s < 3; ++s) {
        const int t = p.type[s];
        const int q = t == IB_TYPE_Q5_K ? 3 : t == IB_TYPE_Q4_K || t == IB_TYPE_Q6_K ? 0
                    : t == IB_TYPE_Q4_0 || t == IB_TYPE_Q8_0 ? 1
                    : t == IB_TYPE_Q5_0 || t == IB_TYPE_Q5_1 ? 2 : -1;
        if (q < 0) return -1;
        if (q == 3 || pr < 0) pr = q;
    }
    return pr;
}

struct OccKey {
    const void* f;
    size_t smem;
    bool operator<(const OccKey& o) const { return f < o.f || (f == o.f && smem < o.smem); }
};

static int max_ctas(const void* f, int threads, size_t smem, int* out) {
    static std::mutex mu;
    static std::map<std::pair<int, OccKey>, int> cache;
    static std::map<std::pair<int, const void*>, size_t> attr;
    int dev = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    auto ak = std::make_pair(dev, f);
    if (smem > 48 * 1024 - 4096 && attr[ak] < smem) {
        IB_CUDA_CHECK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr[ak] = smem;
    }
    auto key = std::make_pair(dev, OccKey{f, smem});
    auto it = cache.find(key);
    if (it == cache.end()) {
        int per_sm = 0, sms = 0;
        IB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, threads, smem));
        IB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        if (per_sm < 1) {
            set_error("fused GEMV: launch configuration does not fit on an SM");
            return IB_ERR_UNSUPPORTED;
        }
        it = cache.emplace(key, per_sm * sms).first;
    }
    *out = it->second;
    return IB_OK;
}

bool fused_gemv_supported(const FusedGemv& p, int epi) {
    if (p.n_seg < 1 || p.n_seg > 3 || p.K <= 0 || !p.slab || ((uintptr_t)p.slab & 15)) return false;
    const int pr = pair_of(p);
    if (pr < 0) return false;
    const int be = (pr == 0 || pr == 3) ? 256 : 32;
    if (p.K % be) return false;
    for (int s = 0; s < p.n_seg; ++s) {
        if (!in_pair(p.type[s], pr) || !p.W[s] || p.rows[s] <= 0) return false;
        if (((uintptr_t)p.W[s] % 16) != 0) return false;
        if (!p.paired && s < p.n_seg - 1 && p.rows[s] % 16) return false;
    }
    for (int s = p.n_seg; s < 3; ++s)
        if (p.rows[s] != 0) return false;
    if (p.paired && (p.n_seg != 2 || p.rows[0] != p.rows[1] || p.type[0] != p.type[1] ||
                     p.rows[0] % 8))
        return false;
    if (epi == EPI_SWIGLU && !p.paired) return false;
    if (epi != EPI_SWIGLU && p.paired) return false;
    if (epi == EPI_QKV && (p.n_seg != 3 || p.head_dim <= 0 || p.head_dim % 2 || p.rows[2] % 16 ||
                           p.rows[0] % p.head_dim || p.rows[1] % p.head_dim ||
                           p.rows[1] != p.rows[2] || !p.pos || !p.rope || !p.q || !p.kc || !p.vc))
        return false;
    if (epi == EPI_ARGMAX && !p.best) return false;
    if (epi == EPI_ALLRED || (epi == EPI_ARGMAX && p.tp.world > 1)) {
        const TpExchange& x = p.tp;
        if (x.world < 2 || x.world > kMaxRanks || x.rank < 0 || x.rank >= x.world || !x.seq ||
            !p.work || p.paired)
            return false;
        if (epi == EPI_ALLRED && p.rows[0] + p.rows[1] + p.rows[2] > x.stride) return false;
        for (int q = 0; q < x.world; ++q)
            if (!x.region[q]) return false;
    }
    if (!p.y && epi != EPI_QKV) return false;
    return true;
}

template <int TA, int TB, int PRO, int EPI>
static int launch_inst(const FusedGemv& p, cudaStream_t st, bool pdl) {
    using P = Pair<TA, TB>;
    const int nb = p.K / P::BE;
    const int n_rg = p.paired ? p.rows[0] / 8 : (p.rows[0] + p.rows[1] + p.rows[2] + 15) / 16;
    bool has_a = false, has_b = false;
    for (int s = 0; s < p.n_seg; ++s) (p.type[s] == TA ? has_a : has_b) = true;
    int r;
    {
        const bool pad_a = has_a && (size_t)nb * Fmt<TA>::BB % 16 != 0;
        const bool pad_b = has_b && (size_t)nb * Fmt<TB>::BB % 16 != 0;
        const bool gen = pad_a || pad_b || nb % P::KB != 0;
        const int slot_a = ring_slot(TA, P::KB * Fmt<TA>::BB, pad_a);
        const int slot_b = ring_slot(TB, P::KB * Fmt<TB>::BB, pad_b);
        const int wbytes = 16 * ((has_b && (!has_a || slot_b > slot_a)) ? slot_b : slot_a);
        const int stage = wbytes + P::SLICE;
        // Ring depth.  Short rows (K-quant rows of <= 4 stages: K <= 8192) run 2 stages
        // at 3-4 CTAs per SM: 215-223 KB in flight per SM, and the row groups spread
        // evenly over the CTAs.  Long Q6_K rows (the down projection: 7 stages per row
        // group at K = 14336) run 3 stages at 2 CTAs per SM, so each CTA keeps a deeper
        // queue through its row.  Measured on the Llama-3-8B decode step at position
        // 2050: 2.26 ms, against 2.45 with 2 stages for the down projection, 2.32 with 3
        // stages for the QKV projection and head too, 2.36 with 4 stages at one CTA per
        // SM for the down projection, and 2.58 with 3 stages for the 4-bit kernels.
        const int spg = (nb + P::KB - 1) / P::KB;  // ring stages per row group
        int S = (has_b && TB == IB_TYPE_Q6_K && spg > 4) ? 3 : 73728 / stage;
        if (S < 2) S = 2;
        if (S > kMaxStages) S = kMaxStages;
        const size_t smem = (size_t)S * stage;
        auto kern = gen ? fused_tma_kernel<TA, TB, PRO, EPI, true>
                        : fused_tma_kernel<TA, TB, PRO, EPI, false>;
        int cap = 0;
        if ((r = max_ctas((const void*)kern, (kNWC + 1) * 32, smem, &cap))) return r;
        // dynamic schedule: every resident slot claims row groups; static: an even split
        const int per = ((k_split<EPI>(p, spg) ? 2 * n_rg : n_rg) + cap - 1) / cap;
        const int n_units = k_split<EPI>(p, spg) ? 2 * n_rg : n_rg;
        const int grid = p.work ? (n_units < cap ? n_units : cap) : (n_units + per - 1) / per;
        IB_CUDA_CHECK(launch_pdl(kern, dim3(grid), dim3((kNWC + 1) * 32), smem, st, pdl, p, S,
                                 slot_a, slot_b, wbytes));
    }
    return IB_OK;
}

template <int TA, int TB>
static int launch_pair(const FusedGemv& p, int pro, int epi, cudaStream_t st, bool pdl) {
    if (pro == PRO_NORM && epi == EPI_QKV) return launch_inst<TA, TB, PRO_NORM, EPI_QKV>(p, st, pdl);
    if (pro == PRO_PLAIN && epi == EPI_RESID) return launch_inst<TA, TB, PRO_PLAIN, EPI_RESID>(p, st, pdl);
    if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_inst<TA, TB, PRO_NORM, EPI_SWIGLU>(p, st, pdl);
    if (pro == PRO_NORM && epi == EPI_ARGMAX) return launch_inst<TA, TB, PRO_NORM, EPI_ARGMAX>(p, st, pdl);
    if (pro == PRO_PLAIN && epi == EPI_STORE) return launch_inst<TA, TB, PRO_PLAIN, EPI_STORE>(p, st, pdl);
    if (pro == PRO_PLAIN && epi == EPI_ALLRED) return launch_inst<TA, TB, PRO_PLAIN, EPI_ALLRED>(p, st, pdl);
    set_error("fused GEMV: unsupported prologue/epilogue combination");
    return IB_ERR_UNSUPPORTED;
}

int fused_gemv_launch(const FusedGemv& p, int pro, int epi, cudaStream_t st, bool pdl) {
    if (!fused_gemv_supported(p, epi)) {
        set_error("fused GEMV: unsupported types or shapes");
        return IB_ERR_UNSUPPORTED;
    }
    if (pro == PRO_NORM && !p.ssq) {
        set_error("fused GEMV: a normed input needs its sums of squares");
        return IB_ERR_INVALID;
    }
    switch (pair_of(p)) {
        case 0: return launch_pair<IB_TYPE_Q4_K, IB_TYPE_Q6_K>(p, pro, epi, st, pdl);
        case 3: return launch_pair<IB_TYPE_Q5_K, IB_TYPE_Q6_K>(p, pro, epi, st, pdl);
        case 1: return launch_pair<IB_TYPE_Q4_0, IB_TYPE_Q8_0>(p, pro, epi, st, pdl);
        case 2: return launch_pair<IB_TYPE_Q5_0, IB_TYPE_Q5_1>(p, pro, epi, st, pdl);
    }
    return IB_ERR_UNSUPPORTED;
}

// ---- self-test of the exchange's bounded wait -----------------------------------------
// Writes the tagged rows rank `src` contributes to exchange 0 (slot 0) of a region.
__global__ void tp_selftest_push_kernel(uint64_t* region, int world, int stride, int src, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        st_tagged(region + (size_t)src * stride + i, 1u, __float_as_uint(0.25f * (float)(src + 1)));
}

// One exchange round's sending side, as the row-split GEMV's epilogue and its last CTA
// do it (every rank's rows, zeros here, into slot [rank] of every rank's region, tagged
// with the exchange number; then the exchange counter advances).  One CTA.
__global__ void tp_probe_push_kernel(const TpExchange x, int n) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t e = __ldcg(x.seq);
    const size_t at = ((size_t)(e & 1u) * x.world + x.rank) * x.stride;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
            if (q < x.world) st_tagged((uint64_t*)x.region[q] + at + i, e + 1, 0u);
    __syncthreads();
    if (threadIdx.x == 0) *x.seq = e + 1;
}

int tp_probe_launch(const TpExchange& x, float* xv, int n, bool kquant, uint8_t* slab,
                    cudaStream_t st) {
    IB_CUDA_CHECK(launch_pdl(tp_probe_push_kernel, dim3(1), dim3(256), 0, st, true, x, n));
    return xq_slab_launch(xv, nullptr, n, kquant, slab, nullptr, st, true, &x);
}

}  // namespace ib

// One exchange on this GPU between rank 0 and a stand-in rank 1 whose rows arrive only
// when `peer_sends` != 0.  The receiving slab kernel either completes x (+0.25 + 0.5 per
// element) or gives up after its bounded wait (2 s), recording fault 21; *fault gets
// the recorded code (0 = none) and *x_out one completed element.  No counterpart in the
// reference: it exercises the failure path of the tensor-parallel exchange without a
// second GPU and without faulting the device.
extern "C" int ib_tp_wait_selftest(int peer_sends, int* fault, float* x_out) {
    using namespace ib;
    IB_REQUIRE(fault && x_out, "null pointer argument");
    const int K = 256, W = 2;
    const size_t rb = tp_region_bytes(W, K);
    uint8_t* region = nullptr;
    uint32_t* seq = nullptr;
    float* x = nullptr;
    uint8_t* slab = nullptr;
    IB_CUDA_CHECK(cudaMalloc(&region, rb));
    IB_CUDA_CHECK(cudaMalloc(&seq, 16));
    IB_CUDA_CHECK(cudaMalloc(&x, K * 4));
    IB_CUDA_CHECK(cudaMalloc(&slab, slab_total_bytes(K, true) + 16));
    int r = IB_OK;
    do {
        if (cudaMemset(region, 0, rb) != cudaSuccess || cudaMemset(x, 0, K * 4) != cudaSuccess) {
            r = IB_ERR_CUDA;
            break;
        }
        const uint32_t one = 1;  // the producing GEMV has advanced the counter past exchange 0
        if (cudaMemcpy(seq, &one, 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            r = IB_ERR_CUDA;
            break;
        }
        tp_selftest_push_kernel<<<1, 256>>>((uint64_t*)region, W, K, 0, K);
        if (peer_sends) tp_selftest_push_kernel<<<1, 256>>>((uint64_t*)region, W, K, 1, K);
        TpExchange t{};
        t.region[0] = region;
        t.region[1] = region;  // the stand-in peer shares this GPU's region
        t.seq = seq;
        t.rank = 0;
        t.world = W;
        t.stride = K;
        if ((r = xq_slab_launch(x, nullptr, K, true, slab, nullptr, nullptr, false, &t))) break;
        if (cudaDeviceSynchronize() != cudaSuccess) {
            r = IB_ERR_CUDA;
            break;
        }
        if ((r = decode_fault_take(fault))) break;
        if (cudaMemcpy(x_out, x, 4, cudaMemcpyDeviceToHost) != cudaSuccess) r = IB_ERR_CUDA;
    } while (false);
    cudaFree(region);
    cudaFree(seq);
    cudaFree(x);
    cudaFree(slab);
    return r;
}

namespace ib {

int decode_fault_take(int* code) {
    int v = 0, z = 0;
    IB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_decode_fault, sizeof(int)));
    if (v) IB_CUDA_CHECK(cudaMemcpyToSymbol(g_decode_fault, &z, sizeof(int)));
    *code = v;
    return IB_OK;
}

}  // namespace ib
