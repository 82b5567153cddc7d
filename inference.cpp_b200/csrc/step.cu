// Persistent decode-step kernel (sm_100a): one launch per batch-1 decode token.
//
// The per-operation decode path (decode.cu, attention.cu) runs a step as ~260 kernels
// chained by programmatic dependent launch; each boundary drains one kernel's tail and
// ramps the next one's weight stream.  Here one persistent grid runs the whole step as
// a task list (the scheme is described in step.cuh).  A CTA is ten warps:
//   producer (warp 8)  claims tasks in order from a global counter (one claim ahead),
//              and for a GEMV task copies each stage's 16 weight rows with 1-D bulk
//              copies (TMA, no multicast) as soon as a ring slot is free, whatever
//              layer or phase the task belongs to; the stage's limb slice follows once
//              its readiness counter says the slice is complete.  Attention and
//              embedding tasks take a slot as scratch.  It describes every task it
//              issues in a per-slot record (row group, rows, per-row byte offsets), so
//              the other warps never wait on the phase table in global memory.
//   math (warps 0-7)  run the int8-MMA block math of gemv_math.cuh on each stage,
//              post each task's per-warp partial sums to a queue of NQ shared-memory
//              buffers and go on with the next task; they also run the attention and
//              embedding tasks.
//   epilogue (warp 9)  reduces each queued task's partials and applies the epilogue
//              (RMSNorm divisor, RoPE + KV write, residual, SwiGLU, argmax), then
//              publishes: the tasks it finished back to back are released with one
//              fence, their counter increments go out together, and a task that
//              completes a limb group of its output builds that group's limbs for the
//              next GEMV.  Fences and counter round trips never stall the math warps.
// Attention (kv head, split) tasks copy the head group's query rows and tiles of K/V
// rows into the slot with bulk copies; each math warp runs an online softmax over its
// own positions of a tile (no barrier per position), the warps' states are merged once
// per split, and the last split of a kv head combines the splits and writes the wo
// input's limb groups.
//
// Memory ordering: data crossing CTAs is written with plain stores, fenced
// (__threadfence) before the counter increment that publishes it; readers acquire the
// counter (ld.acquire.gpu), and a reader that then copies with the async proxy (TMA)
// first executes fence.proxy.async.global.  Plain loads of cross-CTA data use .cg
// (L2), never a possibly stale L1 line.
//
// Waits: mbarrier waits are bounded by poll count, cross-CTA waits by %globaltimer
// (2 s); an expired wait records a code in the step's fault word (read by
// ib_check_fault) and the CTA winds down: the producer still completes every copy it
// started before the CTA exits.
#include <math.h>

#include <string>

#include "common.cuh"
#include "fused_gemv.cuh"
#include "quant.cuh"
#include "step.cuh"

namespace ib {

static __device__ int g_step_fault;

constexpr unsigned long long kStepTimeoutNs = 2000000000ull;
constexpr int kProducer = kNWC;      // warp index of the producer
constexpr int kEpilogue = kNWC + 1;  // warp index of the epilogue warp
constexpr int kStepThreads = (kNWC + 2) * 32;
constexpr int kNQ = 4;               // partial-sum buffers between math and epilogue warps
// CTAs per SM the kernel is built for (registers: 65536 / (CTAs * 320 threads)); the ring
// gets as many stages as fit beside them.
#ifndef IB_STEP_CTAS_PER_SM
#define IB_STEP_CTAS_PER_SM 3
#endif
constexpr int kStepCtasPerSm = IB_STEP_CTAS_PER_SM;

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Waits until *p >= target (one thread); false (fault code) after the time limit or
// when another CTA has raised a fault.
__device__ __forceinline__ bool wait_count(const int* p, int target, int code) {
    unsigned long long t0 = 0ull;
    for (uint32_t i = 0;; ++i) {
        if (ld_acquire_gpu(p) >= target) return true;
        if (i == 0) t0 = globaltimer_ns();
        if (i >= 16) {
            if (fault_raised(&g_step_fault)) return false;
            if (globaltimer_ns() - t0 > kStepTimeoutNs) {
                atomicCAS(&g_step_fault, 0, code);
                return false;
            }
            __nanosleep(64);
        }
    }
}

// Bounded barrier of the math warps (an mbarrier counting one arrival per warp).
__device__ __forceinline__ bool cbar(uint64_t* bar, uint32_t& ph, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
    const bool ok = mbar_wait(bar, ph, &g_step_fault, 30);
    ph ^= 1u;
    __syncwarp();
    return ok;
}

// Copy of a phase descriptor into shared memory by one warp.
__device__ __forceinline__ void load_phase(StepPhase* dst, const StepPhase* src, int lane) {
    static_assert(sizeof(StepPhase) % 4 == 0, "phase descriptor copied as words");
    const int* s = reinterpret_cast<const int*>(src);
    int* d = reinterpret_cast<int*>(dst);
    for (int i = lane; i < (int)(sizeof(StepPhase) / 4); i += 32) d[i] = s[i];
    __syncwarp();
}

// Split geometry of the attention for n_pos positions: `per` positions per split (at
// least kStepAttMinSplit, a multiple of the tile), `live` splits.
__device__ __forceinline__ void att_span(int n_pos, int tile, int& per, int& live) {
    per = (n_pos + kStepAttMaxSplits - 1) / kStepAttMaxSplits;
    if (per < kStepAttMinSplit) per = kStepAttMinSplit;
    per = (per + tile - 1) / tile * tile;
    live = (n_pos + per - 1) / per;
}

// RMSNorm divisor from the per-group sums of squares (warp-wide; cross-CTA data).
template <int GS>
__device__ __forceinline__ float rms_cg(const FusedGemv& g, int lane) {
    float t = 0.f;
    for (int i = lane; i < g.K / GS; i += 32) t += __ldcg(g.ssq + i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return sqrtf(t / (float)g.K + g.eps);
}

// Limb group gi of `src` (optionally times `norm`, with its sum of squares before the
// norm into ssq[gi]) into the slab: the arithmetic of xq_slab_kernel.
template <bool KQ>
__device__ __forceinline__ void build_group(const float* src, const float* norm, float* ssq,
                                            uint8_t* slab, int gi, int lane) {
    constexpr int GS = SlabG<KQ>::GS, PER = GS / 32;
    float v[PER];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = slab_elem<KQ>(gi, j, lane);
        float t = __ldcg(src + i);
        ss = fmaf(t, t, ss);
        if (norm) t *= norm[i];
        v[j] = t;
    }
    if (ssq) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) ssq[gi] = ss;
    }
    slab_write_group<KQ>(v, gi, slab, lane);
}

template <bool KQ>
__device__ __forceinline__ int* ready_ctr(const StepParams& P, int inst, int gi) {
    return P.ctr + P.ready_off + inst * P.max_slices + (gi * SlabG<KQ>::GS) / SlabG<KQ>::SE;
}

// Publishes limb group gi of slab instance inst (the group's writes are fenced first).
template <bool KQ>
__device__ __forceinline__ void publish_group(const StepParams& P, int inst, int gi, int lane) {
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(ready_ctr<KQ>(P, inst, gi), 1);
}

// The kv head whose attention row group rg of a QKV GEMV ([q; k; v] rows) feeds.
__device__ __forceinline__ int qkv_kv_head(const FusedGemv& g, int rg) {
    const int R = rg * 16, HD = g.head_dim;
    const int G = g.rows[0] / g.rows[1];
    if (R < g.rows[0]) return R / HD / G;
    if (R < g.rows[0] + g.rows[1]) return (R - g.rows[0]) / HD;
    return (R - g.rows[0] - g.rows[1]) / HD;
}

// What the producer records about a task in the slot of its first stage.
struct SlotRec {
    int task, phase, kind, rg, n, isb, spg, nb, stride;
    uint8_t off[16];  // byte offset of each tile row in its row slot
};

// Embedding task gi (one warp): elements [gi*GS, (gi+1)*GS) of the token's row,
// bit-exact dequantisation, into x; then the group's limbs of x * norm and its sum of
// squares.
template <int T>
__device__ __forceinline__ void embed_deq(const StepParams& P, int tok, int e0, float* y) {
    using F = Fmt<T>;
    constexpr int BE = F::K ? 256 : 32;
    const int blk = e0 / BE, sub = (e0 % BE) / 8;
    const uint8_t* p = P.emb + ((size_t)tok * (P.dim / BE) + blk) * F::BB;
    deq8<T>(p, sub, y);
}

template <bool KQ>
__device__ void embed_task(const StepParams& P, const StepPhase& ph, int gi, float* tmp, int lane) {
    constexpr int GS = SlabG<KQ>::GS, PER = GS / 32;
    int tok = __ldcg(P.dev_i32);
    if (tok < 0 || tok >= P.vocab) tok = 0;  // as Model::forward (src/models/model.cpp:259)
    for (int l = lane; l < GS / 8; l += 32) {
        float y[8];
        const int e0 = gi * GS + 8 * l;
        switch (P.emb_type) {
            case IB_TYPE_Q4_0: embed_deq<IB_TYPE_Q4_0>(P, tok, e0, y); break;
            case IB_TYPE_Q5_0: embed_deq<IB_TYPE_Q5_0>(P, tok, e0, y); break;
            case IB_TYPE_Q5_1: embed_deq<IB_TYPE_Q5_1>(P, tok, e0, y); break;
            case IB_TYPE_Q8_0: embed_deq<IB_TYPE_Q8_0>(P, tok, e0, y); break;
            case IB_TYPE_Q4_K: embed_deq<IB_TYPE_Q4_K>(P, tok, e0, y); break;
            default: embed_deq<IB_TYPE_Q6_K>(P, tok, e0, y); break;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) tmp[8 * l + i] = y[i];
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < PER; ++j) ph.x[gi * GS + 32 * j + lane] = tmp[32 * j + lane];
    __syncwarp();
    __threadfence();  // x is read back below through L2
    build_group<KQ>(ph.x, ph.norm, ph.ssq, ph.out_slab, gi, lane);
    publish_group<KQ>(P, ph.out_inst, gi, lane);
}

// Attention task (kv head h, split sp) on the eight math warps; scratch = the task's
// ring slot.  J = head_dim / 32 (each lane holds dims lane + 32j).  Warp w serves query
// head w % G of the kv head's group over part w / G of each tile's positions (8 / G
// parts), with its own running online-softmax state; the warps' states are merged
// once per split.  Returns false on an expired wait.
template <bool KQ, int J>
__device__ bool attn_task(const StepParams& P, const StepPhase* gph, int t, uint8_t* slot,
                          uint64_t* cb, uint32_t& cb_ph, uint64_t* abar, uint32_t& a_ph,
                          int* s_flag, int pos, int warp, int lane) {
    constexpr int HD = 32 * J;
    const int tid = warp * 32 + lane;
    const int Hkv = P.Hkv, G = P.H / Hkv, TILE = P.att_tile;
    const int parts = kNWC / G, gw = warp % G, part = warp / G, ppp = TILE / parts;
    const int first = gph->first, layer = gph->layer;
    const int h = (t - first) % Hkv, sp = (t - first) / Hkv;
    const int n_pos = pos + 1;
    int per, live;
    att_span(n_pos, TILE, per, live);
    const int p0 = sp * per, p1 = min(n_pos, p0 + per);
    const int n_out = G * HD;
    float* sK = reinterpret_cast<float*>(slot);
    float* sV = sK + TILE * HD;
    float* sq = sV + TILE * HD;
    const float* kh = gph->kc + (size_t)h * P.max_seq * HD;
    const float* vh = gph->vc + (size_t)h * P.max_seq * HD;
    const float* qh = gph->q + (size_t)h * n_out;
    // the QKV row groups of this kv head's heads have finished
    if (tid == 0)
        *s_flag = wait_count(P.ctr + P.att_ready_off + layer * P.max_kv + h, P.att_target, 41);
    if (!cbar(cb, cb_ph, lane)) return false;
    if (!*s_flag) return false;
    float m = -INFINITY, l = 0.f, acc[J], qr[J];
#pragma unroll
    for (int j = 0; j < J; ++j) acc[j] = 0.f;
    for (int t0 = p0; t0 < p1; t0 += TILE) {
        const int nt = min(TILE, p1 - t0);
        if (tid == 0) {
            const uint32_t kv = (uint32_t)(nt * HD * 4);
            fence_proxy_async_global();  // k/v row `pos` and q were written by other CTAs
            mbar_arrive_expect_tx(abar, 2 * kv + (t0 == p0 ? (uint32_t)(n_out * 4) : 0u));
            if (t0 == p0) bulk_g2s(sq, qh, (uint32_t)(n_out * 4), abar);
            bulk_g2s(sK, kh + (size_t)t0 * HD, kv, abar);
            bulk_g2s(sV, vh + (size_t)t0 * HD, kv, abar);
        }
        const bool got = mbar_wait(abar, a_ph, &g_step_fault, 31);
        a_ph ^= 1u;
        if (!got) return false;
        if (t0 == p0) {
#pragma unroll
            for (int j = 0; j < J; ++j) qr[j] = sq[gw * HD + lane + 32 * j] * P.scale;
        }
        // this warp's positions of the tile, two at a time (their reductions interleaved),
        // one online-softmax update per pair
        const int s_end = min(nt, (part + 1) * ppp);
        for (int s0 = part * ppp; s0 < s_end; s0 += 2) {
            const int s1 = s0 + 1;
            const bool has1 = s1 < s_end;
            float a = 0.f, b = 0.f, v0[J], v1[J];
#pragma unroll
            for (int j = 0; j < J; ++j) {
                const int e = lane + 32 * j;
                a = fmaf(qr[j], sK[s0 * HD + e], a);
                b = has1 ? fmaf(qr[j], sK[s1 * HD + e], b) : b;
                v0[j] = sV[s0 * HD + e];
                v1[j] = has1 ? sV[s1 * HD + e] : 0.f;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                a += __shfl_xor_sync(0xffffffffu, a, o);
                b += __shfl_xor_sync(0xffffffffu, b, o);
            }
            if (!has1) b = -INFINITY;
            const float mn = fmaxf(m, fmaxf(a, b));
            const float al = m == -INFINITY ? 0.f : expf(m - mn);
            const float e0 = expf(a - mn), e1 = has1 ? expf(b - mn) : 0.f;
            l = fmaf(l, al, e0 + e1);
#pragma unroll
            for (int j = 0; j < J; ++j) acc[j] = fmaf(acc[j], al, fmaf(e0, v0[j], e1 * v1[j]));
            m = mn;
        }
        if (!cbar(cb, cb_ph, lane)) return false;  // the tile buffer is free again
    }
    // merge the warps' states: per warp (m, l) and its accumulator, then one partial
    // (max M, sum L, unnormalised accumulator) per query head of this split
    float* sacc = reinterpret_cast<float*>(slot);                 // [kNWC][HD]
    float2* sml = reinterpret_cast<float2*>(sacc + kNWC * HD);  // [kNWC]
#pragma unroll
    for (int j = 0; j < J; ++j) sacc[warp * HD + lane + 32 * j] = acc[j];
    if (lane == 0) sml[warp] = make_float2(m, l);
    if (!cbar(cb, cb_ph, lane)) return false;
    for (int idx = tid; idx < n_out; idx += kNWC * 32) {
        const int g = idx / HD, e = idx - g * HD;
        float M = -INFINITY;
        for (int w = g; w < kNWC; w += G) M = fmaxf(M, sml[w].x);
        float L = 0.f, a = 0.f;
        for (int w = g; w < kNWC; w += G) {
            const float2 v = sml[w];
            const float wt = v.x == -INFINITY ? 0.f : expf(v.x - M);
            L = fmaf(wt, v.y, L);
            a = fmaf(wt, sacc[w * HD + e], a);
        }
        P.att_acc[((size_t)(h * G + g) * kStepAttMaxSplits + sp) * HD + e] = a;
        if (e == 0) P.att_ml[(size_t)(h * G + g) * kStepAttMaxSplits + sp] = make_float2(M, L);
    }
    __threadfence();
    if (!cbar(cb, cb_ph, lane)) return false;
    if (tid == 0) *s_flag = atomicAdd(P.ctr + P.att_done_off + layer * P.max_kv + h, 1) == live - 1;
    if (!cbar(cb, cb_ph, lane)) return false;
    if (!*s_flag) return true;
    __threadfence();
    // the last split combines: weights per split, then the outputs, then the limb groups
    float* wsp = reinterpret_cast<float*>(slot);  // [G][kStepAttMaxSplits]
    float* linv = wsp + G * kStepAttMaxSplits;    // [G]
    float* ov = linv + 8;                         // [G * HD]
    for (int g = warp; g < G; g += kNWC) {
        const float2* ml = P.att_ml + (size_t)(h * G + g) * kStepAttMaxSplits;
        float m4[4], l4[4];
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int ci = lane + 32 * k;
            const float2 v = ci < live ? __ldcg(ml + ci) : make_float2(-INFINITY, 0.f);
            m4[k] = v.x;
            l4[k] = v.y;
            M = fmaxf(M, v.x);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int ci = lane + 32 * k;
            const float w = ci < live ? expf(m4[k] - M) : 0.f;
            wsp[g * kStepAttMaxSplits + ci] = w;
            L = fmaf(w, l4[k], L);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (lane == 0) linv[g] = 1.0f / L;
    }
    if (!cbar(cb, cb_ph, lane)) return false;
    // four threads per four consecutive outputs, each over a quarter of the splits (8
    // loads in flight), combined with two shuffles; the loop runs on whole warps
    for (int i0 = warp * 32; i0 < n_out; i0 += kNWC * 32) {
        const int i = i0 + lane;
        const bool act = i < n_out;
        const int quad = act ? i >> 2 : 0, qtr = i & 3;
        const int g = (quad * 4) / HD, e = quad * 4 - g * HD;
        const float4* src = reinterpret_cast<const float4*>(
            P.att_acc + (size_t)(h * G + g) * kStepAttMaxSplits * HD + e);
        const float* w = wsp + g * kStepAttMaxSplits;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = qtr; act && c0 < live; c0 += 32) {
            float4 b[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int ci = c0 + 4 * u;
                b[u] = ci < live ? __ldcg(src + (size_t)ci * (HD / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int ci = c0 + 4 * u;
                const float wt = ci < live ? w[ci] : 0.f;
                a.x = fmaf(wt, b[u].x, a.x);
                a.y = fmaf(wt, b[u].y, a.y);
                a.z = fmaf(wt, b[u].z, a.z);
                a.w = fmaf(wt, b[u].w, a.w);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            a.x += __shfl_xor_sync(0xffffffffu, a.x, o);
            a.y += __shfl_xor_sync(0xffffffffu, a.y, o);
            a.z += __shfl_xor_sync(0xffffffffu, a.z, o);
            a.w += __shfl_xor_sync(0xffffffffu, a.w, o);
        }
        if (act && qtr == 0) {
            const float inv = linv[g];
            ov[quad * 4 + 0] = a.x * inv;
            ov[quad * 4 + 1] = a.y * inv;
            ov[quad * 4 + 2] = a.z * inv;
            ov[quad * 4 + 3] = a.w * inv;
        }
    }
    if (!cbar(cb, cb_ph, lane)) return false;
    constexpr int GS = SlabG<KQ>::GS, PER = GS / 32;
    const int base_el = h * n_out;
    uint8_t* slab = gph->out_slab;
    const int inst = gph->out_inst;
    for (int gl = warp; gl < n_out / GS; gl += kNWC) {
        float v[PER];
        slab_load<KQ>(ov, gl, lane, v);
        const int gi = (base_el + gl * GS) / GS;
        slab_write_group<KQ>(v, gi, slab, lane);
        publish_group<KQ>(P, inst, gi, lane);
    }
    return true;
}

// Epilogue of one GEMV task on the epilogue warp: lanes 0..15 hold the task's finished
// rows (v, before the RMSNorm divisor).
__device__ __forceinline__ void task_epilogue(const StepPhase& ph, int rg, int lane, float v) {
    const FusedGemv& g = ph.g;
    switch (ph.epi) {
        case EPI_QKV: epilogue<EPI_QKV>(g, rg, lane, v); break;
        case EPI_SWIGLU: epilogue<EPI_SWIGLU>(g, rg, lane, v); break;
        case EPI_ARGMAX: epilogue<EPI_ARGMAX>(g, rg, lane, v); break;
        case EPI_RESID: {  // x += rows; x was last written by another CTA: read it from L2
            const int R = rg * 16 + lane;
            if (lane < group_rows(g, rg)) g.y[R] = __ldcg(g.y + R) + v;
        } break;
        default: epilogue<EPI_STORE>(g, rg, lane, v); break;
    }
}

template <int TA, int TB, int J>
__global__ void __launch_bounds__(kStepThreads, kStepCtasPerSm) decode_step_kernel(const StepParams P) {
    using PR = Pair<TA, TB>;
    constexpr bool KQ = PR::KQ;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kStepMaxStages], empty[kStepMaxStages];
    __shared__ __align__(8) uint64_t qfull[kNQ], qfree[kNQ], cb, abar;
    __shared__ SlotRec rec[kStepMaxStages];
    __shared__ int s_need[kStepMaxStages], s_tgt[kStepMaxStages];
    __shared__ const uint8_t* s_src[kStepMaxStages];
    __shared__ const int* s_rdy[kStepMaxStages];
    __shared__ float red[kNQ][kNWC][16];
    __shared__ int q_task[kNQ], q_phase[kNQ];
    __shared__ __align__(16) StepPhase s_pph, s_eph;  // the producer's / epilogue's phase
    __shared__ int s_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = P.S;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNWC);
        }
        for (int b = 0; b < kNQ; ++b) {
            mbar_init(&qfull[b], kNWC);
            mbar_init(&qfree[b], 1);
        }
        mbar_init(&cb, kNWC);
        mbar_init(&abar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int pos = __ldcg(P.dev_i32 + 1);

    if (warp == kProducer) {
        // ---------------- producer ----------------
        int att_per, att_live;
        att_span(pos + 1, P.att_tile, att_per, att_live);
        int issue = 0, e_slot = 0, e_round = 0;  // stages issued; slot and round of the next
        int sl = 0, s_slot = 0;                  // stages whose slice went out
        int pc = -1, next_first = 0, t_cur = 0, st_cur = 0, spg_cur = 0;
        bool ended = false, ok = true;
        int claim = 0;  // lane 0: the next task index (claimed one task ahead)
        if (lane == 0) claim = atomicAdd(P.ctr, 1);
        unsigned long long t_last = globaltimer_ns();
        while (ok) {
            bool prog = false;
            if (!ended) {
                int fr = issue < S;
                if (!fr && lane == 0) fr = mbar_test_wait(&empty[e_slot], (e_round - 1) & 1);
                fr = __shfl_sync(0xffffffffu, fr, 0);
                if (fr) {
                    while (st_cur == spg_cur) {  // next task
                        const int t = __shfl_sync(0xffffffffu, claim, 0);
                        if (lane == 0) claim = atomicAdd(P.ctr, 1);
                        if (t >= P.n_tasks) {
                            ended = true;
                            break;
                        }
                        if (pc < 0 || t >= next_first) {
                            while (pc + 1 < P.n_phases && t >= P.phases[pc + 1].first) ++pc;
                            load_phase(&s_pph, P.phases + pc, lane);
                            next_first = pc + 1 < P.n_phases ? P.phases[pc + 1].first : P.n_tasks;
                        }
                        if (s_pph.kind == TK_ATTN && (t - s_pph.first) / P.Hkv >= att_live) {
                            // splits past the live ones: every later slot of the phase is too
                            if (lane == 0) atomicMax(P.ctr, s_pph.first + s_pph.n);
                            continue;
                        }
                        t_cur = t;
                        st_cur = 0;
                        spg_cur = s_pph.kind == TK_GEMV ? s_pph.spg : 1;
                    }
                    SlotRec& r = rec[e_slot];
                    if (ended) {
                        if (lane == 0) {
                            r.task = -1;
                            s_need[e_slot] = 0;
                            mbar_arrive(&full[e_slot]);
                        }
                    } else if (s_pph.kind == TK_GEMV) {
                        const FusedGemv& g = s_pph.g;
                        const int rg = t_cur - s_pph.first;
                        const bool isb = group_is_b<TA, TB>(g, rg);
                        const int bb = isb ? Fmt<TB>::BB : Fmt<TA>::BB;
                        const int nbl = min(PR::KB, s_pph.nb - st_cur * PR::KB);
                        const int n = group_rows(g, rg);
                        const int stride = isb ? P.slot_b : P.slot_a;
                        uint32_t len = 0, off = 0;
                        const uint8_t* a0 = nullptr;
                        if (lane < n) {
                            int seg, lr;
                            tile_row(g, rg, lane, seg, lr);
                            const uint8_t* src = g.W[seg] + (size_t)lr * s_pph.nb * bb +
                                                 (size_t)st_cur * PR::KB * bb;
                            off = (uint32_t)((uintptr_t)src & 15u);
                            a0 = src - off;
                            len = (off + (uint32_t)(nbl * bb) + 15u) & ~15u;
                        }
                        uint32_t tot = len;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
                        if (st_cur == 0 && lane < 16) r.off[lane] = (uint8_t)off;
                        __syncwarp();  // the record is complete before lane 0's arrival
                        if (lane == 0) {
                            if (st_cur == 0) {
                                r.task = t_cur;
                                r.phase = pc;
                                r.kind = TK_GEMV;
                                r.rg = rg;
                                r.n = n;
                                r.isb = isb;
                                r.spg = s_pph.spg;
                                r.nb = s_pph.nb;
                                r.stride = stride;
                            }
                            s_need[e_slot] = 1;
                            s_src[e_slot] = g.slab + (size_t)st_cur * PR::SLICE;
                            s_rdy[e_slot] = s_pph.in_inst >= 0
                                                ? P.ctr + P.ready_off + s_pph.in_inst * P.max_slices + st_cur
                                                : nullptr;
                            const int left = g.K - st_cur * PR::SE;
                            s_tgt[e_slot] = (left < PR::SE ? left : PR::SE) / PR::GS;
                            mbar_arrive_expect_tx(&full[e_slot], tot + (uint32_t)PR::SLICE);
                        }
                        __syncwarp();
                        if (lane < n)
                            bulk_g2s(smem + (size_t)e_slot * P.stage_bytes + (size_t)lane * stride, a0,
                                     len, &full[e_slot]);
                        ++st_cur;
                    } else {
                        if (lane == 0) {
                            r.task = t_cur;
                            r.phase = pc;
                            r.kind = s_pph.kind;
                            s_need[e_slot] = 0;
                            mbar_arrive(&full[e_slot]);
                        }
                        ++st_cur;
                    }
                    __syncwarp();
                    ++issue;
                    if (++e_slot == S) {
                        e_slot = 0;
                        ++e_round;
                    }
                    prog = true;
                }
            }
            // limb slices, in stage order, once published
            while (sl < issue) {
                int go = 1;
                if (lane == 0 && s_need[s_slot]) {
                    const int* rp = s_rdy[s_slot];
                    go = !rp || ld_acquire_gpu(rp) >= s_tgt[s_slot];
                    if (go) {
                        fence_proxy_async_global();
                        bulk_g2s(smem + (size_t)s_slot * P.stage_bytes + P.wbytes, s_src[s_slot],
                                 (uint32_t)PR::SLICE, &full[s_slot]);
                    }
                }
                go = __shfl_sync(0xffffffffu, go, 0);
                if (!go) break;
                ++sl;
                if (++s_slot == S) s_slot = 0;
                prog = true;
            }
            if (ended && sl == issue) break;
            if (prog) {
                t_last = globaltimer_ns();
            } else {
                int stop = 0;
                if (lane == 0) {
                    if (fault_raised(&g_step_fault)) stop = 1;
                    else if (globaltimer_ns() - t_last > kStepTimeoutNs) {
                        atomicCAS(&g_step_fault, 0, 40);
                        stop = 1;
                    }
                }
                stop = __shfl_sync(0xffffffffu, stop, 0);
                if (stop) ok = false;
                else __nanosleep(32);
            }
        }
        // every started copy completes before the CTA exits: slices not yet sent (only
        // after a fault) go out now, from the slab as it is
        while (sl < issue) {
            if (lane == 0 && s_need[s_slot])
                bulk_g2s(smem + (size_t)s_slot * P.stage_bytes + P.wbytes, s_src[s_slot],
                         (uint32_t)PR::SLICE, &full[s_slot]);
            ++sl;
            if (++s_slot == S) s_slot = 0;
        }
        for (int j = issue > S ? issue - S : 0; j < issue; ++j)
            mbar_wait(&full[j % S], (j / S) & 1, &g_step_fault, 12);
    } else if (warp == kEpilogue) {
        // ---------------- epilogue ----------------
        int q = 0, cached = -1;
        float rms = 1.0f;
        bool rms_ok = false;
        for (;;) {
            int b = q & (kNQ - 1);
            if (!mbar_wait(&qfull[b], (q / kNQ) & 1, &g_step_fault, 16)) break;
            int t = q_task[b];
            if (t < 0) break;
            const int pc = q_phase[b];
            if (pc != cached) {
                load_phase(&s_eph, P.phases + pc, lane);
                cached = pc;
                rms_ok = false;
            }
            const StepPhase& ph = s_eph;
            if (ph.pro == PRO_NORM && !rms_ok) {
                rms = rms_cg<PR::GS>(ph.g, lane);  // every group of the input is in
                rms_ok = true;
            }
            // the tasks queued back to back in this phase: epilogues first, then one fence
            // and their counter increments together (lane i carries task i's)
            int n = 0, my_ctr = -1, my_gi = 0;
            for (;;) {
                float v = 0.f;
                if (lane < 16) {
#pragma unroll
                    for (int w = 0; w < kNWC; ++w) v += red[b][w][lane];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&qfree[b]);
                const int rg = t - ph.first;
                task_epilogue(ph, rg, lane, ph.pro == PRO_NORM ? v / rms : v);
                int ctr = -1, gi = 0;
                if (ph.epi == EPI_QKV) {
                    ctr = P.att_ready_off + ph.layer * P.max_kv + qkv_kv_head(ph.g, rg);
                } else if (ph.out_inst >= 0) {
                    gi = rg * (ph.epi == EPI_SWIGLU ? 8 : 16) / PR::GS;
                    ctr = P.grp_off + ph.out_inst * P.max_groups + gi;
                }
                if (lane == n) {
                    my_ctr = ctr;
                    my_gi = gi;
                }
                ++q;
                ++n;
                if (n == kNQ) break;
                b = q & (kNQ - 1);
                if (!mbar_test_wait(&qfull[b], (q / kNQ) & 1)) break;
                const int t2 = q_task[b];
                if (t2 < 0 || q_phase[b] != pc) break;  // left for the next round
                t = t2;
            }
            if (!__any_sync(0xffffffffu, lane < n && my_ctr >= 0)) continue;  // nothing to publish
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane < n && my_ctr >= 0) {
                const int old = atomicAdd(P.ctr + my_ctr, 1);
                last = ph.epi != EPI_QKV && old == ph.out_per_group - 1;
            }
            unsigned mask = __ballot_sync(0xffffffffu, last);
            if (mask) {
                __threadfence();  // the other tasks' rows of the group are visible
                for (unsigned mk = mask; mk; mk &= mk - 1) {
                    const int gi = __shfl_sync(0xffffffffu, my_gi, __ffs(mk) - 1);
                    build_group<KQ>(ph.out_src, ph.out_norm, ph.out_ssq, ph.out_slab, gi, lane);
                }
                __threadfence();
                __syncwarp();
                if (last) atomicAdd(ready_ctr<KQ>(P, ph.out_inst, my_gi), 1);
            }
        }
    } else {
        // ---------------- math warps ----------------
        const LaneCtx c = lane_ctx();
        const LeanLane ll = lean_lane(c);
        float acc_a = 0.f, acc_b = 0.f;
        int cs = 0, cpar = 0, q = 0;
        uint32_t cb_ph = 0, a_ph = 0;
        for (;;) {
            if (!mbar_wait(&full[cs], cpar, &g_step_fault, 13)) break;
            const SlotRec& r = rec[cs];
            const int t = r.task;
            if (t < 0) break;
            if (r.kind == TK_GEMV) {
                const int n = r.n, spg = r.spg, nb = r.nb, stride = r.stride, pc = r.phase;
                const bool isb = r.isb;
                const int ra = c.g < n ? c.g : n - 1, rb = c.g + 8 < n ? c.g + 8 : n - 1;
                const int oa = r.off[ra], ob = r.off[rb];
                bool ok = true;
                for (int st = 0; st < spg; ++st) {
                    if (st > 0 && !mbar_wait(&full[cs], cpar, &g_step_fault, 13)) {
                        ok = false;
                        break;
                    }
                    const uint8_t* base = smem + (size_t)cs * P.stage_bytes;
                    const int nbl = min(PR::KB, nb - st * PR::KB);
                    if (isb)
                        stage_math<TB, PR::KB, PR::SE, PR::GS, false>(
                            base, base + P.wbytes, stride, ra, rb, oa, ob, nbl, c, ll, warp, acc_a,
                            acc_b);
                    else
                        stage_math<TA, PR::KB, PR::SE, PR::GS, false>(
                            base, base + P.wbytes, stride, ra, rb, oa, ob, nbl, c, ll, warp, acc_a,
                            acc_b);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[cs]);
                    if (++cs == S) {
                        cs = 0;
                        cpar ^= 1;
                    }
                }
                if (!ok) break;
                // the task's partials to the epilogue warp's queue
                const int b = q & (kNQ - 1);
                if (q >= kNQ && !mbar_wait(&qfree[b], ((q / kNQ) - 1) & 1, &g_step_fault, 15)) break;
                acc_a = quad_sum(acc_a);
                acc_b = quad_sum(acc_b);
                if (c.t == 0) {
                    red[b][warp][c.g] = acc_a;
                    red[b][warp][c.g + 8] = acc_b;
                }
                if (warp == 0 && lane == 0) {
                    q_task[b] = t;
                    q_phase[b] = pc;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&qfull[b]);
                acc_a = 0.f;
                acc_b = 0.f;
                ++q;
            } else {
                uint8_t* slot = smem + (size_t)cs * P.stage_bytes;
                const StepPhase* gph = P.phases + r.phase;
                bool ok = true;
                if (r.kind == TK_ATTN)
                    ok = attn_task<KQ, J>(P, gph, t, slot, &cb, cb_ph, &abar, a_ph, &s_flag, pos, warp,
                                          lane);
                else if (warp == 0)
                    embed_task<KQ>(P, *gph, t - gph->first, reinterpret_cast<float*>(slot), lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[cs]);
                if (++cs == S) {
                    cs = 0;
                    cpar ^= 1;
                }
                if (!ok) break;
            }
        }
        // end of the epilogue warp's queue
        const int b = q & (kNQ - 1);
        const bool fr = q < kNQ || mbar_wait(&qfree[b], ((q / kNQ) - 1) & 1, &g_step_fault, 15);
        if (fr) {
            if (warp == 0 && lane == 0) q_task[b] = -1;
            __syncwarp();
            if (lane == 0) mbar_arrive(&qfull[b]);
        }
    }
    __syncthreads();
    // the last CTA out feeds the greedy token back (every task has completed)
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(P.ctr + 1, 1) == (int)gridDim.x - 1) {
            __threadfence();
            const unsigned long long key = atomicAdd(P.best, 0ull);
            const int next = argmax_key_row(key);
            *P.best = 0ull;
            P.dev_i32[2] = next;
            if (P.tokens && pos >= 0 && pos < P.max_seq) P.tokens[pos] = next;
            P.dev_i32[0] = next;
            P.dev_i32[1] = pos + 1;
        }
    }
}

// ---- host side ----------------------------------------------------------------------
size_t step_counter_bytes(int n_inst, int max_slices, int max_groups, int n_layers, int max_kv) {
    const size_t n = 2 + (size_t)n_inst * (max_slices + max_groups) + 2ull * n_layers * max_kv;
    return (n * 4 + 255) / 256 * 256;
}

// Shared memory an attention task needs (K/V tile + query rows; the warps' merge area;
// the combine's weights and outputs).
static size_t attention_smem(int G, int HD, int tile) {
    const size_t a = (size_t)2 * tile * HD * 4 + (size_t)G * HD * 4;
    const size_t b = (size_t)kNWC * HD * 4 + (size_t)kNWC * 8;
    const size_t c = (size_t)G * kStepAttMaxSplits * 4 + 8 * 4 + (size_t)G * HD * 4;
    return a > b ? (a > c ? a : c) : (b > c ? b : c);
}

// Row stride in a stage: >= the chunk (+16 when rows start unaligned), a multiple of 16,
// congruent to 32 (Q4_K) or 16 modulo 128 (bank spread of the math warps' row loads).
static int step_slot(int type, int chunk, bool pad) {
    const int want = type == IB_TYPE_Q4_K ? 32 : 16;
    int s = (chunk + (pad ? 16 : 0) + 15) / 16 * 16;
    while (s % 128 != want) s += 16;
    return s;
}

template <int TA, int TB, int J>
static int geometry_inst(StepParams& p, int* grid) {
    auto kern = decode_step_kernel<TA, TB, J>;
    int dev = 0, sms = 0, max_optin = 0, per_sm = 0;
    IB_CUDA_CHECK(cudaGetDevice(&dev));
    IB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    IB_CUDA_CHECK(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cudaFuncAttributes fa;
    IB_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
    // kStepCtasPerSm CTAs per SM with as many stages as fit (at most kStepMaxStages),
    // else two stages at whatever fits
    int S = kStepMaxStages;
    for (; S >= 2; --S) {
        const size_t smem = (size_t)S * p.stage_bytes;
        if (smem + fa.sharedSizeBytes > (size_t)max_optin) continue;
        IB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        IB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStepThreads, smem));
        if (per_sm >= kStepCtasPerSm) break;
    }
    if (S < 2) {
        S = 2;
        const size_t smem = (size_t)S * p.stage_bytes;
        IB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        IB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStepThreads, smem));
        if (per_sm < 1) {
            set_error("decode step: ring does not fit on an SM");
            return IB_ERR_UNSUPPORTED;
        }
    }
    p.S = S;
    *grid = per_sm * sms;
    return IB_OK;
}

template <int TA, int TB>
static int geometry_pair(bool pad_a, bool pad_b, int G, int HD, StepParams& p, int* grid) {
    using PR = Pair<TA, TB>;
    p.slot_a = step_slot(TA, PR::KB * Fmt<TA>::BB, pad_a);
    p.slot_b = step_slot(TB, PR::KB * Fmt<TB>::BB, pad_b);
    p.wbytes = 16 * (p.slot_a > p.slot_b ? p.slot_a : p.slot_b);
    const int stage = p.wbytes + PR::SLICE;
    // the attention tile: up to 32 positions whose K and V rows fit the stage
    int tile = 32;
    while (tile > 8 && attention_smem(G, HD, tile) > (size_t)stage) tile -= 8;
    if (attention_smem(G, HD, tile) > (size_t)stage) {
        set_error("decode step: attention scratch does not fit a ring stage");
        return IB_ERR_UNSUPPORTED;
    }
    p.att_tile = tile;
    p.stage_bytes = (stage + 127) / 128 * 128;
    p.kq = PR::KQ ? 1 : 0;
    switch (HD) {
        case 32: return geometry_inst<TA, TB, 1>(p, grid);
        case 64: return geometry_inst<TA, TB, 2>(p, grid);
        case 128: return geometry_inst<TA, TB, 4>(p, grid);
    }
    set_error("decode step: head_dim must be 32, 64 or 128");
    return IB_ERR_UNSUPPORTED;
}

static int pair_index(int type) {
    switch (type) {
        case IB_TYPE_Q4_K:
        case IB_TYPE_Q6_K: return 0;
        case IB_TYPE_Q4_0:
        case IB_TYPE_Q8_0: return 1;
        case IB_TYPE_Q5_0:
        case IB_TYPE_Q5_1: return 2;
    }
    return -1;
}

int step_geometry(int type_a, bool pad_a, bool pad_b, int G, int HD, StepParams& p, int* grid) {
    if (G < 1 || G > 8 || 8 % G || G * HD > 1024) {
        set_error("decode step: 1, 2, 4 or 8 query heads per kv head");
        return IB_ERR_UNSUPPORTED;
    }
    switch (pair_index(type_a)) {
        case 0: return geometry_pair<IB_TYPE_Q4_K, IB_TYPE_Q6_K>(pad_a, pad_b, G, HD, p, grid);
        case 1: return geometry_pair<IB_TYPE_Q4_0, IB_TYPE_Q8_0>(pad_a, pad_b, G, HD, p, grid);
        case 2: return geometry_pair<IB_TYPE_Q5_0, IB_TYPE_Q5_1>(pad_a, pad_b, G, HD, p, grid);
    }
    set_error("decode step: unsupported weight formats");
    return IB_ERR_UNSUPPORTED;
}

template <int TA, int TB>
static int launch_pair(const StepParams& p, int grid, cudaStream_t st) {
    const size_t smem = (size_t)p.S * p.stage_bytes;
    switch (p.HD) {
        case 32: decode_step_kernel<TA, TB, 1><<<grid, kStepThreads, smem, st>>>(p); break;
        case 64: decode_step_kernel<TA, TB, 2><<<grid, kStepThreads, smem, st>>>(p); break;
        case 128: decode_step_kernel<TA, TB, 4><<<grid, kStepThreads, smem, st>>>(p); break;
        default:
            set_error("decode step: head_dim must be 32, 64 or 128");
            return IB_ERR_UNSUPPORTED;
    }
    IB_LAUNCH_CHECK("decode_step_kernel");
    return IB_OK;
}

int step_launch(const StepParams& p, int type_a, int grid, cudaStream_t st) {
    switch (pair_index(type_a)) {
        case 0: return launch_pair<IB_TYPE_Q4_K, IB_TYPE_Q6_K>(p, grid, st);
        case 1: return launch_pair<IB_TYPE_Q4_0, IB_TYPE_Q8_0>(p, grid, st);
        case 2: return launch_pair<IB_TYPE_Q5_0, IB_TYPE_Q5_1>(p, grid, st);
    }
    set_error("decode step: unsupported weight formats");
    return IB_ERR_UNSUPPORTED;
}

int step_fault_take(int* code) {
    int v = 0, z = 0;
    IB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_step_fault, sizeof(int)));
    if (v) IB_CUDA_CHECK(cudaMemcpyToSymbol(g_step_fault, &z, sizeof(int)));
    *code = v;
    return IB_OK;
}

}  // namespace ib
