// Fused decode GEMV (decode.cu).
//
// An activation vector enters a GEMV as a "limb slab": the exact four-int8-limb split
// of its FP32 values (see gemv_math.cuh), laid out in slices of SE elements so that
// the GEMV's producer warp can TMA-copy the slice of each pipeline stage next to the
// stage's weight rows.  Slice layout (bytes): limbs [SE/32][4][32] int8 | scale
// [SE/GS] | sum32 [SE/32] | sum16 [SE/16] (FP32), padded to 16 bytes.  K-quant weights
// use SE = 2048, GS = 256; 32-element blocks SE = 1024, GS = 32.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib {

enum { PRO_PLAIN = 0, PRO_NORM = 1 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4, EPI_ALLRED = 5 };

// Tensor-parallel exchange over peer memory (NVLink): each rank owns a region that
// every rank maps; region[q] is rank q's as seen from this rank.  Region layout:
// tagged rows u64 [2][world][stride] | tagged keys u64 [2][world][2].  Exchange e
// (counted by *seq, identical on every rank since every rank runs the same steps)
// uses slot e & 1: each rank stores its rows, as (e + 1) << 32 | float bits, into slot
// row [rank] of every region; a receiver polls the words of its own region until their
// tags read e + 1 and sums the rows in rank order.  A slot is rewritten two exchanges
// later, after every rank has produced the exchange in between, which it does only
// once its reads of the earlier one are done.
constexpr int kMaxRanks = 8;
struct TpExchange {
    uint8_t* region[kMaxRanks];
    uint32_t* seq;  // this rank's exchange counter (device)
    int rank, world, stride;
};

__host__ __device__ inline size_t tp_keys_offset(int world, int stride) {
    return (size_t)2 * world * stride * 8;
}
__host__ __device__ inline size_t tp_region_bytes(int world, int stride) {
    return (tp_keys_offset(world, stride) + (size_t)2 * world * 2 * 8 + 255) / 256 * 256;
}

struct SlabGeom {
    int SE;           // elements per slice
    int GS;           // elements per limb scale
    int slice_bytes;  // bytes per slice
};

__host__ __device__ inline SlabGeom slab_geom(bool kquant) {
    SlabGeom g;
    g.SE = kquant ? 2048 : 1024;
    g.GS = kquant ? 256 : 32;
    const int b = g.SE * 4 + (g.SE / g.GS + g.SE / 32 + g.SE / 16) * 4;
    g.slice_bytes = (b + 15) / 16 * 16;
    return g;
}

__host__ __device__ inline size_t slab_total_bytes(int K, bool kquant) {
    const SlabGeom g = slab_geom(kquant);
    return (size_t)((K + g.SE - 1) / g.SE) * g.slice_bytes;
}

// True for the K-quant formats (slab geometry SE 2048 / GS 256).
bool slab_kquant(int type);

// True for the formats the fused limb-slab GEMV decodes (the six of gemv_mma and Q5_K).
bool slab_supported(int type);

// slab <- limbs of x (norm == nullptr) or of x * norm; ssq[g] <- sum of x^2 over scale
// group g (when ssq != nullptr; the RMSNorm of x is then applied in the GEMV
// epilogue as 1 / sqrt(sum(ssq) / K + eps)).  K must be a multiple of GS.
// With an exchange (tp, world > 1): x (K <= stride) is first completed with the latest
// exchange's rows, x[i] += their sum over the ranks, and written back.
int xq_slab_launch(const float* x, const float* norm, int K, bool kquant, uint8_t* slab,
                   float* ssq, cudaStream_t st, bool pdl, const TpExchange* tp = nullptr);
// After a head GEMV with an ARGMAX exchange: *best <- the maximum key over the ranks.
int tp_key_max_launch(const TpExchange& x, unsigned long long* best, cudaStream_t st);

struct FusedGemv {
    // Weight rows: segments concatenated in row order (row groups of 16), or, with
    // `paired`, row group i = rows [8i, 8i+8) of segment 0 followed by the same
    // rows of segment 1 (both segments of equal shape and type).
    const uint8_t* W[3];
    int type[3];
    int rows[3];
    int n_seg;
    int paired;
    int K;  // columns of every segment
    // input: limb slab of x (xq_slab_launch); PRO_NORM: sums of squares for RMSNorm
    const uint8_t* slab;
    const float* ssq;
    float eps;
    // epilogue
    // STORE / ARGMAX: y[row]; RESID: y[row] += ; SWIGLU: y[i] = silu(g_i) * u_i;
    // ALLRED: y[row] += the sum over the ranks of their rows (tp exchange)
    float* y;
    float* q;  // QKV: segment 0 after RoPE -> q; segment 1 -> kc; segment 2 -> vc
    float* kc;  // FP32, or FP16 (__half) when kv_half
    float* vc;
    int kv_half;
    const float* rope;  // [max_seq][head_dim / 2][cos, sin]
    const int* pos;     // device position of the token
    int head_dim, max_seq;
    unsigned long long* best;  // ARGMAX: max of (ordered logit << 32 | ~(row_base + row))
    int row_base;              // ARGMAX: global index of this kernel's first row
    // ALLRED, and ARGMAX with tp.world > 1 (the key maximum over the ranks): the exchange;
    // both need `work` (its second counter finds the last CTA, which exchanges)
    TpExchange tp;
    // optional work counters {next row group, CTAs done}, zero between launches: row
    // groups are then claimed dynamically (balanced over SMs); null = static schedule.
    // work_ext = 1: the caller zeroes them between launches, so the CTAs skip counting
    // themselves out on exit (an exchange's last CTA still does)
    int* work;
    int work_ext;
    // optional K split of long rows (EPI_RESID with more than 8 stages per row): every
    // row group is two work units, its first and second half of stages.  A unit's rows go
    // to kpart[rg][half][16]; the unit that finishes second (kcnt[rg], zero between
    // launches) adds the two halves and runs the epilogue.  Null: one unit per row group.
    float* kpart;
    int* kcnt;
};

// Launches the fused GEMV; IB_ERR_UNSUPPORTED when the type mix or shapes have no
// fused kernel (the caller then uses the separate kernels).
int fused_gemv_launch(const FusedGemv& p, int pro, int epi, cudaStream_t st, bool pdl);
bool fused_gemv_supported(const FusedGemv& p, int epi);
// One tensor-parallel exchange round in isolation (the sending side of a row-split
// GEMV's epilogue with zero rows, then the receiving slab kernel that adds every rank's
// rows to xv[0..n) and builds its slab): collective, every rank launches the same rounds.
int tp_probe_launch(const TpExchange& x, float* xv, int n, bool kquant, uint8_t* slab,
                    cudaStream_t st);
// Reads and clears the fused kernels' fault word (0 = no bounded wait expired).
int decode_fault_take(int* code);
// Decodes the ARGMAX key into a row index (resets nothing).
__host__ __device__ inline int argmax_key_row(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}

}  // namespace ib
