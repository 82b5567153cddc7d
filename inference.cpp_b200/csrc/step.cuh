// Persistent decode step (step.cu): one kernel launch runs a whole batch-1 decode
// step of the Llama forward -- embedding, every layer's QKV / attention / wo /
// gate+up / down, the output head with its argmax, and the token feedback.
//
// The step is a list of tasks in dependency order: embedding groups, then per layer
// the QKV row groups, the attention splits, the wo row groups, the gate+up row groups
// and the down row groups, then the head's row groups.  CTAs claim tasks from one
// atomic counter in that order and run the tasks they claimed in claim order, so every
// task's inputs come from tasks with smaller indices that running CTAs have claimed:
// the step cannot deadlock, whatever number of CTAs is resident.  Each CTA's producer
// warp streams the weight bytes of the stages of its claimed tasks into a shared-memory
// ring as soon as a slot is free (weights are constant, so they stream across layer
// and phase boundaries); a stage's activation slice is copied in once the tasks that
// write it have published it.  Readiness is counted per slice of each GEMV input
// ("slab instance"): the task that completes a limb group of an output builds that
// group's limbs and adds one to its slice's counter.  Attention for a kv head starts
// once the QKV row groups of its heads have finished.  Every wait is bounded and
// records a fault code instead of hanging.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode.cuh"

namespace ib {

enum { TK_EMBED = 0, TK_GEMV = 1, TK_ATTN = 2 };

constexpr int kStepMaxStages = 4;
constexpr int kStepAttMaxSplits = 128;  // attention split slots per kv head
constexpr int kStepAttMinSplit = 32;    // positions per split at least

// One phase: a run of consecutive tasks of one kind.
struct StepPhase {
    int kind;   // TK_*
    int first;  // index of the phase's first task
    int n;      // tasks (attention: kStepAttMaxSplits slots per kv head, split-major)
    // ---- GEMV: row groups of g (16 rows; SwiGLU: 8 gate + 8 up rows) ----
    FusedGemv g;
    int pro, epi;
    int nb;        // blocks per row
    int spg;       // ring stages per task (the last may hold fewer blocks)
    int in_inst;   // slab instance of the input (readiness counters)
    // output groups: the task completing a limb group of out_src builds its limbs
    int out_inst;          // slab instance written (-1: none)
    const float* out_src;  // the output vector (x or the SwiGLU product)
    const float* out_norm; // RMSNorm weights of the next GEMV's input (null: none)
    float* out_ssq;        // sums of squares per group for that RMSNorm (null: none)
    uint8_t* out_slab;
    int out_per_group;     // tasks that complete one limb group
    int layer;             // QKV / attention: the layer (counter rows)
    // ---- attention ----
    const float* q;
    const float* kc;
    const float* vc;
    // ---- embedding ----
    float* x;
    const float* norm;
    float* ssq;
};

struct StepParams {
    const StepPhase* phases;
    int n_phases, n_tasks;
    int* ctr;  // counters, zero at the start of every step
    int ready_off, grp_off, att_ready_off, att_done_off;
    int max_slices, max_groups, max_kv;
    int32_t* dev_i32;  // [0] token, [1] position, [2] next token
    int32_t* tokens;   // ids by position (may be null)
    unsigned long long* best;
    int max_seq;
    // embedding table
    const uint8_t* emb;
    int emb_type, vocab, dim;
    // attention shapes
    int H, Hkv, HD;
    float scale;
    float* att_acc;   // [H][kStepAttMaxSplits][HD]
    float2* att_ml;   // [H][kStepAttMaxSplits]
    int att_tile;     // positions per K/V tile in shared memory (multiple of 8)
    int att_target;   // QKV row groups per kv head
    // ring
    int S, stage_bytes, wbytes, slot_a, slot_b;
    int kq;           // slab geometry: 1 = K-quants (SE 2048, GS 256), 0 = 32-element blocks
};

// Bytes of counters a step needs.
size_t step_counter_bytes(int n_inst, int max_slices, int max_groups, int n_layers, int max_kv);
// Launch geometry for the format pair of type_a; rings of shapes with unaligned rows
// (pad_a / pad_b) get 16 more bytes per row.  Fills S, stage_bytes, wbytes, slot_a,
// slot_b, att_tile and the grid size; IB_ERR_UNSUPPORTED when the shapes do not fit.
int step_geometry(int type_a, bool pad_a, bool pad_b, int G, int HD, StepParams& p, int* grid);
// Launches the step kernel (the counters must be zero: the caller clears them first
// on the same stream).
int step_launch(const StepParams& p, int type_a, int grid, cudaStream_t st);
// Reads and clears the step kernel's fault word.
int step_fault_take(int* code);

}  // namespace ib
