// Persistent decode-step kernel: one cooperative launch runs a whole token step.
//
// One block per SM. The last warp of each block is a producer that walks the step's phase
// list and streams this block's share of every weight matrix, in order, through one
// shared-memory ring (1-D bulk copies, full/empty mbarriers). It never waits for
// activations, so HBM streaming continues across phase boundaries and across the grid
// barriers the consumers wait on. The other warps run the phases: fused W4A16 GEMVs (the
// same device math as gemv_w4a16_kernel), Gated-DeltaNet and attention work items, the
// embedding load of a prefill step. Consecutive phases are separated by a grid barrier
// (global arrival counter, bounded spin).
#pragma once

#include "gemv.cuh"
#include "ops.cuh"

namespace xqb {

enum PhaseKind : int { kPhaseGemv = 0, kPhaseDelta = 1, kPhaseAttn = 2, kPhaseEmbed = 3 };

struct PhaseDesc {
    int kind;
    int pro, epi;
    GemvParams g;   // kPhaseGemv (rows_per_chunk and unit filled in)
    DeltaParams d;  // kPhaseDelta
    AttnParams a;   // kPhaseAttn
};

constexpr int kStepConsumers = 384;                    // 12 warps
constexpr int kStepThreads = kStepConsumers + 32;      // + producer warp
constexpr int kStepMaxSlots = 16;
constexpr int kStepSlotBytes = 26112;                  // 12 rows of K=4096 or 4 rows of K=12288
constexpr int kStepAttnDynBytes = 24 * 1024;           // q [group][hd] + scores [group][cmax]
constexpr int kStepHeaderBytes = 8704;                 // barriers, sums, scratch (see stepper.cu)

struct StepParams {
    const PhaseDesc* phases;
    int nphases;
    int nslots;          // ring slots of kStepSlotBytes
    unsigned* grid_bar;  // arrival counter, 0 at launch, reset to 0 by the last arrival
    unsigned* err;
    // kPhaseEmbed
    const int* prompt;
    const uint16_t* emb;
    float* hidden;
    int hidden_size;
    int vocab;
    int* pos;
    int* next_pos;
    // Optional per-phase device timestamps of block 0 ([nphases][3] ns: barrier passed, work
    // done, and — for the last block to arrive — the arrival time) when non-null.
    unsigned long long* trace;
};

// Launch one step (cooperative). kv_fp16 selects the KV-cache element type; meta_kind the
// weight metadata layout (all matrices of a model share one).
cudaError_t launch_decode_step(const StepParams& p, int meta_kind, bool kv_fp16, int num_sms, cudaStream_t s);
size_t step_smem_bytes(int nslots);
// Largest ring that fits next to the kernel's other shared memory on this device.
int step_max_slots();
cudaError_t step_init_device();

}  // namespace xqb
