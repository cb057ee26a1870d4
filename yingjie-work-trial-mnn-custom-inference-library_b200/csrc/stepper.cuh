// Persistent decode-step kernel: one cooperative launch runs a whole token step.
//
// One block per SM. The last warp of each block is a producer that walks the step's phase
// list and streams this block's share of every weight matrix, in order, through one
// shared-memory ring (1-D bulk copies, full/empty mbarriers). It never waits for
// activations, so HBM streaming continues across phase boundaries and across the grid
// barriers the consumers wait on. The other warps run the phases: fused W4A16 GEMVs (on the
// integer tensor cores over 16-row tiles, kMetaMma, or the dp4a row loop of gemv_w4a16_kernel),
// Gated-DeltaNet and attention work items, the embedding load of a prefill step. Consecutive phases are separated by a grid barrier
// (global arrival counter, bounded spin).
#pragma once

#include "gemv.cuh"
#include "ops.cuh"

namespace xqb {

enum PhaseKind : int { kPhaseGemv = 0, kPhaseDelta = 1, kPhaseAttn = 2, kPhaseEmbed = 3 };

struct alignas(16) PhaseDesc {  // copied into shared memory with one bulk copy
    int kind;
    int pro, epi;
    // kPhaseGemv: tensor maps (global memory, 128 bytes each) of x, of the second prologue
    // vector (norm weights or gate) and of the gated norm's head_dim weights, each viewed as
    // [n / 32][32] fp32 rows with 128-byte swizzle.
    const void* tmap[3];
    GemvParams g;   // kPhaseGemv (rows_per_chunk and unit filled in)
    DeltaParams d;  // kPhaseDelta
    AttnParams a;   // kPhaseAttn
};

constexpr int kStepConsumers = 384;                    // 12 warps
constexpr int kStepThreads = kStepConsumers + 32;      // + producer warp
constexpr int kStepMaxSlots = 16;
constexpr int kStepSlotBytes = 26112;                  // dp4a rows: 12 of K=4096 or 4 of K=12288
constexpr int kMmaStepSlotBytes = 34816;               // tensor-core tiles: 32 pairs of groups x 16 rows (default)
constexpr int kStepAttnDynBytes = 24 * 1024;           // q [group][hd] + scores [group][cmax]
constexpr int kStepHeaderBytes = 8704;
constexpr int kStepTraceSlots = 13;
// Shared staging of a GEMV phase's inputs: x and its second vector (norm weights or gate, plus
// the gated norm's head_dim weights) in the activation area; this block's residual rows or conv
// weights + state in the epilogue area.
constexpr int kStepActBytes = 48 * 1024;
constexpr int kStepEpiFloats = 1024;
inline size_t step_act_bytes(int pro, int cols, int head_dim) {
    size_t b = 4u * static_cast<size_t>(cols);
    if (pro == kProRms) b += 4u * static_cast<size_t>(cols);
    if (pro == kProGatedRms) b += 4u * (static_cast<size_t>(cols) + static_cast<size_t>(head_dim));
    if (pro == kProHeadScale) b += 4u * 1024u;  // per-slice sums of squares (<= 1024)
    return b;
}                 // barriers, sums, scratch (see stepper.cu)

struct StepParams {
    const PhaseDesc* phases;
    int nphases;
    int nslots;          // ring slots of slot_bytes
    int slot_bytes;      // kStepSlotBytes (row layout) or kMmaStepSlotBytes (tensor-core tiles)
    int inflight;        // at most this many issued copies not yet landed (1..nslots)
    int l2_prefetch;     // producers warm L2 with each GEMV phase's constant inputs
    int l2_ahead;        // weight chunks prefetched into L2 ahead of the ring, within a phase
    unsigned* grid_bar;  // arrival counter, 0 at launch, reset to 0 by the last arrival
    unsigned* err;
    // Limit of every bounded wait in the launch (ns; 0 = kWaitLimitNs, 2 s).
    unsigned long long wait_ns;
    // Failure-detection test hook, 0 in normal launches: the grid barrier that opens phase 1
    // waits for this many arrivals more than there are blocks. Nothing provides them, so that
    // wait runs out after wait_ns, the kernel records kErrBarrierTimeout and every later wait
    // returns at once; the launch ends and the host reports the error.
    unsigned barrier_extra;
    // kPhaseEmbed
    const int* prompt;
    const uint16_t* emb;
    float* hidden;
    int hidden_size;
    int vocab;
    int* pos;
    int* next_pos;
    // Optional per-phase device timestamps (ns), [nphases][kStepTraceSlots] when non-null:
    // block 0 passed the barrier (0), finished its work (1), the last block arrived (2), and
    // for GEMV phases block 0's constants staged (7), prologue done (3), activation limbs
    // ready (4), first weight chunk landed (5), chunk loop done (6), activations staged (10),
    // block 0 saw the grid barrier complete (11; before the phase start), its activation copies
    // issued (12); and
    // two durations (ns): thread 0's time waiting for weight chunks to land (8), the producer's
    // time waiting for free ring slots while issuing this phase's chunks (9).
    unsigned long long* trace;
    // Optional [nphases][gridDim.x] time (ns) at which each block finished its part of a phase.
    unsigned long long* block_done;
};

// Launch one step (cooperative). kv_fp16 selects the KV-cache element type; meta_kind the
// weight metadata layout (all matrices of a model share one).
cudaError_t launch_decode_step(const StepParams& p, int meta_kind, bool kv_fp16, int num_sms, cudaStream_t s);
size_t step_smem_bytes(int nslots, int slot_bytes);
// Largest ring that fits next to the kernel's other shared memory on this device.
int step_max_slots(int slot_bytes);
cudaError_t step_init_device();
// cudaFuncAttributes::binaryVersion of the loaded step kernel (100 for sm_100a), 0 on error.
int step_kernel_binary_version();
// Tensor map (written to `out`, kStepTmapBytes) of an fp32 vector of n floats (n a multiple of
// 32, n / 32 a multiple of min(32, n / 32)), as the step kernel stages it.
constexpr int kStepTmapBytes = 128;
bool encode_vector_tmap(void* out, const float* ptr, int n);
// Tensor map of a DeltaNet recurrent state [rows][cols] fp32 read in boxes of `box_rows` rows
// x kDeltaCols columns (one work item's state slice).
bool encode_state_tmap(void* out, const float* ptr, int rows, int cols, int box_rows);

}  // namespace xqb
