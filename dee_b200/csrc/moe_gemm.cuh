// moe_gemm.cuh -- grouped (ragged, per-expert) W4A16 GEMM on tcgen05.
//
// One kernel template serves both projections of the routed-expert FFN:
//
//   kGateUp: act[rows, I]  = SwiGLU( X_perm[rows, H] . W1^T , X_perm . W3^T )
//            with FP16 rounding of gate, up, SiLU and the product, exactly
//            the chain of swiglu_expert_batch_fp16_cuda
//            (reference dee.cpp/src/swiglu_cuda.cu:387-431, :46-59).
//   kDown:   raw[pos, H]   = act[rows, I] . W2^T in FP32, each grouped row
//            scattered to its (token, rank) position (engine.cpp:1080-1113).
//
// Roles (one CTA per SM, persistent over a static round-robin work list):
//   warp 0      TMA producer of packed FP4 weight tiles + UE8M0 scale tiles
//   warp 1      TMA producer of the token operand (X_perm or act) tiles
//   warp 2      TMEM allocator and single-thread tcgen05.mma issuer
//   warps 3-10  dequantisers, two warpgroups taking alternate 64-wide K steps:
//               each thread owns one weight row (one TMEM lane), turns 64
//               packed nibbles into 64 FP16 weights per step and writes them
//               to a tensor-memory A buffer with tcgen05.st
//   warps 11-14 epilogue: tcgen05.ld of the FP32 accumulator, SwiGLU or
//               scatter, global stores
//
// The MMA is tcgen05.mma.kind::f16 with A (weights, M = 128 rows) read from
// tensor memory and B (tokens, N = 16..N_MAX rows) from 128B-swizzled shared
// memory; the accumulator lives in tensor memory and is double buffered so
// the epilogue of one work item overlaps the main loop of the next.
//
// Work item = (tile, m): a tile is <= N_MAX consecutive grouped rows of one
// expert (built on device by the permutation kernel), m selects 64 gate+up
// feature pairs (kGateUp) or 128 output features (kDown).  Every output
// element accumulates over K in the same fixed order regardless of how many
// rows share its tile, so per-row results do not depend on group sizes.
#pragma once

#include "sm100.cuh"

namespace dee {

enum class GemmMode : int { kGateUp = 0, kDown = 1 };

struct TileDesc {
    int expert;     // routed expert id
    int row_start;  // first grouped row
    int n_rows;     // valid rows (<= N_MAX)
    int n_pad;      // MMA N: n_rows rounded up to 16
};

struct GemmArgs {
    int hidden;              // H
    int inter;               // I
    int k_total;             // reduction length: H (kGateUp) or I (kDown)
    int m_tiles;             // I/64 (kGateUp) or H/128 (kDown)
    int topk;                // K (positions are token * topk + rank)
    float swiglu_limit;      // > 0 clamps gate/up as the reference does
    const TileDesc* tiles;   // device tile list
    const int* n_tiles;      // device: number of tiles
    const int* slot_of;      // device: expert -> record slot in the bank
    int num_slots;           // slots in the bank (bounds check)
    const uint8_t* records;  // bank base: slot s starts at records + s * record_bytes
    size_t record_bytes;
    int num_experts;
    const int* perm;         // device: grouped row -> position (kDown)
    __half* act;             // kGateUp output [rows, I]
    float* raw;              // kDown output [positions, H]
    uint32_t* status;        // device status word (sm100::StatusBits)
    // Expert-parallel return over NVLink (decode kernel only): when set,
    // output row i -- received from rank i / ep_capacity into slot
    // i % ep_capacity -- is stored at raw_peers[rank] + (ep_rank *
    // ep_capacity + slot) * H, the owner's return buffer, instead of raw.
    float* const* raw_peers;  // device array [ranks] of peer pointers, or null
    int ep_capacity;
    int ep_rank;
    // Official semantics (deepseek_v4_moe_reference.py:87-110): the gate/up
    // epilogue keeps the FP32 chain and multiplies by route_w[position]
    // (route_w null: weight 1, the shared expert); weights dequantise in FP32.
    int official;
    const float* route_w;
};

constexpr int kGemmThreads = 480;     // 15 warps
constexpr int kPkStageBytes = 32768;  // 128 rows x 256 packed bytes (K = 512)
constexpr int kScStageBytes = 2048;   // 128 rows x 16 scale bytes
constexpr int kKStage = 512;          // K elements per packed stage
constexpr int kKBlock = 64;           // K elements per A/B step (one 128B row of FP16)

// N_MAX: largest MMA N (token rows per tile); PK_STAGES: packed-weight
// stages in shared memory; B_STAGES x B_KB: token-operand stages, each
// covering B_KB 64-wide K steps; A_STAGES: tensor-memory A buffers;
// PREFETCH: packed stages prefetched into L2 ahead of the shared-memory ring.
template <int N_MAX, int PK_STAGES, int B_STAGES, int B_KB, int A_STAGES, int PREFETCH>
struct GemmConfig {
    static constexpr int kNMax = N_MAX;
    static constexpr int kPk = PK_STAGES;
    static constexpr int kB = B_STAGES;
    static constexpr int kBKb = B_KB;
    static constexpr int kA = A_STAGES;
    static constexpr int kPrefetch = PREFETCH;
    static constexpr int kBStageBytes = N_MAX * 128 * B_KB;
    static constexpr int kAccBase = A_STAGES * 32;
    static constexpr int kTmemCols = 512;
    static_assert(N_MAX % 16 == 0 && N_MAX <= 256, "N_MAX");
    static_assert(kAccBase + 2 * N_MAX <= kTmemCols, "tensor memory budget");
    static_assert(A_STAGES % 2 == 0, "each A stage must belong to one dequantiser warpgroup");
    static constexpr int kSmemBytes = 1024 /*align slack*/ + PK_STAGES * kPkStageBytes +
                                      B_STAGES * kBStageBytes + PK_STAGES * kScStageBytes +
                                      1024 /*barriers*/;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

}  // namespace dee
