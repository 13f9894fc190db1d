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
//   warp 1      TMA producer of the token operand (X_perm or act): one 3-D
//               box per 128-K step, 16/32/64/128 rows to fit the tile
//   warp 2      TMEM allocator and single-thread tcgen05.mma issuer
//   warps 3-18  dequantisers, four warpgroups taking 128-wide K steps in turn:
//               each thread owns one weight row (one TMEM lane), turns 128
//               packed nibbles into 128 FP16 weights per step and writes them
//               to a tensor-memory A buffer with tcgen05.st
//   warps 19-22 epilogue: tcgen05.ld of the FP32 accumulator, SwiGLU or
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
    // Decode kernel: the scale rows arrive by swizzled tensor copies (set by
    // the launcher from GemmMaps::scale_swz of the gate/up and down maps).
    int scale_swz;
    int dn_scale_swz;
    // Decode kernel, both projections in one launch (launch_moe_decode_layer):
    // tile_done[tile] counts the tile's finished gate/up items (zeroed by the
    // permutation); a down item waits for its tile's count before it loads
    // the SwiGLU rows.  With comb_out set, the kernel also runs the live
    // combine comb_out[t] = sum_r comb_w[t*K + r] * raw[t*K + r] (rank order,
    // FP32), per 128-feature block once the block's K rows are written;
    // comb_cnt [tokens * H/128] counts them (zeroed by the permutation).
    int phases;  // bit 0: gate/up items, bit 1: down items
    uint32_t* tile_done;
    const float* comb_w;
    float* comb_out;
    uint32_t* comb_cnt;
    // Prefill GEMMs: per tile {first tile, tile count} of its expert.  With
    // it the items of one expert run m-major -- all of its token tiles
    // against one weight slice, then the next slice -- so the tiles sharing
    // a weight slice run at the same time and its re-reads hit L2; without
    // it items are tile-major.
    const int2* tile_grp;
};

// Work item -> (tile, m).  The items of an expert's tiles [f, f + c) are
// [f * M, (f + c) * M) in either order, so the tile-major tile of an item
// names its expert group.
__device__ __forceinline__ void item_tile_m(const GemmArgs& a, int item, int& tile, int& m) {
    const int t0 = item / a.m_tiles;
    if (a.tile_grp) {
        const int2 g = a.tile_grp[t0];
        const int j = item - g.x * a.m_tiles;
        m = j / g.y;
        tile = g.x + (j - m * g.y);
    } else {
        tile = t0;
        m = item - t0 * a.m_tiles;
    }
}

constexpr int kDqGroups = 4;          // dequantiser warpgroups
constexpr int kEpilogueWarp = 3 + 4 * kDqGroups;
constexpr int kGemmThreads = 32 * (kEpilogueWarp + 4);  // producers, MMA, dequantisers, epilogue
constexpr int kPkStageBytes = 32768;  // 128 rows x 256 packed bytes (K = 512)
constexpr int kScStageBytes = 2048;   // 128 rows x 16 scale bytes
constexpr int kKStage = 512;          // K elements per packed stage
constexpr int kKBlock = 64;           // K elements per 128-byte row of FP16

// The pipeline between the dequantisers, the token producer and the MMA
// issuer moves in steps of kAK = 128 K: one full/empty handshake per eight
// K = 16 MMAs.  (A handshake costs the single issuing thread one mbarrier
// wait and one tcgen05.commit -- together ~150 cycles in which at most one
// queued MMA keeps the tensor pipe busy -- so per-64-K handshakes idled the
// pipe for over half the time at N <= 128.)
constexpr int kAK = 128;
constexpr int kAStages = 4;                  // tensor-memory A stages, 64 columns each
constexpr int kBStages = 4;                  // token-operand stages in shared memory
constexpr int kNMax = 128;                   // MMA N (token rows per tile)
constexpr int kBStageBytes = kNMax * 128 * (kAK / kKBlock);  // 32 KB
constexpr int kPkStages = 2;
constexpr int kAccBase = kAStages * (kAK / 2);               // first accumulator column
constexpr int kTmemCols = 512;
constexpr int kTokenBoxes = 4;               // token boxes of 16, 32, 64 and 128 rows
static_assert(kAccBase + 2 * kNMax <= kTmemCols, "tensor memory budget");
constexpr int kGemmSmemBytes = 1024 /*align slack*/ + kPkStages * kPkStageBytes + kBStages * kBStageBytes +
                               kPkStages * kScStageBytes + 1024 /*barriers*/;
static_assert(kGemmSmemBytes <= 232448, "shared memory budget");

}  // namespace dee
