// kernels.h -- launchers shared between the kernel files and the engine.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

#include "moe_gemm.cuh"

namespace dee {

// Launch with programmatic stream serialisation (see sm100::pdl_wait).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Opt kernel Kern in to `bytes` of dynamic shared memory on the current
// device, once per device (the attribute belongs to the device's context;
// devices 64 and up set it at every call).
template <auto Kern>
cudaError_t ensure_smem_attr(int bytes) {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t{1} << dev) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
    return e;
}

struct GemmMaps {
    CUtensorMap w0, w1, s0, s1, b;
    CUtensorMap bt[4];  // tcgen05 kernel: token boxes of 16/32/64/128 rows x 128 K
    // decode kernel: s0 / s1 are swizzled scale-row maps (else its scale rows
    // come in by bulk copies)
    int scale_swz = 0;
};

// The MXFP8-activation grouped GEMM (moe_mxfp8.cu): weights E2M1 unpacked by
// the TMA (a), E4M3 token rows in boxes of 16/32/64/128 rows (bt).
struct MxMaps {
    CUtensorMap a;
    CUtensorMap bt[4];
};
cudaError_t launch_moe_mxfp8(bool gate_up, const MxMaps& maps, const GemmArgs& args, const uint8_t* b_scales,
                             int b_rows_cap, int grid, cudaStream_t stream);

// Largest N (rows per expert tile) of the tcgen05 GEMM.
int gemm_n_max();

cudaError_t launch_moe_gemm(bool gate_up, const GemmMaps& maps, const GemmArgs& args, int grid,
                            cudaStream_t stream);

// Decode-sized groups (tiles of at most kDecodeTileRows token rows): register
// dequant + mma.sync kernel of moe_decode.cu.  Its tensor maps come from the
// two encode_decode_* helpers below (maps.s0 / s1 are the swizzled scale-row
// maps when scale_swz is set; otherwise scale rows come by bulk copies).
constexpr int kDecodeTileRows = 8;
constexpr int kDecodeMaxTokens = 64;
constexpr int kDecodeMaxSelections = 384;  // selections (rows) the decode kernel takes
cudaError_t launch_moe_decode(bool gate_up, const GemmMaps& maps, const GemmArgs& args, int grid,
                              cudaStream_t stream);
// The whole decode layer in one launch, for batches decode_front_fits
// accepts (T*K <= kFrontMaxSel, E <= 256; live semantics, one GPU): every
// CTA routes the batch and groups it itself (the router of
// launch_route_topk and the grouping of launch_permute, computed
// redundantly per CTA), loads its token rows straight from x with bulk
// copies, and runs the gate/up and down items and the combine of
// launch_moe_decode_layer.  No kernel runs before it to zero counters: the
// tile counters advance by a fixed amount per launch (a launch waits for
// epoch x target), the (token, block) counters are reset by the add that
// completes them.
constexpr int kFrontMaxSel = 96;
constexpr int kFrontMaxTiles = kFrontMaxSel;  // a tile holds at least one selection
constexpr int kFrontScratchInts = kFrontMaxSel;  // per CTA: the combine weights by position (FP32)
struct DecFront {
    const float* logits;      // [T, E] FP32 router logits, or null: ids_out / weights_out are inputs
    const __half* x;          // [T, H] token rows
    int tokens;
    int32_t* ids_out;         // [T, K]  (written by CTA 0 when routing)
    float* weights_out;       // [T, K]  (written by CTA 0 when routing; may be null without logits and combine)
    int32_t* journal;         // [T*K] or null (written by CTA 0)
    int32_t* scratch;         // [grid * kFrontScratchInts]
    unsigned long long* ctr;  // [kFrontMaxTiles + kFrontMaxSel * H/128], zeroed once at allocation
    uint32_t epoch;           // > 0 and new for every launch on these counters
};
inline bool decode_front_fits(int tokens, int topk, int experts) {
    return tokens > 0 && topk > 0 && topk <= experts && experts <= 256 &&
           static_cast<long long>(tokens) * topk <= kFrontMaxSel;
}
// The engine takes the one-launch layer for batches of at most this many
// selections.  Measured on a B200 (DeepSeek-V4 layer, 256 experts): with
// routing inside it saves ~7 us of ~49 at one token; at eight tokens (48
// selections) it is ~1.5 us slower than the router+grouping kernel, gather
// and two-phase layer (every CTA routes all eight tokens), and on the
// caller's ids ~3 us slower than grouping, gather and layer (the in-kernel
// grouping holds back the first weight copies, which the two-phase layer
// issues while the gather runs).
constexpr int kFrontEngineMaxSel = 24;
cudaError_t launch_moe_decode_front(const GemmMaps& gu, const GemmMaps& dn, const GemmArgs& args,
                                    const DecFront& front, int grid, cudaStream_t stream);
// Both projections in one persistent launch: the gate/up items of every tile,
// then the down items (each waits, bounded, for its tile's gate/up items),
// and, with args.comb_out, the fused rank-order combine.  args.tile_done and
// (with comb_out) args.comb_cnt must have been zeroed by the permutation.
cudaError_t launch_moe_decode_layer(const GemmMaps& gu, const GemmMaps& dn, const GemmArgs& args, int grid,
                                    cudaStream_t stream);

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Weight maps of the decode kernel over a bank of DEE4 records: W1, W3 (gate
// and up) into gu->w0 / gu->w1 and W2 into dn->w0 / dn->w1.
bool encode_decode_weight_maps(EncodeTiledFn fn, const void* records, size_t record_bytes,
                               int n_slots, int hidden, int inter, GemmMaps* gu, GemmMaps* dn);
// Token-row map over a [rows, cols] FP16 buffer: boxes of 8 rows x
// box_chunks 64-wide column chunks (8 for the decode kernel's 512-wide
// stages, 4 for the shared expert's 256-wide ones).
bool encode_decode_token_map(EncodeTiledFn fn, const void* rows_base, int rows, int cols,
                             CUtensorMap* map, int box_chunks = 8);
// The general form: [rows, cols] FP16 viewed as {64, rows, cols/64}, boxes of
// box_rows rows x box_chunks chunks landing as [chunk][row][128 B] (128-byte
// swizzle).
bool encode_token_map(EncodeTiledFn fn, const void* rows_base, int rows, int cols, int box_rows, int box_chunks,
                      CUtensorMap* map);
// The MXFP8 GEMM's maps: E2M1 weights over a bank of records, E4M3 token rows.
bool encode_mx_weight_maps(EncodeTiledFn fn, const void* records, size_t record_bytes, int n_slots, int hidden,
                           int inter, MxMaps* gu, MxMaps* dn);
bool encode_mx_token_maps(EncodeTiledFn fn, const void* rows_base, int rows, int cols, CUtensorMap* maps);
// The tcgen05 GEMM's four token maps (boxes of 16/32/64/128 rows x 128 K).
bool encode_gemm_token_maps(EncodeTiledFn fn, const void* rows_base, int rows, int cols, CUtensorMap* maps);

// The shared expert (moe_shared.cu): dense F8_E4M3 projections W1, W3
// [inter, H] and W2 [H, inter] with E8M0 scales per 128 x 128 tile.
bool encode_shared_weight_maps(EncodeTiledFn fn, const void* w1, const void* w3, const void* w2, int hidden,
                               int inter, CUtensorMap* m1, CUtensorMap* m3, CUtensorMap* m2);
// Gate/up + SwiGLU over x (map_x: [T, H], 4-chunk boxes) into act [T, inter],
// then down (map_act over act) into out [T, H] FP32; official FP32 chain, no
// routing weight.
cudaError_t launch_shared_expert(const CUtensorMap& m1, const CUtensorMap& m3, const CUtensorMap& m2,
                                 const CUtensorMap& map_x, const CUtensorMap& map_act, const uint8_t* s1,
                                 const uint8_t* s3, const uint8_t* s2, int tokens, int hidden, int inter,
                                 float swiglu_limit, __half* act, float* out, uint32_t* status, int grid,
                                 cudaStream_t stream);
// out[t] = sum_r raw[t*K + r] (rank order, FP32) + shared[t] (if non-null):
// the official combination of weighted routed outputs and the shared expert.
cudaError_t launch_combine_sum(const float* raw, const float* shared, int tokens, int topk, int hidden,
                               float* out, cudaStream_t stream);

// Expert-parallel packing (ep.cu): selections [T, K] of global ids over
// ranks x experts_per_rank experts -> per destination rank `capacity` slots of
// FP16 rows and local expert ids (-1 unused), and slot_of_pos [T*K].
constexpr int kEpMaxRanks = 32;
cudaError_t launch_ep_pack(const int32_t* ids, const __half* x, int tokens, int topk, int hidden,
                           int ranks, int epr, int capacity, __half* send_rows, int32_t* send_expert,
                           int32_t* slot_of_pos, int32_t* journal, uint32_t* status,
                           cudaStream_t stream);
// Rank-order FP32 combine of rows returned by the expert owners; with `flags`
// each CTA first waits (bounded by limit_ns, status bit kStatusTimeoutFlag)
// for every owner's return flag to reach `epoch`.
cudaError_t launch_ep_combine(const float* back, const int32_t* slot_of_pos, const float* weights,
                              int tokens, int topk, int hidden, float* out, cudaStream_t stream,
                              const uint32_t* flags = nullptr, int ranks = 0, uint32_t epoch = 0,
                              uint32_t* status = nullptr, uint64_t limit_ns = 0);

// Peer (NVLink) expert parallelism: every rank's exchange buffers, indexed by
// rank (this rank's own entries are local pointers).  Block s of rank d's
// receive buffers holds the rows rank s sent to d; block d of rank s's return
// buffer holds the output rows d computed for s.
struct EpPeers {
    __half* recv_rows[kEpMaxRanks];      // [ranks * capacity, H] FP16
    int32_t* recv_expert[kEpMaxRanks];   // [ranks * capacity], -1 unused
    uint32_t* recv_flag[kEpMaxRanks];    // [ranks] dispatch epoch per source
    float* back_rows[kEpMaxRanks];       // [ranks * capacity, H] FP32
    uint32_t* back_flag[kEpMaxRanks];    // [ranks] return epoch per expert owner
};
// Index + row stores into the owners' receive buffers, then the dispatch flags
// (raised by the rows kernel's last CTA; `done` is its completion counter,
// zero between calls).
cudaError_t launch_ep_peer_dispatch(const int32_t* ids, const __half* x, int tokens, int topk, int hidden,
                                    int ranks, int rank, int epr, int capacity, const EpPeers& peers,
                                    int32_t* slot_of_pos, int32_t* journal, uint32_t* status,
                                    uint32_t* done, uint32_t epoch, cudaStream_t stream);
// Publish `epoch` in slot `rank` of every rank's dispatch (back = false) or
// return (back = true) flags, after the stream's earlier kernels.
cudaError_t launch_ep_signal(const EpPeers& peers, bool back, int ranks, int rank, uint32_t epoch,
                             cudaStream_t stream);
// A wait on an mbarrier nothing arrives on, bounded by limit_ns (sets `code`).
cudaError_t launch_wait_selftest(uint64_t limit_ns, uint32_t* status, uint32_t code, cudaStream_t stream);

// The synthetic stack's dense glue (stack.cu), every per-token result in a
// fixed order independent of the batch.
cudaError_t launch_stack_embed(const __half* table, const int32_t* ids, int tokens, int hidden, int vocab,
                               float* x, uint32_t* status, cudaStream_t stream);
cudaError_t launch_stack_rmsnorm(const float* x, const float* w, float eps, int tokens, int hidden, __half* y,
                                 cudaStream_t stream);
cudaError_t launch_stack_rowdot_f32(const __half* x, const float* w, int tokens, int hidden, int rows,
                                    float* out, cudaStream_t stream);
cudaError_t launch_stack_rowdot_f16(const __half* x, const __half* w, int tokens, int hidden, int rows,
                                    float* out, cudaStream_t stream);
cudaError_t launch_stack_residual_add(float* x, const float* y, size_t n, cudaStream_t stream);
cudaError_t launch_stack_argmax(const float* logits, int tokens, int vocab, int32_t* ids, cudaStream_t stream);
// Block-wise E4M3 quantisation with UE8M0 scales (act_quant.cu): rows of x
// [.., cols] FP16 (row r = perm[r] / topk when perm is given; *rows_dev, if
// given, caps the rows) into q [rows, cols] and scales [rows, cols / block],
// or with per32 one scale byte per 32 columns (the MMA's granularity).
cudaError_t launch_act_quant(const __half* x, int rows, int cols, int block, const int32_t* perm, int topk,
                             const int32_t* rows_dev, uint8_t* q, uint8_t* scales, cudaStream_t stream,
                             bool per32);

cudaError_t launch_records_scramble(const uint8_t* src, uint8_t* dst, int records, size_t record_bytes,
                                    size_t packed_bytes, uint64_t seed, int first_record, cudaStream_t stream);

// Router: logits [T, E] FP32 -> ids [T, K] int32 (rank order), weights [T, K].
cudaError_t launch_route_topk(const float* logits, int tokens, int experts, int topk,
                              int32_t* ids, float* weights, uint32_t* status, cudaStream_t stream);

// DeepSeek-V4 router: sqrt(softplus) scores, bias for selection only (may be
// null), hash selection from tid2eid[input_ids] when tid2eid is non-null.
cudaError_t launch_route_dsv4(const float* logits, const float* bias, const int64_t* tid2eid,
                              const int64_t* input_ids, int tokens, int experts, int topk,
                              float route_scale, int32_t* ids, float* weights, uint32_t* status,
                              cudaStream_t stream);

// Group-by-expert permutation (one CTA): counts/offsets per expert, grouped
// row -> position table, position -> row table, and the GEMM tile list.
struct PermuteOut {
    int32_t* counts;    // [E]
    int32_t* offsets;   // [E + 1]
    int32_t* perm;      // [T*K] grouped row -> position
    int32_t* row_of;    // [T*K] position -> grouped row
    TileDesc* tiles;    // [max_tiles]
    int32_t* n_tiles;   // [1]
    int32_t* journal;   // [T*K] copy of the consumed ids, or null
    // Scratch of the multi-CTA permutation (batches of more than two chunks
    // of 1024 selections); without it one CTA does the whole batch.
    int32_t* chunk_counts = nullptr;  // [max_chunks * E]
    int32_t* lrank = nullptr;         // [T*K]
    long long max_chunks = 0;
    // Expert-parallel receive buffers: before reading ids, wait (bounded)
    // for wait_ranks senders' flags to reach wait_epoch.
    const uint32_t* wait_flags = nullptr;
    int wait_ranks = 0;
    uint32_t wait_epoch = 0;
    uint64_t wait_limit_ns = 0;
    // Counters of the one-launch decode layer, zeroed before grouping
    // (one-CTA permutation only).
    uint32_t* clear = nullptr;
    int clear_n = 0;
    // Per tile: its expert's first tile and tile count (the prefill GEMMs'
    // expert-local m-major item order).
    int2* tile_grp = nullptr;
};
// skip_negative: ids of -1 mark unused rows (expert-parallel receive
// buffers) and are left out without raising kStatusBadExpert.
// Kernels launch_permute issues for this batch: 1 (one CTA) or 2 (the
// multi-CTA passes).
int permute_launch_count(int tokens, int topk, const PermuteOut& out);
cudaError_t launch_permute(const int32_t* ids, int tokens, int topk, int experts, int n_tile_max,
                           int max_tiles, const PermuteOut& out, uint32_t* status,
                           cudaStream_t stream, bool skip_negative = false);

// Softmax top-k routing and the permutation in one single-CTA launch, for
// batches route_permute_fits accepts (at most 16 tokens, T*K <=
// kDecodeMaxSelections, E <= 256): the same ids, weights and grouping as
// launch_route_topk + launch_permute.  More tokens route faster spread over
// SMs by the router kernel (one CTA routing 64 tokens cost ~13 us more on a
// B200, measured at b = 64).
inline bool route_permute_fits(int tokens, int topk, int experts) {
    return tokens > 0 && tokens <= 16 && topk > 0 && topk <= experts && experts <= 256 &&
           static_cast<long long>(tokens) * topk <= kDecodeMaxSelections;
}
cudaError_t launch_route_permute(const float* logits, int tokens, int experts, int topk, int32_t* ids,
                                 float* weights, int n_tile_max, int max_tiles, const PermuteOut& out,
                                 uint32_t* status, cudaStream_t stream);

// X_perm[row] = X[perm[row] / topk] (FP16 rows of H elements).
cudaError_t launch_gather_rows(const __half* x, const int32_t* perm, const int32_t* total_rows_dev,
                               int max_rows, int topk, int hidden, __half* x_perm,
                               cudaStream_t stream);

// Live combine: out[t] = sum_r w[t, r] * raw[t, r] in rank order, FP32.
cudaError_t launch_combine_f32(const float* raw, const float* weights, int tokens, int topk,
                               int hidden, float* out, cudaStream_t stream);
// Exact eager-FP16 combine in stable ascending-expert order.
cudaError_t launch_combine_f16(const float* raw, const float* weights, const int64_t* ids64,
                               int tokens, int topk, int hidden, __half* out,
                               cudaStream_t stream);
// Same as combine_f16 with int32 expert ids.
cudaError_t launch_combine_f16_i32(const float* raw, const float* weights, const int32_t* ids,
                                   int tokens, int topk, int hidden, __half* out,
                                   cudaStream_t stream);

// Standalone FP4 -> FP16 decode of one [out, in] projection.
cudaError_t launch_fp4_decode(const uint8_t* packed, const uint8_t* scale, __half* dst,
                              size_t out, size_t in, cudaStream_t stream);

// N(0, std)-shaped FP32 weights [out, in] -> packed FP4 + UE8M0 scales.
cudaError_t launch_fp4_quantize(const float* w, size_t out, size_t in, uint8_t* packed,
                                uint8_t* scale, cudaStream_t stream);

// Convert int64 ids to int32 (validating range into status).
cudaError_t launch_ids_i64_to_i32(const int64_t* src, int n, int experts, int32_t* dst,
                                  uint32_t* status, cudaStream_t stream);

}  // namespace dee
