/*
 * dee_b200.h -- C ABI of the B200-native routed-expert MoE layer.
 *
 * Drop-in boundary for the routed-expert FFN of so-nerdyy/dee.  Each entry
 * point names the reference interface it replaces (paths relative to the
 * reference project root).  Conventions follow the reference engine:
 *   - the caller owns every input/output buffer; the engine owns expert
 *     banks' descriptors, workspaces and its compute stream
 *     (dee.cpp/include/dee/engine.h:302-326);
 *   - failures return a negative status and record a message readable with
 *     dee_last_error() (Engine::last_error_message, engine.h:434-436);
 *   - one engine per CUDA device, driven from one host thread at a time;
 *   - an engine's workspaces (grouped token rows, SwiGLU rows, internal raw
 *     rows, the decode layer's counters) serve one call at a time: queue an
 *     engine's calls on one stream, or order calls made on different streams
 *     with events.  Separate engines share nothing;
 *   - device pointers are aligned to the widest access the kernels make:
 *     FP16 token rows (x, h_in, rows) and FP32 row buffers (raw, outputs,
 *     returned rows) 16 bytes, int64 ids 8, int32 ids, weights, logits and
 *     index tables 4, FP16 outputs 2.  Rows of a contiguous tensor meet
 *     this whenever its base does; a column slice need not.  An entry
 *     point given a pointer off its alignment returns DEE_ERR_INVALID,
 *     naming the pointer, before it launches anything.
 * No torch types cross this boundary: device pointers, host pointers,
 * sizes and CUDA stream handles (cudaStream_t passed as void*; NULL is the
 * legacy default stream, as in engine.cpp:2011-2013).
 */
#ifndef DEE_B200_H
#define DEE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DEE_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define DEE_API __attribute__((visibility("default")))
#else
#define DEE_API
#endif

/* Status codes. */
#define DEE_OK 0
#define DEE_ERR_INVALID (-1)     /* bad argument or shape                     */
#define DEE_ERR_CUDA (-2)        /* CUDA runtime/driver error                 */
#define DEE_ERR_RANGE (-3)       /* expert id outside [0, num_experts)        */
#define DEE_ERR_UNSUPPORTED (-4) /* configuration this build does not cover   */
#define DEE_ERR_DEVICE (-5)      /* a kernel reported a failure (status word) */
#define DEE_ERR_NO_BANK (-6)     /* no expert bank attached for the layer     */
#define DEE_ERR_SCRATCH_LIMIT (-7) /* request larger than the static scratch  */

typedef struct dee_engine dee_engine;

/* Mirrors the EngineConfig fields the routed-expert path reads
 * (dee.cpp/include/dee/engine.h:84-156). */
typedef struct dee_config {
    int hidden;          /* EngineConfig::hidden                             */
    int inter;           /* EngineConfig::inter                              */
    int num_experts;     /* EngineConfig::num_experts                        */
    int topk;            /* EngineConfig::topk                               */
    int num_layers;      /* EngineConfig::num_layers (bank slots)            */
    int device_id;       /* EngineConfig::device_id                          */
    float swiglu_limit;  /* EngineConfig::swiglu_limit, 0 disables the clamp */
    int max_tokens;      /* initial workspace capacity; grows on demand      */
} dee_config;

/* sizeof(dee_config) of this build; replaces engine_abi_size()
 * (engine.h:771-774) as the guard a binding checks before use. */
DEE_API size_t dee_abi_config_size(void);
DEE_API int dee_abi_version(void);

/* Engine::init (engine.h:237).  Returns DEE_OK and *out on success. */
DEE_API int dee_engine_create(const dee_config* cfg, dee_engine** out);
DEE_API void dee_engine_destroy(dee_engine* engine);

/* Engine::last_error_message (engine.h:434-436, pydee.cpp:768-772). */
DEE_API const char* dee_last_error(const dee_engine* engine);

/* Attach the packed expert records of one layer.  d_records points at
 * n_slots records of record_bytes each in the DEE4 layout
 * [w1][w3][w2][w1.scale][w3.scale][w2.scale]
 * (dee.cpp/include/dee/expert_store.h:28-46; VramCacheManager::data,
 * vram_cache.h:166-215 supplies the same per-expert device pointer).
 * h_slot_of_expert (host, num_experts entries, may be NULL for identity)
 * maps an expert id to its slot, -1 for "not resident". */
DEE_API int dee_expert_bank_attach(dee_engine* engine, int layer, const void* d_records, int n_slots,
                           size_t record_bytes, const int32_t* h_slot_of_expert);

/* Update the slot table of an attached bank (offload tier residency). */
DEE_API int dee_expert_bank_set_slots(dee_engine* engine, int layer, const int32_t* h_slot_of_expert,
                              void* stream);

/* The engine's group-by-expert step on its own (Engine's grouping,
 * engine.cpp:812-823): device ids [tokens, topk] int32 -> perm [T*K]
 * (grouped row -> position t*K + r; the rows of one expert in (rank, token)
 * order, experts by ascending id), row_of [T*K] (position -> grouped row, -1
 * for an id outside [0, E)) and offsets [E + 1].  Ids outside [0, E) are
 * reported by dee_engine_sync_status.  Asynchronous on `stream`. */
DEE_API int dee_group_by_expert_device(dee_engine* engine, const int32_t* d_ids, int tokens, int topk,
                                       int32_t* d_perm, int32_t* d_row_of, int32_t* d_offsets, void* stream);

/* Softmax top-k with renormalised weights on device logits [T, E] FP32 ->
 * ids [T, K] int32 in rank order and weights [T, K] FP32.
 * Engine::route_topk_batch (engine.cpp:2604-2771). */
DEE_API int dee_route_topk_device(dee_engine* engine, const float* d_logits, int tokens,
                          int32_t* d_ids, float* d_weights, void* stream);

/* DeepSeek-V4 router on device logits [T, E] (x . W_gate^T, FP32):
 * score = sqrt(softplus(logit)); d_bias (E floats, may be NULL) shifts only
 * the selection; top-k by biased score, ties to the lower id; weights =
 * selected unbiased scores / their sum * route_scale.  With d_tid2eid
 * ([vocab, K] int64) and d_input_ids ([T] int64) the selection is the hash
 * table row instead (hash layers).  Replaces the torch router of
 * dee.cpp/scripts/deepseek_v4_layer_candidate.py:99-120
 * (deepseek_v4_layer_common.py:349-403). */
DEE_API int dee_route_dsv4_device(dee_engine* engine, const float* d_logits, const float* d_bias,
                                  const int64_t* d_tid2eid, const int64_t* d_input_ids, int tokens,
                                  float route_scale, int32_t* d_ids, float* d_weights, void* stream);

/* Engine::moe_forward_batch_device (engine.h:312-314, pydee.cpp:430-467):
 * FP16 hidden [T, H] on device, host int32 ids [T, K] (validated on the
 * host, fail closed), FP32 raw expert outputs [T, K, H] on device;
 * 1 <= K <= EngineConfig::topk, as the reference accepts (engine.cpp:780-781).
 * Runs on the engine's stream and synchronises it before returning. */
DEE_API int dee_moe_forward_batch_device(dee_engine* engine, int layer, const void* d_h_in, int tokens,
                                 const int32_t* h_expert_ids, int topk, void* d_experts_out);

/* Engine::moe_forward_combined_device (engine.h:322-326,
 * pydee.cpp:468-509): device int64 ids, FP32 weights, FP16 output combined
 * in stable expert order with FP16 rounding (swiglu_cuda.cu:69-116),
 * optional FP32 raw trace [T, K, H].  Work is queued on external_stream
 * without a host synchronisation; invalid ids are reported through
 * dee_engine_sync_status. */
DEE_API int dee_moe_forward_combined_device(dee_engine* engine, int layer, const void* d_h_in, int tokens,
                                    const int64_t* d_expert_ids, int topk,
                                    const float* d_weights_f32, void* d_output_f16,
                                    void* d_raw_trace_out, void* external_stream);

/* The live DeepSeek layer in one call: ids from device (d_ids) or host
 * (h_ids, validated), raw expert rows and the rank-order FP32 combine
 * out[t] = sum_r w[t, r] * raw[t, r] of
 * dee.cpp/scripts/deepseek_v4_layer_candidate.py:616-629.  d_out_f32 and
 * d_raw may each be NULL (not both).  Queued on `stream`, no host sync. */
DEE_API int dee_moe_forward_device(dee_engine* engine, int layer, const void* d_x_f16, int tokens,
                           const int32_t* d_ids, const int32_t* h_ids, int topk,
                           const float* d_weights, float* d_out_f32, float* d_raw, void* stream);

/* Routing and the layer in one call: softmax top-k with renormalised weights
 * on device logits [T, E] FP32 (dee_route_topk_device, Engine::route_topk_batch,
 * engine.cpp:2604-2771) writes d_ids [T, K] int32 and d_weights [T, K] FP32,
 * then the layer of dee_moe_forward_device runs on them (K = the engine's
 * topk).  Small batches (at most 16 tokens, E <= 256) route inside the
 * grouping kernel -- at most 24 selections inside the one-launch layer --
 * one launch and one kernel dependency fewer; results are identical to the
 * two calls.  Queued on `stream`, no host sync. */
DEE_API int dee_moe_forward_routed_device(dee_engine* engine, int layer, const void* d_x_f16, int tokens,
                                          const float* d_logits, int32_t* d_ids, float* d_weights,
                                          float* d_out_f32, float* d_raw, void* stream);

/* The MXFP8-activation variant of dee_moe_forward_device (device ids only):
 * token rows and the SwiGLU output are quantised to E4M3 with UE8M0 scales
 * per act_block columns (128: the official act_quant, 32: MX), and both
 * grouped GEMMs run tcgen05 kind::mxf8f6f4 block-scaled MMAs straight on the
 * records' E2M1 weights and UE8M0 scales (no dequantisation).  Numerics
 * differ from the FP16 path by the activation quantisation; the tolerance
 * is stated with its tests.  DEE_ERR_UNSUPPORTED if the driver cannot encode
 * the unpacked-FP4 tensor maps. */
DEE_API int dee_moe_forward_mxfp8_device(dee_engine* engine, int layer, const void* d_x_f16, int tokens,
                                         const int32_t* d_ids, int topk, const float* d_weights, float* d_out_f32,
                                         float* d_raw, int act_block, void* stream);

/* Synchronise `stream`, read and clear the engine's device status word.
 * Returns DEE_ERR_DEVICE (and *status_out != 0) when a kernel flagged an
 * invalid expert id, a router failure or a pipeline timeout. */
DEE_API int dee_engine_sync_status(dee_engine* engine, void* stream, uint32_t* status_out);

/* The official DeepSeek-V4 MoE FFN semantics
 * (dee.cpp/scripts/deepseek_v4_moe_reference.py:87-203): each routed expert
 * runs the FP32 SwiGLU chain (clamp = the engine's swiglu_limit, 10 in the
 * official model) with the routing weight applied to the intermediate BEFORE
 * w2; the layer's shared expert (dense F8_E4M3 weights, F8_E8M0 scales per
 * 128 x 128 tile, no routing weight) is added; the sum is FP32.  The MMA
 * operands are FP16 (x, the weighted intermediate); weights dequantise
 * exactly.
 *
 * Attach the shared expert of `layer`: device F8_E4M3 W1, W3 [inter, H] and
 * W2 [H, inter] (row-major, 16-byte aligned) and their E8M0 scale bytes
 * [ceil(rows/128), ceil(cols/128)] (the official shared_experts tensors;
 * moe_reference.py:35-84).  inter and H must be multiples of 256. */
DEE_API int dee_shared_expert_attach(dee_engine* engine, int layer, const void* d_w1,
                                     const void* d_w1_scale, const void* d_w3, const void* d_w3_scale,
                                     const void* d_w2, const void* d_w2_scale, int inter_shared);

/* One layer with the official semantics: x FP16 [T, H], device ids [T, K]
 * (global), routing weights FP32 [T, K] -> d_out_f32 [T, H] = sum of weighted
 * routed outputs + shared expert.  d_shared_out (may be NULL) receives the
 * shared expert's FP32 [T, H] output. */
DEE_API int dee_moe_forward_official_device(dee_engine* engine, int layer, const void* d_x_f16,
                                            int tokens, const int32_t* d_ids, const float* d_weights,
                                            float* d_out_f32, float* d_shared_out, void* stream);

/* Expert parallelism over `ranks` GPUs (no counterpart in the reference's
 * engine, which runs one GPU; the split follows the official DeepSeek-V4
 * convention that rank r owns experts [r*epr, (r+1)*epr),
 * benchmark_reports/deepseek-v4-flash-0731-t4/official-source/inference/
 * model.py:625-626).  The engine of each rank is configured with
 * num_experts = experts_per_rank and holds that rank's records.  A layer is
 *   dee_ep_pack_device -> all-to-all of send rows and send experts ->
 *   dee_moe_forward_rows_device -> all-to-all of the FP32 rows back ->
 *   dee_ep_combine_device;
 * the all-to-alls exchange equal blocks of `capacity` rows per rank pair, so
 * no host synchronisation is needed between the steps. */

/* Pack this rank's selections (device global ids [T, K]) by owner rank:
 * d_send_rows FP16 [ranks * capacity, H] (the token's hidden row),
 * d_send_expert int32 [ranks * capacity] (the owner's local expert id, -1 in
 * unused slots), d_slot_of_pos int32 [T * K] (the send row of selection
 * t*K + r).  Within a destination the selections keep ascending t*K + r.
 * capacity must cover the most selections any one rank receives from this
 * one (T * K always does); overflow raises a device status bit.  The ids
 * are also the journal's (dee_journal_ids_host). */
DEE_API int dee_ep_pack_device(dee_engine* engine, const int32_t* d_ids, int tokens,
                               const void* d_x_f16, int ranks, int experts_per_rank, int capacity,
                               void* d_send_rows, int32_t* d_send_expert, int32_t* d_slot_of_pos,
                               void* stream);

/* The grouped expert GEMMs over received rows: row i (FP16 [rows, H]) through
 * local expert d_expert[i] into d_raw FP32 [rows, H]; rows with expert -1 are
 * skipped (their output rows are left as they were).  Same kernels and
 * per-row results as dee_moe_forward_device. */
DEE_API int dee_moe_forward_rows_device(dee_engine* engine, int layer, const void* d_rows_f16,
                                        const int32_t* d_expert, int rows, float* d_raw,
                                        void* stream);

/* out[t] = sum_r w[t, r] * back[slot_of_pos[t*K + r]] in rank order, each
 * multiply and add rounded to FP32 (the live combine of
 * dee.cpp/scripts/deepseek_v4_layer_candidate.py:616-629), over the rows that
 * came back from the expert owners (d_back FP32 [ranks * capacity, H]). */
DEE_API int dee_ep_combine_device(dee_engine* engine, const float* d_back,
                                  const int32_t* d_slot_of_pos, const float* d_weights, int tokens,
                                  float* d_out_f32, void* stream);

/* Expert parallelism over NVLink peer memory (same split and results as the
 * all-to-all path above, no collective library).  Each rank's engine owns an
 * exchange block -- receive rows/experts/flags and return rows/flags -- that
 * the other ranks write directly:
 *   dispatch: the rank's selections are packed straight into the owners'
 *             receive buffers, then a per-source epoch flag is raised;
 *   experts:  a bounded wait for every source's flag, the grouped GEMMs over
 *             the received rows, whose down-projection epilogue stores each
 *             FP32 row straight into the token owner's return buffer, then a
 *             flag per owner;
 *   combine:  a bounded wait for every owner's flag, the rank-order combine.
 * All ranks call the phases the same number of times; waits that run out
 * (2 s) set bit 6 of the device status word and return. */
#define DEE_EP_IPC_HANDLE_BYTES 64

/* Allocate this rank's exchange block for `tokens` tokens per layer call and
 * export it: *ipc_handle_out receives DEE_EP_IPC_HANDLE_BYTES (a CUDA IPC
 * memory handle), *block_out (may be NULL) the block's device address. */
DEE_API int dee_ep_p2p_init(dee_engine* engine, int ranks, int rank, int tokens,
                            void* ipc_handle_out, uint64_t* block_out);

/* Map every rank's block: ipc_handles holds ranks x DEE_EP_IPC_HANDLE_BYTES
 * (rank order); blocks (may be NULL) gives device addresses for ranks that
 * live in this process on this device, used instead of their handle. */
DEE_API int dee_ep_p2p_connect(dee_engine* engine, const void* ipc_handles, const uint64_t* blocks);

/* The three phases (device ids [T, K] of global experts, x FP16 [T, H],
 * weights FP32 [T, K], out FP32 [T, H]); dee_ep_p2p_forward_device runs them
 * in order.  The dispatched ids are the journal's. */
DEE_API int dee_ep_p2p_dispatch_device(dee_engine* engine, const void* d_x_f16, const int32_t* d_ids,
                                       void* stream);
DEE_API int dee_ep_p2p_experts_device(dee_engine* engine, int layer, void* stream);
DEE_API int dee_ep_p2p_combine_device(dee_engine* engine, const float* d_weights, float* d_out_f32,
                                      void* stream);
DEE_API int dee_ep_p2p_forward_device(dee_engine* engine, int layer, const void* d_x_f16,
                                      const int32_t* d_ids, const float* d_weights, float* d_out_f32,
                                      void* stream);

/* Offload tier (configuration 4): the reference's VRAM expert cache over a
 * pinned-host record pool (prepare_fp4_experts -> HostPackCache::get_batch ->
 * H2D, engine.cpp:3133, async_prefetcher.cpp:691-780) with next-use
 * eviction (VramCacheManager::evict_until_free, vram_cache.cpp:113, ranked by
 * NextUseEstimator::victim_rank, include/dee/next_use.h:132-137).  Placement
 * only: it never changes which experts run, so route ids and outputs equal
 * the all-resident ones.
 *
 * Attach: h_records holds every layer's records [layers][num_experts]
 * (pinned host memory, the DEE4 layout); d_pool is a device pool of
 * pool_slots records shared by all layers.  Every layer's bank becomes
 * (d_pool, pool_slots) with no expert resident. */
DEE_API int dee_offload_attach(dee_engine* engine, const void* h_records, size_t record_bytes, int layers,
                               void* d_pool, int pool_slots);
/* Before a layer's forward: read its ids [T, K] (waits for `stream`), keep the
 * resident experts, bring the others in from host memory into free slots or
 * the residents with the largest expected next use (one H2D copy per expert on
 * the engine's copy stream), update the layer's slot table, and make `stream`
 * wait for the copies.  *cold_out (may be NULL) = experts copied. */
DEE_API int dee_offload_prepare_device(dee_engine* engine, int layer, const int32_t* d_ids, int tokens,
                                       void* stream, int* cold_out);
/* Test hook, one-shot: the next cold record copy of dee_offload_prepare_device
 * fails as if it could not be queued (AsyncPrefetcher::debug_fail_next_submit,
 * dee.cpp/include/dee/async_prefetcher.h:232).  That prepare call returns
 * DEE_ERR_CUDA naming the expert, whose slot is invalidated (not resident:
 * a forward run anyway reports it through the status word instead of
 * reading the slot), and a later prepare for it cold-loads it again. */
DEE_API int dee_offload_debug_fail_next_copy(dee_engine* engine);

/* Exactly `bytes` of pinned host memory (for an offload tier's records;
 * allocators that round pinned requests up to powers of two cannot hold a
 * 140 GB stack on a 196 GB host). */
DEE_API int dee_host_alloc_pinned(size_t bytes, void** out);
DEE_API int dee_host_free_pinned(void* p);

/* Totals since attach: out4 = {lookups, hits, cold reads, bytes copied}. */
DEE_API int dee_offload_stats(dee_engine* engine, uint64_t* out4);

/* The dense glue of the synthetic multi-layer stack that drives the routed
 * layer end to end (no counterpart in the reference engine; the stack of the
 * benchmark's configurations 3 and 4: embedding -> [RMSNorm, router, MoE,
 * residual] x L -> RMSNorm -> LM head argmax).  Every per-token result is
 * computed in a fixed order independent of the batch, so route ids and
 * tokens do not depend on how the tokens are spread over GPUs.
 *   embed:        x FP32 [T, H] = table FP16 [V, H] rows of ids [T]
 *   rmsnorm:      y FP16 [T, H] = x * rsqrt(mean(x^2) + eps) * w
 *   router:       logits FP32 [T, E] = y . W_r^T, W_r FP32 [E, H]
 *   residual_add: x += y (FP32 [T, H])
 *   lm_head:      ids [T] = argmax_v (y . W^T), W FP16 [V, H], first index on
 *                 ties; d_logits FP32 [T, V] is scratch */
DEE_API int dee_stack_embed_device(dee_engine* engine, const void* d_table_f16, const int32_t* d_ids,
                                   int tokens, int vocab, float* d_x, void* stream);
DEE_API int dee_stack_rmsnorm_device(dee_engine* engine, const float* d_x, const float* d_w, float eps,
                                     int tokens, void* d_y_f16, void* stream);
DEE_API int dee_stack_router_logits_device(dee_engine* engine, const void* d_h_f16, const float* d_wr,
                                           int tokens, int experts, float* d_logits, void* stream);
DEE_API int dee_stack_residual_add_device(dee_engine* engine, float* d_x, const float* d_y, int tokens,
                                          void* stream);
DEE_API int dee_stack_lm_head_argmax_device(dee_engine* engine, const void* d_h_f16, const void* d_w_f16,
                                            int tokens, int vocab, float* d_logits, int32_t* d_ids_out,
                                            void* stream);
/* Derive a distinct bank: dst record i = src record i with its first
 * packed_bytes (the packed weights) XORed by a hash of (seed, first_record +
 * i); scale bytes copied.  Used to give every layer of a synthetic stack its
 * own experts without quantising each one. */
DEE_API int dee_records_scramble_device(const void* d_src, void* d_dst, int records, size_t record_bytes,
                                        size_t packed_bytes, uint64_t seed, int first_record, void* stream);

/* Host copy of the int32 [T, K] route ids the last forward consumed -- the
 * buffer the route journal records (deepseek_v4_native_generate.py
 * :2196-2216).  Waits for the last forward's stream, then copies.  Returns
 * the number of ids written, or a negative DEE_ERR_* code. */
DEE_API int dee_journal_ids_host(dee_engine* engine, int32_t* h_out, int max_ids);

/* fp4_e2m1_to_f16_cuda (dee.cpp/include/dee/cuda_convert.h:104-134,
 * cuda_convert.cu:252-288): packed [out, in/2] + scales [out, in/32] ->
 * FP16 [out, in]; in must be a multiple of 64. */
DEE_API int dee_fp4_decode_device(const uint8_t* d_packed, const uint8_t* d_scale, void* d_dst_f16,
                          size_t out, size_t in, void* stream);

/* Pack FP32 [out, in] weights as E2M1 + per-32 UE8M0 scales (the layout the
 * reference's repacker writes, repack_to_dee4.py:42-55); used to build
 * synthetic expert banks on the device. */
DEE_API int dee_fp4_quantize_device(const float* d_w, size_t out, size_t in, uint8_t* d_packed,
                            uint8_t* d_scale, void* stream);

/* The official FP8 activation quantisation (act_quant with scale_fmt
 * "ue8m0", official-source/inference/kernel.py:41-103; restated in
 * dee.cpp/scripts/deepseek_v4_layer_common.py:213-240): per row and block of
 * `block` (128 official, 32 MX) columns, amax = max(|x|, 1e-4), scale
 * s = 2^ceil(log2(amax / 448)), q = E4M3(clamp(x / s, +-448)) round to
 * nearest even.  x FP16 [rows, cols] -> q E4M3 bytes [rows, cols] and the
 * UE8M0 scale bytes [rows, cols / block].  cols % 256 == 0. */
DEE_API int dee_act_quant_device(const void* d_x_f16, int rows, int cols, int block, uint8_t* d_q,
                                 uint8_t* d_scales, void* stream);

/* The layer forward for callers that cannot allocate device memory (code
 * inside an allocator or memory-pool callback, or a host whose device memory
 * is entirely owned by its own caching allocator).  No counterpart in the
 * reference: it has no engine handle and allocates nothing.  Same kernels
 * and results as dee_moe_forward_device with device ids and the FP32
 * rank-order combine; every scratch buffer lives in a 4 MiB static device
 * array that the library reserves on each GPU it is loaded on (145
 * selections at H=4096, I=2048, i.e. 24 tokens at top-6).  Larger requests
 * return DEE_ERR_SCRATCH_LIMIT.  d_records holds n_slots records in expert
 * order (slot e = expert e).  d_status_out (may be NULL) receives the
 * kernels' status word (0 = ok).  All calls share the static array: calls
 * that overlap on the GPU race, so serialise them.  The first call on a
 * device resolves the array's device address; make it before any stream
 * capture.  That address is kept for the life of the process: do not call
 * this entry point after cudaDeviceReset.  d_x_f16 and d_out_f32 must be
 * 16-byte aligned, d_ids, d_weights and d_status_out 4-byte aligned; every
 * argument is checked before any CUDA call (DEE_ERR_INVALID, nothing
 * launched). */
DEE_API int dee_moe_forward_noalloc(const dee_config* cfg, const void* d_records,
                                    size_t record_bytes, int n_slots, const void* d_x_f16,
                                    int tokens, const int32_t* d_ids, const float* d_weights,
                                    float* d_out_f32, uint32_t* d_status_out, void* stream);

/* Failure detection.  Every device wait is bounded: a wait that runs out
 * sets a bit in the engine's status word, the kernel unwinds, the context
 * stays usable and dee_engine_sync_status reports DEE_ERR_DEVICE (the
 * fail-closed convention of Engine::last_error_message, engine.h:434-436).
 *
 * Limit of this engine's waits on other ranks' flags (the NVLink expert-
 * parallel phases), in nanoseconds, 100 us .. 2 s (default 2 s): a rank that
 * never dispatches or never returns its rows is reported after this long
 * (status bit 6).  No counterpart in the reference's single-GPU engine. */
DEE_API int dee_engine_set_wait_limit_ns(dee_engine* engine, uint64_t limit_ns);

/* Self-test of the bounded pipeline wait on the current device: one kernel
 * waits on an mbarrier that nothing ever arrives on; after limit_ns (100 us
 * .. 2 s) the wait gives up and ORs bit 0 (a pipeline wait timeout) into
 * *d_status (device memory, 4-byte aligned).  Queued on `stream`.  No
 * counterpart in the reference (its host-side equivalent is the prefetcher's
 * debug_fail_next_submit, include/dee/async_prefetcher.h:232). */
DEE_API int dee_wait_selftest(uint64_t limit_ns, uint32_t* d_status, void* stream);

/* Kernel launches issued by this engine since creation (for the bench's
 * launch accounting). */
DEE_API uint64_t dee_engine_launch_count(const dee_engine* engine);

/* Opt-in stage timing, the role of the reference's StageProfiler
 * (dee.cpp/include/dee/profiling.h:31-46, GpuStage): when enabled every
 * stage of a forward is bracketed by CUDA events on its launch stream.
 * Stages: 0 route, 1 permute, 2 gather, 3 gate/up GEMM, 4 down GEMM,
 * 5 combine, 6 expert-parallel dispatch (the peer rows kernel or the pack
 * before an NCCL exchange), 7 the one-launch decode layer (gate/up, down
 * and the fused combine of decode-sized batches, in place of 3-5). */
DEE_API int dee_engine_set_profiling(dee_engine* engine, int enable);

/* Milliseconds of each stage of the most recent profiled forward (-1 for a
 * stage that did not run).  Waits for the stage events.  Returns the number
 * of entries written. */
DEE_API int dee_engine_stage_ms(dee_engine* engine, float* out_ms, int n);

/* ---- DEE4 expert store on disk -------------------------------------------
 * Dee4ExpertStore (dee.cpp/include/dee/expert_store.h:286-409,
 * dee.cpp/src/expert_store.cpp:786-1230): formats dee4-v2 (one fixed-stride
 * file, dense index (layer - start_layer) * experts_per_layer + expert),
 * dee4-v3-trace (one file with a sorted (layer, expert) record table) and
 * dee4-v4-segmented (one sha256-sealed file per layer bucket).  open() takes
 * a store directory or its metadata.json and fails closed, with the
 * reference's messages, on malformed metadata, missing or mis-sized files,
 * segment paths that leave the store, and (verify_segment_hashes != 0)
 * segments whose sha256 does not match their seal.  Records are read with
 * pread() by `threads` host threads straight into caller memory. */
typedef struct dee_store dee_store;

/* The geometry and component table (Dee4ExpertStore accessors,
 * expert_store.h:349-358, and the per-component views of get()). */
typedef struct dee_store_info {
    int start_layer;
    int num_layers;
    int experts_per_layer;
    int segmented;
    int trace_indexed;
    size_t record_bytes;
    size_t stored_records;
    size_t file_count;
    size_t weight_offsets[3];
    size_t weight_nbytes[3];
    size_t weight_out[3];
    size_t weight_stored_in[3];
    size_t scale_offsets[3];
    size_t scale_nbytes[3];
    size_t scale_out[3];
    size_t scale_in[3];
} dee_store_info;

/* Per-fill accounting (MaterializeResult, expert_store.h:48-61).
 * files_verified: files whose seal a fill checked (verify != 0). */
typedef struct dee_store_read_stats {
    uint64_t bytes_read;
    uint64_t pread_calls;
    uint64_t short_reads;
    uint64_t records;
    uint64_t files_verified;
    double seconds;
} dee_store_read_stats;

/* dee_store_open options (Dee4OpenOptions, expert_store.h:286-306).
 * VERIFY_SEALS: re-hash every segment at open and fail closed on a mismatch
 * (verify_segment_hashes).  SEAL_DROP_PAGES: drop each segment from the page
 * cache after hashing it (the effect of seal_reads_through_page_cache). */
#define DEE_STORE_VERIFY_SEALS 1
#define DEE_STORE_SEAL_DROP_PAGES 2

/* Dee4ExpertStore() / ~Dee4ExpertStore(). */
DEE_API int dee_store_create(dee_store** out);
DEE_API void dee_store_destroy(dee_store* store);
/* Dee4ExpertStore::open(path, Dee4OpenOptions) (expert_store.h:286-306,
 * expert_store.cpp:790); options = DEE_STORE_* bits, `threads` hash segments
 * in parallel.  DEE_ERR_INVALID on any failure; the reason is
 * dee_store_last_error(). */
DEE_API int dee_store_open(dee_store* store, const char* directory_or_metadata, int options, int threads);
DEE_API void dee_store_close(dee_store* store);
DEE_API const char* dee_store_last_error(const dee_store* store);
/* backend_name() ("dee4", "dee4_trace", "dee4_segmented") and
 * integrity_identity() (data_sha256, or for a segmented store the sha256 of
 * the concatenated segment seals). */
DEE_API const char* dee_store_backend(const dee_store* store);
DEE_API const char* dee_store_identity(const dee_store* store);
DEE_API int dee_store_get_info(const dee_store* store, dee_store_info* out);
/* {lookups, lookup failures, records read, bytes read} since open. */
DEE_API int dee_store_stats(const dee_store* store, uint64_t* out4);
/* get() (expert_store.cpp:1176-1215): the record index of (layer, expert);
 * DEE_ERR_RANGE outside the store or, for a trace store, for a pair it does
 * not hold. */
DEE_API int dee_store_lookup(dee_store* store, int layer, int expert, uint64_t* record_index);
/* materialize_ex() (expert_store.h:341-347): one record into dst (nbytes must
 * equal record_bytes). */
DEE_API int dee_store_materialize(dee_store* store, int layer, int expert, void* dst, size_t nbytes,
                                  dee_store_read_stats* stats);
/* Experts [first_expert, first_expert + experts) of layers [first_layer,
 * first_layer + layers) into host memory dst as [layer][expert][record_bytes]
 * (the offload tier's pinned record block; an expert-parallel rank's share),
 * by `threads` parallel preads.  verify != 0: every file the call reads whole
 * (a segment, or the data file of a single-file store) is hashed as it
 * streams in and the call fails closed on a seal mismatch -- the seal check
 * of open() without a second pass over the disk. */
DEE_API int dee_store_read_layers(dee_store* store, int first_layer, int layers, int first_expert, int experts,
                                  void* dst, size_t dst_bytes, int threads, int verify, dee_store_read_stats* stats);
/* The same records into device memory d_dst (a resident expert bank),
 * through 2 * threads pinned staging buffers of staging_bytes / (2 * threads)
 * each: every reader thread preads into one buffer while its other buffer's
 * H2D copy runs on `stream`.  Returns after the copies completed. */
DEE_API int dee_store_upload_layers_device(dee_store* store, int first_layer, int layers, int first_expert,
                                           int experts, void* d_dst, size_t dst_bytes, size_t staging_bytes,
                                           int threads, int verify, void* stream, dee_store_read_stats* stats);
/* SHA-256 of n bytes as 64 lowercase hex digits + NUL (the seal function). */
DEE_API int dee_sha256_hex(const void* data, size_t n, char* out65);

#ifdef __cplusplus
}
#endif

#endif /* DEE_B200_H */
