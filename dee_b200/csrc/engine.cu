// engine.cu -- host orchestration behind the C ABI in include/dee_b200.h.
//
// The engine replaces the per-expert host loop of the reference
// (Engine::moe_forward_batch_device_impl, reference
// dee.cpp/src/engine.cpp:776-1190: host grouping, one D2D copy per gathered
// row, three dequant launches, three cuBLAS calls and one D2D copy per
// scattered row for every active expert) with a fixed sequence of launches
// independent of how many experts are active:
//
//   permute (1 CTA)  -> gather (token rows into grouped order)
//   -> gate/up grouped GEMM (tcgen05, SwiGLU epilogue)
//   -> down grouped GEMM (tcgen05, scatter epilogue)
//   -> combine (optional)
#include "dee_b200.h"
#include "kernels.h"

#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>
#include <vector>
#include <algorithm>
#include <unordered_map>
#include <cmath>

namespace dee {
namespace {

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

struct RecordLayout {
    size_t w1, w3, w2, s1, s3, s2, bytes;
};

RecordLayout record_layout(int hidden, int inter) {
    const size_t ih = static_cast<size_t>(hidden) * inter;
    RecordLayout L{};
    L.w1 = 0;
    L.w3 = ih / 2;
    L.w2 = ih;
    L.s1 = ih + ih / 2;
    L.s3 = L.s1 + ih / 32;
    L.s2 = L.s3 + ih / 32;
    L.bytes = L.s2 + ih / 32;
    return L;
}

// kStageDispatch: the expert-parallel send side (the peer rows kernel, or
// the NCCL path's pack), recorded by the engine that owns the tokens.
// kStageExperts: the one-launch decode layer (gate/up, down and, for the
// live path, the combine in one kernel).
enum Stage : int { kStageRoute = 0, kStagePermute, kStageGather, kStageGateUp, kStageDown,
                   kStageCombine, kStageDispatch, kStageExperts, kStageCount };

struct Bank {
    bool attached = false;
    const uint8_t* records = nullptr;
    int n_slots = 0;
    size_t record_bytes = 0;
    int32_t* d_slot_of = nullptr;  // [E]
    CUtensorMap w1, w3, w2, s1, s3, s2;  // tcgen05 kernel
    GemmMaps dec_gu{}, dec_dn{};         // decode kernel (weight maps)
    bool mx = false;                     // MXFP8 kernel maps encoded
    MxMaps mx_gu{}, mx_dn{};
    // the layer's shared expert (F8_E4M3 + E8M0 per 128 x 128), if attached
    bool shared = false;
    int shared_inter = 0;
    const uint8_t *sh_s1 = nullptr, *sh_s3 = nullptr, *sh_s2 = nullptr;
    CUtensorMap sh_m1, sh_m3, sh_m2;
};

template <class T>
cudaError_t dev_alloc(T** p, size_t n) {
    return cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T) + 16);
}

}  // namespace
}  // namespace dee

namespace dee {
// Peer (NVLink) expert-parallel state of one rank: its exchange block
// (exported with CUDA IPC), every rank's buffer pointers and the epoch that
// numbers layer calls.
struct EpP2P {
    int ranks = 0, rank = 0, tokens = 0, capacity = 0;
    uint8_t* block = nullptr;
    size_t off_recv_rows = 0, off_recv_expert = 0, off_recv_flag = 0, off_back_rows = 0,
           off_back_flag = 0, bytes = 0;
    EpPeers peers{};
    std::vector<void*> opened;        // peer blocks opened from IPC handles
    float** d_back_peers = nullptr;   // device copy of peers.back_rows
    int32_t* d_slot_of_pos = nullptr; // [tokens * K]
    uint32_t* d_done = nullptr;       // dispatch rows kernel's completion counter (in the same allocation)
    uint32_t epoch = 0;
    bool connected = false;
};
}  // namespace dee

namespace dee {
// Offload tier: every layer's records in pinned host memory, a device pool of
// slots shared by all layers, and a next-use ranking of the residents.
//
// The ranking restates the probabilistic-Belady estimator of the reference
// (dee.cpp/include/dee/next_use.h:1-160): decode visits the layers in a fixed
// cycle, an expert of layer L is next needed d = (L - current) mod cycle
// layer calls from now, and with a per-expert reuse probability p (an
// exponentially weighted estimate updated at every visit of its layer) its
// expected next use is d + cycle * (1/p - 1).  The victim is the resident with
// the largest expectation; experts of the running layer rank below all others.
struct Offload {
    bool on = false;
    const uint8_t* host = nullptr;  // [layers][experts] records, pinned
    size_t record_bytes = 0;
    int layers = 0, experts = 0, pool_slots = 0;
    uint8_t* pool = nullptr;        // device [pool_slots] records
    std::vector<int64_t> slot_key;  // slot -> layer * experts + expert, -1 free
    std::vector<int32_t> slot_of;   // [layers * experts] -> slot, -1 absent
    std::vector<uint32_t> visits;   // per layer
    struct Stat { double ewma; uint32_t last_visit; };
    std::unordered_map<int64_t, Stat> stats;
    std::vector<uint32_t> used_visit;  // per slot: the prepare call that last used it
    uint32_t calls = 0;
    int current = 0;
    double alpha = 0.2, p0 = 0.1, p_floor = 1e-3;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t copied = nullptr;
    int32_t* h_ids = nullptr;       // pinned staging of a layer's ids
    size_t h_ids_cap = 0;
    uint64_t lookups = 0, hits = 0, cold = 0, bytes = 0;
    // one-shot test hook: the next cold copy's submission fails
    // (AsyncPrefetcher::debug_fail_next_submit, include/dee/async_prefetcher.h:232)
    bool fail_next_copy = false;
    uint64_t submit_failures = 0;

    double probability(int64_t key) const {
        auto it = stats.find(key);
        if (it == stats.end()) return p0;
        const int layer = static_cast<int>(key / experts);
        int64_t elapsed = static_cast<int64_t>(visits[layer]) - it->second.last_visit;
        if (layer == current) --elapsed;
        double p = it->second.ewma;
        if (elapsed > 0) p *= std::pow(1.0 - alpha, static_cast<double>(elapsed));
        return std::max(p_floor, std::min(1.0, p));
    }
    double victim_rank(int64_t key) const {
        const int layer = static_cast<int>(key / experts);
        if (layer == current) return -1.0;  // the running layer leaves last
        const int d = ((layer - current) % layers + layers) % layers;
        return d + layers * (1.0 / probability(key) - 1.0);
    }
    void on_use(int64_t key) {
        const int layer = static_cast<int>(key / experts);
        const uint32_t visit = visits[layer];
        auto it = stats.find(key);
        if (it == stats.end()) {
            stats.emplace(key, Stat{p0 * (1.0 - alpha) + alpha, visit});
            return;
        }
        if (it->second.last_visit == visit) return;
        it->second.ewma = it->second.ewma * std::pow(1.0 - alpha, visit - it->second.last_visit) + alpha;
        it->second.last_visit = visit;
    }
};
}  // namespace dee

struct dee_engine {
    dee_config cfg{};
    dee::EpP2P ep;
    // limit of the waits on other ranks' flags (dee_engine_set_wait_limit_ns)
    uint64_t wait_limit_ns = dee::sm100::kWaitLimitNs;
    dee::Offload off;
    std::string last_error;
    int num_sms = 148;
    cudaStream_t stream = nullptr;  // the engine's own stream (synchronous API)
    uint32_t* d_status = nullptr;
    uint32_t* h_status = nullptr;  // pinned
    std::vector<dee::Bank> banks;
    // workspaces, capacity in selections (tokens * topk)
    size_t cap_sel = 0;
    int32_t* d_ids = nullptr;
    float* d_weights = nullptr;
    int32_t* d_perm = nullptr;
    int32_t* d_row_of = nullptr;
    int32_t* d_counts = nullptr;
    int32_t* d_offsets = nullptr;
    dee::TileDesc* d_tiles = nullptr;
    int32_t* d_n_tiles = nullptr;
    int max_tiles = 0;
    __half* d_xperm = nullptr;
    __half* d_act = nullptr;
    float* d_raw = nullptr;
    int32_t* h_ids = nullptr;      // pinned staging of host-given ids
    int32_t* d_journal = nullptr;  // ids consumed by the latest forward (written by permute)
    int32_t* d_perm_chunks = nullptr;  // multi-CTA permutation: per-chunk expert counts
    int32_t* d_perm_lrank = nullptr;   // multi-CTA permutation: rank within the chunk
    // one-launch decode layer: [max_tiles] gate/up items done per tile, then
    // [kDecodeMaxSelections * H/128] rows written per (token, feature block)
    uint32_t* d_sync = nullptr;
    int2* d_tile_grp = nullptr;      // [max_tiles] prefill: first tile and tile count of the tile's expert
    // one-launch decode front end: per-CTA grouping scratch and the
    // epoch-tagged counters (zeroed once), with the epoch of the last launch
    int32_t* d_front_scratch = nullptr;
    unsigned long long* d_front_ctr = nullptr;
    uint32_t front_epoch = 0;
    // shared-expert workspaces, capacity in tokens
    // MXFP8 path workspaces (E4M3 rows and per-32 UE8M0 scales), capacity in rows
    size_t cap_mx = 0;
    uint8_t *d_xq = nullptr, *d_xs = nullptr, *d_aq = nullptr, *d_as = nullptr;
    CUtensorMap map_xq_t[4], map_aq_t[4];
    size_t cap_sh = 0;
    int cap_sh_inter = 0;
    __half* d_sh_act = nullptr;
    float* d_sh_out = nullptr;
    cudaStream_t journal_stream = nullptr;
    size_t h_ids_count = 0;
    CUtensorMap map_xperm_t[4], map_act_t[4];  // token boxes of the tcgen05 kernel
    CUtensorMap map_xperm_dec, map_act_dec;  // token rows of the decode kernel
    uint64_t launches = 0;
    // Opt-in stage timing (the role of the reference's StageProfiler,
    // dee.cpp/include/dee/profiling.h:31-46): events recorded on the launch
    // stream around each stage of the most recent forward.
    bool profile = false;
    cudaEvent_t ev_start[dee::kStageCount] = {};
    cudaEvent_t ev_end[dee::kStageCount] = {};
    bool ev_used[dee::kStageCount] = {};
};

namespace dee {
namespace {

constexpr uint64_t kMinWaitLimitNs = 100000;  // 100 us

int fail(dee_engine* e, int code, const std::string& msg) {
    if (e) e->last_error = msg;
    return code;
}

// Stage timing: when profiling is on, each stage of a forward is bracketed
// by two events recorded on the stream the stage is launched on.
void stage_begin(dee_engine* e, int st, cudaStream_t stream) {
    if (!e->profile) return;
    cudaEventRecord(e->ev_start[st], stream);
}

void stage_end(dee_engine* e, int st, cudaStream_t stream) {
    if (!e->profile) return;
    cudaEventRecord(e->ev_end[st], stream);
    e->ev_used[st] = true;
}

int cuda_fail(dee_engine* e, cudaError_t err, const char* what) {
    return fail(e, DEE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

bool encode(dee_engine* e, CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
            const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
            CUtensorMapSwizzle swz, const char* what) {
    auto fn = get_encode_fn();
    if (!fn) {
        e->last_error = "cuTensorMapEncodeTiled unavailable (driver entry point)";
        return false;
    }
    cuuint32_t elem[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(map, dt, rank, const_cast<void*>(base), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        e->last_error = std::string("cuTensorMapEncodeTiled failed for ") + what + " (code " +
                        std::to_string(static_cast<int>(r)) + ")";
        return false;
    }
    return true;
}

void free_workspace(dee_engine* e) {
    cudaFree(e->d_ids); cudaFree(e->d_weights); cudaFree(e->d_perm); cudaFree(e->d_row_of);
    cudaFree(e->d_counts); cudaFree(e->d_offsets); cudaFree(e->d_tiles); cudaFree(e->d_n_tiles);
    cudaFree(e->d_xperm); cudaFree(e->d_act); cudaFree(e->d_raw); cudaFree(e->d_journal);
    cudaFree(e->d_perm_chunks); cudaFree(e->d_perm_lrank); cudaFree(e->d_sync); cudaFree(e->d_tile_grp);
    e->d_perm_chunks = nullptr; e->d_perm_lrank = nullptr; e->d_sync = nullptr; e->d_tile_grp = nullptr;
    if (e->h_ids) cudaFreeHost(e->h_ids);
    e->d_ids = nullptr; e->d_weights = nullptr; e->d_perm = nullptr; e->d_row_of = nullptr;
    e->d_counts = nullptr; e->d_offsets = nullptr; e->d_tiles = nullptr; e->d_n_tiles = nullptr;
    e->d_xperm = nullptr; e->d_act = nullptr; e->d_raw = nullptr; e->h_ids = nullptr;
    e->d_journal = nullptr;
    e->h_ids_count = 0;
    e->cap_sel = 0;
}

// Grow the workspaces to hold `sel` selections.  Growth synchronises
// `stream` first so no queued kernel still reads the old buffers (the
// reference grows its batch buffers the same way, engine.cpp:827-884).
int ensure_capacity(dee_engine* e, size_t sel, cudaStream_t stream) {
    if (sel <= e->cap_sel) return DEE_OK;
    cudaError_t err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "cudaStreamSynchronize(workspace growth)");
    free_workspace(e);
    const size_t cap = ((sel + 255) / 256) * 256;
    const int H = e->cfg.hidden, I = e->cfg.inter, E = e->cfg.num_experts;
    const int max_tiles = E + static_cast<int>(cap / 8) + 1;
    if ((err = dev_alloc(&e->d_ids, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_weights, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_perm, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_row_of, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_counts, static_cast<size_t>(E))) != cudaSuccess ||
        (err = dev_alloc(&e->d_offsets, static_cast<size_t>(E) + 1)) != cudaSuccess ||
        (err = dev_alloc(&e->d_tiles, static_cast<size_t>(max_tiles))) != cudaSuccess ||
        (err = dev_alloc(&e->d_n_tiles, 1)) != cudaSuccess ||
        (err = dev_alloc(&e->d_xperm, cap * H)) != cudaSuccess ||
        (err = dev_alloc(&e->d_act, cap * I)) != cudaSuccess ||
        (err = dev_alloc(&e->d_raw, cap * H)) != cudaSuccess ||
        (err = dev_alloc(&e->d_journal, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_perm_chunks, ((cap + 1023) / 1024) * static_cast<size_t>(E))) != cudaSuccess ||
        (err = dev_alloc(&e->d_perm_lrank, cap)) != cudaSuccess ||
        (err = dev_alloc(&e->d_tile_grp, static_cast<size_t>(max_tiles))) != cudaSuccess ||
        (err = dev_alloc(&e->d_sync, static_cast<size_t>(max_tiles) +
                                         static_cast<size_t>(kDecodeMaxSelections) * (H / 128))) != cudaSuccess ||
        (err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_ids), cap * sizeof(int32_t),
                             cudaHostAllocDefault)) != cudaSuccess) {
        free_workspace(e);
        return cuda_fail(e, err, "workspace allocation");
    }
    e->cap_sel = cap;
    e->max_tiles = max_tiles;
    if (!encode_gemm_token_maps(get_encode_fn(), e->d_xperm, static_cast<int>(cap), H, e->map_xperm_t) ||
        !encode_gemm_token_maps(get_encode_fn(), e->d_act, static_cast<int>(cap), I, e->map_act_t)) {
        e->last_error = "cuTensorMapEncodeTiled failed for the GEMM token maps";
        return DEE_ERR_CUDA;
    }
    if (!encode_decode_token_map(get_encode_fn(), e->d_act, static_cast<int>(cap), I,
                                 &e->map_act_dec) ||
        !encode_decode_token_map(get_encode_fn(), e->d_xperm, static_cast<int>(cap), H,
                                 &e->map_xperm_dec)) {
        e->last_error = "cuTensorMapEncodeTiled failed for the decode token maps";
        return DEE_ERR_CUDA;
    }
    return DEE_OK;
}

int check_engine(dee_engine* e) {
    if (!e) return DEE_ERR_INVALID;
    cudaError_t err = cudaSetDevice(e->cfg.device_id);
    if (err != cudaSuccess) return cuda_fail(e, err, "cudaSetDevice");
    return DEE_OK;
}

// A caller's device pointer and the widest access the kernels make through
// it: FP16 token rows by 16-byte vector loads, bulk copies or tensor maps,
// FP32 rows (raw rows, outputs) by float4, ids, weights and logits by 4-byte
// loads (int64 ids by 8).  A pointer off that alignment (a column slice of a
// tensor, say) would raise a misaligned-address fault inside a kernel and
// lose the context, so the entry points refuse it before any launch.  Null
// passes: each entry checks the pointers it requires.
struct PtrAlign {
    const char* name;
    const void* p;
    uintptr_t align;
};

int check_aligned(dee_engine* e, const char* entry, std::initializer_list<PtrAlign> ptrs) {
    for (const PtrAlign& q : ptrs)
        if ((reinterpret_cast<uintptr_t>(q.p) & (q.align - 1)) != 0)
            return fail(e, DEE_ERR_INVALID, std::string(entry) + ": " + q.name + " must be " +
                                                std::to_string(q.align) + "-byte aligned");
    return DEE_OK;
}

bool host_ids_valid(dee_engine* e, const int32_t* ids, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= e->cfg.num_experts) {
            e->last_error = "expert id " + std::to_string(ids[i]) + " at selection " +
                            std::to_string(i) + " is outside [0," +
                            std::to_string(e->cfg.num_experts) + ")";
            return false;
        }
    }
    return true;
}

// The launch sequence shared by every forward entry point.  d_ids32 holds
// validated-or-device-checked int32 ids [T, K]; raw receives [T*K, H] FP32.
// The expert-parallel rows entry point runs it with K = 1, one row per
// selection, and ids of -1 for unused rows (skip_negative).
struct EpReturn {
    float* const* raw_peers;  // device array [ranks]
    int capacity, rank;
};

// The senders' dispatch flags the permutation waits for (bounded) before it
// reads an expert-parallel receive buffer.
struct EpWait {
    const uint32_t* flags;
    int ranks;
    uint32_t epoch;
    uint64_t limit_ns;
};

// Routing fused into the permutation (decode-sized batches): the router
// reads logits and writes the ids run_experts groups by, and the weights.
struct FusedRoute {
    const float* logits;
    float* weights;
};

// The live combine fused into the decode layer launch: out[t] = sum_r
// weights[t*K + r] * raw[t*K + r] (run_experts reports whether it ran it).
struct FusedCombine {
    const float* weights;
    float* out;
    bool* done;
};

int forward_front(dee_engine* e, int layer, const void* d_x_f16, int tokens, int K, const float* d_logits,
                  int32_t* d_ids, float* d_weights, float* d_out_f32, float* d_raw, cudaStream_t stream);

int run_experts(dee_engine* e, int layer, const __half* d_x, int tokens, const int32_t* d_ids32,
                float* raw, cudaStream_t stream, int K, bool skip_negative, bool write_journal,
                const EpReturn* ret = nullptr, const float* official_route_w = nullptr,
                const EpWait* wait = nullptr, const FusedRoute* route = nullptr,
                const FusedCombine* combine = nullptr) {
    if (layer < 0 || layer >= static_cast<int>(e->banks.size()) || !e->banks[layer].attached)
        return fail(e, DEE_ERR_NO_BANK, "no expert bank attached for layer " + std::to_string(layer));
    const dee::Bank& bank = e->banks[layer];
    const int H = e->cfg.hidden, I = e->cfg.inter, E = e->cfg.num_experts;
    const size_t sel = static_cast<size_t>(tokens) * K;
    // Decode-sized calls use the register-dequant kernel (tiles of <= 8 token
    // rows); larger calls the tcgen05 kernel (tiles of <= 128 rows).
    const bool decode = sel <= static_cast<size_t>(kDecodeMaxSelections);
    if (ret && !decode)
        return fail(e, DEE_ERR_UNSUPPORTED, "the NVLink expert-parallel return needs <= " +
                                                std::to_string(kDecodeMaxSelections) + " rows per rank");
    const int n_max = decode ? kDecodeTileRows : gemm_n_max();

    PermuteOut po{e->d_counts, e->d_offsets, e->d_perm,     e->d_row_of,
                  e->d_tiles,  e->d_n_tiles, write_journal ? e->d_journal : nullptr};
    po.chunk_counts = e->d_perm_chunks;
    po.lrank = e->d_perm_lrank;
    po.max_chunks = static_cast<long long>((e->cap_sel + 1023) / 1024);
    if (wait) {
        po.wait_flags = wait->flags;
        po.wait_ranks = wait->ranks;
        po.wait_epoch = wait->epoch;
        po.wait_limit_ns = wait->limit_ns;
    }
    // the decode layer runs in one launch; its counters are zeroed by the
    // (one-CTA) permutation
    const bool fuse_combine = decode && combine && !ret && !official_route_w;
    if (combine) *combine->done = fuse_combine;
    if (decode) {
        po.clear = e->d_sync;
        po.clear_n = e->max_tiles + (fuse_combine ? tokens * (H / 128) : 0);
    } else {
        po.tile_grp = e->d_tile_grp;
    }
    stage_begin(e, kStagePermute, stream);
    cudaError_t err;
    if (route) {
        err = launch_route_permute(route->logits, tokens, E, K, const_cast<int32_t*>(d_ids32), route->weights,
                                   n_max, e->max_tiles, po, e->d_status, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "route+permute launch");
    } else {
        err = launch_permute(d_ids32, tokens, K, E, n_max, e->max_tiles, po, e->d_status, stream, skip_negative);
        if (err != cudaSuccess) return cuda_fail(e, err, "permute launch");
        e->launches += permute_launch_count(tokens, K, po) - 1;
    }
    stage_end(e, kStagePermute, stream);
    stage_begin(e, kStageGather, stream);
    err = launch_gather_rows(d_x, e->d_perm, e->d_offsets + E, static_cast<int>(sel), K, H, e->d_xperm, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "gather launch");
    stage_end(e, kStageGather, stream);

    GemmArgs a{};
    a.hidden = H;
    a.inter = I;
    a.topk = K;
    a.swiglu_limit = e->cfg.swiglu_limit;
    a.tiles = e->d_tiles;
    a.n_tiles = e->d_n_tiles;
    a.slot_of = bank.d_slot_of;
    a.num_slots = bank.n_slots;
    a.records = bank.records;
    a.record_bytes = bank.record_bytes;
    a.num_experts = E;
    a.perm = e->d_perm;
    a.act = e->d_act;
    a.raw = raw;
    a.status = e->d_status;
    if (!decode) a.tile_grp = e->d_tile_grp;
    if (official_route_w) {
        a.official = 1;
        a.route_w = official_route_w;
    }
    if (ret) {
        a.raw_peers = ret->raw_peers;
        a.ep_capacity = ret->capacity;
        a.ep_rank = ret->rank;
    }

    if (decode) {
        GemmMaps gu = bank.dec_gu, dn = bank.dec_dn;
        gu.b = e->map_xperm_dec;
        dn.b = e->map_act_dec;
        a.tile_done = e->d_sync;
        if (fuse_combine) {
            a.comb_w = combine->weights;
            a.comb_out = combine->out;
            a.comb_cnt = e->d_sync + e->max_tiles;
        }
        stage_begin(e, kStageExperts, stream);
        err = launch_moe_decode_layer(gu, dn, a, e->num_sms, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "decode layer launch");
        stage_end(e, kStageExperts, stream);
        e->launches += 3;
        return DEE_OK;
    }
    GemmMaps gm{};
    {
        gm.w0 = bank.w1; gm.w1 = bank.w3; gm.s0 = bank.s1; gm.s1 = bank.s3;
        for (int i = 0; i < 4; ++i) gm.bt[i] = e->map_xperm_t[i];
    }
    a.k_total = H;
    a.m_tiles = I / 64;
    stage_begin(e, kStageGateUp, stream);
    err = launch_moe_gemm(true, gm, a, e->num_sms, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "gate/up GEMM launch");
    stage_end(e, kStageGateUp, stream);

    gm.w0 = bank.w2; gm.w1 = bank.w2; gm.s0 = bank.s2; gm.s1 = bank.s2;
    for (int i = 0; i < 4; ++i) gm.bt[i] = e->map_act_t[i];
    a.k_total = I;
    a.m_tiles = H / 128;
    stage_begin(e, kStageDown, stream);
    err = launch_moe_gemm(false, gm, a, e->num_sms, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "down GEMM launch");
    stage_end(e, kStageDown, stream);
    e->launches += 4;
    return DEE_OK;
}

// The MXFP8 workspaces for `sel` rows (grown like the FP16 ones).
int ensure_mx_capacity(dee_engine* e, size_t sel, cudaStream_t stream) {
    if (sel <= e->cap_mx) return DEE_OK;
    cudaError_t err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "cudaStreamSynchronize(workspace growth)");
    cudaFree(e->d_xq); cudaFree(e->d_xs); cudaFree(e->d_aq); cudaFree(e->d_as);
    e->d_xq = e->d_xs = e->d_aq = e->d_as = nullptr;
    e->cap_mx = 0;
    const size_t cap = ((sel + 255) / 256) * 256;
    const size_t H = e->cfg.hidden, I = e->cfg.inter;
    if ((err = dev_alloc(&e->d_xq, cap * H)) != cudaSuccess || (err = dev_alloc(&e->d_xs, cap * H / 32)) != cudaSuccess ||
        (err = dev_alloc(&e->d_aq, cap * I)) != cudaSuccess || (err = dev_alloc(&e->d_as, cap * I / 32)) != cudaSuccess)
        return cuda_fail(e, err, "MXFP8 workspace allocation");
    if (!encode_mx_token_maps(get_encode_fn(), e->d_xq, static_cast<int>(cap), static_cast<int>(H), e->map_xq_t) ||
        !encode_mx_token_maps(get_encode_fn(), e->d_aq, static_cast<int>(cap), static_cast<int>(I), e->map_aq_t))
        return fail(e, DEE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the MXFP8 token maps");
    e->cap_mx = cap;
    return DEE_OK;
}

// The layer with E4M3 activations (act_block-column UE8M0 blocks, 32 or
// 128) against the records' E2M1 weights: permute, quantise-and-gather the
// token rows, block-scaled gate/up GEMM (SwiGLU into FP16 act), quantise act,
// block-scaled down GEMM into raw.
int run_experts_mx(dee_engine* e, int layer, const __half* d_x, int tokens, const int32_t* d_ids32, float* raw,
                   cudaStream_t stream, int K, int act_block) {
    if (layer < 0 || layer >= static_cast<int>(e->banks.size()) || !e->banks[layer].attached)
        return fail(e, DEE_ERR_NO_BANK, "no expert bank attached for layer " + std::to_string(layer));
    const dee::Bank& bank = e->banks[layer];
    if (!bank.mx) return fail(e, DEE_ERR_UNSUPPORTED, "the MXFP8 weight maps are unavailable on this driver");
    const int H = e->cfg.hidden, I = e->cfg.inter, E = e->cfg.num_experts;
    if (H % 256 || I % 256) return fail(e, DEE_ERR_UNSUPPORTED, "MXFP8 path needs hidden and inter % 256 == 0");
    const size_t sel = static_cast<size_t>(tokens) * K;
    int rc = ensure_mx_capacity(e, sel, stream);
    if (rc != DEE_OK) return rc;
    PermuteOut po{e->d_counts, e->d_offsets, e->d_perm, e->d_row_of, e->d_tiles, e->d_n_tiles, e->d_journal};
    po.chunk_counts = e->d_perm_chunks;
    po.lrank = e->d_perm_lrank;
    po.max_chunks = static_cast<long long>((e->cap_sel + 1023) / 1024);
    po.tile_grp = e->d_tile_grp;
    stage_begin(e, kStagePermute, stream);
    cudaError_t err = launch_permute(d_ids32, tokens, K, E, gemm_n_max(), e->max_tiles, po, e->d_status, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "permute launch");
    e->launches += permute_launch_count(tokens, K, po) - 1;
    stage_end(e, kStagePermute, stream);
    stage_begin(e, kStageGather, stream);
    err = launch_act_quant(d_x, static_cast<int>(sel), H, act_block, e->d_perm, K, e->d_offsets + E, e->d_xq, e->d_xs,
                           stream, true);
    if (err != cudaSuccess) return cuda_fail(e, err, "activation quantisation launch");
    stage_end(e, kStageGather, stream);

    GemmArgs a{};
    a.hidden = H;
    a.inter = I;
    a.topk = K;
    a.swiglu_limit = e->cfg.swiglu_limit;
    a.tiles = e->d_tiles;
    a.n_tiles = e->d_n_tiles;
    a.slot_of = bank.d_slot_of;
    a.num_slots = bank.n_slots;
    a.records = bank.records;
    a.record_bytes = bank.record_bytes;
    a.num_experts = E;
    a.perm = e->d_perm;
    a.act = e->d_act;
    a.raw = raw;
    a.status = e->d_status;
    a.tile_grp = e->d_tile_grp;
    MxMaps m = bank.mx_gu;
    for (int i = 0; i < 4; ++i) m.bt[i] = e->map_xq_t[i];
    a.k_total = H;
    a.m_tiles = I / 64;
    const int cap = static_cast<int>(e->cap_mx);
    stage_begin(e, kStageGateUp, stream);
    err = launch_moe_mxfp8(true, m, a, e->d_xs, cap, e->num_sms, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "MXFP8 gate/up GEMM launch");
    err = launch_act_quant(e->d_act, static_cast<int>(sel), I, act_block, nullptr, 1, e->d_offsets + E, e->d_aq,
                           e->d_as, stream, true);
    if (err != cudaSuccess) return cuda_fail(e, err, "act quantisation launch");
    stage_end(e, kStageGateUp, stream);
    m = bank.mx_dn;
    for (int i = 0; i < 4; ++i) m.bt[i] = e->map_aq_t[i];
    a.k_total = I;
    a.m_tiles = H / 128;
    stage_begin(e, kStageDown, stream);
    err = launch_moe_mxfp8(false, m, a, e->d_as, cap, e->num_sms, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "MXFP8 down GEMM launch");
    stage_end(e, kStageDown, stream);
    e->launches += 5;
    return DEE_OK;
}

}  // namespace
}  // namespace dee

using namespace dee;

extern "C" {

size_t dee_abi_config_size(void) { return sizeof(dee_config); }
int dee_abi_version(void) { return DEE_B200_ABI_VERSION; }

int dee_engine_create(const dee_config* cfg, dee_engine** out) {
    if (!cfg || !out) return DEE_ERR_INVALID;
    *out = nullptr;
    const int H = cfg->hidden, I = cfg->inter;
    if (H <= 0 || I <= 0 || H % 512 != 0 || I % 512 != 0 || cfg->num_experts <= 0 ||
        cfg->num_experts > 256 || cfg->topk <= 0 || cfg->topk > 32 ||
        cfg->topk > cfg->num_experts || cfg->num_layers <= 0)
        return DEE_ERR_UNSUPPORTED;
    auto* e = new dee_engine();
    e->cfg = *cfg;
    if (e->cfg.max_tokens <= 0) e->cfg.max_tokens = 64;
    cudaError_t err = cudaSetDevice(cfg->device_id);
    if (err == cudaSuccess)
        err = cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, cfg->device_id);
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(&e->d_status), 16);
    if (err == cudaSuccess) err = cudaMemset(e->d_status, 0, 16);
    if (err == cudaSuccess)
        err = cudaHostAlloc(reinterpret_cast<void**>(&e->h_status), 16, cudaHostAllocDefault);
    if (err != cudaSuccess) {
        dee_engine_destroy(e);
        return DEE_ERR_CUDA;
    }
    e->banks.resize(static_cast<size_t>(cfg->num_layers));
    const int rc = ensure_capacity(e, static_cast<size_t>(e->cfg.max_tokens) * cfg->topk, e->stream);
    if (rc != DEE_OK) {
        dee_engine_destroy(e);
        return rc;
    }
    *out = e;
    return DEE_OK;
}

void dee_engine_destroy(dee_engine* e) {
    if (!e) return;
    cudaSetDevice(e->cfg.device_id);
    if (e->stream) cudaStreamSynchronize(e->stream);
    free_workspace(e);
    cudaFree(e->d_sh_act);
    cudaFree(e->d_sh_out);
    cudaFree(e->d_front_scratch);
    cudaFree(e->d_front_ctr);
    cudaFree(e->d_xq);
    cudaFree(e->d_xs);
    cudaFree(e->d_aq);
    cudaFree(e->d_as);
    if (e->off.copy_stream) cudaStreamDestroy(e->off.copy_stream);
    if (e->off.copied) cudaEventDestroy(e->off.copied);
    if (e->off.h_ids) cudaFreeHost(e->off.h_ids);
    for (void* p : e->ep.opened) cudaIpcCloseMemHandle(p);
    cudaFree(e->ep.block);
    cudaFree(e->ep.d_back_peers);
    cudaFree(e->ep.d_slot_of_pos);
    for (auto& b : e->banks) cudaFree(b.d_slot_of);
    for (int i = 0; i < kStageCount; ++i) {
        if (e->ev_start[i]) cudaEventDestroy(e->ev_start[i]);
        if (e->ev_end[i]) cudaEventDestroy(e->ev_end[i]);
    }
    cudaFree(e->d_status);
    if (e->h_status) cudaFreeHost(e->h_status);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

const char* dee_last_error(const dee_engine* e) { return e ? e->last_error.c_str() : "null engine"; }

int dee_expert_bank_attach(dee_engine* e, int layer, const void* d_records, int n_slots,
                           size_t record_bytes, const int32_t* h_slot_of_expert) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    if (layer < 0 || layer >= e->cfg.num_layers || !d_records || n_slots <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid bank arguments");
    const int H = e->cfg.hidden, I = e->cfg.inter, E = e->cfg.num_experts;
    const RecordLayout L = record_layout(H, I);
    if (record_bytes < L.bytes || record_bytes % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(d_records) & 15) != 0)
        return fail(e, DEE_ERR_INVALID, "record_bytes must be >= " + std::to_string(L.bytes) +
                                            " and 16-byte aligned");
    std::vector<int32_t> slots(static_cast<size_t>(E));
    for (int i = 0; i < E; ++i) {
        slots[i] = h_slot_of_expert ? h_slot_of_expert[i] : (i < n_slots ? i : -1);
        if (slots[i] >= n_slots) return fail(e, DEE_ERR_INVALID, "slot index beyond n_slots");
    }
    Bank& b = e->banks[layer];
    if (!b.d_slot_of) {
        cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&b.d_slot_of), sizeof(int32_t) * E);
        if (err != cudaSuccess) return cuda_fail(e, err, "slot table allocation");
    }
    cudaError_t err = cudaMemcpy(b.d_slot_of, slots.data(), sizeof(int32_t) * E,
                                 cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return cuda_fail(e, err, "slot table upload");
    const uint8_t* base = static_cast<const uint8_t*>(d_records);
    const cuuint64_t ns = static_cast<cuuint64_t>(n_slots);
    const cuuint64_t rb = static_cast<cuuint64_t>(record_bytes);
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(H / 2), static_cast<cuuint64_t>(I), ns};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(H / 2), rb};
        const cuuint32_t box[3] = {128, 64, 1};
        if (!encode(e, &b.w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.w1, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B, "w1") ||
            !encode(e, &b.w3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.w3, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B, "w3"))
            return DEE_ERR_CUDA;
    }
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(I / 2), static_cast<cuuint64_t>(H), ns};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(I / 2), rb};
        const cuuint32_t box[3] = {128, 128, 1};
        if (!encode(e, &b.w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.w2, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B, "w2"))
            return DEE_ERR_CUDA;
    }
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(H / 32), static_cast<cuuint64_t>(I), ns};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(H / 32), rb};
        const cuuint32_t box[3] = {16, 64, 1};
        if (!encode(e, &b.s1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.s1, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE, "w1.scale") ||
            !encode(e, &b.s3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.s3, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE, "w3.scale"))
            return DEE_ERR_CUDA;
    }
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(I / 32), static_cast<cuuint64_t>(H), ns};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(I / 32), rb};
        const cuuint32_t box[3] = {16, 128, 1};
        if (!encode(e, &b.s2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base + L.s2, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_NONE, "w2.scale"))
            return DEE_ERR_CUDA;
    }
    if (!encode_decode_weight_maps(get_encode_fn(), base, record_bytes, n_slots, H, I, &b.dec_gu,
                                   &b.dec_dn))
        return fail(e, DEE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the decode weight maps");
    // the MXFP8 path's maps (E2M1 unpacked by the TMA); a driver without
    // that tensor-map type leaves the path unavailable, the rest works
    b.mx = encode_mx_weight_maps(get_encode_fn(), base, record_bytes, n_slots, H, I, &b.mx_gu, &b.mx_dn);
    b.records = base;
    b.n_slots = n_slots;
    b.record_bytes = record_bytes;
    b.attached = true;
    return DEE_OK;
}

int dee_expert_bank_set_slots(dee_engine* e, int layer, const int32_t* h_slot_of_expert,
                              void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (layer < 0 || layer >= e->cfg.num_layers || !e->banks[layer].attached || !h_slot_of_expert)
        return fail(e, DEE_ERR_NO_BANK, "no bank attached for layer");
    Bank& b = e->banks[layer];
    for (int i = 0; i < e->cfg.num_experts; ++i)
        if (h_slot_of_expert[i] >= b.n_slots)
            return fail(e, DEE_ERR_INVALID, "slot index beyond n_slots");
    cudaError_t err = cudaMemcpyAsync(b.d_slot_of, h_slot_of_expert,
                                      sizeof(int32_t) * e->cfg.num_experts, cudaMemcpyHostToDevice,
                                      static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(e, err, "slot table update");
    return DEE_OK;
}

int dee_route_topk_device(dee_engine* e, const float* d_logits, int tokens, int32_t* d_ids,
                          float* d_weights, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_logits || !d_ids || !d_weights || tokens <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid router arguments");
    if ((rc = check_aligned(e, "route_topk_device",
                            {{"d_logits", d_logits, 4}, {"d_ids", d_ids, 4}, {"d_weights", d_weights, 4}})) != DEE_OK)
        return rc;
    stage_begin(e, kStageRoute, static_cast<cudaStream_t>(stream));
    cudaError_t err = launch_route_topk(d_logits, tokens, e->cfg.num_experts, e->cfg.topk, d_ids,
                                        d_weights, e->d_status, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(e, err, "router launch");
    stage_end(e, kStageRoute, static_cast<cudaStream_t>(stream));
    e->launches += 1;
    return DEE_OK;
}

int dee_group_by_expert_device(dee_engine* e, const int32_t* d_ids, int tokens, int topk, int32_t* d_perm,
                               int32_t* d_row_of, int32_t* d_offsets, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_ids || !d_perm || !d_row_of || !d_offsets || tokens <= 0 || topk <= 0 || topk > e->cfg.num_experts)
        return fail(e, DEE_ERR_INVALID, "invalid grouping arguments");
    if ((rc = check_aligned(e, "group_by_expert_device",
                            {{"d_ids", d_ids, 4}, {"d_perm", d_perm, 4}, {"d_row_of", d_row_of, 4},
                             {"d_offsets", d_offsets, 4}})) != DEE_OK)
        return rc;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((rc = ensure_capacity(e, static_cast<size_t>(tokens) * topk, s)) != DEE_OK) return rc;
    PermuteOut po{e->d_counts, d_offsets, d_perm, d_row_of, e->d_tiles, e->d_n_tiles, nullptr};
    po.chunk_counts = e->d_perm_chunks;
    po.lrank = e->d_perm_lrank;
    po.max_chunks = static_cast<long long>((e->cap_sel + 1023) / 1024);
    stage_begin(e, kStagePermute, s);
    cudaError_t err = launch_permute(d_ids, tokens, topk, e->cfg.num_experts, gemm_n_max(), e->max_tiles, po,
                                     e->d_status, s);
    if (err != cudaSuccess) return cuda_fail(e, err, "permute launch");
    stage_end(e, kStagePermute, s);
    e->launches += permute_launch_count(tokens, topk, po);
    return DEE_OK;
}

int dee_route_dsv4_device(dee_engine* e, const float* d_logits, const float* d_bias,
                          const int64_t* d_tid2eid, const int64_t* d_input_ids, int tokens,
                          float route_scale, int32_t* d_ids, float* d_weights, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_logits || !d_ids || !d_weights || tokens <= 0 || (d_tid2eid && !d_input_ids))
        return fail(e, DEE_ERR_INVALID, "invalid DSv4 router arguments");
    if ((rc = check_aligned(e, "route_dsv4_device",
                            {{"d_logits", d_logits, 4}, {"d_bias", d_bias, 4}, {"d_tid2eid", d_tid2eid, 8},
                             {"d_input_ids", d_input_ids, 8}, {"d_ids", d_ids, 4}, {"d_weights", d_weights, 4}})) !=
        DEE_OK)
        return rc;
    stage_begin(e, kStageRoute, static_cast<cudaStream_t>(stream));
    cudaError_t err = launch_route_dsv4(d_logits, d_bias, d_tid2eid, d_input_ids, tokens,
                                        e->cfg.num_experts, e->cfg.topk, route_scale, d_ids,
                                        d_weights, e->d_status, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(e, err, "DSv4 router launch");
    stage_end(e, kStageRoute, static_cast<cudaStream_t>(stream));
    e->launches += 1;
    return DEE_OK;
}

int dee_moe_forward_device(dee_engine* e, int layer, const void* d_x_f16, int tokens,
                           const int32_t* d_ids, const int32_t* h_ids, int topk,
                           const float* d_weights, float* d_out_f32, float* d_raw, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_x_f16 || tokens <= 0 || topk <= 0 || topk > e->cfg.topk || (!d_ids && !h_ids) ||
        (!d_out_f32 && !d_raw) || (d_out_f32 && !d_weights))
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_device arguments");
    if ((rc = check_aligned(e, "moe_forward_device",
                            {{"d_x_f16", d_x_f16, 16}, {"d_ids", d_ids, 4}, {"d_weights", d_weights, 4},
                             {"d_out_f32", d_out_f32, 16}, {"d_raw", d_raw, 16}})) != DEE_OK)
        return rc;
    const size_t sel = static_cast<size_t>(tokens) * topk;
    if (h_ids && !host_ids_valid(e, h_ids, sel)) return DEE_ERR_RANGE;
    if ((rc = ensure_capacity(e, sel, stream)) != DEE_OK) return rc;
    const int32_t* ids32 = d_ids;
    cudaError_t err;
    if (h_ids) {
        std::memcpy(e->h_ids, h_ids, sel * sizeof(int32_t));
        err = cudaMemcpyAsync(e->d_ids, e->h_ids, sel * sizeof(int32_t), cudaMemcpyHostToDevice,
                              stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "ids H2D");
        ids32 = e->d_ids;
    }
    e->h_ids_count = sel;
    if (decode_front_fits(tokens, topk, e->cfg.num_experts) && sel <= static_cast<size_t>(kFrontEngineMaxSel))
        return forward_front(e, layer, d_x_f16, tokens, topk, nullptr, const_cast<int32_t*>(ids32),
                             const_cast<float*>(d_weights), d_out_f32, d_raw, stream);
    float* raw = d_raw ? d_raw : e->d_raw;
    bool combined = false;
    const FusedCombine fc{d_weights, d_out_f32, &combined};
    if ((rc = run_experts(e, layer, static_cast<const __half*>(d_x_f16), tokens, ids32, raw,
                          stream, topk, false, true, nullptr, nullptr, nullptr, nullptr,
                          d_out_f32 ? &fc : nullptr)) != DEE_OK)
        return rc;
    if (d_out_f32 && !combined) {
        stage_begin(e, kStageCombine, stream);
        err = launch_combine_f32(raw, d_weights, tokens, topk, e->cfg.hidden, d_out_f32, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "combine launch");
        stage_end(e, kStageCombine, stream);
        e->launches += 1;
    }
    e->journal_stream = stream;
    return DEE_OK;
}

}  // extern "C"

namespace dee {
namespace {

// A small decode batch's layer in one launch (launch_moe_decode_front):
// grouping, token rows, both projections and the combine, and with d_logits
// the routing too (else d_ids / d_weights are inputs).
int forward_front(dee_engine* e, int layer, const void* d_x_f16, int tokens, int K, const float* d_logits,
                  int32_t* d_ids, float* d_weights, float* d_out_f32, float* d_raw, cudaStream_t stream) {
    if (layer < 0 || layer >= static_cast<int>(e->banks.size()) || !e->banks[layer].attached)
        return fail(e, DEE_ERR_NO_BANK, "no expert bank attached for layer " + std::to_string(layer));
    const dee::Bank& bank = e->banks[layer];
    const int H = e->cfg.hidden;
    cudaError_t err;
    if (!e->d_front_scratch) {
        const size_t n_ctr = kFrontMaxTiles + static_cast<size_t>(kFrontMaxSel) * (H / 128);
        if ((err = dev_alloc(&e->d_front_scratch, static_cast<size_t>(e->num_sms) * kFrontScratchInts)) !=
                cudaSuccess ||
            (err = dev_alloc(&e->d_front_ctr, n_ctr)) != cudaSuccess ||
            (err = cudaMemsetAsync(e->d_front_ctr, 0, n_ctr * sizeof(unsigned long long), stream)) != cudaSuccess) {
            cudaFree(e->d_front_scratch);
            cudaFree(e->d_front_ctr);
            e->d_front_scratch = nullptr;
            e->d_front_ctr = nullptr;
            return cuda_fail(e, err, "decode front-end workspace");
        }
    }
    if (++e->front_epoch == 0) {
        // after 2^32 launches the tags would repeat: start over from zeroed counters
        const size_t n_ctr = kFrontMaxTiles + static_cast<size_t>(kFrontMaxSel) * (H / 128);
        if ((err = cudaMemsetAsync(e->d_front_ctr, 0, n_ctr * sizeof(unsigned long long), stream)) != cudaSuccess)
            return cuda_fail(e, err, "decode front-end counter reset");
        e->front_epoch = 1;
    }
    GemmArgs a{};
    a.hidden = H;
    a.inter = e->cfg.inter;
    a.topk = K;
    a.swiglu_limit = e->cfg.swiglu_limit;
    a.slot_of = bank.d_slot_of;
    a.num_slots = bank.n_slots;
    a.records = bank.records;
    a.record_bytes = bank.record_bytes;
    a.num_experts = e->cfg.num_experts;
    a.act = e->d_act;
    a.raw = d_raw ? d_raw : e->d_raw;
    a.status = e->d_status;
    a.comb_out = d_out_f32;
    DecFront f{};
    f.logits = d_logits;
    f.x = static_cast<const __half*>(d_x_f16);
    f.tokens = tokens;
    f.ids_out = d_ids;
    f.weights_out = d_weights;
    f.journal = e->d_journal;
    f.scratch = e->d_front_scratch;
    f.ctr = e->d_front_ctr;
    f.epoch = e->front_epoch;
    GemmMaps gu = bank.dec_gu, dn = bank.dec_dn;
    dn.b = e->map_act_dec;
    stage_begin(e, kStageExperts, stream);
    err = launch_moe_decode_front(gu, dn, a, f, e->num_sms, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "decode front-end launch");
    stage_end(e, kStageExperts, stream);
    e->launches += 1;
    e->h_ids_count = static_cast<size_t>(tokens) * K;
    e->journal_stream = stream;
    return DEE_OK;
}

}  // namespace
}  // namespace dee

extern "C" {

int dee_moe_forward_routed_device(dee_engine* e, int layer, const void* d_x_f16, int tokens, const float* d_logits,
                                  int32_t* d_ids, float* d_weights, float* d_out_f32, float* d_raw, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_x_f16 || !d_logits || !d_ids || !d_weights || tokens <= 0 || (!d_out_f32 && !d_raw))
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_routed_device arguments");
    if ((rc = check_aligned(e, "moe_forward_routed_device",
                            {{"d_x_f16", d_x_f16, 16}, {"d_logits", d_logits, 4}, {"d_ids", d_ids, 4},
                             {"d_weights", d_weights, 4}, {"d_out_f32", d_out_f32, 16}, {"d_raw", d_raw, 16}})) !=
        DEE_OK)
        return rc;
    const int K = e->cfg.topk;
    const size_t sel = static_cast<size_t>(tokens) * K;
    if ((rc = ensure_capacity(e, sel, stream)) != DEE_OK) return rc;
    if (decode_front_fits(tokens, K, e->cfg.num_experts) && sel <= static_cast<size_t>(kFrontEngineMaxSel))
        return forward_front(e, layer, d_x_f16, tokens, K, d_logits, d_ids, d_weights, d_out_f32, d_raw, stream);
    const bool fuse = route_permute_fits(tokens, K, e->cfg.num_experts);
    if (!fuse && (rc = dee_route_topk_device(e, d_logits, tokens, d_ids, d_weights, stream)) != DEE_OK) return rc;
    e->h_ids_count = sel;
    float* raw = d_raw ? d_raw : e->d_raw;
    const FusedRoute fr{d_logits, d_weights};
    bool combined = false;
    const FusedCombine fc{d_weights, d_out_f32, &combined};
    if ((rc = run_experts(e, layer, static_cast<const __half*>(d_x_f16), tokens, d_ids, raw, stream, K, false, true,
                          nullptr, nullptr, nullptr, fuse ? &fr : nullptr, d_out_f32 ? &fc : nullptr)) != DEE_OK)
        return rc;
    if (d_out_f32 && !combined) {
        stage_begin(e, kStageCombine, stream);
        const cudaError_t err = launch_combine_f32(raw, d_weights, tokens, K, e->cfg.hidden, d_out_f32, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "combine launch");
        stage_end(e, kStageCombine, stream);
        e->launches += 1;
    }
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_moe_forward_mxfp8_device(dee_engine* e, int layer, const void* d_x_f16, int tokens, const int32_t* d_ids,
                                 int topk, const float* d_weights, float* d_out_f32, float* d_raw, int act_block,
                                 void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_x_f16 || tokens <= 0 || topk <= 0 || topk > e->cfg.topk || !d_ids || (!d_out_f32 && !d_raw) ||
        (d_out_f32 && !d_weights) || (act_block != 32 && act_block != 128))
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_mxfp8_device arguments");
    if ((rc = check_aligned(e, "moe_forward_mxfp8_device",
                            {{"d_x_f16", d_x_f16, 16}, {"d_ids", d_ids, 4}, {"d_weights", d_weights, 4},
                             {"d_out_f32", d_out_f32, 16}, {"d_raw", d_raw, 16}})) != DEE_OK)
        return rc;
    const size_t sel = static_cast<size_t>(tokens) * topk;
    if ((rc = ensure_capacity(e, sel, stream)) != DEE_OK) return rc;
    e->h_ids_count = sel;
    float* raw = d_raw ? d_raw : e->d_raw;
    if ((rc = run_experts_mx(e, layer, static_cast<const __half*>(d_x_f16), tokens, d_ids, raw, stream, topk,
                             act_block)) != DEE_OK)
        return rc;
    if (d_out_f32) {
        stage_begin(e, kStageCombine, stream);
        cudaError_t err = launch_combine_f32(raw, d_weights, tokens, topk, e->cfg.hidden, d_out_f32, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "combine launch");
        stage_end(e, kStageCombine, stream);
        e->launches += 1;
    }
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_moe_forward_batch_device(dee_engine* e, int layer, const void* d_h_in, int tokens,
                                 const int32_t* h_expert_ids, int topk, void* d_experts_out) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_h_in || !h_expert_ids || !d_experts_out || tokens <= 0 || topk <= 0 || topk > e->cfg.topk)
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_batch_device arguments");
    cudaError_t err = cudaMemsetAsync(e->d_status, 0, 4, e->stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "status reset");
    rc = dee_moe_forward_device(e, layer, d_h_in, tokens, nullptr, h_expert_ids, topk, nullptr,
                                nullptr, static_cast<float*>(d_experts_out), e->stream);
    if (rc != DEE_OK) return rc;
    uint32_t st = 0;
    return dee_engine_sync_status(e, e->stream, &st);
}

int dee_moe_forward_combined_device(dee_engine* e, int layer, const void* d_h_in, int tokens,
                                    const int64_t* d_expert_ids, int topk,
                                    const float* d_weights_f32, void* d_output_f16,
                                    void* d_raw_trace_out, void* external_stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(external_stream);
    if (!d_h_in || !d_expert_ids || !d_weights_f32 || !d_output_f16 || tokens <= 0 ||
        topk <= 0 || topk > e->cfg.topk)
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_combined_device arguments");
    if ((rc = check_aligned(e, "moe_forward_combined_device",
                            {{"d_h_in", d_h_in, 16}, {"d_expert_ids", d_expert_ids, 8},
                             {"d_weights_f32", d_weights_f32, 4}, {"d_output_f16", d_output_f16, 2},
                             {"d_raw_trace_out", d_raw_trace_out, 16}})) != DEE_OK)
        return rc;
    const size_t sel = static_cast<size_t>(tokens) * topk;
    if ((rc = ensure_capacity(e, sel, stream)) != DEE_OK) return rc;
    cudaError_t err = launch_ids_i64_to_i32(d_expert_ids, static_cast<int>(sel),
                                            e->cfg.num_experts, e->d_ids, e->d_status, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "id conversion launch");
    e->h_ids_count = sel;
    float* raw = d_raw_trace_out ? static_cast<float*>(d_raw_trace_out) : e->d_raw;
    if ((rc = run_experts(e, layer, static_cast<const __half*>(d_h_in), tokens, e->d_ids, raw,
                          stream, topk, false, true)) != DEE_OK)
        return rc;
    stage_begin(e, kStageCombine, stream);
    err = launch_combine_f16(raw, d_weights_f32, d_expert_ids, tokens, topk, e->cfg.hidden,
                             static_cast<__half*>(d_output_f16), stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "FP16 combine launch");
    stage_end(e, kStageCombine, stream);
    e->launches += 2;
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_ep_pack_device(dee_engine* e, const int32_t* d_ids, int tokens, const void* d_x_f16,
                       int ranks, int experts_per_rank, int capacity, void* d_send_rows,
                       int32_t* d_send_expert, int32_t* d_slot_of_pos, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_ids || !d_x_f16 || !d_send_rows || !d_send_expert || !d_slot_of_pos || tokens <= 0 ||
        ranks <= 0 || ranks > kEpMaxRanks || capacity <= 0 || experts_per_rank != e->cfg.num_experts)
        return fail(e, DEE_ERR_INVALID,
                    "invalid ep_pack arguments (ranks 1..32, capacity > 0, experts_per_rank must "
                    "equal the engine's num_experts)");
    if ((rc = check_aligned(e, "ep_pack_device",
                            {{"d_ids", d_ids, 4}, {"d_x_f16", d_x_f16, 16}, {"d_send_rows", d_send_rows, 16},
                             {"d_send_expert", d_send_expert, 4}, {"d_slot_of_pos", d_slot_of_pos, 4}})) != DEE_OK)
        return rc;
    const size_t sel = static_cast<size_t>(tokens) * e->cfg.topk;
    // room for the rows this engine receives next (ranks x capacity), so the
    // rows forward does not regrow the workspace and drop the journal
    const size_t recv = static_cast<size_t>(ranks) * capacity;
    if ((rc = ensure_capacity(e, sel > recv ? sel : recv, stream)) != DEE_OK) return rc;
    stage_begin(e, kStageDispatch, stream);
    cudaError_t err = launch_ep_pack(d_ids, static_cast<const __half*>(d_x_f16), tokens, e->cfg.topk,
                                     e->cfg.hidden, ranks, experts_per_rank, capacity,
                                     static_cast<__half*>(d_send_rows), d_send_expert, d_slot_of_pos,
                                     e->d_journal, e->d_status, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep pack launch");
    stage_end(e, kStageDispatch, stream);
    e->launches += 2;
    e->h_ids_count = sel;
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_moe_forward_rows_device(dee_engine* e, int layer, const void* d_rows_f16,
                                const int32_t* d_expert, int rows, float* d_raw, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_rows_f16 || !d_expert || !d_raw || rows <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_rows_device arguments");
    if ((rc = check_aligned(e, "moe_forward_rows_device",
                            {{"d_rows_f16", d_rows_f16, 16}, {"d_expert", d_expert, 4}, {"d_raw", d_raw, 16}})) !=
        DEE_OK)
        return rc;
    if ((rc = ensure_capacity(e, static_cast<size_t>(rows), stream)) != DEE_OK) return rc;
    return run_experts(e, layer, static_cast<const __half*>(d_rows_f16), rows, d_expert, d_raw, stream,
                       1, true, false);
}

int dee_ep_combine_device(dee_engine* e, const float* d_back, const int32_t* d_slot_of_pos,
                          const float* d_weights, int tokens, float* d_out, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    if (!d_back || !d_slot_of_pos || !d_weights || !d_out || tokens <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid ep_combine arguments");
    if ((rc = check_aligned(e, "ep_combine_device",
                            {{"d_back", d_back, 16}, {"d_slot_of_pos", d_slot_of_pos, 4},
                             {"d_weights", d_weights, 4}, {"d_out", d_out, 16}})) != DEE_OK)
        return rc;
    const auto stream = static_cast<cudaStream_t>(stream_v);
    stage_begin(e, kStageCombine, stream);
    cudaError_t err = launch_ep_combine(d_back, d_slot_of_pos, d_weights, tokens, e->cfg.topk,
                                        e->cfg.hidden, d_out, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep combine launch");
    stage_end(e, kStageCombine, stream);
    e->launches += 1;
    return DEE_OK;
}

int dee_shared_expert_attach(dee_engine* e, int layer, const void* d_w1, const void* d_w1_scale,
                             const void* d_w3, const void* d_w3_scale, const void* d_w2,
                             const void* d_w2_scale, int inter_shared) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    const int H = e->cfg.hidden;
    if (layer < 0 || layer >= e->cfg.num_layers || !d_w1 || !d_w3 || !d_w2 || !d_w1_scale ||
        !d_w3_scale || !d_w2_scale || inter_shared <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid shared-expert arguments");
    if (inter_shared % 256 != 0 || H % 256 != 0)
        return fail(e, DEE_ERR_UNSUPPORTED, "shared expert needs hidden and inter multiples of 256");
    for (const void* p : {d_w1, d_w3, d_w2})
        if (reinterpret_cast<uintptr_t>(p) & 15)
            return fail(e, DEE_ERR_INVALID, "shared-expert weights must be 16-byte aligned");
    Bank& b = e->banks[layer];
    if (!encode_shared_weight_maps(get_encode_fn(), d_w1, d_w3, d_w2, H, inter_shared, &b.sh_m1, &b.sh_m3,
                                   &b.sh_m2))
        return fail(e, DEE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the shared expert");
    b.sh_s1 = static_cast<const uint8_t*>(d_w1_scale);
    b.sh_s3 = static_cast<const uint8_t*>(d_w3_scale);
    b.sh_s2 = static_cast<const uint8_t*>(d_w2_scale);
    b.shared_inter = inter_shared;
    b.shared = true;
    return DEE_OK;
}

int dee_moe_forward_official_device(dee_engine* e, int layer, const void* d_x_f16, int tokens,
                                    const int32_t* d_ids, const float* d_weights, float* d_out_f32,
                                    float* d_shared_out, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!d_x_f16 || tokens <= 0 || !d_ids || !d_weights || !d_out_f32)
        return fail(e, DEE_ERR_INVALID, "invalid moe_forward_official_device arguments");
    if ((rc = check_aligned(e, "moe_forward_official_device",
                            {{"d_x_f16", d_x_f16, 16}, {"d_ids", d_ids, 4}, {"d_weights", d_weights, 4},
                             {"d_out_f32", d_out_f32, 16}, {"d_shared_out", d_shared_out, 16}})) != DEE_OK)
        return rc;
    if (layer < 0 || layer >= static_cast<int>(e->banks.size()) || !e->banks[layer].attached)
        return fail(e, DEE_ERR_NO_BANK, "no expert bank attached for layer " + std::to_string(layer));
    const int K = e->cfg.topk, H = e->cfg.hidden;
    const size_t sel = static_cast<size_t>(tokens) * K;
    if ((rc = ensure_capacity(e, sel, stream)) != DEE_OK) return rc;
    e->h_ids_count = sel;
    if ((rc = run_experts(e, layer, static_cast<const __half*>(d_x_f16), tokens, d_ids, e->d_raw, stream, K,
                          false, true, nullptr, d_weights)) != DEE_OK)
        return rc;
    const Bank& b = e->banks[layer];
    float* shared_out = nullptr;
    if (b.shared) {
        const int Is = b.shared_inter;
        if (static_cast<size_t>(tokens) > e->cap_sh || Is > e->cap_sh_inter) {
            cudaError_t err = cudaStreamSynchronize(stream);
            cudaFree(e->d_sh_act);
            cudaFree(e->d_sh_out);
            e->d_sh_act = nullptr;
            e->d_sh_out = nullptr;
            e->cap_sh = 0;
            const size_t cap = ((static_cast<size_t>(tokens) + 63) / 64) * 64;
            const int ci = Is > e->cap_sh_inter ? Is : e->cap_sh_inter;
            if (err == cudaSuccess) err = dev_alloc(&e->d_sh_act, cap * ci);
            if (err == cudaSuccess) err = dev_alloc(&e->d_sh_out, cap * H);
            if (err != cudaSuccess) return cuda_fail(e, err, "shared-expert workspace");
            e->cap_sh = cap;
            e->cap_sh_inter = ci;
        }
        CUtensorMap map_x, map_act;
        if (!encode_decode_token_map(get_encode_fn(), d_x_f16, tokens, H, &map_x, 4) ||
            !encode_decode_token_map(get_encode_fn(), e->d_sh_act, tokens, Is, &map_act, 4))
            return fail(e, DEE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the shared-expert tokens");
        shared_out = d_shared_out ? d_shared_out : e->d_sh_out;
        cudaError_t err = launch_shared_expert(b.sh_m1, b.sh_m3, b.sh_m2, map_x, map_act, b.sh_s1, b.sh_s3,
                                               b.sh_s2, tokens, H, Is, e->cfg.swiglu_limit, e->d_sh_act,
                                               shared_out, e->d_status, e->num_sms, stream);
        if (err != cudaSuccess) return cuda_fail(e, err, "shared-expert launch");
        e->launches += 2;
    }
    cudaError_t err = launch_combine_sum(e->d_raw, shared_out, tokens, K, H, d_out_f32, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "official combine launch");
    e->launches += 1;
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_ep_p2p_init(dee_engine* e, int ranks, int rank, int tokens, void* ipc_handle_out,
                    uint64_t* block_out) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    if (ranks <= 0 || ranks > kEpMaxRanks || rank < 0 || rank >= ranks || tokens <= 0 ||
        !ipc_handle_out || e->ep.block)
        return fail(e, DEE_ERR_INVALID, "invalid ep_p2p_init arguments (or already initialised)");
    EpP2P& p = e->ep;
    const size_t H = static_cast<size_t>(e->cfg.hidden);
    const int cap = tokens * e->cfg.topk;
    const size_t n = static_cast<size_t>(ranks) * cap;
    auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
    p.off_recv_rows = 0;
    p.off_recv_expert = up(p.off_recv_rows + n * H * 2);
    p.off_recv_flag = up(p.off_recv_expert + n * 4);
    p.off_back_rows = up(p.off_recv_flag + static_cast<size_t>(ranks) * 4);
    p.off_back_flag = up(p.off_back_rows + n * H * 4);
    p.bytes = up(p.off_back_flag + static_cast<size_t>(ranks) * 4);
    cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&p.block), p.bytes);
    if (err == cudaSuccess) err = cudaMemset(p.block, 0, p.bytes);  // flags start below epoch 1
    const size_t sop_bytes = up(sizeof(int32_t) * cap);
    if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(&p.d_slot_of_pos), sop_bytes + 256);
    if (err == cudaSuccess) {
        p.d_done = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.d_slot_of_pos) + sop_bytes);
        err = cudaMemset(p.d_done, 0, 256);
    }
    if (err == cudaSuccess)
        err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle_out), p.block);
    if (err != cudaSuccess) {
        cudaFree(p.block);
        cudaFree(p.d_slot_of_pos);
        p = EpP2P{};
        return cuda_fail(e, err, "ep_p2p_init");
    }
    p.ranks = ranks;
    p.rank = rank;
    p.tokens = tokens;
    p.capacity = cap;
    if (block_out) *block_out = reinterpret_cast<uint64_t>(p.block);
    return DEE_OK;
}

int dee_ep_p2p_connect(dee_engine* e, const void* ipc_handles, const uint64_t* blocks) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    EpP2P& p = e->ep;
    if (!p.block || p.connected || (!ipc_handles && !blocks))
        return fail(e, DEE_ERR_INVALID, "ep_p2p_connect needs ep_p2p_init first and handles or blocks");
    for (int d = 0; d < p.ranks; ++d) {
        uint8_t* base = nullptr;
        if (d == p.rank) {
            base = p.block;
        } else if (blocks && blocks[d]) {
            base = reinterpret_cast<uint8_t*>(blocks[d]);  // same process, same device
        } else {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(ipc_handles) + sizeof(h) * d, sizeof(h));
            void* q = nullptr;
            cudaError_t err = cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess);
            if (err != cudaSuccess)
                return cuda_fail(e, err, ("cudaIpcOpenMemHandle (peer " + std::to_string(d) + ")").c_str());
            p.opened.push_back(q);
            base = static_cast<uint8_t*>(q);
        }
        p.peers.recv_rows[d] = reinterpret_cast<__half*>(base + p.off_recv_rows);
        p.peers.recv_expert[d] = reinterpret_cast<int32_t*>(base + p.off_recv_expert);
        p.peers.recv_flag[d] = reinterpret_cast<uint32_t*>(base + p.off_recv_flag);
        p.peers.back_rows[d] = reinterpret_cast<float*>(base + p.off_back_rows);
        p.peers.back_flag[d] = reinterpret_cast<uint32_t*>(base + p.off_back_flag);
    }
    cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&p.d_back_peers), sizeof(float*) * p.ranks);
    if (err == cudaSuccess)
        err = cudaMemcpy(p.d_back_peers, p.peers.back_rows, sizeof(float*) * p.ranks,
                         cudaMemcpyHostToDevice);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep_p2p_connect");
    p.connected = true;
    return DEE_OK;
}

int dee_ep_p2p_dispatch_device(dee_engine* e, const void* d_x_f16, const int32_t* d_ids, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    EpP2P& p = e->ep;
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!p.connected || !d_x_f16 || !d_ids)
        return fail(e, DEE_ERR_INVALID, "ep_p2p_dispatch needs a connected engine, x and ids");
    if ((rc = check_aligned(e, "ep_p2p_dispatch_device", {{"d_x_f16", d_x_f16, 16}, {"d_ids", d_ids, 4}})) !=
        DEE_OK)
        return rc;
    const size_t sel = static_cast<size_t>(p.tokens) * e->cfg.topk;
    const size_t recv = static_cast<size_t>(p.ranks) * p.capacity;
    if ((rc = ensure_capacity(e, sel > recv ? sel : recv, stream)) != DEE_OK) return rc;
    ++p.epoch;
    stage_begin(e, kStageDispatch, stream);
    cudaError_t err = launch_ep_peer_dispatch(d_ids, static_cast<const __half*>(d_x_f16), p.tokens,
                                              e->cfg.topk, e->cfg.hidden, p.ranks, p.rank,
                                              e->cfg.num_experts, p.capacity, p.peers, p.d_slot_of_pos,
                                              e->d_journal, e->d_status, p.d_done, p.epoch, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep peer dispatch launch");
    stage_end(e, kStageDispatch, stream);
    e->launches += 2;
    e->h_ids_count = sel;
    e->journal_stream = stream;
    return DEE_OK;
}

int dee_ep_p2p_experts_device(dee_engine* e, int layer, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    EpP2P& p = e->ep;
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!p.connected || p.epoch == 0)
        return fail(e, DEE_ERR_INVALID, "ep_p2p_experts before any dispatch");
    // the permutation waits (bounded) for every sender's dispatch flag
    const EpReturn ret{p.d_back_peers, p.capacity, p.rank};
    const EpWait wait{p.peers.recv_flag[p.rank], p.ranks, p.epoch, e->wait_limit_ns};
    if ((rc = run_experts(e, layer, p.peers.recv_rows[p.rank], p.ranks * p.capacity,
                          p.peers.recv_expert[p.rank], e->d_raw, stream, 1, true, false, &ret, nullptr,
                          &wait)) != DEE_OK)
        return rc;
    cudaError_t err = launch_ep_signal(p.peers, true, p.ranks, p.rank, p.epoch, stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep signal launch");
    e->launches += 1;
    return DEE_OK;
}

int dee_ep_p2p_combine_device(dee_engine* e, const float* d_weights, float* d_out_f32, void* stream_v) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    EpP2P& p = e->ep;
    auto stream = static_cast<cudaStream_t>(stream_v);
    if (!p.connected || p.epoch == 0 || !d_weights || !d_out_f32)
        return fail(e, DEE_ERR_INVALID, "ep_p2p_combine needs a dispatched layer, weights and out");
    if ((rc = check_aligned(e, "ep_p2p_combine_device", {{"d_weights", d_weights, 4}, {"d_out_f32", d_out_f32, 16}})) !=
        DEE_OK)
        return rc;
    // every combine CTA waits (bounded) for every owner's return flag
    stage_begin(e, kStageCombine, stream);
    const cudaError_t err = launch_ep_combine(p.peers.back_rows[p.rank], p.d_slot_of_pos, d_weights, p.tokens,
                                              e->cfg.topk, e->cfg.hidden, d_out_f32, stream,
                                              p.peers.back_flag[p.rank], p.ranks, p.epoch, e->d_status,
                                              e->wait_limit_ns);
    if (err != cudaSuccess) return cuda_fail(e, err, "ep combine launch");
    stage_end(e, kStageCombine, stream);
    e->launches += 1;
    return DEE_OK;
}

int dee_ep_p2p_forward_device(dee_engine* e, int layer, const void* d_x_f16, const int32_t* d_ids,
                              const float* d_weights, float* d_out_f32, void* stream) {
    int rc = dee_ep_p2p_dispatch_device(e, d_x_f16, d_ids, stream);
    if (rc == DEE_OK) rc = dee_ep_p2p_experts_device(e, layer, stream);
    if (rc == DEE_OK) rc = dee_ep_p2p_combine_device(e, d_weights, d_out_f32, stream);
    return rc;
}

int dee_offload_attach(dee_engine* e, const void* h_records, size_t record_bytes, int layers,
                       void* d_pool, int pool_slots) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    e->last_error.clear();
    Offload& o = e->off;
    const int E = e->cfg.num_experts;
    if (!h_records || !d_pool || layers <= 0 || layers > e->cfg.num_layers || pool_slots <= 0 || o.on)
        return fail(e, DEE_ERR_INVALID, "invalid offload_attach arguments (or already attached)");
    o.host = static_cast<const uint8_t*>(h_records);
    o.record_bytes = record_bytes;
    o.layers = layers;
    o.experts = E;
    o.pool = static_cast<uint8_t*>(d_pool);
    o.pool_slots = pool_slots;
    o.slot_key.assign(static_cast<size_t>(pool_slots), -1);
    o.used_visit.assign(static_cast<size_t>(pool_slots), 0);
    o.slot_of.assign(static_cast<size_t>(layers) * E, -1);
    o.visits.assign(static_cast<size_t>(layers), 0);
    cudaError_t err = cudaStreamCreateWithFlags(&o.copy_stream, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&o.copied, cudaEventDisableTiming);
    if (err != cudaSuccess) return cuda_fail(e, err, "offload streams");
    for (int l = 0; l < layers; ++l) {
        std::vector<int32_t> none(static_cast<size_t>(E), -1);
        if ((rc = dee_expert_bank_attach(e, l, d_pool, pool_slots, record_bytes, none.data())) != DEE_OK)
            return rc;
    }
    o.on = true;
    return DEE_OK;
}

int dee_offload_prepare_device(dee_engine* e, int layer, const int32_t* d_ids, int tokens, void* stream_v,
                               int* cold_out) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    Offload& o = e->off;
    auto stream = static_cast<cudaStream_t>(stream_v);
    const int E = o.experts, K = e->cfg.topk;
    if (!o.on || layer < 0 || layer >= o.layers || !d_ids || tokens <= 0)
        return fail(e, DEE_ERR_INVALID, "offload_prepare needs an attached offload tier and a layer's ids");
    if ((rc = check_aligned(e, "offload_prepare_device", {{"d_ids", d_ids, 4}})) != DEE_OK) return rc;
    const size_t sel = static_cast<size_t>(tokens) * K;
    if (sel > o.h_ids_cap) {
        if (o.h_ids) cudaFreeHost(o.h_ids);
        o.h_ids = nullptr;
        cudaError_t err = cudaHostAlloc(reinterpret_cast<void**>(&o.h_ids), sel * sizeof(int32_t),
                                        cudaHostAllocDefault);
        if (err != cudaSuccess) return cuda_fail(e, err, "offload ids staging");
        o.h_ids_cap = sel;
    }
    // The ids, and with them everything queued before on `stream`: once this
    // returns, no earlier kernel still reads a slot that is about to be refilled.
    cudaError_t err = cudaMemcpyAsync(o.h_ids, d_ids, sel * sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "offload ids readback");
    o.current = layer;
    const uint32_t visit = ++o.visits[layer];
    std::vector<int> need;
    for (size_t i = 0; i < sel; ++i) {
        const int ex = o.h_ids[i];
        if (ex < 0 || ex >= E) return fail(e, DEE_ERR_RANGE, "offload_prepare: expert id out of range");
        if (std::find(need.begin(), need.end(), ex) == need.end()) need.push_back(ex);
    }
    const uint32_t stamp = ++o.calls;  // "used by this layer call"
    std::vector<int> miss;
    for (int ex : need) {
        const int64_t key = static_cast<int64_t>(layer) * E + ex;
        o.on_use(key);
        ++o.lookups;
        const int32_t slot = o.slot_of[static_cast<size_t>(key)];
        if (slot >= 0) {
            ++o.hits;
            o.used_visit[static_cast<size_t>(slot)] = stamp;
        } else {
            miss.push_back(ex);
        }
    }
    // slots for the misses: free ones first, then the residents with the
    // largest expected next use (never one this layer call uses)
    std::vector<int> take;
    std::vector<std::pair<double, int>> cand;
    for (int s2 = 0; s2 < o.pool_slots && take.size() < miss.size(); ++s2)
        if (o.slot_key[static_cast<size_t>(s2)] < 0) take.push_back(s2);
    if (take.size() < miss.size()) {
        for (int s2 = 0; s2 < o.pool_slots; ++s2) {
            const int64_t k2 = o.slot_key[static_cast<size_t>(s2)];
            if (k2 < 0 || o.used_visit[static_cast<size_t>(s2)] == stamp) continue;
            cand.emplace_back(o.victim_rank(k2), s2);
        }
        const size_t want = miss.size() - take.size();
        if (cand.size() < want) return fail(e, DEE_ERR_INVALID, "offload pool smaller than one layer's experts");
        std::nth_element(cand.begin(), cand.begin() + (want - 1), cand.end(),
                         [](const auto& a, const auto& b) { return a.first > b.first; });
        for (size_t i = 0; i < want; ++i) take.push_back(cand[i].second);
    }
    int cold = 0;
    int failed_expert = -1;
    for (size_t i = 0; i < miss.size(); ++i) {
        const int64_t key = static_cast<int64_t>(layer) * E + miss[i];
        const int victim = take[i];
        const int64_t old = o.slot_key[static_cast<size_t>(victim)];
        if (old >= 0) o.slot_of[static_cast<size_t>(old)] = -1;
        o.slot_key[static_cast<size_t>(victim)] = key;
        o.slot_of[static_cast<size_t>(key)] = victim;
        o.used_visit[static_cast<size_t>(victim)] = stamp;
        err = cudaSuccess;
        if (o.fail_next_copy) {
            o.fail_next_copy = false;
            err = cudaErrorLaunchFailure;  // as if the copy could not be queued
        } else {
            err = cudaMemcpyAsync(o.pool + static_cast<size_t>(victim) * o.record_bytes,
                                  o.host + static_cast<size_t>(key) * o.record_bytes, o.record_bytes,
                                  cudaMemcpyHostToDevice, o.copy_stream);
        }
        if (err != cudaSuccess) {
            // the slot holds no valid record: invalidate it so no later lookup
            // can hit it (a later call for the expert cold-loads again), and
            // report the failure once this layer's table is consistent
            o.slot_key[static_cast<size_t>(victim)] = -1;
            o.slot_of[static_cast<size_t>(key)] = -1;
            ++o.submit_failures;
            if (failed_expert < 0) failed_expert = miss[i];
            continue;
        }
        ++cold;
        o.bytes += o.record_bytes;
    }
    o.cold += static_cast<uint64_t>(cold);
    // this layer's slot table, after its records, then the compute stream waits
    Bank& b = e->banks[layer];
    err = cudaMemcpyAsync(b.d_slot_of, o.slot_of.data() + static_cast<size_t>(layer) * E, sizeof(int32_t) * E,
                          cudaMemcpyHostToDevice, o.copy_stream);
    if (err == cudaSuccess) err = cudaEventRecord(o.copied, o.copy_stream);
    if (err == cudaSuccess) err = cudaStreamWaitEvent(stream, o.copied, 0);
    if (err != cudaSuccess) return cuda_fail(e, err, "offload slot table");
    if (cold_out) *cold_out = cold;
    if (failed_expert >= 0)
        return fail(e, DEE_ERR_CUDA, "offload H2D copy of layer " + std::to_string(layer) + " expert " +
                                         std::to_string(failed_expert) +
                                         " could not be queued; the expert is not resident");
    return DEE_OK;
}

int dee_offload_debug_fail_next_copy(dee_engine* e) {
    if (!e || !e->off.on) return DEE_ERR_INVALID;
    e->off.fail_next_copy = true;
    return DEE_OK;
}

int dee_host_alloc_pinned(size_t bytes, void** out) {
    if (!out || bytes == 0) return DEE_ERR_INVALID;
    return cudaHostAlloc(out, bytes, cudaHostAllocDefault) == cudaSuccess ? DEE_OK : DEE_ERR_CUDA;
}

int dee_host_free_pinned(void* p) { return cudaFreeHost(p) == cudaSuccess ? DEE_OK : DEE_ERR_CUDA; }

int dee_offload_stats(dee_engine* e, uint64_t* out4) {
    if (!e || !out4) return DEE_ERR_INVALID;
    out4[0] = e->off.lookups;
    out4[1] = e->off.hits;
    out4[2] = e->off.cold;
    out4[3] = e->off.bytes;
    return DEE_OK;
}

int dee_stack_embed_device(dee_engine* e, const void* d_table_f16, const int32_t* d_ids, int tokens,
                           int vocab, float* d_x, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_table_f16 || !d_ids || !d_x || tokens <= 0 || vocab <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid stack_embed arguments");
    cudaError_t err = launch_stack_embed(static_cast<const __half*>(d_table_f16), d_ids, tokens, e->cfg.hidden,
                                         vocab, d_x, e->d_status, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : cuda_fail(e, err, "stack_embed launch");
}

int dee_stack_rmsnorm_device(dee_engine* e, const float* d_x, const float* d_w, float eps, int tokens,
                             void* d_y_f16, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_x || !d_w || !d_y_f16 || tokens <= 0) return fail(e, DEE_ERR_INVALID, "invalid stack_rmsnorm arguments");
    cudaError_t err = launch_stack_rmsnorm(d_x, d_w, eps, tokens, e->cfg.hidden, static_cast<__half*>(d_y_f16),
                                           static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : cuda_fail(e, err, "stack_rmsnorm launch");
}

int dee_stack_router_logits_device(dee_engine* e, const void* d_h_f16, const float* d_wr, int tokens,
                                   int experts, float* d_logits, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_h_f16 || !d_wr || !d_logits || tokens <= 0 || experts <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid stack_router_logits arguments");
    cudaError_t err = launch_stack_rowdot_f32(static_cast<const __half*>(d_h_f16), d_wr, tokens, e->cfg.hidden,
                                              experts, d_logits, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : cuda_fail(e, err, "stack_router_logits launch");
}

int dee_stack_residual_add_device(dee_engine* e, float* d_x, const float* d_y, int tokens, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_x || !d_y || tokens <= 0) return fail(e, DEE_ERR_INVALID, "invalid stack_residual_add arguments");
    cudaError_t err = launch_stack_residual_add(d_x, d_y, static_cast<size_t>(tokens) * e->cfg.hidden,
                                                static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : cuda_fail(e, err, "stack_residual_add launch");
}

int dee_stack_lm_head_argmax_device(dee_engine* e, const void* d_h_f16, const void* d_w_f16, int tokens,
                                    int vocab, float* d_logits, int32_t* d_ids_out, void* stream) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!d_h_f16 || !d_w_f16 || !d_logits || !d_ids_out || tokens <= 0 || vocab <= 0)
        return fail(e, DEE_ERR_INVALID, "invalid stack_lm_head_argmax arguments");
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t err = launch_stack_rowdot_f16(static_cast<const __half*>(d_h_f16),
                                              static_cast<const __half*>(d_w_f16), tokens, e->cfg.hidden, vocab,
                                              d_logits, s);
    if (err == cudaSuccess) err = launch_stack_argmax(d_logits, tokens, vocab, d_ids_out, s);
    return err == cudaSuccess ? DEE_OK : cuda_fail(e, err, "stack_lm_head_argmax launch");
}

int dee_records_scramble_device(const void* d_src, void* d_dst, int records, size_t record_bytes,
                                size_t packed_bytes, uint64_t seed, int first_record, void* stream) {
    if (!d_src || !d_dst || records <= 0 || packed_bytes > record_bytes) return DEE_ERR_INVALID;
    cudaError_t err = launch_records_scramble(static_cast<const uint8_t*>(d_src), static_cast<uint8_t*>(d_dst),
                                              records, record_bytes, packed_bytes, seed, first_record,
                                              static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : DEE_ERR_CUDA;
}

int dee_engine_set_wait_limit_ns(dee_engine* e, uint64_t limit_ns) {
    if (!e) return DEE_ERR_INVALID;
    if (limit_ns < kMinWaitLimitNs || limit_ns > sm100::kWaitLimitNs)
        return fail(e, DEE_ERR_INVALID, "wait limit must lie in [100 us, 2 s]");
    e->wait_limit_ns = limit_ns;
    return DEE_OK;
}

int dee_wait_selftest(uint64_t limit_ns, uint32_t* d_status, void* stream) {
    if (!d_status || (reinterpret_cast<uintptr_t>(d_status) & 3) != 0 || limit_ns < kMinWaitLimitNs ||
        limit_ns > sm100::kWaitLimitNs)
        return DEE_ERR_INVALID;
    const cudaError_t err =
        launch_wait_selftest(limit_ns, d_status, sm100::kStatusTimeoutTma, static_cast<cudaStream_t>(stream));
    return err == cudaSuccess ? DEE_OK : DEE_ERR_CUDA;
}

int dee_engine_sync_status(dee_engine* e, void* stream, uint32_t* status_out) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemcpyAsync(e->h_status, e->d_status, 4, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_fail(e, err, "status readback");
    const uint32_t st = *e->h_status;
    if (status_out) *status_out = st;
    if (st != 0) {
        cudaMemsetAsync(e->d_status, 0, 4, s);
        // a launch that gave up may have left the decode front end's counters
        // short of their per-launch totals: start them over
        if (e->d_front_ctr) {
            cudaMemsetAsync(e->d_front_ctr, 0,
                            (kFrontMaxTiles + static_cast<size_t>(kFrontMaxSel) * (e->cfg.hidden / 128)) *
                                sizeof(unsigned long long),
                            s);
            e->front_epoch = 0;
        }
        cudaStreamSynchronize(s);
        char buf[320];
        std::snprintf(buf, sizeof(buf),
                      "device status 0x%08x (bit0-3: pipeline wait timeout, bit4: expert id out "
                      "of range or not resident, bit5: tile overflow, bit6: a peer rank's flag "
                      "did not arrive in time, bit7: router failure)",
                      st);
        e->last_error = buf;
        return DEE_ERR_DEVICE;
    }
    return DEE_OK;
}

// The permutation kernel copies the ids it consumes into d_journal; reading
// them waits for the stream of the latest forward.
int dee_journal_ids_host(dee_engine* e, int32_t* h_out, int max_ids) {
    if (!e || !h_out || max_ids < 0) return DEE_ERR_INVALID;
    const size_t n = e->h_ids_count < static_cast<size_t>(max_ids) ? e->h_ids_count
                                                                   : static_cast<size_t>(max_ids);
    if (n == 0) return 0;
    if (cudaSetDevice(e->cfg.device_id) != cudaSuccess) return DEE_ERR_CUDA;
    cudaError_t err = cudaStreamSynchronize(e->journal_stream);
    if (err == cudaSuccess)
        err = cudaMemcpy(h_out, e->d_journal, n * sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) {
        cuda_fail(e, err, "journal ids readback");
        return DEE_ERR_CUDA;
    }
    return static_cast<int>(n);
}

int dee_fp4_decode_device(const uint8_t* d_packed, const uint8_t* d_scale, void* d_dst_f16,
                          size_t out, size_t in, void* stream) {
    if (!d_packed || !d_scale || !d_dst_f16 || out == 0 || in % 64 != 0) return DEE_ERR_INVALID;
    return launch_fp4_decode(d_packed, d_scale, static_cast<__half*>(d_dst_f16), out, in,
                             static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? DEE_OK
               : DEE_ERR_CUDA;
}

int dee_fp4_quantize_device(const float* d_w, size_t out, size_t in, uint8_t* d_packed,
                            uint8_t* d_scale, void* stream) {
    if (!d_w || !d_packed || !d_scale || out == 0 || in % 32 != 0) return DEE_ERR_INVALID;
    return launch_fp4_quantize(d_w, out, in, d_packed, d_scale,
                               static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? DEE_OK
               : DEE_ERR_CUDA;
}

int dee_act_quant_device(const void* d_x_f16, int rows, int cols, int block, uint8_t* d_q, uint8_t* d_scales,
                         void* stream) {
    if (!d_x_f16 || !d_q || !d_scales || rows < 0 || cols <= 0 || cols % 256 != 0 || (block != 32 && block != 128))
        return DEE_ERR_INVALID;
    return launch_act_quant(static_cast<const __half*>(d_x_f16), rows, cols, block, nullptr, 1, nullptr, d_q,
                            d_scales, static_cast<cudaStream_t>(stream), false) == cudaSuccess
               ? DEE_OK
               : DEE_ERR_CUDA;
}

uint64_t dee_engine_launch_count(const dee_engine* e) { return e ? e->launches : 0; }

int dee_engine_set_profiling(dee_engine* e, int enable) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (enable && !e->ev_start[0]) {
        for (int i = 0; i < kStageCount; ++i) {
            cudaError_t err = cudaEventCreate(&e->ev_start[i]);
            if (err == cudaSuccess) err = cudaEventCreate(&e->ev_end[i]);
            if (err != cudaSuccess) return cuda_fail(e, err, "profiling event creation");
        }
    }
    e->profile = enable != 0;
    for (int i = 0; i < kStageCount; ++i) e->ev_used[i] = false;
    return DEE_OK;
}

int dee_engine_stage_ms(dee_engine* e, float* out_ms, int n) {
    int rc = check_engine(e);
    if (rc != DEE_OK) return rc;
    if (!out_ms || n < 0) return DEE_ERR_INVALID;
    const int m = n < kStageCount ? n : kStageCount;
    for (int i = 0; i < m; ++i) {
        out_ms[i] = -1.0f;
        if (!e->profile || !e->ev_used[i]) continue;
        cudaError_t err = cudaEventSynchronize(e->ev_end[i]);
        if (err == cudaSuccess) err = cudaEventElapsedTime(&out_ms[i], e->ev_start[i], e->ev_end[i]);
        if (err != cudaSuccess) return cuda_fail(e, err, "stage timing readback");
    }
    return m;
}

}  // extern "C"
