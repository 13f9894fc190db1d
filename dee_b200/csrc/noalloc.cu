// noalloc.cu -- the MoE layer forward for callers that cannot allocate
// device memory.
//
// Some callers cannot call cudaMalloc: code running inside an allocator or
// memory-pool callback (allocating there would re-enter the allocator), or a
// host that has handed all device memory to its own caching allocator (a
// second allocator would fail or fragment it).  For them
// dee_moe_forward_noalloc runs the same kernels as dee_moe_forward_device,
// but every scratch buffer (grouped row tables, the tile list, the gathered
// token rows, the SwiGLU activations and the raw per-selection rows) lives in
// one statically sized device array defined in this file.  The call itself
// allocates nothing.
//
// Limits and sharing:
//   * kNoAllocScratchBytes (4 MiB) of device memory is reserved on every GPU
//     that loads the library, for the life of the process.  At H=4096,
//     I=2048 that holds 145 token-expert selections (24 tokens at top-6);
//     larger requests are rejected with DEE_ERR_SCRATCH_LIMIT.
//   * All calls share the one array and it keeps the last call's contents;
//     the per-call state that must start at zero (the status word) is
//     cleared on the caller's stream at the start of each call.  Calls whose
//     work overlaps on the GPU (different streams, or different host threads)
//     race on the array and must be serialised by the caller.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current).  Make
//     that first call before any stream capture begins.  The address is kept
//     for the life of the process, so a process that calls cudaDeviceReset
//     must not call this entry point again afterwards (the reset unloads the
//     module that holds the array).
//   * Every argument is checked on the host before any CUDA call: the token
//     rows and the output are read and written with 16-byte vector accesses
//     and must be 16-byte aligned (a column slice of a wider tensor is not),
//     ids, weights and the status word 4-byte aligned.  A request that fails
//     a check returns an error without launching anything.
#include "dee_b200.h"
#include "kernels.h"

#include <cstdio>
#include <mutex>

namespace dee {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;

// The scratch array.  In host code `g_noalloc_scratch` names a host-side
// stand-in, not device memory: the device address comes from
// cudaGetSymbolAddress below and only that address is handed to kernels.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Once per device, with that device current.
cudaError_t scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return cudaSuccess;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct ScratchPlan {
    size_t status, slots, counts, offsets, n_tiles, perm, row_of, tiles, xperm, act, raw, total;
    int max_tiles;
};

ScratchPlan plan(int H, int I, int E, size_t sel) {
    ScratchPlan p{};
    size_t o = 0;
    p.status = o; o = align256(o + 16);
    p.slots = o; o = align256(o + sizeof(int32_t) * E);
    p.counts = o; o = align256(o + sizeof(int32_t) * E);
    p.offsets = o; o = align256(o + sizeof(int32_t) * (E + 1));
    p.n_tiles = o; o = align256(o + sizeof(int32_t));
    p.perm = o; o = align256(o + sizeof(int32_t) * sel);
    p.row_of = o; o = align256(o + sizeof(int32_t) * sel);
    p.max_tiles = E + static_cast<int>(sel / 8) + 1;
    p.tiles = o; o = align256(o + sizeof(TileDesc) * p.max_tiles);
    p.xperm = o; o = align256(o + sel * H * sizeof(__half));
    p.act = o; o = align256(o + sel * I * sizeof(__half));
    p.raw = o; o = align256(o + sel * H * sizeof(float));
    p.total = o;
    return p;
}

__global__ void identity_slots_kernel(int32_t* slots, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) slots[i] = i;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeFn>(p);
    });
    return fn;
}

bool enc(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
         const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz) {
    const EncodeFn fn = encode_fn();
    if (!fn) return false;
    const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
    return fn(m, dt, rank, const_cast<void*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int report(int code, const char* msg) {
    std::fprintf(stderr, "[dee_moe_forward_noalloc] %s\n", msg);
    return code;
}

}  // namespace
}  // namespace dee

using namespace dee;

extern "C" DEE_API int dee_moe_forward_noalloc(const dee_config* cfg, const void* d_records,
                                               size_t record_bytes, int n_slots,
                                               const void* d_x_f16, int tokens,
                                               const int32_t* d_ids, const float* d_weights,
                                               float* d_out_f32, uint32_t* d_status_out,
                                               void* stream_v) {
    if (!cfg || !d_records || !d_x_f16 || !d_ids || !d_weights || !d_out_f32 || tokens <= 0 ||
        n_slots <= 0)
        return report(DEE_ERR_INVALID, "null pointer or empty batch");
    const int H = cfg->hidden, I = cfg->inter, E = cfg->num_experts, K = cfg->topk;
    if (H <= 0 || I <= 0 || H % 512 != 0 || I % 512 != 0 || E <= 0 || E > 256 || K <= 0 ||
        K > 32 || K > E || n_slots < E)
        return report(DEE_ERR_UNSUPPORTED, "unsupported shape (H, I multiples of 512; E <= 256)");
    const size_t ih = static_cast<size_t>(H) * I;
    const size_t need_record = ih + ih / 2 + 3 * (ih / 32);
    if (record_bytes < need_record || record_bytes % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(d_records) & 15) != 0)
        return report(DEE_ERR_INVALID, "record_bytes too small or records not 16-byte aligned");
    // gather_rows_kernel copies token rows and combine_f32_kernel writes the
    // output with 16-byte vectors; ids, weights and the status are 4-byte words.
    if (((reinterpret_cast<uintptr_t>(d_x_f16) | reinterpret_cast<uintptr_t>(d_out_f32)) & 15) != 0)
        return report(DEE_ERR_INVALID, "token rows and output must be 16-byte aligned");
    if (((reinterpret_cast<uintptr_t>(d_ids) | reinterpret_cast<uintptr_t>(d_weights) |
          reinterpret_cast<uintptr_t>(d_status_out)) & 3) != 0)
        return report(DEE_ERR_INVALID, "ids, weights and status must be 4-byte aligned");
    const size_t sel = static_cast<size_t>(tokens) * K;
    const ScratchPlan sp = plan(H, I, E, sel);
    if (sp.total > kNoAllocScratchBytes) {
        char buf[200];
        std::snprintf(buf, sizeof(buf),
                      "request needs %zu bytes of scratch for %zu selections; the static scratch "
                      "holds %zu bytes",
                      sp.total, sel, kNoAllocScratchBytes);
        return report(DEE_ERR_SCRATCH_LIMIT, buf);
    }
    auto stream = static_cast<cudaStream_t>(stream_v);
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return report(DEE_ERR_CUDA, "cudaGetDevice failed");
    void* base_v = nullptr;
    err = scratch_address(dev, &base_v);
    if (err != cudaSuccess) return report(DEE_ERR_CUDA, cudaGetErrorString(err));
    uint8_t* base = static_cast<uint8_t*>(base_v);
    auto* status = reinterpret_cast<uint32_t*>(base + sp.status);
    auto* slots = reinterpret_cast<int32_t*>(base + sp.slots);

    const bool decode = static_cast<size_t>(tokens) * K <= static_cast<size_t>(kDecodeMaxSelections);
    // Tensor maps over the caller's records and the scratch rows (host work).
    const uint8_t* rec = static_cast<const uint8_t*>(d_records);
    const cuuint64_t ns = static_cast<cuuint64_t>(n_slots), rb = record_bytes;
    const size_t s1 = ih + ih / 2, s3 = s1 + ih / 32, s2 = s3 + ih / 32;
    GemmMaps gu{}, dn{};
    bool ok = true;
    {
        const cuuint64_t d[3] = {static_cast<cuuint64_t>(H / 2), static_cast<cuuint64_t>(I), ns};
        const cuuint64_t st[2] = {static_cast<cuuint64_t>(H / 2), rb};
        const cuuint32_t box[3] = {128, 64, 1};
        ok = ok && enc(&gu.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
        ok = ok && enc(&gu.w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec + ih / 2, d, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    }
    {
        const cuuint64_t d[3] = {static_cast<cuuint64_t>(H / 32), static_cast<cuuint64_t>(I), ns};
        const cuuint64_t st[2] = {static_cast<cuuint64_t>(H / 32), rb};
        const cuuint32_t box[3] = {16, 64, 1};
        ok = ok && enc(&gu.s0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec + s1, d, st, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        ok = ok && enc(&gu.s1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec + s3, d, st, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    {
        const cuuint64_t d[3] = {static_cast<cuuint64_t>(I / 2), static_cast<cuuint64_t>(H), ns};
        const cuuint64_t st[2] = {static_cast<cuuint64_t>(I / 2), rb};
        const cuuint32_t box[3] = {128, 128, 1};
        ok = ok && enc(&dn.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec + ih, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
        dn.w1 = dn.w0;
    }
    {
        const cuuint64_t d[3] = {static_cast<cuuint64_t>(I / 32), static_cast<cuuint64_t>(H), ns};
        const cuuint64_t st[2] = {static_cast<cuuint64_t>(I / 32), rb};
        const cuuint32_t box[3] = {16, 128, 1};
        ok = ok && enc(&dn.s0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, rec + s2, d, st, box, CU_TENSOR_MAP_SWIZZLE_NONE);
        dn.s1 = dn.s0;
    }
    {
        const cuuint64_t d[2] = {static_cast<cuuint64_t>(H), sel};
        const cuuint64_t st[1] = {static_cast<cuuint64_t>(H) * 2};
        const cuuint32_t box[2] = {64, decode ? 8u : 16u};
        ok = ok && enc(&gu.b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base + sp.xperm, d, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    }
    {
        const cuuint64_t d[2] = {static_cast<cuuint64_t>(I), sel};
        const cuuint64_t st[1] = {static_cast<cuuint64_t>(I) * 2};
        const cuuint32_t box[2] = {64, decode ? 8u : 16u};
        ok = ok && enc(&dn.b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base + sp.act, d, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (!decode) {
        ok = ok && encode_gemm_token_maps(encode_fn(), base + sp.xperm, static_cast<int>(sel), H, gu.bt);
        ok = ok && encode_gemm_token_maps(encode_fn(), base + sp.act, static_cast<int>(sel), I, dn.bt);
    }
    if (decode) {
        ok = ok && encode_decode_weight_maps(encode_fn(), rec, record_bytes, n_slots, H, I, &gu, &dn);
        ok = ok && encode_decode_token_map(encode_fn(), base + sp.xperm, static_cast<int>(sel), H, &gu.b);
        ok = ok && encode_decode_token_map(encode_fn(), base + sp.act, static_cast<int>(sel), I, &dn.b);
    }
    if (!ok) return report(DEE_ERR_CUDA, "tensor map encoding failed");

    // Per-call state that must start from zero: the status word.
    err = cudaMemsetAsync(status, 0, 4, stream);
    if (err != cudaSuccess) return report(DEE_ERR_CUDA, cudaGetErrorString(err));
    identity_slots_kernel<<<1, 256, 0, stream>>>(slots, E);
    if ((err = cudaGetLastError()) != cudaSuccess) return report(DEE_ERR_CUDA, cudaGetErrorString(err));

    PermuteOut po{reinterpret_cast<int32_t*>(base + sp.counts),
                  reinterpret_cast<int32_t*>(base + sp.offsets),
                  reinterpret_cast<int32_t*>(base + sp.perm),
                  reinterpret_cast<int32_t*>(base + sp.row_of),
                  reinterpret_cast<TileDesc*>(base + sp.tiles),
                  reinterpret_cast<int32_t*>(base + sp.n_tiles),
                  nullptr};
    err = launch_permute(d_ids, tokens, K, E, decode ? kDecodeTileRows : gemm_n_max(),
                         sp.max_tiles, po, status, stream);
    if (err == cudaSuccess)
        err = launch_gather_rows(static_cast<const __half*>(d_x_f16), po.perm, po.offsets + E,
                                 static_cast<int>(sel), K, H,
                                 reinterpret_cast<__half*>(base + sp.xperm), stream);
    if (err != cudaSuccess) return report(DEE_ERR_CUDA, cudaGetErrorString(err));

    int num_sms = 148;
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    GemmArgs a{};
    a.hidden = H;
    a.inter = I;
    a.topk = K;
    a.swiglu_limit = cfg->swiglu_limit;
    a.tiles = po.tiles;
    a.n_tiles = po.n_tiles;
    a.slot_of = slots;
    a.num_slots = n_slots;
    a.records = rec;
    a.record_bytes = record_bytes;
    a.num_experts = E;
    a.perm = po.perm;
    a.act = reinterpret_cast<__half*>(base + sp.act);
    a.raw = reinterpret_cast<float*>(base + sp.raw);
    a.status = status;
    a.k_total = H;
    a.m_tiles = I / 64;
    err = decode ? launch_moe_decode(true, gu, a, num_sms, stream)
                 : launch_moe_gemm(true, gu, a, num_sms, stream);
    if (err == cudaSuccess) {
        a.k_total = I;
        a.m_tiles = H / 128;
        err = decode ? launch_moe_decode(false, dn, a, num_sms, stream)
                     : launch_moe_gemm(false, dn, a, num_sms, stream);
    }
    if (err == cudaSuccess)
        err = launch_combine_f32(a.raw, d_weights, tokens, K, H, d_out_f32, stream);
    if (err == cudaSuccess && d_status_out)
        err = cudaMemcpyAsync(d_status_out, status, 4, cudaMemcpyDeviceToDevice, stream);
    if (err != cudaSuccess) return report(DEE_ERR_CUDA, cudaGetErrorString(err));
    return DEE_OK;
}
