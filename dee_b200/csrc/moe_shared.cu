// moe_shared.cu -- the DeepSeek-V4 shared expert: a dense SwiGLU FFN over
// every token, weights stored F8_E4M3 with F8_E8M0 scales per 128 x 128 tile
// (deepseek_v4_moe_reference.py:35-84: dequantised in FP32, no routing
// weight, the official FP32 chain).
//
// Same shape of kernel as moe_decode.cu: one CTA per SM, a TMA producer warp
// feeding a ring of 256-wide K stages (128 weight rows x 256 B through one
// 4-D copy per projection, and the tile's 8 token rows through one 3-D copy),
// sixteen consumer warps in pairs over the two 128-wide halves of a stage.
// A half is exactly one 128-wide scale block, so each fragment row's scale
// is applied once per stage to the FP32 partial sum (exact: E4M3 values are
// exact in FP16, the scale is a power of two).  Work items are (8-token tile,
// 64 gate + 64 up rows) or (tile, 128 output rows).
#include "decode_common.cuh"
#include "kernels.h"

namespace dee {
namespace {

using namespace sm100;

constexpr int kShConsumerWarps = 16;
constexpr int kShThreads = 32 * (1 + kShConsumerWarps);
constexpr int kShK = 256;                     // K per stage
constexpr int kShWBytes = 32768;              // 128 rows x 256 FP8
constexpr int kShBBytes = 4096;               // 8 token rows x 256 FP16 (4 chunks of 8 x 128 B)
constexpr int kShStageBytes = kShWBytes + kShBBytes;
constexpr int kShStages = 5;
constexpr int kShRedBytes = 2 * 8 * 32 * 4 * 4 + 2 * 2 * 8 * 4;
constexpr int kShSmem = 1024 + kShStages * kShStageBytes + 256 + kShRedBytes;
static_assert(kShSmem <= 232448, "shared memory budget");

struct SharedArgs {
    int tokens, hidden, inter;  // T, H, shared intermediate size
    int k_total, m_tiles;
    float swiglu_limit;
    const uint8_t* scale0;      // E8M0 [ceil(rows/128), ceil(K/128)]: W1 (gate/up) or W2 (down)
    const uint8_t* scale1;      // W3 scales (gate/up)
    __half* act;                // gate/up output [T, inter]
    float* out;                 // down output [T, H]
    uint32_t* status;
};

// Four E4M3 bytes -> two f16x2 (exact: every E4M3 value is a binary16).
__device__ __forceinline__ void cvt_e4m3x4(uint32_t w, uint32_t& o0, uint32_t& o1) {
    asm("{\n\t.reg .b16 lo, hi;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(o0), "=r"(o1)
        : "r"(w));
}

__device__ __forceinline__ uint2 lds_v2u(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

template <bool kGU>
__global__ void __launch_bounds__(kShThreads, 1)
    shared_fp8_kernel(const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1,
                      const __grid_constant__ CUtensorMap map_b, const SharedArgs args) {
    const int n_tiles = (args.tokens + 7) / 8;
    const int n_items = n_tiles * args.m_tiles;
    if (static_cast<int>(blockIdx.x) >= n_items) {
        pdl_wait();
        pdl_trigger();
        return;
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kShStages * kShStageBytes);
    uint64_t* empty = full + kShStages;
    float* red = reinterpret_cast<float*>(smem + kShStages * kShStageBytes + 256);
    int* red_ok = reinterpret_cast<int*>(red + 2 * 8 * 32 * 4);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kShStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kShConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_wait();  // tokens (gate/up) or the gate/up output (down)
    pdl_trigger();
    const int k_stages = args.k_total / kShK;
    uint32_t* status = args.status;

    if (warp == 0) {
        if (lane != 0) return;
        const uint64_t pol_w = policy_evict_last();  // re-read by every token tile
        const uint64_t pol_b = policy_evict_last();
        int st = 0;
        uint32_t ph = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const int tile = item / args.m_tiles, m = item - tile * args.m_tiles;
            for (int s = 0; s < k_stages; ++s) {
                if (!mbar_wait(&empty[st], ph ^ 1, status, kStatusTimeoutTma)) return;
                mbar_arrive_expect_tx(&full[st], kShStageBytes);
                uint8_t* pk = smem + st * kShStageBytes;
                if (kGU) {
                    tma_load_4d(pk, &map_w0, &full[st], 0, m * 64, 2 * s, 0, pol_w);
                    tma_load_4d(pk + 16384, &map_w1, &full[st], 0, m * 64, 2 * s, 0, pol_w);
                } else {
                    tma_load_4d(pk, &map_w0, &full[st], 0, m * 128, 2 * s, 0, pol_w);
                }
                tma_load_3d(pk + kShWBytes, &map_b, &full[st], 0, tile * 8, 4 * s, pol_b);
                if (++st == kShStages) { st = 0; ph ^= 1; }
            }
        }
        return;
    }

    // consumers: as in moe_decode.cu, thread q owns K 8q..8q+7 of every
    // 32-wide block (one 8-byte load per fragment row), MMA column n reads
    // token row 4*(n&1) + n/2
    const int cw = (warp - 1) & 7;
    const int kh = (warp - 1) >> 3;
    const int g = lane >> 2;
    const int q = lane & 3;
    const int row_lo = kGU ? (8 * cw + g) : (16 * cw + g);
    constexpr uint32_t kHalf = kGU ? 8192 : 16384;  // bytes of one 128-wide K chunk of a projection
    constexpr uint32_t kHi = kGU ? 16384 : 8 * 128;
    const int brow = ((g & 1) << 2) | (g >> 1);
    const uint32_t w_row = kh * kHalf + row_lo * 128 + (q & 1) * 8;
    const uint32_t b_off0 = kShWBytes + 2 * kh * 1024 + brow * 128 + ((q ^ brow) << 4);
    const uint32_t b_off1 = kShWBytes + 2 * kh * 1024 + brow * 128 + (((4 + q) ^ brow) << 4);
    const int kb_count = (args.k_total + 127) / 128;
    const uint32_t smem_base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    int st = 0, parity = 0;
    uint32_t ph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int tile = item / args.m_tiles, m = item - tile * args.m_tiles;
        // global weight rows of the lo / hi fragment rows and their scale rows
        const int grow_lo = kGU ? m * 64 + 8 * cw + g : m * 128 + 16 * cw + g;
        const uint8_t* sc_lo = args.scale0 + static_cast<size_t>(grow_lo / 128) * kb_count;
        const uint8_t* sc_hi = kGU ? args.scale1 + static_cast<size_t>(grow_lo / 128) * kb_count
                                   : args.scale0 + static_cast<size_t>((grow_lo + 8) / 128) * kb_count;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        bool ok = true;
        for (int s = 0; s < k_stages; ++s) {
            ok = mbar_wait(&full[st], ph, status, kStatusTimeoutDequant);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            const uint32_t sb = smem_base + st * kShStageBytes;
            const uint32_t wb = sb + w_row;
            const float f_lo = e8m0_value(__ldg(sc_lo + 2 * s + kh));
            const float f_hi = e8m0_value(__ldg(sc_hi + 2 * s + kh));
            float t[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t unit = static_cast<uint32_t>(((2 * j + (q >> 1)) ^ g) << 4);
                const uint2 wl = lds_v2u(wb + unit);
                const uint2 wh = lds_v2u(wb + kHi + unit);
                const uint4 bv = lds_v4(sb + ((j & 1) ? b_off1 : b_off0) + (j >> 1) * 1024);
                uint32_t a[8];
                cvt_e4m3x4(wl.x, a[0], a[1]);
                cvt_e4m3x4(wl.y, a[2], a[3]);
                cvt_e4m3x4(wh.x, a[4], a[5]);
                cvt_e4m3x4(wh.y, a[6], a[7]);
                if (j == 0)
                    mma_16816_zero(t, a[0], a[4], a[1], a[5], bv.x, bv.y);
                else
                    mma_16816_acc(t, a[0], a[4], a[1], a[5], bv.x, bv.y);
                mma_16816_acc(t, a[2], a[6], a[3], a[7], bv.z, bv.w);
            }
            c[0] = fmaf(f_lo, t[0], c[0]);
            c[1] = fmaf(f_lo, t[1], c[1]);
            c[2] = fmaf(f_hi, t[2], c[2]);
            c[3] = fmaf(f_hi, t[3], c[3]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            if (++st == kShStages) { st = 0; ph ^= 1; }
        }
        // Pair reduction: the second warp (kh == 1) hands its partial sums to
        // the first through a slot double buffered by item parity.  Both warps
        // wait on the pair's named barrier once per item, so neither runs an
        // item ahead of the other.  (A second warp that only arrived could,
        // when an item has fewer K stages than the ring holds, reach the
        // barrier twice while its partner was in an epilogue, complete a
        // phase on its own and leave the partner's last wait unmatched.)
        // Each warp publishes whether its waits succeeded before the barrier;
        // after it both read the partner's flag and leave together, so no
        // barrier ever waits on a warp that has gone.
        float* rslot = red + ((parity * 8 + cw) * 32 + lane) * 4;
        if (kh == 1) *reinterpret_cast<float4*>(rslot) = make_float4(c[0], c[1], c[2], c[3]);
        if (lane == 0) red_ok[(parity * 2 + kh) * 8 + cw] = ok ? 1 : 0;
        named_bar_sync(1 + cw, 64);
        const bool ok_pair = red_ok[(parity * 2 + (kh ^ 1)) * 8 + cw] != 0;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (kh == 0) o = *reinterpret_cast<const float4*>(rslot);
        parity ^= 1;
        if (!ok || !ok_pair) break;
        if (kh == 1) continue;
        c[0] += o.x;
        c[1] += o.y;
        c[2] += o.z;
        c[3] += o.w;
        const int row0 = tile * 8;
        const int n_rows = min(8, args.tokens - row0);
        const int n0 = q, n1 = 4 + q;  // tokens of MMA columns 2q and 2q+1
        if (kGU) {
            const int feat = m * 64 + 8 * cw + g;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                args.act[static_cast<size_t>(row0 + n) * args.inter + feat] =
                    swiglu_out(c[h], c[2 + h], args.swiglu_limit, true, 1.0f);
            }
        } else {
            const int f_lo = m * 128 + 16 * cw + g;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                float* dst = args.out + static_cast<size_t>(row0 + n) * args.hidden;
                dst[f_lo] = c[h];
                dst[f_lo + 8] = c[2 + h];
            }
        }
    }
}

template <bool kGU>
cudaError_t launch_sh(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& b,
                      const SharedArgs& args, int grid, cudaStream_t stream) {
    auto kern = shared_fp8_kernel<kGU>;
    const cudaError_t e = ensure_smem_attr<shared_fp8_kernel<kGU>>(kShSmem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kShThreads), kShSmem, stream, w0, w1, b, args);
}

}  // namespace

// Weight maps over dense FP8 [rows, K] projections: {128 B, rows, K/128
// chunks, 1} with the chunk stride (128 B) below the row stride; one box
// {128, 64 or 128, 2, 1} is a 256-wide stage.
bool encode_shared_weight_maps(EncodeTiledFn fn, const void* w1, const void* w3, const void* w2, int hidden,
                               int inter, CUtensorMap* m1, CUtensorMap* m3, CUtensorMap* m2) {
    if (!fn) return false;
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    auto enc = [&](CUtensorMap* m, const void* base, int rows, int k, cuuint32_t box_rows) {
        const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(k / 128), 1};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(k), 128,
                                       static_cast<cuuint64_t>(rows) * static_cast<cuuint64_t>(k)};
        const cuuint32_t box[4] = {128, box_rows, 2, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    return enc(m1, w1, inter, hidden, 64) && enc(m3, w3, inter, hidden, 64) && enc(m2, w2, hidden, inter, 128);
}

cudaError_t launch_shared_expert(const CUtensorMap& m1, const CUtensorMap& m3, const CUtensorMap& m2,
                                 const CUtensorMap& map_x, const CUtensorMap& map_act, const uint8_t* s1,
                                 const uint8_t* s3, const uint8_t* s2, int tokens, int hidden, int inter,
                                 float swiglu_limit, __half* act, float* out, uint32_t* status, int grid,
                                 cudaStream_t stream) {
    if (tokens <= 0 || hidden % kShK != 0 || inter % kShK != 0 || inter % 64 != 0 || hidden % 128 != 0)
        return cudaErrorInvalidValue;
    SharedArgs a{};
    a.tokens = tokens;
    a.hidden = hidden;
    a.inter = inter;
    a.swiglu_limit = swiglu_limit;
    a.act = act;
    a.out = out;
    a.status = status;
    a.k_total = hidden;
    a.m_tiles = inter / 64;
    a.scale0 = s1;
    a.scale1 = s3;
    const int tiles = (tokens + 7) / 8;
    const int g1 = tiles * a.m_tiles < grid ? tiles * a.m_tiles : grid;
    cudaError_t err = launch_sh<true>(m1, m3, map_x, a, g1, stream);
    if (err != cudaSuccess) return err;
    a.k_total = inter;
    a.m_tiles = hidden / 128;
    a.scale0 = s2;
    a.scale1 = s2;
    const int g2 = tiles * a.m_tiles < grid ? tiles * a.m_tiles : grid;
    return launch_sh<false>(m2, m2, map_act, a, g2, stream);
}

}  // namespace dee
