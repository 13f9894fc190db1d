// moe_mxfp8.cu -- the MXFP8-activation variant of the grouped expert GEMMs:
// tcgen05.mma kind::mxf8f6f4.block_scale with the weights' own E2M1 values
// and UE8M0 block-32 scales (the DEE4 record as it is: no dequantisation)
// against E4M3 activations with UE8M0 block scales (act_quant.cu).
//
// Roles (one CTA per SM, persistent over the (tile, m) items of the W4A16
// kernel):
//   warp 0     TMA producer of the packed E2M1 weights, spread by the TMA
//              to 16-byte groups of 8 data bytes and an 8-byte gap
//              (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, the MMA's operand
//              form; the transaction counts the 8 packed bytes);
//              for gate/up the 5-D map lands w1 and w3 rows interleaved in
//              groups of 16 so the accumulator lanes pair gate and up rows
//              the way the W4A16 epilogue expects
//   warp 1     TMA producer of the E4M3 token rows (16/32/64/128-row boxes)
//   warp 2     MMA issuer (whole warp, one elected lane): per 256-K step,
//              four tcgen05.cp of the step's scales from shared memory into
//              tensor memory, then eight K = 32 MMAs, in issue order
//   warps 3-4  scale stagers, taking alternate steps: the weights' and the
//              tokens' UE8M0 bytes of the step, loaded from L2 two of the
//              warp's steps ahead, stored to shared memory in the layout
//              tcgen05.cp.32x128b.warpx4 turns into the one the block-scaled
//              MMA reads (per 128 rows and 4 K blocks, 512 bytes: row
//              32c + l at byte 16l + 4c, one byte per K block; in tensor
//              memory lane l of column c, the same in all four quadrants)
//   warps 5-12 epilogue, two warps per lane quadrant taking alternate
//              32-column chunks: as the W4A16 kernel (SwiGLU into FP16 act,
//              or the FP32 scatter to the selections' rows); a K step here
//              is four times shorter than a W4A16 one, so the epilogue needs
//              twice the warps to stay hidden
#include "decode_common.cuh"
#include "kernels.h"
#include "moe_gemm.cuh"

namespace dee {
namespace {

using namespace sm100;

constexpr int kMxSfWarps = 2;                   // scale stagers, alternate steps
constexpr int kMxEpiWarp = 3 + kMxSfWarps;       // first epilogue warp
constexpr int kMxThreads = 32 * (kMxEpiWarp + 8);
constexpr int kMxStepK = 256;                   // K per pipeline step: 8 MMAs of K = 32
constexpr int kMxStages = 3;
constexpr int kMxAStageBytes = 128 * kMxStepK;  // 128 rows x 256 E2M1 in byte containers
constexpr int kMxBStageBytes = 128 * kMxStepK;  // up to 128 token rows x 256 E4M3
constexpr int kMxSfAtom = 512;                  // scales of 128 rows x 4 K blocks
constexpr int kMxSfStageBytes = 4 * kMxSfAtom;  // weights and tokens, 2 atoms each
constexpr int kMxNMax = 128;
constexpr int kMxSfBase = 2 * kMxNMax;          // after the double-buffered accumulator
constexpr int kMxSfCols = 16;                   // per stage: A scales 8 columns, token scales 8
constexpr int kMxSmemBytes =
    1024 + kMxStages * (kMxAStageBytes + kMxBStageBytes + kMxSfStageBytes) + 1024;
static_assert(kMxSmemBytes <= 232448, "shared memory budget");
static_assert(kMxSfBase + kMxStages * kMxSfCols <= 512, "tensor memory budget");

// Instruction descriptor of kind::mxf8f6f4: A E2M1 (5) at bits 7-9, B E4M3
// (0) at 10-12, UE8M0 scales (bit 23), N >> 3 at 17, M >> 4 at 24, K = 32;
// the scale-factor byte ids (bits 29-30 for A, 4-5 for B) are added per MMA.
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(int M, int N) {
    return (5u << 7) | (0u << 10) | (1u << 23) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                       uint32_t sfb, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ int mx_token_box(int n_pad) { return n_pad <= 16 ? 0 : n_pad <= 32 ? 1 : n_pad <= 64 ? 2 : 3; }

struct MxItem {
    int tile, m, slot;
    TileDesc td;
};

__device__ __forceinline__ bool mx_load_item(const GemmArgs& a, int item, MxItem& out) {
    item_tile_m(a, item, out.tile, out.m);
    out.td = a.tiles[out.tile];
    const int e = out.td.expert;
    int slot = -1;
    if (e >= 0 && e < a.num_experts) slot = a.slot_of[e];
    out.slot = slot;
    return slot >= 0 && slot < a.num_slots && out.td.n_pad >= 16 && out.td.n_pad % 16 == 0;
}

template <GemmMode MODE>
__global__ void __launch_bounds__(kMxThreads, 1)
    moe_mxfp8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b16,
                     const __grid_constant__ CUtensorMap map_b32, const __grid_constant__ CUtensorMap map_b64,
                     const __grid_constant__ CUtensorMap map_b128, const GemmArgs args,
                     const uint8_t* __restrict__ b_scales, int b_rows_cap) {
    constexpr bool kGU = MODE == GemmMode::kGateUp;
    pdl_wait();
    const int n_tiles = *args.n_tiles;
    const int n_items = n_tiles * args.m_tiles;
    pdl_trigger();
    if (static_cast<int>(blockIdx.x) >= n_items) return;  // uniform per CTA

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* a_smem = smem;
    uint8_t* b_smem = a_smem + kMxStages * kMxAStageBytes;
    uint8_t* sf_smem = b_smem + kMxStages * kMxBStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sf_smem + kMxStages * kMxSfStageBytes);
    uint64_t* full = bars;                 // weights + tokens landed, scales staged
    uint64_t* empty = full + kMxStages;    // step consumed by the MMAs
    uint64_t* acc_full = empty + kMxStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMxStages; ++i) { mbar_init(&full[i], 3); mbar_init(&empty[i], 1); }  // 2 TMA + 1 stager
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 8); }  // 8 epilogue warps
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&map_a);
    if (warp == 1 && lane == 0) {
        prefetch_tmap(&map_b16);
        prefetch_tmap(&map_b32);
        prefetch_tmap(&map_b64);
        prefetch_tmap(&map_b128);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int steps = args.k_total / kMxStepK;
    uint32_t* status = args.status;

    if (warp == 0) {
        // ---------------- weight producer ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            uint32_t g = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                MxItem it;
                if (!mx_load_item(args, item, it)) atomicOr(status, kStatusBadExpert);
                const int slot = (it.slot < 0 || it.slot >= args.num_slots) ? 0 : it.slot;
                for (int st = 0; st < steps; ++st, ++g) {
                    const uint32_t s = g % kMxStages;
                    if (!mbar_wait(&empty[s], ((g / kMxStages) & 1u) ^ 1u, status, kStatusTimeoutTma)) {
                        ok = false;
                        break;
                    }
                    // the TMA counts the packed bytes it reads (half the padded footprint)
                    mbar_arrive_expect_tx(&full[s], kMxAStageBytes / 2);
                    uint8_t* dst = a_smem + s * kMxAStageBytes;
                    for (int c = 0; c < kMxStepK / 128; ++c) {
                        const int x = st * kMxStepK + c * 128;  // K element (a multiple of 128)
                        if (kGU)
                            tma_load_5d(dst + c * 16384, &map_a, &full[s], x, 0, 0, it.m * 4, slot, pol);
                        else
                            tma_load_3d(dst + c * 16384, &map_a, &full[s], x, it.m * 128, slot, pol);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- token producer ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_last();
            uint32_t g = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                MxItem it;
                mx_load_item(args, item, it);
                const int box = mx_token_box(min(it.td.n_pad, kMxNMax));
                const int rows = 16 << box;
                const CUtensorMap* map = box == 0 ? &map_b16 : box == 1 ? &map_b32 : box == 2 ? &map_b64 : &map_b128;
                for (int st = 0; st < steps; ++st, ++g) {
                    const uint32_t s = g % kMxStages;
                    if (!mbar_wait(&empty[s], ((g / kMxStages) & 1u) ^ 1u, status, kStatusTimeoutTma)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], rows * kMxStepK);
                    tma_load_3d(b_smem + s * kMxBStageBytes, map, &full[s], 0, it.td.row_start, st * (kMxStepK / 128),
                                pol);
                }
            }
        }
    } else if (warp == 2) {
        // ---------------- MMA issuer ----------------
        uint32_t g = 0;
        bool ok = true;
        int local = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
            MxItem it;
            mx_load_item(args, item, it);
            const int n_pad = min(it.td.n_pad, kMxNMax);
            const uint32_t b_chunk = static_cast<uint32_t>(16 << mx_token_box(n_pad)) * 128u;
            const int acc = local & 1;
            ok = mbar_wait(&acc_empty[acc], (((local >> 1) & 1) ^ 1), status, kStatusTimeoutMma);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * kMxNMax;
            const uint32_t idesc = idesc_mxf8f6f4(128, n_pad);
            for (int st = 0; st < steps; ++st, ++g) {
                const uint32_t s = g % kMxStages;
                ok = mbar_wait(&full[s], (g / kMxStages) & 1u, status, kStatusTimeoutMma);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint64_t da = smem_desc_k128(smem_u32(a_smem + s * kMxAStageBytes));
                const uint64_t db = smem_desc_k128(smem_u32(b_smem + s * kMxBStageBytes));
                const uint32_t sf = tmem_base + kMxSfBase + s * kMxSfCols;
                const uint32_t sf_src = smem_u32(sf_smem + s * kMxSfStageBytes);
                if (elect_one()) {
                    // weight scales to columns sf + 0..7, token scales to sf + 8..15
#pragma unroll
                    for (int a = 0; a < 4; ++a) tmem_cp_32x128b_x4(sf + 4 * a, smem_desc_plain(sf_src + a * kMxSfAtom, 128));
#pragma unroll
                    for (int kb = 0; kb < kMxStepK / 32; ++kb) {
                        const uint32_t c = kb >> 2, id = kb & 3;
                        mma_mx(d_tmem, da + ((c * 16384u + id * 32u) >> 4), db + ((c * b_chunk + id * 32u) >> 4),
                               idesc | (id << 29) | (id << 4), (sf + c * 4) | (id << 30), (sf + 8 + c * 4) | (id << 30),
                               (st | kb) != 0 ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&acc_full[acc]);
            __syncwarp();
        }
    } else if (warp < kMxEpiWarp) {
        // ---------------- scale stagers ----------------
        const int grp = warp - 3;  // takes the steps g with g % kMxSfWarps == grp
        const size_t ih = static_cast<size_t>(args.hidden) * args.inter;
        const size_t s1 = ih + ih / 2, s3 = s1 + ih / 32, s2 = s3 + ih / 32;
        const int kb_row = args.k_total / 32;  // scale bytes per row
        uint32_t g = 0;
        bool ok = true;
        // The scale rows of an item (weights: 128 rows, tokens: up to 128)
        // are contiguous; one thread pulls the next item's into L2 while the
        // current one runs, so the per-step loads below hit L2, not HBM.
        auto prefetch_scales = [&](int item) {
            if (item >= n_items || grp != 0 || lane != 0) return;
            MxItem pi;
            mx_load_item(args, item, pi);
            const int ps = (pi.slot < 0 || pi.slot >= args.num_slots) ? 0 : pi.slot;
            const uint8_t* prec = args.records + static_cast<size_t>(ps) * args.record_bytes;
            if (kGU) {
                bulk_prefetch_l2(prec + s1 + static_cast<size_t>(pi.m * 64) * kb_row, 64 * kb_row);
                bulk_prefetch_l2(prec + s3 + static_cast<size_t>(pi.m * 64) * kb_row, 64 * kb_row);
            } else {
                bulk_prefetch_l2(prec + s2 + static_cast<size_t>(pi.m * 128) * kb_row, 128 * kb_row);
            }
            const int r0 = min(pi.td.row_start, b_rows_cap - 1);
            const int nr = min(min(pi.td.n_pad, kMxNMax), b_rows_cap - r0);
            bulk_prefetch_l2(b_scales + static_cast<size_t>(r0) * kb_row, nr * kb_row);
        };
        prefetch_scales(blockIdx.x);
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            MxItem it;
            mx_load_item(args, item, it);
            prefetch_scales(item + gridDim.x);
            const int slot = (it.slot < 0 || it.slot >= args.num_slots) ? 0 : it.slot;
            const uint8_t* rec = args.records + static_cast<size_t>(slot) * args.record_bytes;
            const uint8_t* arow[4];
            const uint8_t* brow[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int r = 32 * c + lane;  // accumulator row / token row of the tile
                if (kGU) {
                    const int wrow = it.m * 64 + 16 * (r >> 5) + (r & 15);
                    arow[c] = rec + ((r & 16) ? s3 : s1) + static_cast<size_t>(wrow) * kb_row;
                } else {
                    arow[c] = rec + s2 + static_cast<size_t>(it.m * 128 + r) * kb_row;
                }
                const int trow = min(it.td.row_start + r, b_rows_cap - 1);
                brow[c] = b_scales + static_cast<size_t>(trow) * kb_row;
            }
            auto load = [&](uint2 (&av)[4], uint2 (&bv)[4], int st) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    av[c] = __ldg(reinterpret_cast<const uint2*>(arow[c] + st * 8));
                    bv[c] = __ldg(reinterpret_cast<const uint2*>(brow[c] + st * 8));
                }
            };
            // Lane l writes the 16 bytes of rows l, 32 + l, 64 + l, 96 + l of
            // each atom (four K blocks each): 512 contiguous bytes per atom.
            auto put = [&](const uint2 (&av)[4], const uint2 (&bv)[4], uint32_t gi) -> bool {
                const uint32_t s = gi % kMxStages;
                const bool got = mbar_wait(&empty[s], ((gi / kMxStages) & 1u) ^ 1u, status, kStatusTimeoutDequant);
                if (!__all_sync(0xffffffffu, got)) return false;
                uint4* dst = reinterpret_cast<uint4*>(sf_smem + s * kMxSfStageBytes) + lane;
                dst[0] = make_uint4(av[0].x, av[1].x, av[2].x, av[3].x);
                dst[32] = make_uint4(av[0].y, av[1].y, av[2].y, av[3].y);
                dst[64] = make_uint4(bv[0].x, bv[1].x, bv[2].x, bv[3].x);
                dst[96] = make_uint4(bv[0].y, bv[1].y, bv[2].y, bv[3].y);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                return true;
            };
            // This warp's steps of the item are st = grp + kMxSfWarps * k.
            // Two register sets alternate over k, each loaded two of the
            // warp's steps ahead of its use.
            const int n_my = (steps - grp + kMxSfWarps - 1) / kMxSfWarps;
            auto step_of = [&](int k) { return grp + kMxSfWarps * k; };
            uint2 a0[4], b0[4], a1[4], b1[4];
            if (n_my > 0) load(a0, b0, step_of(0));
            if (n_my > 1) load(a1, b1, step_of(1));
            for (int k = 0; k < n_my && ok; k += 2) {
                ok = put(a0, b0, g + step_of(k));
                if (!ok) break;
                if (k + 2 < n_my) load(a0, b0, step_of(k + 2));
                if (k + 1 >= n_my) break;
                ok = put(a1, b1, g + step_of(k + 1));
                if (ok && k + 3 < n_my) load(a1, b1, step_of(k + 3));
            }
            g += steps;
        }
    } else {
        // ---------------- epilogue ----------------
        const int quad = warp & 3;
        const int half = (warp - kMxEpiWarp) >> 2;  // which of the quadrant's two warps
        const int L = quad * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        int local = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++local) {
            MxItem it;
            const bool valid = mx_load_item(args, item, it);
            const int n_rows = min(it.td.n_rows, kMxNMax);
            const int n_pad = min(it.td.n_pad, kMxNMax);
            const int acc = local & 1;
            const bool got = mbar_wait(&acc_full[acc], (local >> 1) & 1, status, kStatusTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t col0 = tmem_base + lane_addr + acc * kMxNMax;
            for (int c = 32 * half; c < n_pad; c += 64) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(col0 + c, v);
                tmem_wait_ld();
                if (!valid) continue;
                const int prow = c + lane < n_rows ? args.perm[it.td.row_start + c + lane] : 0;
                if (kGU) {
                    const bool is_gate = lane < 16;
                    const int feat = it.m * 64 + 16 * quad + (lane & 15);
                    const float lim = args.swiglu_limit;
                    const bool off = args.official != 0;
                    const float wl = (off && args.route_w && c + lane < n_rows) ? args.route_w[prow] : 1.0f;
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float lo = __uint_as_float(v[i]), hi = __uint_as_float(v[i + 1]);
                        const float recv = __shfl_xor_sync(0xffffffffu, is_gate ? hi : lo, 16);
                        const int j = is_gate ? i : i + 1;
                        const float w = __shfl_sync(0xffffffffu, wl, j);
                        const int col = c + j;
                        if (col < n_rows)
                            args.act[static_cast<size_t>(it.td.row_start + col) * args.inter + feat] =
                                swiglu_out(is_gate ? lo : recv, is_gate ? recv : hi, lim, off, w);
                    }
                } else {
                    const int feat = it.m * 128 + L;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int pos = __shfl_sync(0xffffffffu, prow, i);
                        if (c + i < n_rows)
                            args.raw[static_cast<size_t>(pos) * args.hidden + feat] = __uint_as_float(v[i]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

template <GemmMode MODE>
cudaError_t launch_mx(const MxMaps& maps, const GemmArgs& args, const uint8_t* b_scales, int b_rows_cap, int grid,
                      cudaStream_t stream) {
    auto kern = moe_mxfp8_kernel<MODE>;
    const cudaError_t e = ensure_smem_attr<moe_mxfp8_kernel<MODE>>(kMxSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kMxThreads), kMxSmemBytes, stream, maps.a, maps.bt[0], maps.bt[1],
                      maps.bt[2], maps.bt[3], args, b_scales, b_rows_cap);
}

}  // namespace

cudaError_t launch_moe_mxfp8(bool gate_up, const MxMaps& maps, const GemmArgs& args, const uint8_t* b_scales,
                             int b_rows_cap, int grid, cudaStream_t stream) {
    if (args.k_total % kMxStepK || b_rows_cap <= 0) return cudaErrorInvalidValue;
    return gate_up ? launch_mx<GemmMode::kGateUp>(maps, args, b_scales, b_rows_cap, grid, stream)
                   : launch_mx<GemmMode::kDown>(maps, args, b_scales, b_rows_cap, grid, stream);
}

// Weight maps over a bank of DEE4 records, E2M1 unpacked into byte
// containers by the TMA.  Gate/up: 5-D {K, 16 rows, 2 matrices (w1, w3),
// row groups, slots} so a box {128, 16, 2, 4, 1} lands rows of w1 and w3
// interleaved in groups of 16; down: 3-D {K, rows, slots}.
bool encode_mx_weight_maps(EncodeTiledFn fn, const void* records, size_t record_bytes, int n_slots, int hidden,
                           int inter, MxMaps* gu, MxMaps* dn) {
    if (!fn) return false;
    const uint8_t* base = static_cast<const uint8_t*>(records);
    const size_t ih = static_cast<size_t>(hidden) * inter;
    const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
    {
        const cuuint64_t dims[5] = {static_cast<cuuint64_t>(hidden), 16, 2, static_cast<cuuint64_t>(inter / 16),
                                    static_cast<cuuint64_t>(n_slots)};
        const cuuint64_t strides[4] = {static_cast<cuuint64_t>(hidden / 2), ih / 2,
                                       static_cast<cuuint64_t>(16) * (hidden / 2), record_bytes};
        const cuuint32_t box[5] = {128, 16, 2, 4, 1};
        if (fn(&gu->a, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 5, const_cast<uint8_t*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(inter), static_cast<cuuint64_t>(hidden),
                                    static_cast<cuuint64_t>(n_slots)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(inter / 2), record_bytes};
        const cuuint32_t box[3] = {128, 128, 1};
        if (fn(&dn->a, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<uint8_t*>(base + ih), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

// E4M3 token rows [rows, cols] viewed as {128, rows, cols/128}: boxes of
// 16/32/64/128 rows x 2 chunks of 128 columns (one 256-K step).
bool encode_mx_token_maps(EncodeTiledFn fn, const void* rows_base, int rows, int cols, CUtensorMap* maps) {
    if (!fn) return false;
    for (int b = 0; b < 4; ++b) {
        const cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols / 128)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols), 128};
        const cuuint32_t box[3] = {128, static_cast<cuuint32_t>(16 << b), 2};
        const cuuint32_t elem[3] = {1, 1, 1};
        if (fn(&maps[b], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(rows_base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

}  // namespace dee
