// moe_gemm.cu -- the grouped tcgen05 W4A16 kernels (see moe_gemm.cuh).
#include "moe_gemm.cuh"
#include "decode_common.cuh"
#include "kernels.h"

#include <cstdio>

namespace dee {
namespace {

using namespace sm100;

// ---------------------------------------------------------------------------
// FP4 E2M1 x 32 + UE8M0 scale -> 32 FP16 values packed as 16 f16x2 words.
// Element order: word k holds elements 2k (low half) and 2k+1 (high half),
// the low nibble of each byte being the even element (cuda_convert.cu:241).
// Values equal __float2half_rn(e2m1 * 2^(b-127)) with the scale clamps of
// fp4_scale_value (cuda_convert.cu:217-223).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cvt_e2m1x8(uint32_t w, uint32_t& o0, uint32_t& o1, uint32_t& o2,
                                           uint32_t& o3) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
        : "r"(w));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ float scale_value(uint32_t b) {
    const int e = static_cast<int>(b) - 127;
    if (e >= 127) return __int_as_float(0x7F7FFFFF);
    if (e <= -127) return 0.0f;
    return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

__device__ __forceinline__ void dequant_block32(const uint4& q, uint32_t sbyte, uint32_t* out) {
    uint32_t r[16];
    cvt_e2m1x8(q.x, r[0], r[1], r[2], r[3]);
    cvt_e2m1x8(q.y, r[4], r[5], r[6], r[7]);
    cvt_e2m1x8(q.z, r[8], r[9], r[10], r[11]);
    cvt_e2m1x8(q.w, r[12], r[13], r[14], r[15]);
    if (sbyte >= 103u && sbyte <= 142u) {
        // 2^(b-127) is an exact binary16 (normal or subnormal): one correctly
        // rounded f16x2 multiply equals FP16(value * scale) computed in FP32.
        const int e = static_cast<int>(sbyte) - 127;
        const uint32_t sh = e >= -14 ? static_cast<uint32_t>(e + 15) << 10 : 1u << (e + 24);
        const uint32_t s2 = sh | (sh << 16);
#pragma unroll
        for (int i = 0; i < 16; ++i) out[i] = hmul2_u32(r[i], s2);
    } else {
        const float s = scale_value(sbyte);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const __half2 h = *reinterpret_cast<const __half2*>(&r[i]);
            const float2 f = __half22float2(h);
            const __half lo = __float2half_rn(f.x * s);
            const __half hi = __float2half_rn(f.y * s);
            out[i] = static_cast<uint32_t>(__half_as_ushort(lo)) |
                     (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
        }
    }
}


struct ItemInfo {
    int tile;
    int m;
    TileDesc td;
    int slot;
};

__device__ __forceinline__ bool load_item(const GemmArgs& a, int item, ItemInfo& out) {
    item_tile_m(a, item, out.tile, out.m);
    out.td = a.tiles[out.tile];
    const int e = out.td.expert;
    int slot = -1;
    if (e >= 0 && e < a.num_experts) slot = a.slot_of[e];
    out.slot = slot;
    return slot >= 0 && slot < a.num_slots && out.td.n_pad >= 16 && out.td.n_pad % 16 == 0;
}

// Token box for a tile of n_pad rows: index into the 16/32/64/128-row maps.
__device__ __forceinline__ int token_box(int n_pad) {
    return n_pad <= 16 ? 0 : n_pad <= 32 ? 1 : n_pad <= 64 ? 2 : 3;
}

template <GemmMode MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_w0,   // w1 (gate/up) or w2 (down)
                    const __grid_constant__ CUtensorMap map_w1,   // w3 (gate/up only)
                    const __grid_constant__ CUtensorMap map_s0,   // s1 or s2
                    const __grid_constant__ CUtensorMap map_s1,   // s3 (gate/up only)
                    const __grid_constant__ CUtensorMap map_b16,  // X_perm or act, 16-row boxes
                    const __grid_constant__ CUtensorMap map_b32,
                    const __grid_constant__ CUtensorMap map_b64,
                    const __grid_constant__ CUtensorMap map_b128,
                    const GemmArgs args) {
    constexpr bool kGU = MODE == GemmMode::kGateUp;
    constexpr int kPrefetch = 2;  // packed stages prefetched into L2 beyond the ring

    // The gate/up GEMM follows the kernels that write its tile list and
    // token rows, so it waits before reading anything.  The down GEMM
    // follows the gate/up GEMM, which triggers only after its own wait, so
    // the tile list (written two kernels back) is complete when the down
    // GEMM starts: its weight producer streams W2 at once, every other role
    // waits for the gate/up results first.
    if (kGU) pdl_wait();
    const int n_tiles = *args.n_tiles;
    const int n_items = n_tiles * args.m_tiles;
    if (static_cast<int>(blockIdx.x) >= n_items) {  // uniform per CTA
        if (!kGU) pdl_wait();
        pdl_trigger();
        return;
    }

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* pk_smem = smem;
    uint8_t* b_smem = pk_smem + kPkStages * kPkStageBytes;
    uint8_t* sc_smem = b_smem + kBStages * kBStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sc_smem + kPkStages * kScStageBytes);
    uint64_t* pk_full = bars;                  // packed weight stage landed (TMA)
    uint64_t* pk_empty = pk_full + kPkStages;  // all 8 dequantiser warps done with it
    uint64_t* full = pk_empty + kPkStages;     // 128-K step: A written (4 warps) + B landed (TMA)
    uint64_t* empty = full + kAStages;         // 128-K step consumed by the MMAs (commit)
    uint64_t* acc_full = empty + kAStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        // pk_empty: each of the four warps of a step's warpgroup, per step
        for (int i = 0; i < kPkStages; ++i) { mbar_init(&pk_full[i], 1); mbar_init(&pk_empty[i], 4 * (kKStage / kAK)); }
        for (int i = 0; i < kAStages; ++i) { mbar_init(&full[i], 5); mbar_init(&empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&map_w0);
        prefetch_tmap(&map_s0);
        if (kGU) { prefetch_tmap(&map_w1); prefetch_tmap(&map_s1); }
    }
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

    const int k_stages = args.k_total / kKStage;  // packed weight stages per item
    const int a_steps = args.k_total / kAK;       // 128-K steps per item (even)
    uint32_t* status = args.status;
    if (!kGU && warp != 0) pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        // ---------------- packed weight + scale producer ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int ps = 0;
            uint32_t pphase = 0;
            bool ok = true;
            // L2 prefetch cursor: runs kPrefetch stages ahead of the loads
            int pf_item = blockIdx.x, pf_s = 0, pf_slot = 0, pf_m = 0;
            bool pf_valid = false;
            auto pf_advance = [&]() {
                if (pf_valid && ++pf_s < k_stages) return;
                if (pf_valid) pf_item += gridDim.x;
                pf_s = 0;
                pf_valid = pf_item < n_items;
                if (pf_valid) {
                    ItemInfo pit;
                    load_item(args, pf_item, pit);
                    pf_slot = (pit.slot < 0 || pit.slot >= args.num_slots) ? 0 : pit.slot;
                    pf_m = pit.m;
                }
            };
            auto pf_issue = [&]() {
                if (!pf_valid) return;
                const int xk = pf_s * (kKStage / 2);
                if (kGU) {
                    tma_prefetch_3d(&map_w0, xk, pf_m * 64, pf_slot);
                    tma_prefetch_3d(&map_w1, xk, pf_m * 64, pf_slot);
                    tma_prefetch_3d(&map_w0, xk + 128, pf_m * 64, pf_slot);
                    tma_prefetch_3d(&map_w1, xk + 128, pf_m * 64, pf_slot);
                } else {
                    tma_prefetch_3d(&map_w0, xk, pf_m * 128, pf_slot);
                    tma_prefetch_3d(&map_w0, xk + 128, pf_m * 128, pf_slot);
                }
            };
            pf_advance();
            for (int i = 0; i < kPkStages + kPrefetch && pf_valid; ++i) {
                pf_issue();
                pf_advance();
            }
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                ItemInfo it;
                if (!load_item(args, item, it)) { atomicOr(status, kStatusBadExpert); }
                const int slot = (it.slot < 0 || it.slot >= args.num_slots) ? 0 : it.slot;
                for (int s = 0; s < k_stages; ++s) {
                    pf_issue();
                    pf_advance();
                    if (!mbar_wait(&pk_empty[ps], pphase ^ 1, status, kStatusTimeoutTma)) { ok = false; break; }
                    mbar_arrive_expect_tx(&pk_full[ps], kPkStageBytes + kScStageBytes);
                    uint8_t* dst = pk_smem + ps * kPkStageBytes;
                    uint8_t* sdst = sc_smem + ps * kScStageBytes;
                    const int xk = s * (kKStage / 2);  // packed byte column
                    if (kGU) {
                        const int row = it.m * 64;
                        tma_load_3d(dst, &map_w0, &pk_full[ps], xk, row, slot, pol);
                        tma_load_3d(dst + 8192, &map_w1, &pk_full[ps], xk, row, slot, pol);
                        tma_load_3d(dst + 16384, &map_w0, &pk_full[ps], xk + 128, row, slot, pol);
                        tma_load_3d(dst + 16384 + 8192, &map_w1, &pk_full[ps], xk + 128, row, slot, pol);
                        tma_load_3d(sdst, &map_s0, &pk_full[ps], s * 16, row, slot, pol);
                        tma_load_3d(sdst + 1024, &map_s1, &pk_full[ps], s * 16, row, slot, pol);
                    } else {
                        const int row = it.m * 128;
                        tma_load_3d(dst, &map_w0, &pk_full[ps], xk, row, slot, pol);
                        tma_load_3d(dst + 16384, &map_w0, &pk_full[ps], xk + 128, row, slot, pol);
                        tma_load_3d(sdst, &map_s0, &pk_full[ps], s * 16, row, slot, pol);
                    }
                    if (++ps == kPkStages) { ps = 0; pphase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- token operand producer ----------------
        // Step g (a CTA-wide count of 128-K steps) lands in buffer g % 3 and
        // completes full[g % 4]; the buffer is free again once the MMAs of
        // step g - 3 have completed, i.e. after empty[(g - 3) % 4] phase
        // (g - 3) / 4.  (That barrier cannot run two phases ahead: its next
        // phase needs step g + 1, whose tokens this thread has not loaded.)
        if (lane == 0) {
            const uint64_t pol = policy_evict_last();
            uint32_t g = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                ItemInfo it;
                load_item(args, item, it);
                const int n_pad = min(it.td.n_pad, kNMax);
                const int box = token_box(n_pad);
                const int rows = 16 << box;
                const CUtensorMap* map = box == 0 ? &map_b16 : box == 1 ? &map_b32 : box == 2 ? &map_b64 : &map_b128;
                for (int st = 0; st < a_steps; ++st, ++g) {
                    if (g >= static_cast<uint32_t>(kBStages)) {
                        const uint32_t gp = g - kBStages;
                        if (!mbar_wait(&empty[gp % kAStages], (gp / kAStages) & 1u, status, kStatusTimeoutTma)) {
                            ok = false;
                            break;
                        }
                    }
                    uint64_t* bar = &full[g % kAStages];
                    mbar_arrive_expect_tx(bar, rows * 128 * (kAK / kKBlock));
                    tma_load_3d(b_smem + (g % kBStages) * kBStageBytes, map, bar, 0, it.td.row_start,
                                st * (kAK / kKBlock), pol);
                }
            }
        }
    } else if (warp == 2) {
        // ---------------- MMA issuer ----------------
        // The whole warp runs the loop, so descriptors and addresses are
        // warp-uniform values; one elected lane issues the MMAs and commits.
        uint32_t g = 0;
        bool ok = true;
        int local = 0;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
            ItemInfo it;
            load_item(args, item, it);
            const int n_pad = min(it.td.n_pad, kNMax);
            const uint32_t chunk_bytes = static_cast<uint32_t>(16 << token_box(n_pad)) * 128u;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            ok = mbar_wait(&acc_empty[acc], acc_phase ^ 1, status, kStatusTimeoutMma);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + kAccBase + acc * kNMax;
            const uint32_t idesc = idesc_f16_f32(128, n_pad);
            for (int st = 0; st < a_steps; ++st, ++g) {
                const uint32_t s = g % kAStages;
                ok = mbar_wait(&full[s], (g / kAStages) & 1u, status, kStatusTimeoutMma);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_tmem = tmem_base + s * (kAK / 2);
                const uint64_t desc0 = smem_desc_k128(smem_u32(b_smem + (g % kBStages) * kBStageBytes));
                if (elect_one()) {
#pragma unroll
                    for (int c = 0; c < kAK / kKBlock; ++c) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            // +16-byte units in the descriptor's start-address field
                            mma_f16_ts(d_tmem, a_tmem + c * 32 + q * 8, desc0 + ((c * chunk_bytes + q * 32) >> 4),
                                       idesc, (st | c | q) != 0 ? 1u : 0u);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&acc_full[acc]);
            __syncwarp();
        }
    } else if (warp < kEpilogueWarp) {
        // ---------------- dequantisers (TMEM lane = thread's weight row) ----------------
        // Warpgroup wg takes the 128-K steps g with g % kDqGroups == wg; each
        // thread owns one weight row, i.e. one TMEM lane, and writes its 128
        // FP16 weights to A stage g % 4.
        const int wg = (warp - 3) >> 2;
        const int quad = warp & 3;
        const int L = quad * 32 + lane;  // TMEM lane / A row
        int srow;
        if (kGU) {
            const int f = 16 * (L >> 5) + (L & 15);
            srow = (L & 31) < 16 ? f : 64 + f;
        } else {
            srow = L;
        }
        const int sw = srow & 7;
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        int ps = 0;
        uint32_t pphase = 0;
        uint32_t g = 0;  // 128-K steps so far in this CTA (all warpgroups)
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            for (int s = 0; s < k_stages && ok; ++s) {
                ok = mbar_wait(&pk_full[ps], pphase, status, kStatusTimeoutDequant);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                const uint8_t* stg = pk_smem + ps * kPkStageBytes;
#pragma unroll 1
                for (int a = 0; a < kKStage / kAK; ++a) {
                    const uint32_t gi = g + static_cast<uint32_t>(a);
                    if (gi % kDqGroups != static_cast<uint32_t>(wg)) continue;
                    // this step's packed bytes and scales, then the stage can be refilled
                    const uint8_t* rowp = stg + (a >> 1) * 16384 + srow * 128;
                    const int c0 = (a & 1) * 4;
                    uint4 q[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) q[b] = *reinterpret_cast<const uint4*>(rowp + (((c0 + b) ^ sw) << 4));
                    const uint32_t scw = *reinterpret_cast<const uint32_t*>(sc_smem + ps * kScStageBytes + srow * 16 + 4 * a);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&pk_empty[ps]);
                    uint32_t v[32];
                    dequant_block32(q[0], scw & 0xFFu, v);
                    dequant_block32(q[1], (scw >> 8) & 0xFFu, v + 16);
                    const uint32_t as = gi % kAStages;
                    const bool got = mbar_wait(&empty[as], ((gi / kAStages) & 1u) ^ 1u, status, kStatusTimeoutDequant);
                    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t col = tmem_base + lane_addr + as * (kAK / 2);
                    tmem_st_32x32b_x32(col, v);
                    dequant_block32(q[2], (scw >> 16) & 0xFFu, v);
                    dequant_block32(q[3], scw >> 24, v + 16);
                    tmem_st_32x32b_x32(col + 32, v);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[as]);
                }
                g += kKStage / kAK;
                if (++ps == kPkStages) { ps = 0; pphase ^= 1; }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int quad = warp & 3;
        const int L = quad * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
        int local = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++local) {
            ItemInfo it;
            const bool valid = load_item(args, item, it);
            const int n_rows = min(it.td.n_rows, kNMax);
            const int n_pad = min(it.td.n_pad, kNMax);
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            const bool got = mbar_wait(&acc_full[acc], acc_phase, status, kStatusTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t col0 = tmem_base + lane_addr + kAccBase + acc * kNMax;
            // 32 columns (token rows) per load; the accumulator holds kNMax
            // columns, so a chunk past n_pad stays inside it.
            for (int c = 0; c < n_pad; c += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(col0 + c, v);
                tmem_wait_ld();
                if (!valid) continue;
                // lane j holds the grouped position of chunk row j
                const int prow = c + lane < n_rows ? args.perm[it.td.row_start + c + lane] : 0;
                if (kGU) {
                    // Lanes 0-15 hold gate rows, 16-31 the matching up rows.
                    // Per column pair (i, i+1) the gate lane finishes column i
                    // and the up lane column i+1: one exchange, every lane busy.
                    const bool is_gate = lane < 16;
                    const int feat = it.m * 64 + 16 * quad + (lane & 15);
                    const float lim = args.swiglu_limit;
                    const bool off = args.official != 0;
                    const float wl = (off && args.route_w && c + lane < n_rows) ? args.route_w[prow] : 1.0f;
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float lo = __uint_as_float(v[i]), hi = __uint_as_float(v[i + 1]);
                        const float recv = __shfl_xor_sync(0xffffffffu, is_gate ? hi : lo, 16);
                        const int j = is_gate ? i : i + 1;  // column this lane finishes
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
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <GemmMode MODE>
cudaError_t launch_one(const GemmMaps& maps, const GemmArgs& args, int grid, cudaStream_t stream) {
    auto kern = moe_gemm_kernel<MODE>;
    const cudaError_t e = ensure_smem_attr<moe_gemm_kernel<MODE>>(kGemmSmemBytes);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kGemmThreads), kGemmSmemBytes, stream, maps.w0, maps.w1, maps.s0,
                      maps.s1, maps.bt[0], maps.bt[1], maps.bt[2], maps.bt[3], args);
}

}  // namespace

int gemm_n_max() { return kNMax; }

cudaError_t launch_moe_gemm(bool gate_up, const GemmMaps& maps, const GemmArgs& args, int grid, cudaStream_t stream) {
    if (args.k_total % kKStage || (args.k_total / kAK) % 2) return cudaErrorInvalidValue;
    return gate_up ? launch_one<GemmMode::kGateUp>(maps, args, grid, stream)
                   : launch_one<GemmMode::kDown>(maps, args, grid, stream);
}

bool encode_gemm_token_maps(EncodeTiledFn fn, const void* rows_base, int rows, int cols, CUtensorMap* maps) {
    for (int b = 0; b < kTokenBoxes; ++b)
        if (!encode_token_map(fn, rows_base, rows, cols, 16 << b, kAK / kKBlock, &maps[b])) return false;
    return true;
}

}  // namespace dee
