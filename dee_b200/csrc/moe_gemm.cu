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
    out.tile = item / a.m_tiles;
    out.m = item - out.tile * a.m_tiles;
    out.td = a.tiles[out.tile];
    const int e = out.td.expert;
    int slot = -1;
    if (e >= 0 && e < a.num_experts) slot = a.slot_of[e];
    out.slot = slot;
    return slot >= 0 && slot < a.num_slots && out.td.n_pad >= 16 && out.td.n_pad % 16 == 0;
}

template <class Cfg, GemmMode MODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_w0,   // w1 (gate/up) or w2 (down)
                    const __grid_constant__ CUtensorMap map_w1,   // w3 (gate/up only)
                    const __grid_constant__ CUtensorMap map_s0,   // s1 or s2
                    const __grid_constant__ CUtensorMap map_s1,   // s3 (gate/up only)
                    const __grid_constant__ CUtensorMap map_b,    // X_perm or act
                    const GemmArgs args) {
    constexpr int NMAX = Cfg::kNMax;
    constexpr int PK = Cfg::kPk;
    constexpr int BS = Cfg::kB;
    constexpr int AS = Cfg::kA;
    constexpr bool kGU = MODE == GemmMode::kGateUp;

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
    uint8_t* b_smem = pk_smem + PK * kPkStageBytes;
    uint8_t* sc_smem = b_smem + BS * Cfg::kBStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sc_smem + PK * kScStageBytes);
    uint64_t* pk_full = bars;
    uint64_t* pk_empty = pk_full + PK;
    uint64_t* b_full = pk_empty + PK;
    uint64_t* b_empty = b_full + BS;
    uint64_t* a_full = b_empty + BS;
    uint64_t* a_empty = a_full + AS;
    uint64_t* acc_full = a_empty + AS;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < PK; ++i) { mbar_init(&pk_full[i], 1); mbar_init(&pk_empty[i], 8); }
        for (int i = 0; i < BS; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < AS; ++i) { mbar_init(&a_full[i], 4); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&map_w0);
        prefetch_tmap(&map_s0);
        prefetch_tmap(&map_b);
        if (kGU) { prefetch_tmap(&map_w1); prefetch_tmap(&map_s1); }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    const int k_stages = args.k_total / kKStage;
    const int k_blocks = args.k_total / kKBlock;
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
            // L2 prefetch cursor: runs Cfg::kPrefetch stages ahead of the loads
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
            if (Cfg::kPrefetch > 0) {
                pf_advance();
                for (int i = 0; i < PK + Cfg::kPrefetch && pf_valid; ++i) {
                    pf_issue();
                    pf_advance();
                }
            }
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                ItemInfo it;
                if (!load_item(args, item, it)) { atomicOr(status, kStatusBadExpert); }
                const int slot = (it.slot < 0 || it.slot >= args.num_slots) ? 0 : it.slot;
                for (int s = 0; s < k_stages; ++s) {
                    if (Cfg::kPrefetch > 0) {
                        pf_issue();
                        pf_advance();
                    }
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
                    if (++ps == PK) { ps = 0; pphase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- token operand producer ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_last();
            int bs = 0;
            uint32_t bphase = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                ItemInfo it;
                load_item(args, item, it);
                const int n_pad = min(it.td.n_pad, NMAX);
                for (int kb0 = 0; kb0 < k_blocks; kb0 += Cfg::kBKb) {
                    if (!mbar_wait(&b_empty[bs], bphase ^ 1, status, kStatusTimeoutTma)) { ok = false; break; }
                    mbar_arrive_expect_tx(&b_full[bs], n_pad * 128 * Cfg::kBKb);
                    uint8_t* dst = b_smem + bs * Cfg::kBStageBytes;
                    for (int j = 0; j < Cfg::kBKb; ++j)
                        for (int r = 0; r < n_pad; r += 16)
                            tma_load_2d(dst + j * (NMAX * 128) + r * 128, &map_b, &b_full[bs],
                                        (kb0 + j) * kKBlock, it.td.row_start + r, pol);
                    if (++bs == BS) { bs = 0; bphase ^= 1; }
                }
            }
        }
    } else if (warp == 2) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int as = 0, bs = 0;
            uint32_t aphase = 0, bphase = 0;
            bool ok = true;
            int local = 0;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
                ItemInfo it;
                load_item(args, item, it);
                const int n_pad = min(it.td.n_pad, NMAX);
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, status, kStatusTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + Cfg::kAccBase + acc * NMAX;
                const uint32_t idesc = idesc_f16_f32(128, n_pad);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const int j = kb % Cfg::kBKb;  // K step within the token-operand stage
                    if (!mbar_wait(&a_full[as], aphase, status, kStatusTimeoutMma) ||
                        (j == 0 && !mbar_wait(&b_full[bs], bphase, status, kStatusTimeoutMma))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem_base + as * 32;
                    const uint32_t b_addr = smem_u32(b_smem + bs * Cfg::kBStageBytes + j * (NMAX * 128));
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        mma_f16_ts(d_tmem, a_tmem + q * 8, smem_desc_k128(b_addr + q * 32), idesc,
                                   (kb | q) != 0 ? 1u : 0u);
                    }
                    mma_commit(&a_empty[as]);
                    if (++as == AS) { as = 0; aphase ^= 1; }
                    if (j == Cfg::kBKb - 1) {
                        mma_commit(&b_empty[bs]);
                        if (++bs == BS) { bs = 0; bphase ^= 1; }
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
            }
        }
    } else if (warp <= 10) {
        // ---------------- dequantisers (TMEM lane = thread's weight row) ----------------
        // Two warpgroups split the eight 64-wide K steps of a packed stage
        // (even steps: warps 3-6, odd steps: warps 7-10); each thread owns
        // one weight row, i.e. one TMEM lane.
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
        uint32_t g = 0;  // K steps issued so far by this CTA (both warpgroups)
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            for (int s = 0; s < k_stages && ok; ++s) {
                ok = mbar_wait(&pk_full[ps], pphase, status, kStatusTimeoutDequant);
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                const uint8_t* st = pk_smem + ps * kPkStageBytes;
                const uint4 sc = *reinterpret_cast<const uint4*>(sc_smem + ps * kScStageBytes + srow * 16);
                const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
                const uint32_t sshift = 16u * static_cast<uint32_t>(wg);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = 2 * jj + wg;  // K step within the stage
                    const int c0 = (j & 3) * 2;
                    const uint8_t* rowp = st + (jj >> 1) * 16384 + srow * 128;
                    const uint4 q0 = *reinterpret_cast<const uint4*>(rowp + ((c0 ^ sw) << 4));
                    const uint4 q1 = *reinterpret_cast<const uint4*>(rowp + (((c0 + 1) ^ sw) << 4));
                    const uint32_t sb0 = (scw[jj] >> sshift) & 0xFFu;
                    const uint32_t sb1 = (scw[jj] >> (sshift + 8)) & 0xFFu;
                    uint32_t v[32];
                    dequant_block32(q0, sb0, v);
                    dequant_block32(q1, sb1, v + 16);
                    const uint32_t gi = g + static_cast<uint32_t>(j);
                    const int as = static_cast<int>(gi % AS);
                    const uint32_t aphase = (gi / AS) & 1u;
                    const bool got = mbar_wait(&a_empty[as], aphase ^ 1, status, kStatusTimeoutDequant);
                    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                    tc_fence_after();
                    tmem_st_32x32b_x32(tmem_base + lane_addr + as * 32, v);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[as]);
                }
                g += 8;
                __syncwarp();
                if (lane == 0) mbar_arrive(&pk_empty[ps]);
                if (++ps == PK) { ps = 0; pphase ^= 1; }
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
            const int n_rows = min(it.td.n_rows, NMAX);
            const int n_pad = min(it.td.n_pad, NMAX);
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            const bool got = mbar_wait(&acc_full[acc], acc_phase, status, kStatusTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t col0 = tmem_base + lane_addr + Cfg::kAccBase + acc * NMAX;
            for (int c = 0; c < n_pad; c += 16) {
                uint32_t v[16];
                tmem_ld_32x32b_x16(col0 + c, v);
                tmem_wait_ld();
                if (!valid) continue;
                if (kGU) {
                    const bool is_gate = lane < 16;
                    const int feat = it.m * 64 + 16 * quad + (lane & 15);
                    const float lim = args.swiglu_limit;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float mine = __uint_as_float(v[i]);
                        const float other = __shfl_xor_sync(0xffffffffu, mine, 16);
                        // columns alternate between the two half-warps
                        if ((i & 1) != (is_gate ? 0 : 1)) continue;
                        const int col = c + i;
                        if (col >= n_rows) continue;
                        const float w = (args.official && args.route_w)
                                            ? args.route_w[args.perm[it.td.row_start + col]]
                                            : 1.0f;
                        args.act[static_cast<size_t>(it.td.row_start + col) * args.inter + feat] =
                            swiglu_out(is_gate ? mine : other, is_gate ? other : mine, lim,
                                       args.official != 0, w);
                    }
                } else {
                    const int feat = it.m * 128 + L;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int col = c + i;
                        if (col >= n_rows) break;
                        const int pos = args.perm[it.td.row_start + col];
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
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

template <class Cfg, GemmMode MODE>
cudaError_t launch_one(const GemmMaps& maps, const GemmArgs& args, int grid, cudaStream_t stream) {
    auto kern = moe_gemm_kernel<Cfg, MODE>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Cfg::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    return launch_pdl(kern, dim3(grid), dim3(kGemmThreads), Cfg::kSmemBytes, stream, maps.w0,
                      maps.w1, maps.s0, maps.s1, maps.b, args);
}

// Decode-sized tiles: token rows for a whole 512-wide K stage per load (the
// token operand then costs one TMA round trip per eight K steps) and packed
// weights prefetched into L2 four stages beyond the shared-memory ring.
using CfgSmall = GemmConfig<16, 4, 4, 8, 8, 4>;
using CfgLarge = GemmConfig<128, 3, 6, 1, 4, 2>;

}  // namespace

int gemm_n_max(bool large) { return large ? CfgLarge::kNMax : CfgSmall::kNMax; }

cudaError_t launch_moe_gemm(bool gate_up, bool large, const GemmMaps& maps, const GemmArgs& args,
                            int grid, cudaStream_t stream) {
    if (gate_up) {
        return large ? launch_one<CfgLarge, GemmMode::kGateUp>(maps, args, grid, stream)
                     : launch_one<CfgSmall, GemmMode::kGateUp>(maps, args, grid, stream);
    }
    return large ? launch_one<CfgLarge, GemmMode::kDown>(maps, args, grid, stream)
                 : launch_one<CfgSmall, GemmMode::kDown>(maps, args, grid, stream);
}

}  // namespace dee
