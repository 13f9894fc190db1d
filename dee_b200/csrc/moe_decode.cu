// moe_decode.cu -- grouped W4A16 GEMM for decode-sized expert groups.
//
// For groups of at most 8 token rows per expert (decode), every packed
// weight byte is used by only a handful of tokens, so the kernel is bound
// by how fast weights can be streamed and turned into tensor-core operands.
// Measured on B200, the tensor-memory A path of moe_gemm.cu pays about 110
// cycles per 128x16 A slice whatever N is, and staging dequantised weights in
// shared memory would need ~5 bytes of shared-memory traffic per weight.
// Here the dequantised weights never leave registers:
//
//   warp 0       TMA producer: per 512-wide K stage, the packed FP4 rows
//                (128 rows x 256 B), their UE8M0 scales and the stage's token
//                rows (8 rows x 1 KB, 128-byte swizzled)
//   warp 17      scale checker: decides per stage whether every block scale
//                allows the exact FP32 scaling below
//   warps 1-16   consumers: warp w owns the 16 weight rows (w-1)%8 of the
//                128-row work item over one half of each stage's K (warps
//                1-8 the first 256, warps 9-16 the second), reads its packed
//                bytes from shared memory, converts them (cvt.rn.f16x2.e2m1x2)
//                into mma.sync.m16n8k16 A fragments and accumulates FP32 in
//                registers, applying each 32-wide block's power-of-two scale to
//                the block's partial sum.  At the end of an item the second
//                warp of each pair hands its sums to the first through shared
//                memory (one fixed two-term add), and the first runs the
//                epilogue.
//
// Gate/up items pair 8 gate rows with the same 8 up rows in each 16-row MMA
// tile, so one thread holds the gate and up accumulators of the same
// (feature, token) and applies the reference's FP16 SwiGLU chain in
// registers (swiglu_cuda.cu:46-59).  Down items scatter FP32 rows to
// raw[token * K + rank] (engine.cpp:1080-1113).
#include "kernels.h"

namespace dee {
namespace {

using namespace sm100;

constexpr int kDecConsumerWarps = 16;
constexpr int kDecCheckerWarp = 1 + kDecConsumerWarps;
constexpr int kDecThreads = 32 * (kDecCheckerWarp + 1);  // producer, 8 pairs of consumers, checker
constexpr int kDecStages = 5;
constexpr int kDecPkBytes = 32768;         // 128 rows x 256 packed bytes (K = 512)
constexpr int kDecScBytes = 2048;          // 128 rows x 16 scale bytes
constexpr int kDecBBytes = 8 * 1024;       // 8 token rows x 512 FP16 (8 boxes of 8 x 128 B)
constexpr int kDecStageBytes = kDecPkBytes + kDecScBytes + kDecBBytes;
constexpr int kDecBarBytes = 256;  // full, ready, empty barriers + per-stage fast flags
static_assert(kDecStages * (3 * 8 + 4) <= kDecBarBytes, "barrier area");
constexpr int kDecRedBytes = 2 * 8 * 32 * 4 * 4 + 2 * 8 * 4;  // [parity][pair][lane][4] sums + flags
constexpr int kDecSmem = 1024 + kDecStages * kDecStageBytes + kDecBarBytes + kDecRedBytes;
static_assert(kDecSmem <= 232448, "shared memory budget");

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
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

// Block scale for the FP16-rounded dequant path: FP16(value * 2^(s-127)).
struct Scale {
    uint32_t h2;   // f16x2 scale when 2^(s-127) is an exact binary16
    float f;       // FP32 scale otherwise
    bool fast;
};

__device__ __forceinline__ Scale make_scale(uint32_t sbyte) {
    Scale s;
    s.fast = sbyte >= 103u && sbyte <= 142u;
    const int e = static_cast<int>(sbyte) - 127;
    const uint32_t sh = s.fast ? (e >= -14 ? static_cast<uint32_t>(e + 15) << 10 : 1u << (e + 24)) : 0u;
    s.h2 = sh | (sh << 16);
    s.f = scale_value(sbyte);
    return s;
}

// Four packed bytes -> four f16x2 (unscaled E2M1 values, exact in FP16).
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

// f16x2 of unscaled E2M1 values -> FP16(value * 2^(s-127)), as the reference
// dequant kernel rounds them (cuda_convert.cu:245).
__device__ __forceinline__ uint32_t dequant_f16(uint32_t r, const Scale& s) {
    if (s.fast) return hmul2(r, s.h2);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r));
    const __half lo = __float2half_rn(f.x * s.f);
    const __half hi = __float2half_rn(f.y * s.f);
    return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

__device__ __forceinline__ void mma_16816_acc(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816_zero(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Per byte of w: bit 7 of the result is set iff the byte lies in [104, 140]
// (SWAR: add 24 to every byte without carries between bytes, then the byte
// must read 128..164).
__device__ __forceinline__ uint32_t scale_bytes_exact(uint32_t w) {
    const uint32_t y = ((w & 0x7F7F7F7Fu) + 0x18181818u) ^ (w & 0x80808080u);
    const uint32_t z = (y & 0x7F7F7F7Fu) + 0x5B5B5B5Bu;
    return y & ~z & 0x80808080u;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ float silu_ref(float g) {
    return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
}

struct DecItem {
    int m;
    TileDesc td;
    int slot;
    bool valid;
};

__device__ __forceinline__ DecItem dec_item(const GemmArgs& a, int item) {
    DecItem d;
    const int tile = item / a.m_tiles;
    d.m = item - tile * a.m_tiles;
    d.td = a.tiles[tile];
    const int e = d.td.expert;
    int slot = -1;
    if (e >= 0 && e < a.num_experts) slot = a.slot_of[e];
    d.valid = slot >= 0 && slot < a.num_slots && d.td.n_rows > 0 && d.td.n_rows <= 8;
    d.slot = (slot < 0 || slot >= a.num_slots) ? 0 : slot;
    return d;
}

template <GemmMode MODE>
__global__ void __launch_bounds__(kDecThreads, 1)
    moe_decode_kernel(const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1,
                      const __grid_constant__ CUtensorMap map_s0, const __grid_constant__ CUtensorMap map_s1,
                      const __grid_constant__ CUtensorMap map_b, const GemmArgs args) {
    constexpr bool kGU = MODE == GemmMode::kGateUp;
    if (kGU) pdl_wait();
    const int n_items = *args.n_tiles * args.m_tiles;
    if (static_cast<int>(blockIdx.x) >= n_items) {
        if (!kGU) pdl_wait();
        pdl_trigger();
        return;
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
    uint64_t* ready = full + kDecStages;
    uint64_t* empty = ready + kDecStages;
    volatile int* fast_flag = reinterpret_cast<volatile int*>(empty + kDecStages);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kDecStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&ready[i], 1);
            mbar_init(&empty[i], kDecConsumerWarps);
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&map_w0);
        prefetch_tmap(&map_s0);
        prefetch_tmap(&map_b);
        if (kGU) { prefetch_tmap(&map_w1); prefetch_tmap(&map_s1); }
    }
    __syncthreads();
    if (!kGU && warp != 0) pdl_wait();
    pdl_trigger();
    const int k_stages = args.k_total / kKStage;
    uint32_t* status = args.status;
    const uint32_t smem_base = smem_u32(smem);

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane != 0) return;
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_b = policy_evict_last();
        // the down GEMM's token operand is the gate/up output
        if (!kGU) pdl_wait();
        int st = 0;
        uint32_t ph = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const DecItem it = dec_item(args, item);
            if (!it.valid) atomicOr(status, kStatusBadExpert);
            for (int s = 0; s < k_stages; ++s) {
                if (!mbar_wait(&empty[st], ph ^ 1, status, kStatusTimeoutTma)) return;
                mbar_arrive_expect_tx(&full[st], kDecStageBytes);
                uint8_t* pk = smem + st * kDecStageBytes;
                uint8_t* sc = pk + kDecPkBytes;
                uint8_t* bt = sc + kDecScBytes;
                const int xk = s * (kKStage / 2);
                if (kGU) {
                    const int row = it.m * 64;
                    tma_load_3d(pk, &map_w0, &full[st], xk, row, it.slot, pol_w);
                    tma_load_3d(pk + 8192, &map_w1, &full[st], xk, row, it.slot, pol_w);
                    tma_load_3d(pk + 16384, &map_w0, &full[st], xk + 128, row, it.slot, pol_w);
                    tma_load_3d(pk + 24576, &map_w1, &full[st], xk + 128, row, it.slot, pol_w);
                    tma_load_3d(sc, &map_s0, &full[st], s * 16, row, it.slot, pol_w);
                    tma_load_3d(sc + 1024, &map_s1, &full[st], s * 16, row, it.slot, pol_w);
                } else {
                    const int row = it.m * 128;
                    tma_load_3d(pk, &map_w0, &full[st], xk, row, it.slot, pol_w);
                    tma_load_3d(pk + 16384, &map_w0, &full[st], xk + 128, row, it.slot, pol_w);
                    tma_load_3d(sc, &map_s0, &full[st], s * 16, row, it.slot, pol_w);
                }
                for (int j = 0; j < 8; ++j)
                    tma_load_2d(bt + j * 1024, &map_b, &full[st], s * kKStage + j * 64,
                                it.td.row_start, pol_b);
                if (++st == kDecStages) { st = 0; ph ^= 1; }
            }
        }
        return;
    }

    if (warp == kDecCheckerWarp) {
        // ---------------- scale checker ----------------
        // Scale bytes 104..140 make every E2M1 x 2^(s-127) product an exact,
        // finite binary16, so scaling a block's FP32 partial sum equals
        // summing the reference's FP16-rounded weights.  Byte 103 rounds
        // 0.5 x 2^-24 and bytes >= 141 overflow in the reference dequant.  The
        // checker reads each stage's 2 KB of scale bytes once and publishes
        // whether all of them are in range; the consumers start the stage
        // only after that.
        int st = 0;
        uint32_t ph = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            for (int s = 0; s < k_stages; ++s) {
                const bool ok = mbar_wait(&full[st], ph, status, kStatusTimeoutDequant);
                if (!__all_sync(0xffffffffu, ok)) return;
                const uint32_t sc = smem_base + st * kDecStageBytes + kDecPkBytes + lane * 64;
                uint32_t acc = 0x80808080u;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = lds_v4(sc + i * 16);
                    acc &= scale_bytes_exact(v.x) & scale_bytes_exact(v.y) & scale_bytes_exact(v.z) &
                           scale_bytes_exact(v.w);
                }
                const bool fast = __all_sync(0xffffffffu, acc == 0x80808080u);
                if (lane == 0) {
                    fast_flag[st] = fast ? 1 : 0;
                    mbar_arrive(&ready[st]);
                }
                if (++st == kDecStages) { st = 0; ph ^= 1; }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    // K inside each 32-wide scale block is assigned so that thread q owns
    // packed bytes 4q..4q+3 (K 8q..8q+7): its A fragments come from one
    // 32-bit word per row and its token fragments for both k16 steps from
    // one 16-byte slice of the token row.  A and B use the same assignment,
    // so the MMA's sum is unchanged.  MMA column n reads token row
    // pi(n) = 4*(n&1) + n/2 of the stage, which puts the two lane groups of
    // each 128-bit shared-memory phase in opposite halves of the swizzle.
    const int cw = (warp - 1) & 7;  // 16-row MMA tile of the item
    const int kh = (warp - 1) >> 3;  // half of each stage's K
    const int g = lane >> 2;        // fragment row within 8 / MMA column
    const int q = lane & 3;
    const int row_lo = kGU ? (8 * cw + g) : (16 * cw + g);
    constexpr uint32_t kHi = kGU ? 64 * 128 : 8 * 128;  // byte distance of the hi row
    const int brow = ((g & 1) << 2) | (g >> 1);
    // Stage-relative byte offsets.  Rows are 128 B and row & 7 == g, so chunk
    // j of a weight row sits at (j ^ g) * 16: with g * 16 folded into w_off
    // (whose bits 4-6 are otherwise zero) the address of chunk j is
    // (stage + w_off) ^ (j * 16), for the lo and hi rows alike.
    const uint32_t w_off = kh * 16384 + row_lo * 128 + (g << 4) + q * 4;
    const uint32_t s_off = kDecPkBytes + row_lo * 16 + kh * 8;
    const uint32_t b_off0 = kDecPkBytes + kDecScBytes + kh * 4096 + brow * 128 + ((q ^ brow) << 4);
    const uint32_t b_off1 = kDecPkBytes + kDecScBytes + kh * 4096 + brow * 128 + (((4 + q) ^ brow) << 4);
    float* red = reinterpret_cast<float*>(smem + kDecStages * kDecStageBytes + kDecBarBytes);
    int* red_ok = reinterpret_cast<int*>(red + 2 * 8 * 32 * 4);
    int st = 0, parity = 0;
    uint32_t ph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const DecItem it = dec_item(args, item);
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        bool ok = true;
        for (int s = 0; s < k_stages; ++s) {
            ok = mbar_wait(&ready[st], ph, status, kStatusTimeoutDequant);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            const uint32_t sb = smem_base + st * kDecStageBytes;
            const bool fast = fast_flag[st] != 0;
            const uint2 slo = lds_v2(sb + s_off);
            const uint2 shi = lds_v2(sb + s_off + kHi / 8);
            const uint32_t wb = sb + w_off;
            const uint32_t bb0 = sb + b_off0, bb1 = sb + b_off1;
            if (fast) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t wa = wb ^ static_cast<uint32_t>(j << 4);
                    const uint32_t wlo = lds_u32(wa);
                    const uint32_t whi = lds_u32(wa + kHi);
                    const uint4 bv = lds_v4(((j & 1) ? bb1 : bb0) + (j >> 1) * 1024);
                    uint32_t a[8];  // [lo b0..b3, hi b0..b3] as f16x2
                    cvt_e2m1x8(wlo, a[0], a[1], a[2], a[3]);
                    cvt_e2m1x8(whi, a[4], a[5], a[6], a[7]);
                    float t[4];
                    mma_16816_zero(t, a[0], a[4], a[1], a[5], bv.x, bv.y);
                    mma_16816_acc(t, a[2], a[6], a[3], a[7], bv.z, bv.w);
                    const uint32_t sl = ((j < 4 ? slo.x : slo.y) >> (8 * (j & 3))) & 0xFFu;
                    const uint32_t sh = ((j < 4 ? shi.x : shi.y) >> (8 * (j & 3))) & 0xFFu;
                    const float flo = __uint_as_float(sl << 23);
                    const float fhi = __uint_as_float(sh << 23);
                    c[0] = fmaf(flo, t[0], c[0]);
                    c[1] = fmaf(flo, t[1], c[1]);
                    c[2] = fmaf(fhi, t[2], c[2]);
                    c[3] = fmaf(fhi, t[3], c[3]);
                }
            } else {
#pragma unroll 1
                for (int j = 0; j < 8; ++j) {
                    const uint32_t wa = wb ^ static_cast<uint32_t>(j << 4);
                    const uint32_t wlo = lds_u32(wa);
                    const uint32_t whi = lds_u32(wa + kHi);
                    const uint4 bv = lds_v4(((j & 1) ? bb1 : bb0) + (j >> 1) * 1024);
                    const Scale s_lo = make_scale(((j < 4 ? slo.x : slo.y) >> (8 * (j & 3))) & 0xFFu);
                    const Scale s_hi = make_scale(((j < 4 ? shi.x : shi.y) >> (8 * (j & 3))) & 0xFFu);
                    uint32_t a[8];
                    cvt_e2m1x8(wlo, a[0], a[1], a[2], a[3]);
                    cvt_e2m1x8(whi, a[4], a[5], a[6], a[7]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        a[i] = dequant_f16(a[i], s_lo);
                        a[4 + i] = dequant_f16(a[4 + i], s_hi);
                    }
                    mma_16816_acc(c, a[0], a[4], a[1], a[5], bv.x, bv.y);
                    mma_16816_acc(c, a[2], a[6], a[3], a[7], bv.z, bv.w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            if (++st == kDecStages) { st = 0; ph ^= 1; }
        }
        // Pair reduction.  The slot is double buffered by item parity: the
        // second warp can only write it again after passing the next item's
        // barrier, which the first warp reaches after reading this one.  The
        // flag carries a timeout of the second warp, so neither warp waits on
        // a partner that has left.
        float* slot = red + ((parity * 8 + cw) * 32 + lane) * 4;
        if (kh == 1) {
            *reinterpret_cast<float4*>(slot) = make_float4(c[0], c[1], c[2], c[3]);
            if (lane == 0) red_ok[parity * 8 + cw] = ok ? 1 : 0;
            named_bar_arrive(1 + cw, 64);
            parity ^= 1;
            if (!ok) break;
            continue;
        }
        named_bar_sync(1 + cw, 64);
        const float4 o = *reinterpret_cast<const float4*>(slot);
        const bool ok_pair = red_ok[parity * 8 + cw] != 0;
        parity ^= 1;
        if (!ok || !ok_pair) break;
        c[0] += o.x;
        c[1] += o.y;
        c[2] += o.z;
        c[3] += o.w;
        if (!it.valid) continue;
        const int n_rows = it.td.n_rows;
        const int n0 = q, n1 = 4 + q;  // tokens of MMA columns 2q and 2q+1
        if (kGU) {
            const int feat = it.m * 64 + 8 * cw + g;
            const float lim = args.swiglu_limit;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                float gv = __half2float(__float2half_rn(c[h]));
                float uv = __half2float(__float2half_rn(c[2 + h]));
                if (lim > 0.0f) {
                    gv = fminf(gv, lim);
                    uv = fminf(fmaxf(uv, -lim), lim);
                }
                const __half sv = __float2half_rn(silu_ref(gv));
                args.act[static_cast<size_t>(it.td.row_start + n) * args.inter + feat] =
                    __float2half_rn(__fmul_rn(__half2float(sv), uv));
            }
        } else {
            const int f_lo = it.m * 128 + 16 * cw + g;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                const size_t pos = static_cast<size_t>(args.perm[it.td.row_start + n]);
                args.raw[pos * args.hidden + f_lo] = c[h];
                args.raw[pos * args.hidden + f_lo + 8] = c[2 + h];
            }
        }
    }
}

template <GemmMode MODE>
cudaError_t launch_dec(const GemmMaps& maps, const GemmArgs& args, int grid, cudaStream_t stream) {
    auto kern = moe_decode_kernel<MODE>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    return launch_pdl(kern, dim3(grid), dim3(kDecThreads), kDecSmem, stream, maps.w0, maps.w1, maps.s0,
                      maps.s1, maps.b, args);
}

}  // namespace

cudaError_t launch_moe_decode(bool gate_up, const GemmMaps& maps, const GemmArgs& args, int grid,
                              cudaStream_t stream) {
    return gate_up ? launch_dec<GemmMode::kGateUp>(maps, args, grid, stream)
                   : launch_dec<GemmMode::kDown>(maps, args, grid, stream);
}

}  // namespace dee
