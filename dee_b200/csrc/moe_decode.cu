// moe_decode.cu -- the routed-expert layer for decode-sized batches.
//
// For groups of at most 8 token rows per expert (decode), every packed
// weight byte is used by only a handful of tokens, so the kernel is bound
// by how fast weights can be streamed and turned into tensor-core operands.
// Measured on B200, the tensor-memory A path of moe_gemm.cu pays about 110
// cycles per 128x16 A slice whatever N is, and staging dequantised weights in
// shared memory would need ~5 bytes of shared-memory traffic per weight.
// Here the dequantised weights never leave registers.
//
// One persistent kernel runs a work list of gate/up items (per tile: I/64
// items of 64 gate + 64 up rows) and then down items (per tile: H/128 items
// of 128 rows), or either part alone:
//
//   warp 0       producer: per 512-wide K stage, the packed FP4 rows
//                (128 rows x 256 B) and the stage's token rows (8 rows x 1 KB)
//                into a 4-deep ring, one tensor copy per operand (the front
//                end: one bulk copy per token row, straight from x); per
//                item, the rows' UE8M0 scales by a swizzled tensor copy
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
//   warp 17      scale checker: decides per item whether every block scale
//                allows the exact FP32 scaling
//   warp 18      signal: publishes each finished item to the grid (tile
//                counters for the down items' dependency; with the fused
//                combine, per (token, 128-feature block) counters, the
//                completing row summing the block's K rows in rank order)
//   warp 19      dependency: waits (bounded) for each down item's tile to
//                have all of its gate/up items published
//
// Gate/up items pair 8 gate rows with the same 8 up rows in each 16-row MMA
// tile, so one thread holds the gate and up accumulators of the same
// (feature, token) and applies the reference's FP16 SwiGLU chain in
// registers (swiglu_cuda.cu:46-59).  Down items scatter FP32 rows to
// raw[token * K + rank] (engine.cpp:1080-1113).  The "front end" form
// (launch_moe_decode_front) also routes and groups the batch inside the
// kernel, so a small decode layer is one launch.
#include "decode_common.cuh"
#include "kernels.h"
#include "routing.cuh"

namespace dee {
namespace {

using namespace sm100;

constexpr int kDecConsumerWarps = 16;
constexpr int kDecCheckerWarp = 1 + kDecConsumerWarps;
constexpr int kDecSignalWarp = kDecCheckerWarp + 1;
constexpr int kDecDepWarp = kDecSignalWarp + 1;
constexpr int kDecThreads = 32 * (kDecDepWarp + 1);  // producer, 8 pairs of consumers, checker, signal, dependency
constexpr int kDecMaxStages = 4;
constexpr int kDecPkBytes = 32768;         // 128 rows x 256 packed bytes (K = 512)
constexpr int kDecBBytes = 8 * 1024;       // 8 token rows x 512 FP16 (8 boxes of 8 x 128 B)
constexpr int kDecStageBytes = kDecPkBytes + kDecBBytes;
constexpr int kDecBarBytes = 256;  // stage, scale-slot and signal barriers, per-slot flags and item records
constexpr int kDecRedBytes = 2 * 8 * 32 * 4 * 4 + 2 * 2 * 8 * 4;  // [parity][pair][lane][4] sums + flags
constexpr uint32_t kSmemLimit = 232448;
constexpr int kDecScSlots = 3;  // per-item scale rows: the consumed item, the next, the one after
// The front end's tables in shared memory: per tile the token of each row
// (u8), the tile (expert | row_start << 8 | n_rows << 16) and the expert's
// record slot; per grouped row its position t*K + r (u8).
constexpr int kFtTok = 0;
constexpr int kFtTile = kFtTok + kFrontMaxTiles * 8;
constexpr int kFtSlot = kFtTile + kFrontMaxTiles * 4;
constexpr int kFtPerm = kFtSlot + kFrontMaxTiles * 4;
constexpr int kDecTokBytes = (kFtPerm + kFrontMaxSel + 15) & ~15;
static_assert(kFrontMaxSel <= 256 && kFrontMaxTiles <= 256, "front-end tables hold u8 rows and positions");

// Shared-memory plan: a ring of 512-wide K stages (packed weights + token
// rows), three slots of per-item scale rows (128 rows x K/32 bytes), the
// barriers and the pair-reduction buffer.  The ring is 4 deep unless the
// scale rows are too long for that (K > 5120 takes 3).
struct DecLayout {
    int stages;
    uint32_t sc_slot;  // bytes per scale slot
    uint32_t sc_off, bar_off, red_off, bytes;
};

__host__ __device__ inline DecLayout dec_layout(int k_total) {
    DecLayout L;
    L.sc_slot = (static_cast<uint32_t>(128 * (k_total / 32)) + 1023u) & ~1023u;
    const uint32_t fixed = 1024 + kDecScSlots * L.sc_slot + kDecBarBytes + kDecRedBytes + kDecTokBytes;
    const uint32_t room = fixed < kSmemLimit ? (kSmemLimit - fixed) / kDecStageBytes : 0;
    L.stages = room < kDecMaxStages ? static_cast<int>(room) : kDecMaxStages;
    L.sc_off = L.stages * kDecStageBytes;
    L.bar_off = L.sc_off + kDecScSlots * L.sc_slot;
    L.red_off = L.bar_off + kDecBarBytes;
    L.bytes = 1024 + L.red_off + kDecRedBytes + kDecTokBytes;
    return L;
}

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

// Per byte of w: bit 7 of the result is set iff the byte lies in [104, 140]
// (SWAR: add 24 to every byte without carries between bytes, then the byte
// must read 128..164).
__device__ __forceinline__ uint32_t scale_bytes_exact(uint32_t w) {
    const uint32_t y = ((w & 0x7F7F7F7Fu) + 0x18181818u) ^ (w & 0x80808080u);
    const uint32_t z = (y & 0x7F7F7F7Fu) + 0x5B5B5B5Bu;
    return y & ~z & 0x80808080u;
}

// The tensor maps of both projections.  A one-projection launch fills the
// other projection's maps with copies it never uses.
struct DecMaps {
    CUtensorMap gw1, gw3, gx, gs1, gs3;  // gate/up: W1 and W3 rows, token rows, scale rows
    CUtensorMap dw2, dact, ds2;          // down: W2 rows, SwiGLU rows, scale rows
};

// The launch's work list: the gate/up items of every tile (tile-major, I/64
// per tile), then the down items (tile-major, H/128 per tile), either part
// empty when its phase bit is clear.
struct DecPlan {
    int n_gu, n_items, mg, md;
};

__device__ __forceinline__ DecPlan dec_plan(const GemmArgs& a, int nt) {
    DecPlan p;
    p.mg = a.inter / 64;
    p.md = a.hidden / 128;
    p.n_gu = (a.phases & 1) ? nt * p.mg : 0;
    p.n_items = p.n_gu + ((a.phases & 2) ? nt * p.md : 0);
    return p;
}

// The layout's K: the longer reduction of the phases the launch runs.
__host__ __device__ inline int dec_layout_k(const GemmArgs& a) {
    int k = 0;
    if (a.phases & 1) k = a.hidden;
    if ((a.phases & 2) && a.inter > k) k = a.inter;
    return k;
}

struct DecItem {
    int m, tile;
    TileDesc td;
    int slot;
    bool valid, gu;
};

__device__ __forceinline__ TileDesc load_tile(const TileDesc* tiles, const DecPlan& p, int item) {
    return item < p.n_gu ? tiles[item / p.mg] : tiles[(item - p.n_gu) / p.md];
}

// A tile from the front end's shared-memory table (n_pad is not used by
// the decode kernel).
__device__ __forceinline__ TileDesc front_tile(const uint8_t* ft, int tile) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(ft + kFtTile)[tile];
    TileDesc td;
    td.expert = static_cast<int>(w & 0xFFu);
    td.row_start = static_cast<int>((w >> 8) & 0xFFu);
    td.n_rows = static_cast<int>((w >> 16) & 0xFFu);
    td.n_pad = 0;
    return td;
}

// The front end's item: tile and record slot from the shared-memory tables.
__device__ __forceinline__ DecItem front_item(const GemmArgs& a, const DecPlan& p, const uint8_t* ft, int item) {
    DecItem d;
    d.gu = item < p.n_gu;
    const int j = d.gu ? item : item - p.n_gu;
    const int mt = d.gu ? p.mg : p.md;
    d.tile = j / mt;
    d.m = j - d.tile * mt;
    d.td = front_tile(ft, d.tile);
    const int slot = reinterpret_cast<const int32_t*>(ft + kFtSlot)[d.tile];
    d.valid = slot >= 0 && slot < a.num_slots && d.td.n_rows > 0 && d.td.n_rows <= 8;
    d.slot = d.valid ? slot : 0;
    return d;
}

// Completes an item from its tile descriptor: the expert's record slot and
// whether the item can run (an expert id that is out of range or not
// resident leaves the item's outputs unwritten and raises kStatusBadExpert).
__device__ __forceinline__ DecItem finish_item(const GemmArgs& a, const DecPlan& p, int item, const TileDesc& td) {
    DecItem d;
    d.gu = item < p.n_gu;
    const int j = d.gu ? item : item - p.n_gu;
    const int mt = d.gu ? p.mg : p.md;
    d.tile = j / mt;
    d.m = j - d.tile * mt;
    d.td = td;
    const int e = td.expert;
    int slot = -1;
    if (e >= 0 && e < a.num_experts) slot = a.slot_of[e];
    d.valid = slot >= 0 && slot < a.num_slots && td.n_rows > 0 && td.n_rows <= 8;
    d.slot = (slot < 0 || slot >= a.num_slots) ? 0 : slot;
    return d;
}

// What the consumers need of an item, handed over in shared memory with the
// item's scale rows.
struct ItemRec {
    int m, row_start, n_rows, valid;
};

// Bounded wait (gpu-scope acquire) for *p >= target; false and `code` in
// *status when the limit expires.
__device__ __forceinline__ bool wait_count_geq(const uint32_t* p, uint32_t target, uint32_t* status,
                                               uint32_t code) {
    const uint64_t t0 = global_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= target) return true;
        if (global_ns() - t0 > kWaitLimitNs) {
            atomicOr(status, code);
            return false;
        }
        __nanosleep(128);
    }
}

// Bounded wait (cta-scope acquire) for the shared word *p >= target.
__device__ __forceinline__ bool wait_smem_geq(const uint32_t* p, uint32_t target, uint32_t* status,
                                              uint32_t code) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    if (v >= target) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        __nanosleep(64);
        asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
        if (v >= target) return true;
        if (global_ns() - t0 > kWaitLimitNs) {
            atomicOr(status, code);
            return false;
        }
    }
}

// gpu-scope release add (no result) and acquire-release add (old value).
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_acq_rel_add(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned long long atom_acq_rel_add(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// The front end's counters advance by a fixed amount per launch: a tile
// counter by I/64 (its gate/up items, or one filler add for a tile the
// launch does not have), a (token, feature block) counter by K (its rows, or
// a filler add for a token beyond the batch).  After launch number `epoch`
// they read epoch * I/64 and epoch * K, so nothing is zeroed between calls.
// Bounded wait (gpu-scope acquire) for *p >= target.
__device__ __forceinline__ bool wait_u64_geq(const unsigned long long* p, unsigned long long target,
                                             uint32_t* status, uint32_t code) {
    const uint64_t t0 = global_ns();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
        if (v >= target) return true;
        if (global_ns() - t0 > kWaitLimitNs) {
            atomicOr(status, code);
            return false;
        }
        __nanosleep(128);
    }
}

// Address of a thread's token slice j (see consume_item).
template <bool kRowsB>
__device__ __forceinline__ uint32_t b_addr(uint32_t bb0, uint32_t bb1, int j) {
    if constexpr (kRowsB) return j == 7 ? bb1 : bb0 + (j >> 1) * 128 + (j & 1) * 64;
    else return ((j & 1) ? bb1 : bb0) + (j >> 1) * 1024;
}

// Shared-memory handles of the consumers.
struct DecSmem {
    uint8_t* smem;
    uint32_t base;
    uint64_t *full, *empty, *sready, *sempty, *stored, *sfree;
    volatile int* fast_flag;
    volatile ItemRec* item_rec;
    float* red;
    int* red_ok;
};

// One work item of one consumer warp: the K stages, the pair reduction and
// (first warp of the pair) the epilogue; with `signal`, the first warps then
// hand the item to the signal warp.  Returns false when a wait gave up.
// kRowsB: the gate/up token rows sit row-major in the stage (one 1 KB row
// per token, rows 4-7 rotated by 64 bytes within their row) as the bulk
// copies from x place them, instead of the 128-byte-swizzled box.  kPerm8:
// grouped positions come from the front end's shared-memory table.
template <bool kGU, bool kOfficial, bool kRowsB, bool kPerm8>
__device__ __forceinline__ bool consume_item(const GemmArgs& args, const DecLayout& L, const DecSmem& S, int li,
                                             int& st, uint32_t& ph, int& parity, int n_stages, bool signal,
                                             int warp, int lane, const int* perm, const uint8_t* perm8) {
    uint32_t* status = args.status;
    const int k_total = kGU ? args.hidden : args.inter;
    const int k_stages = k_total / kKStage;
    const uint32_t rb = static_cast<uint32_t>(k_total / 32);  // scale bytes per weight row
    const int swz = kGU ? args.scale_swz : args.dn_scale_swz;
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
    // Stage weights: gate/up as [W1: K half 0 | K half 1][W3: ...], 64 rows
    // of 128 B each; down as [K half 0 | K half 1] of 128 rows.
    constexpr uint32_t kHalf = kGU ? 8192 : 16384;     // bytes per K half of one projection
    constexpr uint32_t kHiRows = kGU ? 64 : 8;         // rows between the lo and hi fragment rows
    constexpr uint32_t kHi = kGU ? 16384 : 8 * 128;    // their byte distance in a stage
    const int brow = ((g & 1) << 2) | (g >> 1);
    // Stage-relative byte offsets.  Rows are 128 B and row & 7 == g, so chunk
    // j of a weight row sits at (j ^ g) * 16: with g * 16 folded into w_off
    // (whose bits 4-6 are otherwise zero) the address of chunk j is
    // (stage + w_off) ^ (j * 16), for the lo and hi rows alike.
    const uint32_t w_off = kh * kHalf + row_lo * 128 + (g << 4) + q * 4;
    // Token fragments: the 16-byte slice j of this thread's row.  Swizzled
    // box: chunk (j>>1) of the half at b_off0 / b_off1 by the parity of j.
    // Row-major rows: K offset kh*512 + (j>>1)*128 + (j&1)*64 + q*16 plus the
    // row's rotation, which wraps (to q*16) only for j = 7 of the second half
    // of a rotated row, so j = 7 gets its own base.  Rows brow and brow + 4
    // of a shared-memory phase differ by 64 bytes: distinct banks.
    uint32_t b_off0, b_off1;
    if constexpr (kGU && kRowsB) {
        const uint32_t rot = (brow & 4) ? 64u : 0u;
        b_off0 = kDecPkBytes + brow * 1024 + kh * 512 + rot + q * 16;
        b_off1 = kDecPkBytes + brow * 1024 + ((kh * 512 + 448 + q * 16 + rot) & 1023u);
    } else {
        b_off0 = kDecPkBytes + kh * 4096 + brow * 128 + ((q ^ brow) << 4);
        b_off1 = kDecPkBytes + kh * 4096 + brow * 128 + (((4 + q) ^ brow) << 4);
    }
    // this thread's scale bytes of stage s: row_lo * rb + s * 16 + kh * 8 in
    // the slot, the 16-byte chunk s moved to s ^ sw when the rows came in
    // swizzled (sw from the row's address bits 7 and up, as the tensor copy
    // placed them; the hi row, 64 or 8 rows on, has the same sw)
    const uint32_t s_off = L.sc_off + row_lo * rb + kh * 8;
    const uint32_t s_hi = kHiRows * rb;
    const uint32_t s_sw = swz ? ((row_lo * rb) >> 7) & (rb / 16 - 1) : 0u;

    const int slot = li % kDecScSlots;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = mbar_wait(&S.sready[slot], (li / kDecScSlots) & 1, status, kStatusTimeoutDequant);
    ok = __all_sync(0xffffffffu, ok);
    // official semantics dequantise in FP32: the scaled FP32 partial sum
    // is exact for every scale byte
    const bool fast = ok && (kOfficial || S.fast_flag[slot] != 0);
    const int it_m = S.item_rec[slot].m;
    const int it_row_start = S.item_rec[slot].row_start;
    const int it_n_rows = S.item_rec[slot].n_rows;
    const bool it_valid = S.item_rec[slot].valid != 0;
    const uint32_t sc_base = S.base + s_off + slot * L.sc_slot;
    for (int s = 0; s < k_stages && ok; ++s) {
        ok = mbar_wait(&S.full[st], ph, status, kStatusTimeoutDequant);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        const uint32_t sb = S.base + st * kDecStageBytes;
        const uint32_t s_chunk = (static_cast<uint32_t>(s) ^ s_sw) << 4;
        const uint2 slo = lds_v2(sc_base + s_chunk);
        const uint2 shi = lds_v2(sc_base + s_chunk + s_hi);
        const uint32_t wb = sb + w_off;
        const uint32_t bb0 = sb + b_off0, bb1 = sb + b_off1;
        if (fast) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t wa = wb ^ static_cast<uint32_t>(j << 4);
                const uint32_t wlo = lds_u32(wa);
                const uint32_t whi = lds_u32(wa + kHi);
                const uint4 bv = lds_v4(b_addr<kGU && kRowsB>(bb0, bb1, j));
                uint32_t a[8];  // [lo b0..b3, hi b0..b3] as f16x2
                cvt_e2m1x8(wlo, a[0], a[1], a[2], a[3]);
                cvt_e2m1x8(whi, a[4], a[5], a[6], a[7]);
                float t[4];
                mma_16816_zero(t, a[0], a[4], a[1], a[5], bv.x, bv.y);
                mma_16816_acc(t, a[2], a[6], a[3], a[7], bv.z, bv.w);
                const uint32_t sl = ((j < 4 ? slo.x : slo.y) >> (8 * (j & 3))) & 0xFFu;
                const uint32_t sh = ((j < 4 ? shi.x : shi.y) >> (8 * (j & 3))) & 0xFFu;
                const float flo = kOfficial ? e8m0_value(sl) : __uint_as_float(sl << 23);
                const float fhi = kOfficial ? e8m0_value(sh) : __uint_as_float(sh << 23);
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
                const uint4 bv = lds_v4(b_addr<kGU && kRowsB>(bb0, bb1, j));
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
        if (lane == 0) mbar_arrive(&S.empty[st]);
        if (++st == n_stages) { st = 0; ph ^= 1; }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.sempty[slot]);
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
    float* rslot = S.red + ((parity * 8 + cw) * 32 + lane) * 4;
    if (kh == 1) *reinterpret_cast<float4*>(rslot) = make_float4(c[0], c[1], c[2], c[3]);
    if (lane == 0) S.red_ok[(parity * 2 + kh) * 8 + cw] = ok ? 1 : 0;
    named_bar_sync(1 + cw, 64);
    const bool ok_pair = S.red_ok[(parity * 2 + (kh ^ 1)) * 8 + cw] != 0;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kh == 0) o = *reinterpret_cast<const float4*>(rslot);
    parity ^= 1;
    if (!ok || !ok_pair) return false;
    if (kh == 1) return true;
    c[0] += o.x;
    c[1] += o.y;
    c[2] += o.z;
    c[3] += o.w;
    if (it_valid) {
        const int n_rows = it_n_rows;
        const int n0 = q, n1 = 4 + q;  // tokens of MMA columns 2q and 2q+1
        if (kGU) {
            const int feat = it_m * 64 + 8 * cw + g;
            const float lim = args.swiglu_limit;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                const float w = (kOfficial && args.route_w)
                                    ? args.route_w[kPerm8 ? perm8[it_row_start + n] : perm[it_row_start + n]]
                                    : 1.0f;
                args.act[static_cast<size_t>(it_row_start + n) * args.inter + feat] =
                    swiglu_out(c[h], c[2 + h], lim, kOfficial, w);
            }
        } else {
            const int f_lo = it_m * 128 + 16 * cw + g;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int n = h ? n1 : n0;
                if (n >= n_rows) continue;
                const int pos = kPerm8 ? static_cast<int>(perm8[it_row_start + n]) : perm[it_row_start + n];
                float* dst;
                if (args.raw_peers) {  // straight into the token owner's return buffer
                    const int src = pos / args.ep_capacity;
                    const int rslot_ep = pos - src * args.ep_capacity;
                    dst = args.raw_peers[src] +
                          static_cast<size_t>(args.ep_rank * args.ep_capacity + rslot_ep) * args.hidden;
                } else {
                    dst = args.raw + static_cast<size_t>(pos) * args.hidden;
                }
                dst[f_lo] = c[h];
                dst[f_lo + 8] = c[2 + h];
            }
        }
    }
    if (signal) {
        // the item's stores are done in this warp; the signal warp publishes
        // them (one arrival per first warp; a buffer is reused two items on,
        // after the signal warp has released it)
        __syncwarp();
        bool sok = true;
        if (lane == 0) {
            const int b = li & 1;
            if (li >= 2) sok = mbar_wait(&S.sfree[b], ((li >> 1) - 1) & 1, status, kStatusTimeoutEpilogue);
            if (sok) mbar_arrive(&S.stored[b]);
        }
        if (!__shfl_sync(0xffffffffu, sok, 0)) return false;  // the whole warp leaves together
    }
    return true;
}

// The front end's router and grouping, run by every thread of every CTA on
// the same inputs (so every CTA derives the same tile list without a grid
// barrier).  The scratch lives in the stage ring, which nothing uses yet.
// Routing: route_token per token (one warp each), as route_topk_kernel.
// Grouping: selections enumerated j = rank * T + token and placed stably by
// expert id (engine.cpp:812-823), tiles of at most kDecodeTileRows rows split
// evenly, as permute_block.  Outputs: the shared-memory tables (each tile,
// its record slot and its rows' tokens; each grouped row's position) and the
// combine weights by position in this CTA's slice of the scratch; CTA 0 also writes
// the caller's ids, weights and journal.  Returns the number of tiles.
__device__ int front_route_group(const GemmArgs& a, const DecFront& f, uint8_t* smem, uint8_t* ft) {
    const int T = f.tokens, K = a.topk, E = a.num_experts, sel = T * K;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int32_t* s_ids = reinterpret_cast<int32_t*>(smem);              // [kFrontMaxSel] by position
    float* s_w = reinterpret_cast<float*>(s_ids + kFrontMaxSel);    // [kFrontMaxSel] by position
    int* s_ej = reinterpret_cast<int*>(s_w + kFrontMaxSel);         // [kFrontMaxSel] expert of selection j
    int* cnt = s_ej + kFrontMaxSel;                                 // [256]
    int* off = cnt + 256;                                           // [257]
    int* toff = off + 257;                                          // [257]
    float* sp = reinterpret_cast<float*>(smem + 8192);              // [warps][256] router scratch
    if (f.logits) {
        for (int t = warp; t < T; t += kDecThreads / 32)
            route_token<8>(f.logits + static_cast<size_t>(t) * E, E, K, lane, sp + warp * 256, s_ids + t * K,
                           s_w + t * K, nullptr, a.status);
    } else {
        // ids and weights from the caller (or a router kernel before this
        // one); an id outside [0, E) is reported and its selection left out
        for (int p = tid; p < sel; p += kDecThreads) {
            const int e = f.ids_out[p];
            if (e < 0 || e >= E) atomicOr(a.status, kStatusBadExpert);
            s_ids[p] = (e < 0 || e >= E) ? -1 : e;
            s_w[p] = f.weights_out ? f.weights_out[p] : 0.0f;
        }
    }
    __syncthreads();
    for (int j = tid; j < sel; j += kDecThreads) {
        const int r = j / T, t = j - r * T;
        s_ej[j] = s_ids[t * K + r];
    }
    for (int e = tid; e < E; e += kDecThreads) {
        int c = 0;
        for (int p = 0; p < sel; ++p) c += s_ids[p] == e;
        cnt[e] = c;
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scans of the group sizes and of the tiles per group
        const int per = (E + 31) / 32;
        int sum = 0, sum_t = 0;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < E) {
                sum += cnt[e];
                sum_t += (cnt[e] + kDecodeTileRows - 1) / kDecodeTileRows;
            }
        }
        int incl = sum, incl_t = sum_t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, o);
            const int y = __shfl_up_sync(0xffffffffu, incl_t, o);
            if (lane >= o) { incl += x; incl_t += y; }
        }
        int run = incl - sum, run_t = incl_t - sum_t;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < E) {
                off[e] = run;
                toff[e] = run_t;
                run += cnt[e];
                run_t += (cnt[e] + kDecodeTileRows - 1) / kDecodeTileRows;
            }
        }
        if (lane == 31) { off[E] = incl; toff[E] = incl_t; }
    }
    __syncthreads();
    // combine weights by position: this CTA's slice of the scratch
    float* scr_w = reinterpret_cast<float*>(f.scratch + static_cast<size_t>(blockIdx.x) * kFrontScratchInts);
    uint8_t* ft_tok = ft + kFtTok;
    uint32_t* ft_tile = reinterpret_cast<uint32_t*>(ft + kFtTile);
    int32_t* ft_slot = reinterpret_cast<int32_t*>(ft + kFtSlot);
    uint8_t* ft_perm = ft + kFtPerm;
    for (int j = tid; j < sel; j += kDecThreads) {
        const int e = s_ej[j];
        if (e < 0) continue;  // a bad caller id: left out (reported above)
        int rank = 0;
        for (int j2 = 0; j2 < j; ++j2) rank += s_ej[j2] == e;
        const int r = j / T, t = j - r * T;
        ft_perm[off[e] + rank] = static_cast<uint8_t>(t * K + r);
        scr_w[t * K + r] = s_w[t * K + r];
        // the row's token, by tile and row within the tile (tiles split the
        // expert's rows evenly, as below)
        const int c = cnt[e];
        const int ntl = (c + kDecodeTileRows - 1) / kDecodeTileRows;
        const int sz = (c + ntl - 1) / ntl;
        ft_tok[(toff[e] + rank / sz) * 8 + rank % sz] = static_cast<uint8_t>(t);
    }
    for (int e = tid; e < E; e += kDecThreads) {
        const int c = cnt[e];
        if (c == 0) continue;
        const int ntl = (c + kDecodeTileRows - 1) / kDecodeTileRows;
        const int sz = (c + ntl - 1) / ntl;
        const int slot = a.slot_of[e];
        for (int i = 0; i < ntl; ++i) {
            const int n = min(sz, c - i * sz);
            ft_tile[toff[e] + i] = static_cast<uint32_t>(e) | static_cast<uint32_t>(off[e] + i * sz) << 8 |
                                   static_cast<uint32_t>(n) << 16;
            ft_slot[toff[e] + i] = slot;
        }
    }
    const int nt = toff[E];
    if (blockIdx.x == 0) {
        for (int p = tid; p < sel; p += kDecThreads) {
            if (f.logits) {
                f.ids_out[p] = s_ids[p];
                f.weights_out[p] = s_w[p];
            }
            if (f.journal) f.journal[p] = f.logits ? s_ids[p] : f.ids_out[p];
        }
        // filler adds: the counters of tiles this launch does not have
        // advance like the others (relaxed; nothing waits on them in this
        // launch, and the next launch starts after this one completes)
        const int md = a.hidden / 128;
        for (int t = nt + tid; t < kFrontMaxTiles; t += kDecThreads)
            atomicAdd(f.ctr + t, static_cast<unsigned long long>(a.inter / 64));
        // a selection left out still counts for its token's blocks; the add
        // that completes a block resets it, as the combining one does.  (A
        // launch without the combine adds nothing to these counters, so
        // neither does its filler: a raw-only call leaves them at zero.)
        for (int i = tid; a.comb_out && i < sel * md; i += kDecThreads) {
            if (s_ids[i / md] >= 0) continue;
            unsigned long long* c = f.ctr + kFrontMaxTiles + (i / md / K) * md + i % md;
            if (atomicAdd(c, 1ull) + 1 == static_cast<unsigned long long>(K)) atomicExch(c, 0ull);
        }
    }
    __syncthreads();
    return nt;
}

// Token rows of a launch: kModeBox, the grouped rows (gather kernel) by one
// swizzled box per stage; kModeFront, the front end (routing and grouping
// inside, token rows straight from x by bulk copies).  (Bulk copies from x
// after the permutation kernel, without the gather, measured slower at
// b = 8 -- 137.7 against 129.8 us on one B200, reproduced: eight 1 KB
// copies per stage cost more than one 8 KB box -- and equal at b = 1.)
constexpr int kModeBox = 0, kModeFront = 1;

template <bool kOfficial, int kMode>
__global__ void __launch_bounds__(kDecThreads, 1)
    moe_decode_kernel(const __grid_constant__ DecMaps maps, const GemmArgs args,
                      const __grid_constant__ DecFront front) {
    constexpr bool kFront = kMode == kModeFront;
    constexpr bool kRows = kMode != kModeBox;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    // The work list.  Without the front end the tile list comes from the
    // permutation kernel, which has completed whenever this kernel runs: its
    // predecessor (gather or gate/up) only signals its dependents after its
    // own griddepcontrol.wait.  Everything that reads weights or the tile
    // list may therefore start before this kernel's wait; only the token rows
    // (the predecessor's output) and the counters the permutation zeroed
    // wait.  The front end waits first and derives the list itself, into
    // shared-memory tables (after the barriers are set up and the tensor
    // maps prefetched, so that the first copies follow the grouping at once).
    const DecLayout L = dec_layout(dec_layout_k(args));
    DecPlan P;
    if constexpr (!kFront) {
        P = dec_plan(args, *args.n_tiles);
        if (static_cast<int>(blockIdx.x) >= P.n_items) {
            pdl_wait();
            pdl_trigger();
            return;
        }
    }
    uint8_t* ft = smem + L.red_off + kDecRedBytes;  // front-end tables
    const int n_stages = L.stages;
    DecSmem S;
    S.smem = smem;
    S.base = smem_u32(smem);
    S.full = reinterpret_cast<uint64_t*>(smem + L.bar_off);  // [stages] TMA landed
    S.empty = S.full + kDecMaxStages;                         // [stages] consumers done
    uint64_t* sfull = S.empty + kDecMaxStages;                // [slots] scale rows landed
    S.sready = sfull + kDecScSlots;                           // [slots] scale rows checked
    S.sempty = S.sready + kDecScSlots;                        // [slots] item consumed
    S.fast_flag = reinterpret_cast<volatile int*>(S.sempty + kDecScSlots);            // [slots]
    S.item_rec = reinterpret_cast<volatile ItemRec*>(smem + L.bar_off + 160);         // [slots]
    S.stored = reinterpret_cast<uint64_t*>(smem + L.bar_off + 208);  // [2] an item's outputs stored
    S.sfree = S.stored + 2;                                          // [2] signal warp done with it
    // down items of this CTA whose tiles' gate/up items are all published
    uint32_t* dep_ready = reinterpret_cast<uint32_t*>(smem + L.bar_off + 240);
    S.red = reinterpret_cast<float*>(smem + L.red_off);
    S.red_ok = reinterpret_cast<int*>(S.red + 2 * 8 * 32 * 4);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool gu_on = (args.phases & 1) != 0, dn_on = (args.phases & 2) != 0;
    // the down items of a two-phase launch wait for their tile's gate/up items
    const bool dep = gu_on && dn_on && (kFront || args.tile_done != nullptr);
    const bool signal = dep || args.comb_out != nullptr;
    if (threadIdx.x == 0) {
        for (int i = 0; i < n_stages; ++i) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], kDecConsumerWarps);
        }
        for (int i = 0; i < kDecScSlots; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&S.sready[i], 1);
            mbar_init(&S.sempty[i], kDecConsumerWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.stored[i], kDecConsumerWarps / 2);
            mbar_init(&S.sfree[i], 1);
        }
        *dep_ready = 0u;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        if (gu_on) {
            prefetch_tmap(&maps.gw1);
            prefetch_tmap(&maps.gw3);
            prefetch_tmap(&maps.gx);
            if (args.scale_swz) {
                prefetch_tmap(&maps.gs1);
                prefetch_tmap(&maps.gs3);
            }
        }
        if (dn_on) {
            prefetch_tmap(&maps.dw2);
            prefetch_tmap(&maps.dact);
            if (args.dn_scale_swz) prefetch_tmap(&maps.ds2);
        }
    }
    __syncthreads();
    if constexpr (kFront) {
        pdl_wait();
        pdl_trigger();
        P = dec_plan(args, front_route_group(args, front, smem, ft));
        if (static_cast<int>(blockIdx.x) >= P.n_items) return;
    } else {
        if (warp != 0) pdl_wait();
        pdl_trigger();
    }
    const int n_items = P.n_items;
    const TileDesc* tiles = args.tiles;
    const int* perm = args.perm;
    const float* comb_w = kFront ? reinterpret_cast<const float*>(front.scratch + static_cast<size_t>(blockIdx.x) *
                                                                                     kFrontScratchInts)
                                 : args.comb_w;
    const uint8_t* ft_perm = ft + kFtPerm;
    uint32_t* status = args.status;
    const int H = args.hidden, I = args.inter;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane != 0) return;
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_b = policy_evict_last();
        const size_t ih = static_cast<size_t>(H) * I;
        const size_t off_s1 = ih + ih / 2, off_s3 = off_s1 + ih / 32, off_s2 = off_s3 + ih / 32;
        // Scale rows of one item are contiguous in the record: one copy per
        // projection into the item's slot, after the item's record for the
        // consumers.  With scale maps (rows of 32, 64 or 128 bytes) the copy
        // is a tensor load whose swizzle span is the row length, so the
        // 16-byte chunk j of row r lands at chunk j ^ f(r) and the
        // consumers' per-stage reads of eight rows hit distinct banks;
        // otherwise a plain bulk copy.
        auto issue_scales = [&](const DecItem& d, int li) -> bool {
            const int slot = li % kDecScSlots;
            if (!mbar_wait(&S.sempty[slot], ((li / kDecScSlots) & 1) ^ 1, status, kStatusTimeoutTma))
                return false;
            S.item_rec[slot].m = d.m;
            S.item_rec[slot].row_start = d.td.row_start;
            S.item_rec[slot].n_rows = d.td.n_rows;
            S.item_rec[slot].valid = d.valid ? 1 : 0;
            const uint32_t rb = static_cast<uint32_t>((d.gu ? H : I) / 32);
            mbar_arrive_expect_tx(&sfull[slot], 128 * rb);
            uint8_t* dst = smem + L.sc_off + slot * L.sc_slot;
            const uint8_t* rec = args.records + static_cast<size_t>(d.slot) * args.record_bytes;
            if (d.gu) {
                if (args.scale_swz) {
                    tma_load_3d(dst, &maps.gs1, &sfull[slot], 0, d.m * 64, d.slot, pol_w);
                    tma_load_3d(dst + 64 * rb, &maps.gs3, &sfull[slot], 0, d.m * 64, d.slot, pol_w);
                } else {
                    const size_t r0 = static_cast<size_t>(d.m) * 64 * rb;
                    bulk_load(dst, rec + off_s1 + r0, 64 * rb, &sfull[slot]);
                    bulk_load(dst + 64 * rb, rec + off_s3 + r0, 64 * rb, &sfull[slot]);
                }
            } else if (args.dn_scale_swz) {
                tma_load_3d(dst, &maps.ds2, &sfull[slot], 0, d.m * 128, d.slot, pol_w);
            } else {
                bulk_load(dst, rec + off_s2 + static_cast<size_t>(d.m) * 128 * rb, 128 * rb, &sfull[slot]);
            }
            return true;
        };
        // weights: {128 B, rows, two 128-byte K chunks, slot} per projection;
        // tokens: {64, 8 rows, eight 64-wide K chunks}
        auto issue_weights = [&](const DecItem& d, int s, int st) {
            uint8_t* pk = smem + st * kDecStageBytes;
            if (d.gu) {
                tma_load_4d(pk, &maps.gw1, &S.full[st], 0, d.m * 64, 2 * s, d.slot, pol_w);
                tma_load_4d(pk + 16384, &maps.gw3, &S.full[st], 0, d.m * 64, 2 * s, d.slot, pol_w);
            } else {
                tma_load_4d(pk, &maps.dw2, &S.full[st], 0, d.m * 128, 2 * s, d.slot, pol_w);
            }
        };
        // front end, gate/up: each token row's 1 KB of the stage by bulk copy
        // straight from x into row n of the stage (rows 4-7 rotated by 64
        // bytes: two copies); otherwise one box of the grouped rows
        auto issue_tokens = [&](const DecItem& d, int s, int st) {
            uint8_t* bdst = smem + st * kDecStageBytes + kDecPkBytes;
            if (kRows && d.gu) {
                const uint8_t* x = reinterpret_cast<const uint8_t*>(front.x);
                const uint8_t* toks = ft + kFtTok + d.tile * 8;  // the tile rows' tokens
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    if (n >= d.td.n_rows) break;
                    const int tok = toks[n];
                    const uint8_t* src = x + (static_cast<size_t>(tok) * H + static_cast<size_t>(kKStage) * s) * 2;
                    uint8_t* dst = bdst + n * 1024;
                    if (n & 4) {
                        bulk_load(dst + 64, src, 960, &S.full[st]);
                        bulk_load(dst, src + 960, 64, &S.full[st]);
                    } else {
                        bulk_load(dst, src, 1024, &S.full[st]);
                    }
                }
            } else {
                tma_load_3d(bdst, d.gu ? &maps.gx : &maps.dact, &S.full[st], 0, d.td.row_start, 8 * s, pol_b);
            }
        };
        auto stage_bytes = [&](const DecItem& d) -> uint32_t {
            return (kRows && d.gu) ? static_cast<uint32_t>(kDecPkBytes + d.td.n_rows * 1024) : kDecStageBytes;
        };
        auto stages_of = [&](const DecItem& d) { return (d.gu ? H : I) / kKStage; };
        // The next item's scale rows are issued when an item starts, so they
        // have a whole item's worth of stage traffic to land behind.  Item
        // metadata is pipelined so that no dependent global load sits on the
        // issue path: while item li is issued, the slot of item li+2 and the
        // tile descriptor of item li+3 are in flight.
        const int G = gridDim.x;
        int item = blockIdx.x;
        auto meta = [&](int it, const TileDesc& td) -> DecItem {
            if constexpr (kFront) return front_item(args, P, ft, it);
            else return finish_item(args, P, it, td);
        };
        auto ltile = [&](int it) -> TileDesc {
            if constexpr (kFront) return TileDesc{};  // read with the item from shared memory
            else return load_tile(tiles, P, it);
        };
        DecItem cur = meta(item, ltile(item));
        DecItem n1{};
        if (item + G < n_items) n1 = meta(item + G, ltile(item + G));
        TileDesc td2{};
        if (item + 2 * G < n_items) td2 = ltile(item + 2 * G);
        // Before the wait: the first two items' scale rows and the weights of
        // the first ring's worth of stages.  (The front end has its token
        // rows at hand too; issuing each stage's weights and tokens together
        // instead landed the first stage sooner but made the layer slower:
        // 138.5 against 132.7 us at b = 8, measured on one B200.)
        if (!issue_scales(cur, 0)) return;
        if (item + G < n_items && !issue_scales(n1, 1)) return;
        const int k0 = stages_of(cur);
        const int pre = n_stages < k0 ? n_stages : k0;
        if (kFront) fence_proxy_async_smem();  // the ring held the front end's generic scratch
        for (int s = 0; s < pre; ++s) {  // first use of ring slots 0..pre-1
            mbar_arrive_expect_tx(&S.full[s], stage_bytes(cur));
            issue_weights(cur, s, s);
        }
        // (Prefetching the rest of the first two items' weights into L2 here,
        // 57 MB over all CTAs, made the layer slower: 133.6 against 129.9 us at
        // b = 8 and 52.5 against 45.0 us at b = 1, measured on one B200 -- the
        // prefetches queue ahead of the first stages.)
        pdl_wait();
        int st = 0;
        uint32_t ph = 0;
        uint32_t dk = 0;  // down items of this CTA issued so far
        for (int li = 0; item < n_items; item += G, ++li) {
            if (li > 0 && item + G < n_items && !issue_scales(n1, li + 1)) return;
            DecItem n2{};
            if (item + 2 * G < n_items) n2 = meta(item + 2 * G, td2);
            if (item + 3 * G < n_items) td2 = ltile(item + 3 * G);
            if (!cur.valid) atomicOr(status, kStatusBadExpert);
            const int ks = stages_of(cur);
            for (int s = 0; s < ks; ++s) {
                if (li > 0 || s >= pre) {
                    if (!mbar_wait(&S.empty[st], ph ^ 1, status, kStatusTimeoutTma)) return;
                    mbar_arrive_expect_tx(&S.full[st], stage_bytes(cur));
                    issue_weights(cur, s, st);
                }
                if (s == 0 && dep && !cur.gu) {
                    // the SwiGLU rows of this tile: the dependency warp has
                    // seen every gate/up item of the tile publish its stores
                    // (generic proxy), which the tensor copies below read
                    // through the async proxy
                    if (!wait_smem_geq(dep_ready, ++dk, status, kStatusTimeoutTma)) return;
                    fence_proxy_async_global();
                }
                issue_tokens(cur, s, st);
                if (++st == n_stages) { st = 0; ph ^= 1; }
            }
            cur = n1;
            n1 = n2;
        }
        return;
    }

    if (warp == kDecCheckerWarp) {
        // ---------------- scale checker ----------------
        // Scale bytes 104..140 make every E2M1 x 2^(s-127) product an exact,
        // finite binary16, so scaling a block's FP32 partial sum equals
        // summing the reference's FP16-rounded weights.  Byte 103 rounds
        // 0.5 x 2^-24 and bytes >= 141 overflow in the reference dequant.  The
        // checker reads each item's scale rows once and publishes whether all
        // of them are in range; the consumers start the item after that.
        int li = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
            const int slot = li % kDecScSlots;
            const uint32_t sc_item = 128u * static_cast<uint32_t>((item < P.n_gu ? H : I) / 32);
            const bool ok = mbar_wait(&sfull[slot], (li / kDecScSlots) & 1, status, kStatusTimeoutDequant);
            if (!__all_sync(0xffffffffu, ok)) return;
            const uint32_t sc = S.base + L.sc_off + slot * L.sc_slot;
            uint32_t acc = 0x80808080u;
#pragma unroll 4
            for (uint32_t i = lane; i < sc_item / 16; i += 32) {
                const uint4 v = lds_v4(sc + i * 16);
                acc &= scale_bytes_exact(v.x) & scale_bytes_exact(v.y) & scale_bytes_exact(v.z) &
                       scale_bytes_exact(v.w);
            }
            const bool fast = __all_sync(0xffffffffu, acc == 0x80808080u);
            if (lane == 0) {
                S.fast_flag[slot] = fast ? 1 : 0;
                mbar_arrive(&S.sready[slot]);
            }
        }
        return;
    }

    if (warp == kDecDepWarp) {
        // ---------------- dependency warp ----------------
        // Walks this CTA's down items in order, waits (bounded, gpu-scope
        // acquire) until each one's tile has all its gate/up items
        // published and counts it in dep_ready (shared, release), so the
        // producer's check is a shared-memory read and the global round
        // trips run ahead of the TMA issue.
        if (!dep || lane != 0) return;
        uint32_t dk = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            if (item < P.n_gu) continue;
            const int tile = (item - P.n_gu) / P.md;
            const bool ready =
                kFront ? wait_u64_geq(front.ctr + tile, static_cast<unsigned long long>(front.epoch) * P.mg, status,
                                      kStatusTimeoutTma)
                       : wait_count_geq(&args.tile_done[tile], static_cast<uint32_t>(P.mg), status, kStatusTimeoutTma);
            if (!ready) return;
            ++dk;
            asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(dep_ready)), "r"(dk)
                         : "memory");
        }
        return;
    }

    if (warp == kDecSignalWarp) {
        // ---------------- signal warp ----------------
        // Publishes each item's stores to the grid once the item's first
        // warps have stored them (mbarrier, CTA scope): a gpu-scope fence,
        // then for a gate/up item one increment of its tile's count, for a
        // down item (fused combine) one increment per row of its
        // (token, feature block) count.  The row that completes a count --
        // all K selections of the token written for this block -- runs the
        // block's combine, reading the K rows in rank order.  Which CTA that
        // is does not change the result.
        if (!signal) return;
        const int K = args.topk;
        int li = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
            const int b = li & 1;
            const bool ok = mbar_wait(&S.stored[b], (li >> 1) & 1, status, kStatusTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, ok)) return;
            if (item < P.n_gu) {
                if (dep && lane == 0) {
                    // release-add: publishes the stores this lane acquired
                    // through the mbarrier (the act rows, read next through
                    // the async proxy)
                    fence_proxy_async_global();
                    if (kFront)
                        red_release_add(front.ctr + item / P.mg, 1ull);
                    else
                        red_release_add(&args.tile_done[item / P.mg], 1u);
                }
            } else if (args.comb_out) {
                const int j = item - P.n_gu;
                const int tile = j / P.md;
                const int m = j - tile * P.md;
                const TileDesc td = kFront ? front_tile(ft, tile) : tiles[tile];
                int tok = 0;
                bool last = false;
                if (lane < td.n_rows) {
                    // acquire-release add: publishes the rows this lane
                    // acquired through the mbarrier, and the lane that
                    // completes a block acquires every other CTA's rows of it
                    tok = (kFront ? static_cast<int>(ft_perm[td.row_start + lane]) : perm[td.row_start + lane]) / K;
                    if (kFront) {
                        // (token, block) counters start each launch at zero:
                        // the add that completes a block resets it
                        unsigned long long* c = front.ctr + kFrontMaxTiles + tok * P.md + m;
                        last = atom_acq_rel_add(c, 1ull) + 1 == static_cast<unsigned long long>(K);
                        if (last) atomicExch(c, 0ull);
                    } else
                        last = atom_acq_rel_add(&args.comb_cnt[tok * P.md + m], 1u) == static_cast<uint32_t>(K - 1);
                }
                uint32_t mask = __ballot_sync(0xffffffffu, last);
                if (mask) {
                    // the other lanes read rows the completing lane acquired:
                    // the warp barrier orders their loads after its acquire
                    __syncwarp();
                    const int h0 = m * 128 + lane * 4;
                    while (mask) {
                        const int n = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const int t = __shfl_sync(0xffffffffu, tok, n);
                        const size_t s0 = static_cast<size_t>(t) * K;
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int r0 = 0; r0 < K; r0 += 8) {
                            // all loads of up to eight rows first (one round
                            // trip), then the rank-order sum
                            float wr[8];
                            float4 v[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                if (r0 + i < K) {
                                    wr[i] = comb_w[s0 + r0 + i];
                                    v[i] = __ldcg(reinterpret_cast<const float4*>(args.raw + (s0 + r0 + i) * H + h0));
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                if (r0 + i < K) {
                                    acc.x = __fadd_rn(acc.x, __fmul_rn(wr[i], v[i].x));
                                    acc.y = __fadd_rn(acc.y, __fmul_rn(wr[i], v[i].y));
                                    acc.z = __fadd_rn(acc.z, __fmul_rn(wr[i], v[i].z));
                                    acc.w = __fadd_rn(acc.w, __fmul_rn(wr[i], v[i].w));
                                }
                            }
                        }
                        *reinterpret_cast<float4*>(args.comb_out + static_cast<size_t>(t) * H + h0) = acc;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.sfree[b]);
        }
        return;
    }

    // ---------------- consumers ----------------
    int st = 0, parity = 0, li = 0;
    uint32_t ph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
        const bool go = item < P.n_gu
                            ? consume_item<true, kOfficial, kRows, kFront>(args, L, S, li, st, ph, parity, n_stages, signal,
                                                                    warp, lane, perm, ft_perm)
                            : consume_item<false, kOfficial, kRows, kFront>(args, L, S, li, st, ph, parity, n_stages,
                                                                     signal, warp, lane, perm, ft_perm);
        if (!go) break;
    }
}

template <bool kOfficial, int kMode>
cudaError_t launch_dec(const DecMaps& maps, const GemmArgs& args, const DecFront& front, int grid,
                       cudaStream_t stream) {
    constexpr bool kFront = kMode == kModeFront;
    auto kern = moe_decode_kernel<kOfficial, kMode>;
    const cudaError_t e = ensure_smem_attr<moe_decode_kernel<kOfficial, kMode>>(static_cast<int>(kSmemLimit));
    if (e != cudaSuccess) return e;
    const DecLayout L = dec_layout(dec_layout_k(args));
    if (L.stages < 2 || L.bytes > kSmemLimit || args.phases < 1 || args.phases > 3 || args.hidden % kKStage ||
        args.inter % kKStage || args.inter % 64 || args.hidden % 128)
        return cudaErrorInvalidValue;
    if (!kFront && args.comb_out &&
        (!(args.phases & 2) || !args.comb_w || !args.comb_cnt || !args.raw || args.raw_peers))
        return cudaErrorInvalidValue;
    return launch_pdl(kern, dim3(grid), dim3(kDecThreads), L.bytes, stream, maps, args, front);
}

cudaError_t launch_decode(const DecMaps& maps, const GemmArgs& args, int grid, cudaStream_t stream) {
    const DecFront none{};
    return args.official ? launch_dec<true, kModeBox>(maps, args, none, grid, stream)
                         : launch_dec<false, kModeBox>(maps, args, none, grid, stream);
}

}  // namespace

// The weight maps view a projection [rows, K/2 bytes] of every record as
// {128 B, rows, K/256 chunks, slot} with the chunk stride (128 B) below the
// row stride: one box {128, rows, 2, 1} is a whole 512-wide stage of 64 or
// 128 rows, landing as [chunk][row][128 B] with the 128-byte swizzle.
bool encode_decode_weight_maps(EncodeTiledFn fn, const void* records, size_t record_bytes,
                               int n_slots, int hidden, int inter, GemmMaps* gu, GemmMaps* dn) {
    if (!fn) return false;
    const uint8_t* rec = static_cast<const uint8_t*>(records);
    const size_t ih = static_cast<size_t>(hidden) * inter;
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    auto enc = [&](CUtensorMap* m, const uint8_t* base, int rows, int k, cuuint32_t box_rows) {
        const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(k / 256),
                                    static_cast<cuuint64_t>(n_slots)};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(k / 2), 128,
                                       static_cast<cuuint64_t>(record_bytes)};
        const cuuint32_t box[4] = {128, box_rows, 2, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(base), dims, strides, box,
                  elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    *gu = GemmMaps{};
    *dn = GemmMaps{};
    if (!enc(&gu->w0, rec, inter, hidden, 64) || !enc(&gu->w1, rec + ih / 2, inter, hidden, 64) ||
        !enc(&dn->w0, rec + ih, hidden, inter, 128))
        return false;
    dn->w1 = dn->w0;
    // Scale rows [rows, K/32 bytes] of every record as {K/32, rows, slot},
    // boxes of a work item's 64 (gate/up) or 128 (down) rows, swizzled with
    // the span of one row when that is 32, 64 or 128 bytes.
    auto enc_sc = [&](CUtensorMap* m, const uint8_t* base, int rows, int k, cuuint32_t box_rows) {
        const cuuint32_t rbytes = static_cast<cuuint32_t>(k / 32);
        const CUtensorMapSwizzle swz = rbytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : rbytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_32B;
        const cuuint64_t dims[3] = {rbytes, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(n_slots)};
        const cuuint64_t strides[2] = {rbytes, static_cast<cuuint64_t>(record_bytes)};
        const cuuint32_t box[3] = {rbytes, box_rows, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    auto swizzles = [](int k) { return k / 32 == 32 || k / 32 == 64 || k / 32 == 128; };
    const size_t off_s1 = ih + ih / 2, off_s3 = off_s1 + ih / 32, off_s2 = off_s3 + ih / 32;
    if (swizzles(hidden) && record_bytes % 16 == 0 && enc_sc(&gu->s0, rec + off_s1, inter, hidden, 64) &&
        enc_sc(&gu->s1, rec + off_s3, inter, hidden, 64))
        gu->scale_swz = 1;
    if (swizzles(inter) && record_bytes % 16 == 0 && enc_sc(&dn->s0, rec + off_s2, hidden, inter, 128)) {
        dn->s1 = dn->s0;
        dn->scale_swz = 1;
    }
    return true;
}

// Token rows [rows, cols] FP16 viewed as {64, rows, cols/64 chunks} (chunk
// stride 128 B): one box {64, 8, box_chunks} is the 8 rows of a tile over a
// stage, landing as [chunk][row][128 B] with the 128-byte swizzle.
bool encode_decode_token_map(EncodeTiledFn fn, const void* rows_base, int rows, int cols,
                             CUtensorMap* map, int box_chunks) {
    return encode_token_map(fn, rows_base, rows, cols, 8, box_chunks, map);
}

bool encode_token_map(EncodeTiledFn fn, const void* rows_base, int rows, int cols, int box_rows, int box_chunks,
                      CUtensorMap* map) {
    if (!fn) return false;
    const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols / 64)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2, 128};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(box_chunks)};
    const cuuint32_t elem[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(rows_base), dims, strides, box,
              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_moe_decode(bool gate_up, const GemmMaps& maps, const GemmArgs& args, int grid,
                              cudaStream_t stream) {
    // one projection: the other projection's map slots hold copies
    DecMaps m;
    m.gw1 = maps.w0;
    m.gw3 = maps.w1;
    m.gx = maps.b;
    m.gs1 = maps.s0;
    m.gs3 = maps.s1;
    m.dw2 = maps.w0;
    m.dact = maps.b;
    m.ds2 = maps.s0;
    GemmArgs a = args;
    a.phases = gate_up ? 1 : 2;
    a.scale_swz = gate_up ? maps.scale_swz : 0;
    a.dn_scale_swz = gate_up ? 0 : maps.scale_swz;
    a.tile_done = nullptr;
    a.comb_out = nullptr;
    a.comb_w = nullptr;
    a.comb_cnt = nullptr;
    return launch_decode(m, a, grid, stream);
}

cudaError_t launch_moe_decode_front(const GemmMaps& gu, const GemmMaps& dn, const GemmArgs& args,
                                    const DecFront& front, int grid, cudaStream_t stream) {
    if (args.official || args.raw_peers || !front.x || !front.scratch || !front.ctr || !front.ids_out ||
        (front.logits && !front.weights_out) || (args.comb_out && !front.weights_out) || front.epoch == 0 ||
        !decode_front_fits(front.tokens, args.topk, args.num_experts) || grid <= 0)
        return cudaErrorInvalidValue;
    if (args.comb_out && !args.raw) return cudaErrorInvalidValue;
    DecMaps m;
    m.gw1 = gu.w0;
    m.gw3 = gu.w1;
    m.gx = gu.w0;  // token rows come by bulk copy
    m.gs1 = gu.s0;
    m.gs3 = gu.s1;
    m.dw2 = dn.w0;
    m.dact = dn.b;
    m.ds2 = dn.s0;
    GemmArgs a = args;
    a.phases = 3;
    a.scale_swz = gu.scale_swz;
    a.dn_scale_swz = dn.scale_swz;
    a.tile_done = nullptr;
    a.comb_cnt = nullptr;
    return launch_dec<false, kModeFront>(m, a, front, grid, stream);
}

cudaError_t launch_moe_decode_layer(const GemmMaps& gu, const GemmMaps& dn, const GemmArgs& args, int grid,
                                    cudaStream_t stream) {
    if (!args.tile_done) return cudaErrorInvalidValue;
    DecMaps m;
    m.gw1 = gu.w0;
    m.gw3 = gu.w1;
    m.gx = gu.b;
    m.gs1 = gu.s0;
    m.gs3 = gu.s1;
    m.dw2 = dn.w0;
    m.dact = dn.b;
    m.ds2 = dn.s0;
    GemmArgs a = args;
    a.phases = 3;
    a.scale_swz = gu.scale_swz;
    a.dn_scale_swz = dn.scale_swz;
    return launch_decode(m, a, grid, stream);
}

}  // namespace dee
