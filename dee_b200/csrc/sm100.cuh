// sm100.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a) features
// the MoE kernels use: mbarriers, TMA tensor loads, tcgen05 TMEM allocation,
// tcgen05.mma (A operand in tensor memory), tcgen05.ld/st and the async
// fences.  Every wait is bounded: after kWaitLimitNs of global time a wait
// gives up, records a code in the kernel's status word and returns false so
// the kernel can unwind instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace dee {
namespace sm100 {

// A wait that has not completed after this much global time is treated as a
// deadlock: the kernel records an error and unwinds.  Normal waits finish in
// microseconds; a full 4096-token layer takes about a millisecond.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Status word bits written by kernels (host reads them after a sync).
enum StatusBits : uint32_t {
    kStatusTimeoutTma = 1u << 0,
    kStatusTimeoutDequant = 1u << 1,
    kStatusTimeoutMma = 1u << 2,
    kStatusTimeoutEpilogue = 1u << 3,
    kStatusBadExpert = 1u << 4,
    kStatusBadShape = 1u << 5,
    kStatusTimeoutFlag = 1u << 6,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// is suspended (up to the hint) instead of spinning, so waiting roles do not
// take issue slots from the warps doing the work.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// The blocking part of mbar_wait, kept out of line: a loop in the caller's
// body costs the tensor-core issuer ~50 cycles per wait even when the phase
// is already complete (measured: 120 vs 84 cycles per M=128, N=128 MMA with
// one wait per four MMAs), enough to starve the MMA pipe between K steps.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                                   uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait_sleep(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns) {
            atomicOr(status, code);
            return false;
        }
    }
}

// Bounded wait for the phase with the given parity.  Returns false (and
// sets `code` in *status) when the limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          uint32_t code) {
    if (__builtin_expect(mbar_try_wait(bar, parity), 1)) return true;
    return mbar_wait_slow(bar, parity, status, code, kWaitLimitNs);
}

// The same wait with an explicit limit.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                              uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, status, code, limit_ns);
}

// Bounded wait of thread i < n for flags[i] to reach `epoch` (system-scope
// acquire: the flags are raised by kernels on other GPUs after their
// stores).  A flag that has not arrived after limit_ns sets `code` in
// *status and the thread goes on.  Callers follow it with a CTA barrier, so
// every thread of the CTA is ordered after the acquires.
__device__ __forceinline__ void wait_flags_bounded(const uint32_t* flags, int n, uint32_t epoch,
                                                   uint64_t limit_ns, uint32_t* status, uint32_t code) {
    const int i = threadIdx.x;
    if (i >= n) return;
    const uint64_t t0 = global_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
        if (static_cast<int32_t>(v - epoch) >= 0) return;
        if (global_ns() - t0 > limit_ns) {
            atomicOr(status, code);
            return;
        }
        __nanosleep(200);
    }
}

// ---------------------------------------------------------------- PDL

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while its predecessor in the stream still runs;
// pdl_wait() blocks until the predecessor has completed and its writes are
// visible, pdl_trigger() lets the successor launch.  Every kernel here calls
// pdl_wait() before touching data a predecessor produces and pdl_trigger()
// only after that wait, so a kernel that starts early can rely on the kernel
// two places back having completed.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 2-D tiled load into CTA shared memory; completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// 3-D tiled load (x innermost).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
        "l"(policy)
        : "memory");
}

// 5-D tiled load (x innermost).
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z, int32_t w, int32_t v, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v),
        "l"(policy)
        : "memory");
}

// 4-D tiled load (x innermost).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z, int32_t w,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w),
        "l"(policy)
        : "memory");
}

// Prefetch a 3-D tile into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int32_t x, int32_t y,
                                                int32_t z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// Contiguous global -> shared copy completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Prefetch a contiguous global range into L2 (16-byte aligned address, size a
// multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (FP16 or BF16 inputs,
// FP32 accumulate), one CTA.  Issued by a single thread.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Each thread writes 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// Each thread writes 4 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, uint32_t v0, uint32_t v1, uint32_t v2,
                                                  uint32_t v3) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v0), "r"(v1),
                 "r"(v2), "r"(v3)
                 : "memory");
}

// Each thread reads 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// Each thread reads 16 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30)
// (unused for this layout), stride byte offset >> 4 [32,46), descriptor
// version 1 [46,48), swizzle mode 2 = 128B [61,64).
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Shared-memory descriptor of a tile without swizzle: core matrices of 8 rows
// x 16 bytes (128 contiguous bytes), the next 8 rows `sbo` bytes further on.
// Used as the source of tcgen05.cp for 16-byte-wide tiles, so the leading
// byte offset (between core matrices along the row) is never stepped over.
__device__ __forceinline__ uint64_t smem_desc_plain(uint32_t smem_addr, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((128u >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    return d;
}

// tcgen05.cp of 32 rows x 128 bits from shared memory into tensor memory
// columns taddr..taddr+3, row i to lane i of each of the four 32-lane
// quadrants.  Asynchronous: it runs in issue order with this thread's later
// tcgen05.mma, and tcgen05.commit tracks it.
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Make this thread's ordinary shared-memory stores visible to the async
// proxy (TMA, tcgen05.mma and tcgen05.cp reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Instruction descriptor for kind::f16: D FP32 (bits 4-5 = 1), A and B FP16
// (formats 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ __forceinline__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace sm100
}  // namespace dee
