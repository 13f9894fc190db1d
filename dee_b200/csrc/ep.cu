// ep.cu -- expert-parallel dispatch packing, peer transfers and combine.
//
// With the experts split into contiguous ranges of `experts_per_rank` over
// `ranks` GPUs (rank r owns experts [r*epr, (r+1)*epr), the official
// convention of the DeepSeek-V4 reference, inference/model.py:625-626), a
// token's K selections go to the ranks that own their experts.  The owner of
// the tokens packs, per destination rank, a fixed-capacity block of rows
// (FP16 hidden row + local expert id, -1 for an unused slot), so the
// all-to-all needs no host-side split sizes and no host synchronisation.
// Within a destination block the selections keep ascending position order
// p = t*K + r.  After the experts ran and the rows came back, the combine
// reads each (token, rank) row through the same slot map, in rank order.
#include "kernels.h"

namespace dee {
namespace {

using sm100::kStatusBadExpert;
using sm100::kStatusBadShape;

constexpr int kPackThreads = 1024;

// One CTA.  Chunk by chunk of 1024 selections: per destination a warp
// ballot gives each selection its place among its warp's, a scan over the
// warps' counts its place in the chunk, and a running base per destination
// its slot.  kPeer = false writes the local send block (ranks x capacity
// local expert ids, -1 unused); kPeer = true writes this rank's block of every
// owner's receive buffer over NVLink, including -1 for the unused slots.
template <bool kPeer>
__global__ void __launch_bounds__(kPackThreads, 1)
    ep_index_kernel(const int32_t* __restrict__ ids, int sel, int ranks, int rank, int epr, int capacity,
                    int32_t* __restrict__ send_expert, EpPeers peers, int32_t* __restrict__ slot_of_pos,
                    int32_t* __restrict__ journal, uint32_t* status) {
    __shared__ int wc[kEpMaxRanks][32];    // per destination, per warp: selections in the chunk
    __shared__ int wpre[kEpMaxRanks][32];  // exclusive prefix over warps
    __shared__ int chunk_total[kEpMaxRanks];
    __shared__ int base[kEpMaxRanks];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const unsigned lt = (1u << lane) - 1u;
    if (!kPeer)
        for (int i = tid; i < ranks * capacity; i += kPackThreads) send_expert[i] = -1;
    if (tid < ranks) base[tid] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < sel; c0 += kPackThreads) {
        const int p = c0 + tid;
        int d = -1, le = -1;
        if (p < sel) {
            const int e = ids[p];
            if (journal) journal[p] = e;
            if (e >= 0 && e < ranks * epr) {
                d = e / epr;
                le = e - d * epr;
            } else {
                atomicOr(status, kStatusBadExpert);
                slot_of_pos[p] = -1;
            }
        }
        int my_rank = 0;
        for (int dd = 0; dd < ranks; ++dd) {
            const unsigned m = __ballot_sync(0xffffffffu, d == dd);
            if (lane == 0) wc[dd][warp] = __popc(m);
            if (d == dd) my_rank = __popc(m & lt);
        }
        __syncthreads();
        if (warp < ranks) {
            const int v = wc[warp][lane];
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += a;
            }
            wpre[warp][lane] = incl - v;
            if (lane == 31) chunk_total[warp] = incl;
        }
        __syncthreads();
        if (d >= 0) {
            const int s = base[d] + wpre[d][warp] + my_rank;
            if (s < capacity) {
                slot_of_pos[p] = d * capacity + s;
                if (kPeer)
                    peers.recv_expert[d][rank * capacity + s] = le;
                else
                    send_expert[d * capacity + s] = le;
            } else {
                atomicOr(status, kStatusBadShape);
                slot_of_pos[p] = -1;
            }
        }
        __syncthreads();
        if (tid < ranks) base[tid] += chunk_total[tid];
        __syncthreads();
    }
    if (kPeer)  // this rank's unused slots in every owner's block
        for (int d = 0; d < ranks; ++d)
            for (int s = base[d] + tid; s < capacity; s += kPackThreads)
                peers.recv_expert[d][rank * capacity + s] = -1;
}

// One warp per selection: its token's hidden row into its send slot.
__global__ void ep_pack_rows_kernel(const __half* __restrict__ x, const int32_t* __restrict__ slot_of_pos,
                                    int sel, int topk, int hidden, __half* __restrict__ send_rows) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int warps_total = gridDim.x * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    const int vec = hidden / 8;
    for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < sel; p += warps_total) {
        const int s = slot_of_pos[p];
        if (s < 0) continue;
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(p / topk) * hidden);
        uint4* dst = reinterpret_cast<uint4*>(send_rows + static_cast<size_t>(s) * hidden);
        for (int i = lane; i < vec; i += 32) dst[i] = __ldg(src + i);
    }
}

// The live combine (deepseek_v4_layer_candidate.py:616-629) over rows that
// came back from the expert owners: out = 0, then for each rank in order
// out += w * row, the multiply and the add each rounded to FP32.
// With `flags` set (the NVLink path) every CTA first waits (bounded) for each
// expert owner's return flag to reach `epoch`.
__global__ void ep_combine_kernel(const float* __restrict__ back, const int32_t* __restrict__ slot_of_pos,
                                  const float* __restrict__ w, int tokens, int topk, int hidden,
                                  float* __restrict__ out, const uint32_t* flags, int ranks, uint32_t epoch,
                                  uint32_t* status, uint64_t limit_ns) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    if (flags) {
        sm100::wait_flags_bounded(flags, ranks, epoch, limit_ns, status, sm100::kStatusTimeoutFlag);
        __syncthreads();
    }
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = (i * 4) / hidden;
        const size_t h = i * 4 - t * hidden;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < topk; ++r) {
            const size_t p = t * topk + r;
            const int s = slot_of_pos[p];
            if (s < 0) continue;
            const float wr = w[p];
            const float4 v = *reinterpret_cast<const float4*>(back + static_cast<size_t>(s) * hidden + h);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wr, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wr, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wr, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wr, v.w));
        }
        *reinterpret_cast<float4*>(out + t * hidden + h) = acc;
    }
}

// ---------------------------------------------------------------- peer path
//
// Rows and local expert ids go straight into the owners' receive buffers
// over NVLink (peer pointers from CUDA IPC); block `rank` of every owner's
// buffer belongs to this rank.

// The rows, then the dispatch flags: every CTA fences its stores and counts
// itself on `done`; the CTA that completes the count resets it and raises
// `epoch` in slot `rank` of every owner's flag array (what ep_signal_kernel
// does as a launch of its own).
__global__ void ep_peer_rows_kernel(const __half* __restrict__ x, const int32_t* __restrict__ slot_of_pos,
                                    int sel, int topk, int hidden, int rank, int capacity, EpPeers peers,
                                    int ranks, uint32_t* done, uint32_t epoch) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int warps_total = gridDim.x * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    const int vec = hidden / 8;
    for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < sel; p += warps_total) {
        const int s = slot_of_pos[p];
        if (s < 0) continue;
        const int d = s / capacity;
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(p / topk) * hidden);
        uint4* dst = reinterpret_cast<uint4*>(peers.recv_rows[d] +
                                              static_cast<size_t>(rank * capacity + (s - d * capacity)) * hidden);
        for (int i = lane; i < vec; i += 32) dst[i] = __ldg(src + i);
    }
    // the CTA barrier orders every thread's stores before thread 0's fence,
    // which is cumulative: one system fence per CTA, then its count
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    if (atomicAdd(done, 1u) != gridDim.x - 1) return;
    *done = 0;
    __threadfence_system();
    for (int d = 0; d < ranks; ++d)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.recv_flag[d] + rank), "r"(epoch) : "memory");
}

// After the kernels before it on the stream have completed: make their
// stores visible system-wide, then publish `epoch` in slot `rank` of every
// peer's flag array.
__global__ void ep_signal_kernel(EpPeers peers, bool back, int ranks, int rank, uint32_t epoch) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int d = 0; d < ranks; ++d) {
        uint32_t* f = (back ? peers.back_flag[d] : peers.recv_flag[d]) + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
    }
}

int grid_cap(size_t work, int per_block, int cap) {
    size_t g = (work + per_block - 1) / per_block;
    if (g < 1) g = 1;
    return static_cast<int>(g < static_cast<size_t>(cap) ? g : cap);
}

}  // namespace

cudaError_t launch_ep_pack(const int32_t* ids, const __half* x, int tokens, int topk, int hidden,
                           int ranks, int epr, int capacity, __half* send_rows, int32_t* send_expert,
                           int32_t* slot_of_pos, int32_t* journal, uint32_t* status,
                           cudaStream_t stream) {
    if (tokens <= 0 || topk <= 0 || ranks <= 0 || ranks > kEpMaxRanks || epr <= 0 || capacity <= 0 ||
        hidden % 8 != 0)
        return cudaErrorInvalidValue;
    const int sel = tokens * topk;
    cudaError_t err = launch_pdl(ep_index_kernel<false>, dim3(1), dim3(kPackThreads), 0, stream, ids, sel,
                                 ranks, 0, epr, capacity, send_expert, EpPeers{}, slot_of_pos, journal,
                                 status);
    if (err != cudaSuccess) return err;
    return launch_pdl(ep_pack_rows_kernel, dim3(grid_cap(static_cast<size_t>(sel), 8, 148 * 8)), dim3(256), 0,
                      stream, x, static_cast<const int32_t*>(slot_of_pos), sel, topk, hidden, send_rows);
}

cudaError_t launch_ep_peer_dispatch(const int32_t* ids, const __half* x, int tokens, int topk, int hidden,
                                    int ranks, int rank, int epr, int capacity, const EpPeers& peers,
                                    int32_t* slot_of_pos, int32_t* journal, uint32_t* status,
                                    uint32_t* done, uint32_t epoch, cudaStream_t stream) {
    if (tokens <= 0 || topk <= 0 || ranks <= 0 || ranks > kEpMaxRanks || rank < 0 || rank >= ranks ||
        epr <= 0 || capacity <= 0 || hidden % 8 != 0)
        return cudaErrorInvalidValue;
    const int sel = tokens * topk;
    cudaError_t err = launch_pdl(ep_index_kernel<true>, dim3(1), dim3(kPackThreads), 0, stream, ids, sel,
                                 ranks, rank, epr, capacity, static_cast<int32_t*>(nullptr), peers,
                                 slot_of_pos, journal, status);
    if (err != cudaSuccess) return err;
    return launch_pdl(ep_peer_rows_kernel, dim3(grid_cap(static_cast<size_t>(sel), 8, 148 * 8)), dim3(256), 0,
                      stream, x, static_cast<const int32_t*>(slot_of_pos), sel, topk, hidden, rank, capacity,
                      peers, ranks, done, epoch);
}

cudaError_t launch_ep_signal(const EpPeers& peers, bool back, int ranks, int rank, uint32_t epoch,
                             cudaStream_t stream) {
    return launch_pdl(ep_signal_kernel, dim3(1), dim3(32), 0, stream, peers, back, ranks, rank, epoch);
}

namespace {
// One thread waits on an mbarrier that nothing arrives on: the bounded wait
// every pipeline kernel uses must give up after limit_ns and report `code`.
__global__ void wait_selftest_kernel(uint64_t limit_ns, uint32_t* status, uint32_t code) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) sm100::mbar_wait_for(&bar, 0, status, code, limit_ns);
}
}  // namespace

cudaError_t launch_wait_selftest(uint64_t limit_ns, uint32_t* status, uint32_t code, cudaStream_t stream) {
    wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns, status, code);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const float* back, const int32_t* slot_of_pos, const float* weights,
                              int tokens, int topk, int hidden, float* out, cudaStream_t stream,
                              const uint32_t* flags, int ranks, uint32_t epoch, uint32_t* status,
                              uint64_t limit_ns) {
    if (tokens <= 0 || topk <= 0 || hidden % 4 != 0 || (flags && (ranks <= 0 || ranks > 256)))
        return cudaErrorInvalidValue;
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    return launch_pdl(ep_combine_kernel, dim3(grid_cap(n4, 256, 148 * 4)), dim3(256), 0, stream, back,
                      slot_of_pos, weights, tokens, topk, hidden, out, flags, ranks, epoch, status, limit_ns);
}

}  // namespace dee
