// routing.cu -- router top-k, group-by-expert permutation, token gather and
// the route-weighted combines.
#include "kernels.h"
#include "routing.cuh"

namespace dee {
namespace {

using sm100::kStatusBadExpert;
using sm100::kStatusBadShape;
using Cand = RouteCand;

template <int NPER>
__global__ void route_topk_kernel(const float* __restrict__ logits, int tokens, int experts,
                                  int topk, int32_t* __restrict__ ids, float* __restrict__ weights,
                                  uint32_t* status) {
    extern __shared__ float route_smem[];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= tokens) return;
    route_token<NPER>(logits + static_cast<size_t>(t) * experts, experts, topk, lane, route_smem + warp * experts,
                      ids + static_cast<size_t>(t) * topk, weights + static_cast<size_t>(t) * topk, nullptr,
                      status);
}

__global__ void route_dsv4_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                  const int64_t* __restrict__ tid2eid,
                                  const int64_t* __restrict__ input_ids, int tokens, int experts,
                                  int topk, float route_scale, int32_t* __restrict__ ids,
                                  float* __restrict__ weights, uint32_t* status) {
    extern __shared__ float dsv4_smem[];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= tokens) return;
    float* sc = dsv4_smem + warp * experts;  // unbiased scores
    const float* l = logits + static_cast<size_t>(t) * experts;
    const int nper = (experts + 31) >> 5;
    Cand mine[kRouteMaxPerLane];
#pragma unroll
    for (int j = 0; j < kRouteMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        if (j < nper && e < experts) {
            const float x = l[e];
            const float sp = x > 20.0f ? x : log1pf(expf(x));
            const float s = sqrtf(sp);
            sc[e] = s;
            mine[j].p = bias ? __fadd_rn(s, bias[e]) : s;
            mine[j].id = e;
        } else {
            mine[j].p = -INFINITY;
            mine[j].id = 0x7fffffff;
        }
    }
    __syncwarp();
    int sel_id[32];
    if (tid2eid) {
        const int64_t tok = input_ids[t];
        for (int k = 0; k < topk; ++k) {
            const int64_t e = tid2eid[tok * topk + k];
            sel_id[k] = (e >= 0 && e < experts) ? static_cast<int>(e) : -1;
        }
    } else {
        for (int k = 0; k < topk; ++k) {
            Cand best{-INFINITY, 0x7fffffff};
            int best_j = -1;
#pragma unroll
            for (int j = 0; j < kRouteMaxPerLane; ++j) {
                if (mine[j].id != 0x7fffffff && (best_j < 0 || route_better(mine[j], best))) {
                    best = mine[j];
                    best_j = j;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                Cand other;
                other.p = __shfl_xor_sync(0xffffffffu, best.p, o);
                other.id = __shfl_xor_sync(0xffffffffu, best.id, o);
                if (other.id != 0x7fffffff && (best.id == 0x7fffffff || route_better(other, best))) best = other;
            }
            sel_id[k] = best.id;
#pragma unroll
            for (int j = 0; j < kRouteMaxPerLane; ++j)
                if (mine[j].id == best.id) mine[j].id = 0x7fffffff;
        }
    }
    if (lane == 0) {
        float sum = 0.0f;
        bool ok = true;
        for (int k = 0; k < topk; ++k) {
            if (sel_id[k] < 0 || sel_id[k] >= experts) { ok = false; break; }
            sum = __fadd_rn(sum, sc[sel_id[k]]);
        }
        if (!ok || !(sum > 0.0f)) atomicOr(status, kStatusBadRouter);
        for (int k = 0; k < topk; ++k) {
            const bool good = ok && sum > 0.0f;
            ids[static_cast<size_t>(t) * topk + k] = good ? sel_id[k] : 0;
            weights[static_cast<size_t>(t) * topk + k] =
                good ? __fmul_rn(__fdiv_rn(sc[sel_id[k]], sum), route_scale) : 0.0f;
        }
    }
}

// ---------------------------------------------------------------------------
// Permutation.  Selections are enumerated in the reference's grouping order
// j = rank * T + token (engine.cpp:812-823: for each expert, rank-major then
// token) and placed with a stable counting sort by expert id, so the rows of
// one expert keep (rank, token) order and experts appear by ascending id.
// ---------------------------------------------------------------------------
constexpr int kPermThreads = 1024;
constexpr int kPermMaxExperts = 256;

// The whole permutation in one CTA of kPermThreads threads.  ids may be in
// global or shared memory; wcnt is a [32][kPermMaxExperts] shared scratch
// (per-warp group sizes), which this function zeroes before use.
__device__ void permute_block(const int32_t* ids, int tokens, int topk, int experts, int n_tile_max,
                              int max_tiles, const PermuteOut& out, uint32_t* status, bool skip_negative,
                              int (*wcnt)[kPermMaxExperts]) {
    __shared__ int cnt[kPermMaxExperts];
    __shared__ int off[kPermMaxExperts + 1];
    __shared__ int cursor[kPermMaxExperts];
    __shared__ int ntile_off[kPermMaxExperts + 1];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int sel = tokens * topk;
    for (int e = tid; e < experts; e += kPermThreads) { cnt[e] = 0; cursor[e] = 0; }
    for (int i = tid; i < 32 * kPermMaxExperts; i += kPermThreads) (&wcnt[0][0])[i] = 0;
    for (int i = tid; i < out.clear_n; i += kPermThreads) out.clear[i] = 0u;
    __syncthreads();
    for (int p = tid; p < sel; p += kPermThreads) {
        const int e = ids[p];
        if (out.journal) out.journal[p] = e;
        if (e < 0 || e >= experts) {
            if (!(skip_negative && e == -1)) atomicOr(status, kStatusBadExpert);
            out.row_of[p] = -1;
        } else {
            atomicAdd(&cnt[e], 1);
        }
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan of counts and of per-expert tile counts
        const int per = (experts + 31) / 32;
        int s = 0, st = 0;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < experts) {
                s += cnt[e];
                st += cnt[e] > 0 ? (cnt[e] + n_tile_max - 1) / n_tile_max : 0;
            }
        }
        int incl = s, incl_t = st;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, incl, o);
            const int b = __shfl_up_sync(0xffffffffu, incl_t, o);
            if (lane >= o) { incl += a; incl_t += b; }
        }
        int run = incl - s, run_t = incl_t - st;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < experts) {
                off[e] = run;
                ntile_off[e] = run_t;
                run += cnt[e];
                run_t += cnt[e] > 0 ? (cnt[e] + n_tile_max - 1) / n_tile_max : 0;
            }
        }
        if (lane == 31) { off[experts] = incl; ntile_off[experts] = incl_t; }
    }
    __syncthreads();
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int base = 0; base < sel; base += kPermThreads) {
        const int j = base + tid;
        int key = -1 - lane;  // unique per lane when not a valid selection
        int p = -1;
        if (j < sel) {
            const int r = j / tokens;
            const int t = j - r * tokens;
            p = t * topk + r;
            const int e = ids[p];
            if (e >= 0 && e < experts) key = e;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank_w = __popc(peers & lt_mask);
        const bool leader = rank_w == 0;
        if (key >= 0 && leader) wcnt[warp][key] = __popc(peers);
        __syncthreads();
        if (key >= 0) {
            int pre = 0;
            for (int w = 0; w < warp; ++w) pre += wcnt[w][key];
            const int row = off[key] + cursor[key] + pre + rank_w;
            out.perm[row] = p;
            out.row_of[p] = row;
        }
        __syncthreads();
        if (key >= 0 && leader) {
            atomicAdd(&cursor[key], __popc(peers));
            wcnt[warp][key] = 0;
        }
        __syncthreads();
    }
    for (int e = tid; e < experts; e += kPermThreads) {
        out.counts[e] = cnt[e];
        out.offsets[e] = off[e];
        const int c = cnt[e];
        if (c == 0) continue;
        const int nt = (c + n_tile_max - 1) / n_tile_max;
        const int sz = (c + nt - 1) / nt;
        for (int i = 0; i < nt; ++i) {
            const int slot = ntile_off[e] + i;
            if (slot >= max_tiles) { atomicOr(status, kStatusBadShape); break; }
            const int start = i * sz;
            const int n = min(sz, c - start);
            TileDesc td;
            td.expert = e;
            td.row_start = off[e] + start;
            td.n_rows = n;
            td.n_pad = (n + 15) & ~15;
            out.tiles[slot] = td;
            if (out.tile_grp) out.tile_grp[slot] = make_int2(ntile_off[e], nt);
        }
    }
    if (tid == 0) {
        out.offsets[experts] = off[experts];
        *out.n_tiles = min(ntile_off[experts], max_tiles);
    }
}

__global__ void __launch_bounds__(kPermThreads, 1)
    permute_kernel(const int32_t* __restrict__ ids, int tokens, int topk, int experts,
                   int n_tile_max, int max_tiles, PermuteOut out, uint32_t* status,
                   bool skip_negative) {
    __shared__ int wcnt[32][kPermMaxExperts];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    // expert-parallel receive buffer: the senders' rows and ids have landed
    // once their flags reach the epoch (the __syncthreads in permute_block
    // orders every thread's reads after the acquires)
    if (out.wait_flags)
        sm100::wait_flags_bounded(out.wait_flags, out.wait_ranks, out.wait_epoch, out.wait_limit_ns, status,
                                  sm100::kStatusTimeoutFlag);
    permute_block(ids, tokens, topk, experts, n_tile_max, max_tiles, out, status, skip_negative, wcnt);
}

// Router and permutation in one CTA, for decode-sized batches (T <= 16,
// T*K <= 384, E <= 256): the warps route the tokens (one warp per token, as
// route_topk_kernel) into ids/weights and a shared copy of the ids, and the
// CTA then groups them exactly as permute_kernel does.  One launch and one
// dependency instead of two.  The per-warp probability scratch of the router
// and the permutation's per-warp counts share one buffer.
__global__ void __launch_bounds__(kPermThreads, 1)
    route_permute_kernel(const float* __restrict__ logits, int tokens, int experts, int topk,
                         int32_t* __restrict__ ids, float* __restrict__ weights, int n_tile_max, int max_tiles,
                         PermuteOut out, uint32_t* status) {
    __shared__ int32_t s_ids[kDecodeMaxSelections];
    __shared__ int scratch[32][kPermMaxExperts];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    float* sp = reinterpret_cast<float*>(&scratch[warp][0]);
    for (int t = warp; t < tokens; t += kPermThreads / 32)
        route_token<8>(logits + static_cast<size_t>(t) * experts, experts, topk, lane, sp,
                       ids + static_cast<size_t>(t) * topk, weights + static_cast<size_t>(t) * topk,
                       s_ids + t * topk, status);
    __syncthreads();
    permute_block(s_ids, tokens, topk, experts, n_tile_max, max_tiles, out, status, false, scratch);
}

// The same permutation over many CTAs, for batches of more than two chunks
// of kPermChunk selections.  Pass 1 (one CTA per chunk of the (rank, token)
// enumeration): validation, the journal copy, each selection's stable rank
// among the chunk's selections of its expert, and the chunk's per-expert
// counts.  Pass 2 (one CTA per chunk): every CTA sums the chunk counts into
// expert totals and the prefix over earlier chunks, scans the totals into
// expert offsets and places its chunk; CTA 0 also writes counts, offsets and
// the tile list.  Rows come out exactly as the single-CTA kernel places them.
constexpr int kPermChunk = 1024;

__global__ void __launch_bounds__(kPermChunk, 1)
    permute_count_kernel(const int32_t* __restrict__ ids, int tokens, int topk, int experts, PermuteOut out,
                         uint32_t* status, bool skip_negative) {
    __shared__ int wcnt[32][kPermMaxExperts];  // per-warp group sizes
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int sel = tokens * topk;
    sm100::pdl_wait();
    sm100::pdl_trigger();
    if (out.wait_flags)  // as in permute_kernel; the place pass runs after this one completes
        sm100::wait_flags_bounded(out.wait_flags, out.wait_ranks, out.wait_epoch, out.wait_limit_ns, status,
                                  sm100::kStatusTimeoutFlag);
    for (int i = tid; i < 32 * kPermMaxExperts; i += kPermChunk) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int j = blockIdx.x * kPermChunk + tid;
    int key = -1 - lane;  // unique per lane when not a valid selection
    if (j < sel) {
        const int r = j / tokens;
        const int t = j - r * tokens;
        const int p = t * topk + r;
        const int e = ids[p];
        if (out.journal) out.journal[p] = e;
        if (e < 0 || e >= experts) {
            if (!(skip_negative && e == -1)) atomicOr(status, kStatusBadExpert);
            out.row_of[p] = -1;
        } else {
            key = e;
        }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    if (key >= 0 && rank_w == 0) wcnt[warp][key] = __popc(peers);
    __syncthreads();
    if (key >= 0) {
        int pre = 0;
        for (int w = 0; w < warp; ++w) pre += wcnt[w][key];
        out.lrank[j] = pre + rank_w;
    }
    for (int e = tid; e < experts; e += kPermChunk) {
        int c = 0;
#pragma unroll 8
        for (int w = 0; w < 32; ++w) c += wcnt[w][e];
        out.chunk_counts[static_cast<size_t>(blockIdx.x) * experts + e] = c;
    }
}

__global__ void __launch_bounds__(kPermChunk, 1)
    permute_place_kernel(const int32_t* __restrict__ ids, int tokens, int topk, int experts, int n_tile_max,
                         int max_tiles, PermuteOut out, uint32_t* status) {
    __shared__ int tot[kPermMaxExperts];
    __shared__ int before[kPermMaxExperts];  // this chunk's prefix over earlier chunks
    __shared__ int off[kPermMaxExperts + 1];
    __shared__ int ntile_off[kPermMaxExperts + 1];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int sel = tokens * topk;
    const int chunks = (sel + kPermChunk - 1) / kPermChunk;
    const int me = blockIdx.x;
    sm100::pdl_wait();
    sm100::pdl_trigger();
    for (int e = tid; e < experts; e += kPermChunk) {
        int s = 0, b = 0;
        for (int k = 0; k < chunks; ++k) {
            const int v = out.chunk_counts[static_cast<size_t>(k) * experts + e];
            if (k < me) b += v;
            s += v;
        }
        tot[e] = s;
        before[e] = b;
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan of totals and of per-expert tile counts
        const int per = (experts + 31) / 32;
        int s = 0, st = 0;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < experts) {
                s += tot[e];
                st += tot[e] > 0 ? (tot[e] + n_tile_max - 1) / n_tile_max : 0;
            }
        }
        int incl = s, incl_t = st;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, incl, o);
            const int b = __shfl_up_sync(0xffffffffu, incl_t, o);
            if (lane >= o) { incl += a; incl_t += b; }
        }
        int run = incl - s, run_t = incl_t - st;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < experts) {
                off[e] = run;
                ntile_off[e] = run_t;
                run += tot[e];
                run_t += tot[e] > 0 ? (tot[e] + n_tile_max - 1) / n_tile_max : 0;
            }
        }
        if (lane == 31) { off[experts] = incl; ntile_off[experts] = incl_t; }
    }
    __syncthreads();
    const int j = me * kPermChunk + tid;
    if (j < sel) {
        const int r = j / tokens;
        const int t = j - r * tokens;
        const int p = t * topk + r;
        const int e = ids[p];
        if (e >= 0 && e < experts) {
            const int row = off[e] + before[e] + out.lrank[j];
            out.perm[row] = p;
            out.row_of[p] = row;
        }
    }
    if (me != 0) return;
    for (int e = tid; e < experts; e += kPermChunk) {
        out.counts[e] = tot[e];
        out.offsets[e] = off[e];
        const int c = tot[e];
        if (c == 0) continue;
        const int nt = (c + n_tile_max - 1) / n_tile_max;
        const int sz = (c + nt - 1) / nt;
        for (int i = 0; i < nt; ++i) {
            const int slot = ntile_off[e] + i;
            if (slot >= max_tiles) { atomicOr(status, kStatusBadShape); break; }
            const int start = i * sz;
            const int n = min(sz, c - start);
            TileDesc td;
            td.expert = e;
            td.row_start = off[e] + start;
            td.n_rows = n;
            td.n_pad = (n + 15) & ~15;
            out.tiles[slot] = td;
            if (out.tile_grp) out.tile_grp[slot] = make_int2(ntile_off[e], nt);
        }
    }
    if (tid == 0) {
        out.offsets[experts] = off[experts];
        *out.n_tiles = min(ntile_off[experts], max_tiles);
    }
}

// One CTA per grouped row (grid-stride): every thread issues all of its
// loads of the row before its stores, so a row costs one memory round trip
// instead of one per 16 bytes of a thread.
constexpr int kGatherThreads = 128;
constexpr int kGatherUnroll = 4;

__global__ void __launch_bounds__(kGatherThreads)
    gather_rows_kernel(const __half* __restrict__ x, const int32_t* __restrict__ perm,
                       const int32_t* __restrict__ total_rows_dev, int max_rows, int topk, int hidden,
                       __half* __restrict__ x_perm) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int rows = min(*total_rows_dev, max_rows);
    const int vec = hidden / 8;  // uint4 per row
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
        const int t = perm[row] / topk;
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * hidden);
        uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<size_t>(row) * hidden);
        for (int base = 0; base < vec; base += kGatherThreads * kGatherUnroll) {
            uint4 v[kGatherUnroll];
#pragma unroll
            for (int k = 0; k < kGatherUnroll; ++k) {
                const int i = base + k * kGatherThreads + threadIdx.x;
                if (i < vec) v[k] = __ldg(src + i);
            }
#pragma unroll
            for (int k = 0; k < kGatherUnroll; ++k) {
                const int i = base + k * kGatherThreads + threadIdx.x;
                if (i < vec) dst[i] = v[k];
            }
        }
    }
}

// Live DeepSeek combine (deepseek_v4_layer_candidate.py:616-629): out = 0,
// then for each rank in order out += w * raw, each multiply and add rounded
// to FP32 separately.
__global__ void combine_f32_kernel(const float* __restrict__ raw, const float* __restrict__ w,
                                   int tokens, int topk, int hidden, float* __restrict__ out) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = (i * 4) / hidden;
        const size_t h = i * 4 - t * hidden;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < topk; ++r) {
            const size_t s = t * topk + r;
            const float wr = w[s];
            const float4 v = *reinterpret_cast<const float4*>(raw + s * hidden + h);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wr, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wr, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wr, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wr, v.w));
        }
        *reinterpret_cast<float4*>(out + t * hidden + h) = acc;
    }
}

// Exact eager-FP16 combine (weighted_combine_fp16_kernel,
// reference swiglu_cuda.cu:69-116): ranks visited in stable ascending expert
// order; raw, product and running sum each rounded to FP16.
template <class IdT>
__global__ void combine_f16_kernel(const float* __restrict__ raw, const float* __restrict__ w,
                                   const IdT* __restrict__ ids, int tokens, int topk, int hidden,
                                   __half* __restrict__ out) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const size_t n = static_cast<size_t>(tokens) * hidden;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / hidden;
        const size_t h = i - t * hidden;
        const IdT* te = ids + t * topk;
        __half acc = __float2half_rn(0.0f);
        bool ok = true;
        for (int rank = 0; rank < topk && ok; ++rank) {
            int pos = -1;
            for (int p = 0; p < topk && pos < 0; ++p) {
                int sr = 0;
                for (int o = 0; o < topk; ++o)
                    if (te[o] < te[p] || (te[o] == te[p] && o < p)) ++sr;
                if (sr == rank) pos = p;
            }
            if (pos < 0) { ok = false; break; }
            const size_t s = t * topk + pos;
            const __half rv = __float2half_rn(raw[s * hidden + h]);
            const __half wv = __float2half_rn(__fmul_rn(__half2float(rv), w[s]));
            acc = __float2half_rn(__fadd_rn(__half2float(acc), __half2float(wv)));
        }
        if (ok) out[i] = acc;
    }
}

// The official combination (deepseek_v4_moe_reference.py:186-194): routed
// outputs already carry their weights; out = their sum, then + the shared
// expert.  Rank order, FP32.
__global__ void combine_sum_kernel(const float* __restrict__ raw, const float* __restrict__ shared,
                                   int tokens, int topk, int hidden, float* __restrict__ out) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = (i * 4) / hidden;
        const size_t h = i * 4 - t * hidden;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < topk; ++r) {
            const float4 v = *reinterpret_cast<const float4*>(raw + (t * topk + r) * hidden + h);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (shared) {
            const float4 v = *reinterpret_cast<const float4*>(shared + t * hidden + h);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        *reinterpret_cast<float4*>(out + t * hidden + h) = acc;
    }
}

__global__ void ids_i64_to_i32_kernel(const int64_t* __restrict__ src, int n, int experts,
                                      int32_t* __restrict__ dst, uint32_t* status) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int64_t e = src[i];
        if (e < 0 || e >= experts) {
            atomicOr(status, kStatusBadExpert);
            dst[i] = -1;
        } else {
            dst[i] = static_cast<int32_t>(e);
        }
    }
}

int grid_for(size_t n, int threads, int cap) {
    size_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > static_cast<size_t>(cap)) g = cap;
    return static_cast<int>(g);
}

}  // namespace

cudaError_t launch_route_topk(const float* logits, int tokens, int experts, int topk,
                              int32_t* ids, float* weights, uint32_t* status,
                              cudaStream_t stream) {
    if (tokens <= 0 || experts <= 0 || experts > 32 * kRouteMaxPerLane || topk <= 0 ||
        topk > 32 || topk > experts)
        return cudaErrorInvalidValue;
    const int warps = 4;
    const int grid = (tokens + warps - 1) / warps;
    const size_t smem = static_cast<size_t>(warps) * experts * sizeof(float);
    if (experts <= 256)
        return launch_pdl(route_topk_kernel<8>, dim3(grid), dim3(warps * 32), smem, stream, logits,
                          tokens, experts, topk, ids, weights, status);
    return launch_pdl(route_topk_kernel<kRouteMaxPerLane>, dim3(grid), dim3(warps * 32), smem, stream,
                      logits, tokens, experts, topk, ids, weights, status);
}

cudaError_t launch_route_dsv4(const float* logits, const float* bias, const int64_t* tid2eid,
                              const int64_t* input_ids, int tokens, int experts, int topk,
                              float route_scale, int32_t* ids, float* weights, uint32_t* status,
                              cudaStream_t stream) {
    if (tokens <= 0 || experts <= 0 || experts > 32 * kRouteMaxPerLane || topk <= 0 ||
        topk > 32 || topk > experts || (tid2eid && !input_ids))
        return cudaErrorInvalidValue;
    const int warps = 4;
    const int grid = (tokens + warps - 1) / warps;
    const size_t smem = static_cast<size_t>(warps) * experts * sizeof(float);
    return launch_pdl(route_dsv4_kernel, dim3(grid), dim3(warps * 32), smem, stream, logits, bias,
                      tid2eid, input_ids, tokens, experts, topk, route_scale, ids, weights, status);
}

int permute_launch_count(int tokens, int topk, const PermuteOut& out) {
    const long long chunks = (static_cast<long long>(tokens) * topk + kPermChunk - 1) / kPermChunk;
    return chunks > 2 && out.chunk_counts && out.lrank && chunks <= out.max_chunks ? 2 : 1;
}

cudaError_t launch_permute(const int32_t* ids, int tokens, int topk, int experts, int n_tile_max,
                           int max_tiles, const PermuteOut& out, uint32_t* status,
                           cudaStream_t stream, bool skip_negative) {
    if (experts <= 0 || experts > kPermMaxExperts || tokens <= 0 || topk <= 0 || n_tile_max < 8)
        return cudaErrorInvalidValue;
    if (permute_launch_count(tokens, topk, out) == 2) {
        const long long chunks = (static_cast<long long>(tokens) * topk + kPermChunk - 1) / kPermChunk;
        cudaError_t err = launch_pdl(permute_count_kernel, dim3(static_cast<unsigned>(chunks)), dim3(kPermChunk), 0,
                                     stream, ids, tokens, topk, experts, out, status, skip_negative);
        if (err != cudaSuccess) return err;
        return launch_pdl(permute_place_kernel, dim3(static_cast<unsigned>(chunks)), dim3(kPermChunk), 0, stream,
                          ids, tokens, topk, experts, n_tile_max, max_tiles, out, status);
    }
    return launch_pdl(permute_kernel, dim3(1), dim3(kPermThreads), 0, stream, ids, tokens, topk,
                      experts, n_tile_max, max_tiles, out, status, skip_negative);
}

cudaError_t launch_route_permute(const float* logits, int tokens, int experts, int topk, int32_t* ids,
                                 float* weights, int n_tile_max, int max_tiles, const PermuteOut& out,
                                 uint32_t* status, cudaStream_t stream) {
    if (!route_permute_fits(tokens, topk, experts) || n_tile_max < 8 || topk > 32)
        return cudaErrorInvalidValue;
    return launch_pdl(route_permute_kernel, dim3(1), dim3(kPermThreads), 0, stream, logits, tokens, experts, topk,
                      ids, weights, n_tile_max, max_tiles, out, status);
}

cudaError_t launch_gather_rows(const __half* x, const int32_t* perm, const int32_t* total_rows_dev,
                               int max_rows, int topk, int hidden, __half* x_perm,
                               cudaStream_t stream) {
    if (hidden % 8 != 0 || max_rows <= 0) return cudaErrorInvalidValue;
    const int grid = max_rows < 148 * 8 ? max_rows : 148 * 8;
    return launch_pdl(gather_rows_kernel, dim3(grid), dim3(kGatherThreads), 0, stream, x, perm, total_rows_dev,
                      max_rows, topk, hidden, x_perm);
}

cudaError_t launch_combine_f32(const float* raw, const float* weights, int tokens, int topk,
                               int hidden, float* out, cudaStream_t stream) {
    if (hidden % 4 != 0) return cudaErrorInvalidValue;
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    return launch_pdl(combine_f32_kernel, dim3(grid_for(n4, 256, 148 * 16)), dim3(256), 0, stream,
                      raw, weights, tokens, topk, hidden, out);
}

cudaError_t launch_combine_f16(const float* raw, const float* weights, const int64_t* ids64,
                               int tokens, int topk, int hidden, __half* out,
                               cudaStream_t stream) {
    const size_t n = static_cast<size_t>(tokens) * hidden;
    return launch_pdl(combine_f16_kernel<int64_t>, dim3(grid_for(n, 256, 148 * 16)), dim3(256), 0,
                      stream, raw, weights, ids64, tokens, topk, hidden, out);
}

cudaError_t launch_combine_f16_i32(const float* raw, const float* weights, const int32_t* ids,
                                   int tokens, int topk, int hidden, __half* out,
                                   cudaStream_t stream) {
    const size_t n = static_cast<size_t>(tokens) * hidden;
    return launch_pdl(combine_f16_kernel<int32_t>, dim3(grid_for(n, 256, 148 * 16)), dim3(256), 0,
                      stream, raw, weights, ids, tokens, topk, hidden, out);
}

cudaError_t launch_combine_sum(const float* raw, const float* shared, int tokens, int topk, int hidden,
                               float* out, cudaStream_t stream) {
    if (hidden % 4 != 0) return cudaErrorInvalidValue;
    const size_t n4 = static_cast<size_t>(tokens) * hidden / 4;
    return launch_pdl(combine_sum_kernel, dim3(grid_for(n4, 256, 148 * 4)), dim3(256), 0, stream, raw,
                      shared, tokens, topk, hidden, out);
}

cudaError_t launch_ids_i64_to_i32(const int64_t* src, int n, int experts, int32_t* dst,
                                  uint32_t* status, cudaStream_t stream) {
    return launch_pdl(ids_i64_to_i32_kernel, dim3(grid_for(n, 256, 1024)), dim3(256), 0, stream, src,
                      n, experts, dst, status);
}

}  // namespace dee
