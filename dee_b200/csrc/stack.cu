// stack.cu -- the dense glue of the synthetic 43-layer stack that exercises
// the routed-expert layer end to end (embedding, RMSNorm, router logits,
// residual add, LM head argmax), and the scrambler that derives distinct
// expert banks per layer.
//
// Every per-token result is computed in a fixed order that does not depend
// on how many tokens share the launch, so a token's outputs -- and with them
// the route ids the journal records -- are bit-identical whether the tokens
// are decoded on one GPU or spread over several.
#include "kernels.h"

namespace dee {
namespace {

constexpr int kNormThreads = 256;

// Fixed-order sum of one warp's lane partials.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void embed_kernel(const __half* __restrict__ table, const int32_t* __restrict__ ids, int tokens,
                             int hidden, int vocab, float* __restrict__ x, uint32_t* status) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int t = blockIdx.x;
    if (t >= tokens) return;
    int id = ids[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) atomicOr(status, sm100::kStatusBadShape);
        id = 0;
    }
    for (int h = threadIdx.x; h < hidden; h += blockDim.x)
        x[static_cast<size_t>(t) * hidden + h] = __half2float(table[static_cast<size_t>(id) * hidden + h]);
}

// One CTA per token: y = fp16(x * rsqrt(mean(x^2) + eps) * w).  Each thread
// sums a fixed strided subset, warps reduce by a fixed tree, warp totals are
// added in warp order.
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                               int tokens, int hidden, __half* __restrict__ y) {
    __shared__ float part[kNormThreads / 32];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int t = blockIdx.x;
    if (t >= tokens) return;
    const float* xr = x + static_cast<size_t>(t) * hidden;
    float s = 0.0f;
    for (int h = threadIdx.x; h < hidden; h += kNormThreads) s = fmaf(xr[h], xr[h], s);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < kNormThreads / 32; ++i) tot += part[i];
    const float r = rsqrtf(tot / static_cast<float>(hidden) + eps);
    for (int h = threadIdx.x; h < hidden; h += kNormThreads)
        y[static_cast<size_t>(t) * hidden + h] = __float2half_rn(xr[h] * r * w[h]);
}

// One warp per (token, output row): out = sum_h x[t, h] * W[row, h] (W FP32
// or FP16 [rows, H]), lane-strided partials then a fixed tree.
template <class WT>
__global__ void rowdot_kernel(const __half* __restrict__ x, const WT* __restrict__ w, int tokens, int hidden,
                              int rows, float* __restrict__ out) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int lane = threadIdx.x & 31;
    const size_t pairs = static_cast<size_t>(tokens) * rows;
    const size_t warps_total = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x >> 5) + (threadIdx.x >> 5); i < pairs;
         i += warps_total) {
        const size_t t = i / rows, r = i - t * rows;
        const __half* xr = x + t * hidden;
        const WT* wr = w + r * hidden;
        float s = 0.0f;
        for (int h = lane; h < hidden; h += 32) s = fmaf(__half2float(xr[h]), static_cast<float>(wr[h]), s);
        s = warp_sum(s);
        if (lane == 0) out[t * rows + r] = s;
    }
}

__global__ void residual_add_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        x[i] = __fadd_rn(x[i], y[i]);
}

// One CTA per token: the first index of the maximum logit.
__global__ void argmax_kernel(const float* __restrict__ logits, int tokens, int vocab, int32_t* __restrict__ ids) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int t = blockIdx.x;
    if (t >= tokens) return;
    const float* l = logits + static_cast<size_t>(t) * vocab;
    float best = -INFINITY;
    int idx = vocab;
    for (int v = threadIdx.x; v < vocab; v += blockDim.x)
        if (l[v] > best) { best = l[v]; idx = v; }  // strided ascending: first max per thread
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) { bv[warp] = best; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < nw; ++i)
            if (bv[i] > best || (bv[i] == best && bi[i] < idx)) { best = bv[i]; idx = bi[i]; }
        ids[t] = idx < vocab ? idx : 0;
    }
}

__device__ __forceinline__ uint32_t mix32(uint64_t v) {
    v ^= v >> 33;
    v *= 0xff51afd7ed558ccdull;
    v ^= v >> 33;
    v *= 0xc4ceb9fe1a85ec53ull;
    v ^= v >> 33;
    return static_cast<uint32_t>(v);
}

// dst record i = src record i with its packed weight bytes [0, packed_bytes)
// XORed by a hash of (seed, first_record + i, word): valid E2M1 codes of the
// same scale, a distinct bank per seed.  Scales are copied.
__global__ void scramble_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int records,
                                size_t record_bytes, size_t packed_bytes, uint64_t seed, int first_record) {
    const size_t words = record_bytes / 16;
    const size_t total = static_cast<size_t>(records) * words;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i / words, w = i - r * words;
        uint4 v = reinterpret_cast<const uint4*>(src + r * record_bytes)[w];
        if (w * 16 < packed_bytes) {
            const uint64_t base = (seed << 40) ^ (static_cast<uint64_t>(first_record + r) << 24) ^ (w * 4);
            v.x ^= mix32(base);
            v.y ^= mix32(base + 1);
            v.z ^= mix32(base + 2);
            v.w ^= mix32(base + 3);
        }
        reinterpret_cast<uint4*>(dst + r * record_bytes)[w] = v;
    }
}

}  // namespace

cudaError_t launch_stack_embed(const __half* table, const int32_t* ids, int tokens, int hidden, int vocab,
                               float* x, uint32_t* status, cudaStream_t stream) {
    return launch_pdl(embed_kernel, dim3(tokens), dim3(256), 0, stream, table, ids, tokens, hidden, vocab, x,
                      status);
}

cudaError_t launch_stack_rmsnorm(const float* x, const float* w, float eps, int tokens, int hidden, __half* y,
                                 cudaStream_t stream) {
    return launch_pdl(rmsnorm_kernel, dim3(tokens), dim3(kNormThreads), 0, stream, x, w, eps, tokens, hidden, y);
}

cudaError_t launch_stack_rowdot_f32(const __half* x, const float* w, int tokens, int hidden, int rows,
                                    float* out, cudaStream_t stream) {
    const size_t pairs = static_cast<size_t>(tokens) * rows;
    const int grid = static_cast<int>(pairs / 8 + 1 < 148 * 16 ? pairs / 8 + 1 : 148 * 16);
    return launch_pdl(rowdot_kernel<float>, dim3(grid), dim3(256), 0, stream, x, w, tokens, hidden, rows, out);
}

cudaError_t launch_stack_rowdot_f16(const __half* x, const __half* w, int tokens, int hidden, int rows,
                                    float* out, cudaStream_t stream) {
    const size_t pairs = static_cast<size_t>(tokens) * rows;
    const int grid = static_cast<int>(pairs / 8 + 1 < 148 * 16 ? pairs / 8 + 1 : 148 * 16);
    return launch_pdl(rowdot_kernel<__half>, dim3(grid), dim3(256), 0, stream, x, w, tokens, hidden, rows, out);
}

cudaError_t launch_stack_residual_add(float* x, const float* y, size_t n, cudaStream_t stream) {
    const int grid = static_cast<int>((n + 255) / 256 < 148 * 4 ? (n + 255) / 256 : 148 * 4);
    return launch_pdl(residual_add_kernel, dim3(grid), dim3(256), 0, stream, x, y, n);
}

cudaError_t launch_stack_argmax(const float* logits, int tokens, int vocab, int32_t* ids, cudaStream_t stream) {
    return launch_pdl(argmax_kernel, dim3(tokens), dim3(1024), 0, stream, logits, tokens, vocab, ids);
}

cudaError_t launch_records_scramble(const uint8_t* src, uint8_t* dst, int records, size_t record_bytes,
                                    size_t packed_bytes, uint64_t seed, int first_record, cudaStream_t stream) {
    if (record_bytes % 16 || packed_bytes % 16) return cudaErrorInvalidValue;
    scramble_kernel<<<148 * 8, 256, 0, stream>>>(src, dst, records, record_bytes, packed_bytes, seed,
                                                 first_record);
    return cudaGetLastError();
}

}  // namespace dee
