// act_quant.cu -- block-wise FP8 activation quantisation with power-of-two
// (UE8M0) scales, the official act_quant of the DeepSeek-V4 inference code
// (official-source/inference/kernel.py:41-103 with scale_fmt = "ue8m0";
// restated in dee.cpp/scripts/deepseek_v4_layer_common.py:160-240):
//
//   amax  = max(|x| over the block, 1e-4)                 (FP32)
//   s     = 2^ceil(log2(amax * (1/448)))                  (exponent bits)
//   q     = e4m3_rn(clamp(x / s, -448, 448))
//   scale = the UE8M0 byte of s, log2(s) + 127
//
// block = 128 is the official granularity; block = 32 is the MX form, one
// scale per 32 K, the granularity tcgen05.mma kind::mxf8f6f4 consumes (a
// block-128 scale is the same value repeated over its four 32-blocks).
// With a permutation the kernel gathers token rows (row r of the output is
// token perm[r] / topk) while it quantises -- the MXFP8 counterpart of the
// FP16 row gather of the grouped GEMMs.
#include <cuda_fp8.h>

#include "kernels.h"

namespace dee {
namespace {

// One warp per four 256-column segments of a row (its loads are all issued
// before the first is used, so each warp keeps four 512-byte reads in
// flight); lane j owns columns 8j..8j+7 of a segment (one 16-byte load), so a
// block of 32 spans 4 lanes and a block of 128 spans 16.
constexpr int kSegsPerWarp = 4;

template <int BLOCK>
__device__ __forceinline__ void quantise_segment(const uint4 raw, int lane, uint8_t* __restrict__ q_row,
                                                 uint8_t* __restrict__ s_row, int col, bool per32) {
    constexpr int kLanes = BLOCK / 8;  // lanes per block
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < kLanes; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1e-4f);
    // ceil(log2(amax / 448)) from the exponent and mantissa bits
    const uint32_t b = __float_as_uint(amax * (1.0f / 448.0f));
    const int e = static_cast<int>((b >> 23) & 0xFFu) - 127 + ((b & 0x7FFFFFu) != 0 ? 1 : 0);
    const float inv_s = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e, exact
    uint32_t packed[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = fminf(fmaxf(v[2 * i] * inv_s, -448.0f), 448.0f);
        const float c = fminf(fmaxf(v[2 * i + 1] * inv_s, -448.0f), 448.0f);
        const __nv_fp8x2_storage_t p = __nv_cvt_float2_to_fp8x2(make_float2(a, c), __NV_SATFINITE, __NV_E4M3);
        const uint32_t pv = static_cast<uint32_t>(p);
        if (i & 1) packed[i >> 1] |= pv << 16;
        else packed[i >> 1] = pv;
    }
    *reinterpret_cast<uint2*>(q_row + col) = make_uint2(packed[0], packed[1]);
    if (per32) {
        // one byte per 32 columns (a block of 128 repeats its scale four times)
        if ((lane & 3) == 0) s_row[col / 32] = static_cast<uint8_t>(e + 127);
    } else if ((lane % kLanes) == 0) {
        s_row[col / BLOCK] = static_cast<uint8_t>(e + 127);
    }
}

template <int BLOCK>
__global__ void act_quant_kernel(const __half* __restrict__ x, int rows, int cols, const int32_t* __restrict__ perm,
                                 int topk, const int32_t* __restrict__ rows_dev, uint8_t* __restrict__ q,
                                 uint8_t* __restrict__ scales, bool per32) {
    sm100::pdl_wait();
    sm100::pdl_trigger();
    const int n_rows = rows_dev ? min(*rows_dev, rows) : rows;
    const int segs = cols / 256;
    const int chunks = (segs + kSegsPerWarp - 1) / kSegsPerWarp;
    const int lane = threadIdx.x & 31;
    const int s_cols = per32 ? cols / 32 : cols / BLOCK;  // scale bytes per row
    const long long warps_total = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long w = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
         w < static_cast<long long>(n_rows) * chunks; w += warps_total) {
        const int row = static_cast<int>(w / chunks);
        const int s0 = static_cast<int>(w - static_cast<long long>(row) * chunks) * kSegsPerWarp;
        const int ns = min(kSegsPerWarp, segs - s0);
        const int src_row = perm ? perm[row] / topk : row;
        const __half* src = x + static_cast<size_t>(src_row) * cols + lane * 8;
        uint4 raw[kSegsPerWarp];
#pragma unroll
        for (int i = 0; i < kSegsPerWarp; ++i)
            if (i < ns) raw[i] = __ldg(reinterpret_cast<const uint4*>(src + (s0 + i) * 256));
        uint8_t* q_row = q + static_cast<size_t>(row) * cols;
        uint8_t* s_row = scales + static_cast<size_t>(row) * s_cols;
#pragma unroll
        for (int i = 0; i < kSegsPerWarp; ++i)
            if (i < ns) quantise_segment<BLOCK>(raw[i], lane, q_row, s_row, (s0 + i) * 256 + lane * 8, per32);
    }
}

}  // namespace

cudaError_t launch_act_quant(const __half* x, int rows, int cols, int block, const int32_t* perm, int topk,
                             const int32_t* rows_dev, uint8_t* q, uint8_t* scales, cudaStream_t stream, bool per32) {
    if (rows < 0 || cols % 256 != 0 || (block != 32 && block != 128) || (perm && topk <= 0))
        return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    const long long warps = static_cast<long long>(rows) * ((cols / 256 + kSegsPerWarp - 1) / kSegsPerWarp);
    const int grid = static_cast<int>(warps / 8 + 1 < 148 * 8 ? warps / 8 + 1 : 148 * 8);
    return block == 32
               ? launch_pdl(act_quant_kernel<32>, dim3(grid), dim3(256), 0, stream, x, rows, cols, perm, topk,
                            rows_dev, q, scales, per32)
               : launch_pdl(act_quant_kernel<128>, dim3(grid), dim3(256), 0, stream, x, rows, cols, perm, topk,
                            rows_dev, q, scales, per32);
}

}  // namespace dee
