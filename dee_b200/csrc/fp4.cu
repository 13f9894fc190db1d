// fp4.cu -- standalone FP4 E2M1 + UE8M0 decode (the unit-testable twin of
// the GEMM's in-register dequant) and a device quantiser that packs FP32
// weights into the same record format for synthetic benchmarks.
#include "kernels.h"

namespace dee {
namespace {

__device__ __forceinline__ uint32_t cvt_e2m1x2(uint32_t byte) {
    uint32_t o;
    asm("{\n\t.reg .b8 b0;\n\t"
        "cvt.u8.u32 b0, %1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
        : "=r"(o)
        : "r"(byte));
    return o;
}

__device__ __forceinline__ float scale_value(uint32_t b) {
    const int e = static_cast<int>(b) - 127;
    if (e >= 127) return __int_as_float(0x7F7FFFFF);
    if (e <= -127) return 0.0f;
    return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// fp4_e2m1_to_f16_kernel semantics (reference dee.cpp/src/cuda_convert.cu
// :231-245): W[o, i] = FP16_RN(table[nibble] * 2^(s - 127)) with the scale
// clamps of :217-223; the table's negative-zero entry decodes to +0.
// One thread per packed byte (two outputs).
__global__ void fp4_decode_kernel(const uint8_t* __restrict__ packed,
                                  const uint8_t* __restrict__ scale, __half* __restrict__ dst,
                                  size_t out, size_t in) {
    const size_t half_in = in >> 1;
    const size_t n = out * half_in;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t o = i / half_in;
        const size_t c = i - o * half_in;  // byte column: elements 2c, 2c+1
        const uint32_t byte = packed[i];
        const float s = scale_value(scale[o * (in >> 5) + ((2 * c) >> 5)]);
        // nibble 8 decodes to -0 in E2M1 but the reference table holds +0
        // there (cuda_convert.cu:212-215): clear that sign before scaling.
        uint32_t pair = cvt_e2m1x2(byte);
        if ((pair & 0xFFFFu) == 0x8000u) pair &= 0xFFFF0000u;
        if ((pair >> 16) == 0x8000u) pair &= 0x0000FFFFu;
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&pair));
        const __half lo = __float2half_rn(__fmul_rn(v.x, s));
        const __half hi = __float2half_rn(__fmul_rn(v.y, s));
        reinterpret_cast<__half2*>(dst)[i] = __halves2half2(lo, hi);
    }
}

// Per 32-element block: scale = 2^ceil(log2(max(amax, 6*2^-126) / 6)) as a
// UE8M0 byte, q = clamp(w / scale, -6, 6) rounded to the E2M1 grid with
// ties to the even grid entry (the recipe of the reference's quantisation
// helpers, dee.cpp/scripts/deepseek_v4_layer_common.py:160-211).
__global__ void fp4_quantize_kernel(const float* __restrict__ w, size_t out, size_t in,
                                    uint8_t* __restrict__ packed, uint8_t* __restrict__ scale) {
    const size_t blocks = out * (in >> 5);
    for (size_t b = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; b < blocks;
         b += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float* src = w + b * 32;
        float v[32];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 f = *reinterpret_cast<const float4*>(src + i);
            v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, 6.0f * 1.1754943508222875e-38f);
        const uint32_t bits = __float_as_uint(__fmul_rn(amax, 1.0f / 6.0f));
        const int e = static_cast<int>((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0 ? 1 : 0);
        const float s = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
        uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float q = __fdiv_rn(v[i], s);
            q = fminf(fmaxf(q, -6.0f), 6.0f);
            const float a = fabsf(q);
            uint32_t m;
            if (a <= 0.25f) m = 0;
            else if (a < 0.75f) m = 1;
            else if (a <= 1.25f) m = 2;
            else if (a < 1.75f) m = 3;
            else if (a <= 2.5f) m = 4;
            else if (a < 3.5f) m = 5;
            else if (a <= 5.0f) m = 6;
            else m = 7;
            const uint32_t nib = m | ((q < 0.0f && m != 0) ? 8u : 0u);
            words[i >> 3] |= nib << ((i & 7) * 4);
        }
        uint4* dst = reinterpret_cast<uint4*>(packed + b * 16);
        *dst = make_uint4(words[0], words[1], words[2], words[3]);
        scale[b] = static_cast<uint8_t>(e + 127);
    }
}

}  // namespace

cudaError_t launch_fp4_decode(const uint8_t* packed, const uint8_t* scale, __half* dst,
                              size_t out, size_t in, cudaStream_t stream) {
    if (in % 64 != 0 || out == 0) return cudaErrorInvalidValue;
    const size_t n = out * (in / 2);
    size_t grid = (n + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    fp4_decode_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(packed, scale, dst, out, in);
    return cudaGetLastError();
}

cudaError_t launch_fp4_quantize(const float* w, size_t out, size_t in, uint8_t* packed,
                                uint8_t* scale, cudaStream_t stream) {
    if (in % 32 != 0 || out == 0) return cudaErrorInvalidValue;
    const size_t blocks = out * (in / 32);
    size_t grid = (blocks + 127) / 128;
    if (grid > 148 * 32) grid = 148 * 32;
    fp4_quantize_kernel<<<static_cast<unsigned>(grid), 128, 0, stream>>>(w, out, in, packed, scale);
    return cudaGetLastError();
}

}  // namespace dee
