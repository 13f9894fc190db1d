// decode_common.cuh -- device helpers shared by the register-dequant GEMMs
// (moe_decode.cu for packed FP4 records, moe_shared.cu for the FP8 shared
// expert): mma.sync fragments, 32-bit shared-memory loads, named barriers and
// the SwiGLU epilogues.
#pragma once

#include "sm100.cuh"

namespace dee {

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

// FP32 scale of a UE8M0 byte: 2^(b - 127) for every byte (b = 0 is the
// subnormal 2^-127, b = 255 is +inf), as decode_e8m0 of the reference
// (dee.cpp/scripts/deepseek_v4_expert_reference.py:49-62).
__device__ __forceinline__ float e8m0_value(uint32_t b) {
    return b ? __uint_as_float(b << 23) : __uint_as_float(0x00400000u);
}

// One SwiGLU output of the gate/up epilogue.
//  live:     the reference engine's FP16 chain (swiglu_cuda.cu:46-59):
//            gate and up rounded to FP16, optional clamp, SiLU rounded to
//            FP16, the product rounded to FP16;
//  official: the FP32 chain of the official expert
//            (deepseek_v4_moe_reference.py:87-110): clamp, SiLU, product and
//            the routing weight (1 for the shared expert) in FP32, rounded
//            once to FP16 as the down projection's operand.
__device__ __forceinline__ __half swiglu_out(float g, float u, float lim, bool official, float w) {
    if (!official) {
        g = __half2float(__float2half_rn(g));
        u = __half2float(__float2half_rn(u));
        if (lim > 0.0f) {
            g = fminf(g, lim);
            u = fminf(fmaxf(u, -lim), lim);
        }
        const __half sv = __float2half_rn(silu_ref(g));
        return __float2half_rn(__fmul_rn(__half2float(sv), u));
    }
    if (lim > 0.0f) {
        g = fminf(g, lim);
        u = fminf(fmaxf(u, -lim), lim);
    }
    return __float2half_rn(__fmul_rn(__fmul_rn(silu_ref(g), u), w));
}

}  // namespace dee
