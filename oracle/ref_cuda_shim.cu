// ref_cuda_shim.cu -- a C entry point over the reference project's own GPU
// expert path, for parity tests on the B200.
//
// TEST INFRASTRUCTURE ONLY (a checker; never the product path).
// oracle/Makefile (target ref_cuda) compiles this file together with the
// reference's sources where they lie:
//   dee.cpp/src/cuda_convert.cu  -> dee::fp4_e2m1_to_f16_cuda
//                                   (cuda_convert.cu:252-288)
//   dee.cpp/src/swiglu_cuda.cu   -> dee::swiglu_expert_batch_fp16_cuda
//                                   (swiglu_cuda.cu:387-431: cuBLAS FP16 gate
//                                   and up GEMMs to FP16, the FP16 SwiGLU
//                                   kernel, cuBLAS down GEMM to FP32)
//   dee.cpp/src/profiling.cpp    -> StageProfiler (a dependency of the above)
// into oracle/_ref/libdee_ref_cuda.so, linked with cuBLAS.  The layer loop
// below is the engine's routed-expert device path
// (Engine::moe_forward_batch_device_impl, engine.cpp:776-1190): group the
// selections by expert in (rank, token) order (:812-823), and per active
// expert in ascending id gather its token rows, decode its record's three
// projections into FP16 scratch (decode_fp4_cache_block_to_scratch,
// :3797-3845), run the batched FP16 SwiGLU and scatter the FP32 rows to
// raw[token * K + rank] (:1080-1113).  Nothing here re-implements reference
// arithmetic; the adapter only sequences the reference's own functions.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

#include "dee/cuda_convert.h"
#include "dee/swiglu_cuda.h"

namespace {

struct Layout {
    size_t w1, w3, w2, s1, s3, s2, bytes;
};

Layout record_layout(size_t hidden, size_t inter) {
    const size_t ih = hidden * inter;
    Layout L{};
    L.w1 = 0;
    L.w3 = ih / 2;
    L.w2 = ih;
    L.s1 = ih + ih / 2;
    L.s3 = L.s1 + ih / 32;
    L.s2 = L.s3 + ih / 32;
    L.bytes = L.s2 + ih / 32;
    return L;
}

}  // namespace

// d_records: device, `experts` records of record_bytes in the DEE4 layout.
// h_x: host FP16 bits [tokens, hidden]; h_ids: host int32 [tokens, topk];
// h_raw: host FP32 [tokens, topk, hidden] (every selection written).
// Returns 0, or -1 (bad id) / -2 (CUDA or cuBLAS failure).
extern "C" int dee_refcuda_moe_layer(const uint8_t* d_records, size_t record_bytes, int hidden, int inter,
                                     int experts, int topk, const uint16_t* h_x, int tokens,
                                     const int32_t* h_ids, float swiglu_limit, float* h_raw) {
    const Layout L = record_layout(static_cast<size_t>(hidden), static_cast<size_t>(inter));
    // group: positions t*K + r of each expert in (rank, token) order
    std::vector<std::vector<int>> rows(static_cast<size_t>(experts));
    for (int r = 0; r < topk; ++r)
        for (int t = 0; t < tokens; ++t) {
            const int e = h_ids[static_cast<size_t>(t) * topk + r];
            if (e < 0 || e >= experts) return -1;
            rows[static_cast<size_t>(e)].push_back(t * topk + r);
        }
    size_t max_n = 1;
    for (const auto& v : rows) max_n = v.size() > max_n ? v.size() : max_n;
    const size_t ih = static_cast<size_t>(hidden) * inter;
    cudaStream_t stream = nullptr;
    cublasHandle_t handle = nullptr;
    void *d_w = nullptr, *d_x = nullptr, *d_gate = nullptr, *d_up = nullptr, *d_act = nullptr;
    float* d_y = nullptr;
    int rc = 0;
    std::vector<uint16_t> xe;
    std::vector<float> ye;
    if (cudaStreamCreate(&stream) != cudaSuccess || cublasCreate(&handle) != CUBLAS_STATUS_SUCCESS ||
        cublasSetStream(handle, stream) != CUBLAS_STATUS_SUCCESS ||
        cudaMalloc(&d_w, 3 * ih * sizeof(uint16_t)) != cudaSuccess ||
        cudaMalloc(&d_x, max_n * hidden * sizeof(uint16_t)) != cudaSuccess ||
        cudaMalloc(&d_gate, max_n * inter * sizeof(uint16_t)) != cudaSuccess ||
        cudaMalloc(&d_up, max_n * inter * sizeof(uint16_t)) != cudaSuccess ||
        cudaMalloc(&d_act, max_n * inter * sizeof(uint16_t)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&d_y), max_n * hidden * sizeof(float)) != cudaSuccess) {
        rc = -2;
    }
    auto* w16 = static_cast<uint16_t*>(d_w);
    for (int e = 0; e < experts && rc == 0; ++e) {
        const auto& pos = rows[static_cast<size_t>(e)];
        if (pos.empty()) continue;
        const int n = static_cast<int>(pos.size());
        xe.resize(static_cast<size_t>(n) * hidden);
        for (int i = 0; i < n; ++i)
            for (int h = 0; h < hidden; ++h)
                xe[static_cast<size_t>(i) * hidden + h] =
                    h_x[static_cast<size_t>(pos[static_cast<size_t>(i)] / topk) * hidden + h];
        const uint8_t* rec = d_records + static_cast<size_t>(e) * record_bytes;
        if (cudaMemcpyAsync(d_x, xe.data(), xe.size() * sizeof(uint16_t), cudaMemcpyHostToDevice, stream) !=
                cudaSuccess ||
            !dee::fp4_e2m1_to_f16_cuda(rec + L.w1, rec + L.s1, w16, static_cast<size_t>(inter),
                                       static_cast<size_t>(hidden), stream) ||
            !dee::fp4_e2m1_to_f16_cuda(rec + L.w3, rec + L.s3, w16 + ih, static_cast<size_t>(inter),
                                       static_cast<size_t>(hidden), stream) ||
            !dee::fp4_e2m1_to_f16_cuda(rec + L.w2, rec + L.s2, w16 + 2 * ih, static_cast<size_t>(hidden),
                                       static_cast<size_t>(inter), stream) ||
            !dee::swiglu_expert_batch_fp16_cuda(handle, d_w, d_x, d_gate, d_up, d_act, d_y, n, inter, hidden,
                                                stream, nullptr, swiglu_limit)) {
            rc = -2;
            break;
        }
        ye.resize(static_cast<size_t>(n) * hidden);
        if (cudaMemcpyAsync(ye.data(), d_y, ye.size() * sizeof(float), cudaMemcpyDeviceToHost, stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess) {
            rc = -2;
            break;
        }
        for (int i = 0; i < n; ++i)
            for (int h = 0; h < hidden; ++h)
                h_raw[static_cast<size_t>(pos[static_cast<size_t>(i)]) * hidden + h] =
                    ye[static_cast<size_t>(i) * hidden + h];
    }
    cudaFree(d_w);
    cudaFree(d_x);
    cudaFree(d_gate);
    cudaFree(d_up);
    cudaFree(d_act);
    cudaFree(d_y);
    if (handle) cublasDestroy(handle);
    if (stream) cudaStreamDestroy(stream);
    return rc;
}
