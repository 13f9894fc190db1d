// ref_shim.cpp -- C entry points over the reference project's own CPU code.
//
// TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline; never
// the product path).  oracle/Makefile compiles this file together with the
// reference's sources where they lie:
//   dee.cpp/src/weight_mmap.cpp + dee.cpp/src/json_min.cpp
//       -> dee::fp4_e2m1_dequantize (weight_mmap.cpp:101-117)
//   dee.cpp/experiments/kt_cpu_bridge/src/reference_cpu_executor.cpp
//       -> dee::ktbridge::ReferenceCpuExecutor::execute (:100-151), the
//          reference's portable FP32 routed-expert executor
// into oracle/_ref/libdee_ref.so.  Nothing here re-implements reference
// arithmetic; it only adapts the C++ interfaces to a C ABI and fans the
// per-(token, expert) executor calls out over host threads.
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

#include "dee/weight_mmap.h"
#include "kt_bridge/reference_cpu_executor.hpp"

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

dee::ktbridge::PackedExpertView view_of(const uint8_t* rec, size_t hidden, size_t inter) {
    const Layout L = record_layout(hidden, inter);
    dee::ktbridge::PackedExpertView v;
    v.gate = {rec + L.w1, rec + L.s1, inter, hidden, inter * hidden / 2, inter * hidden / 32};
    v.up = {rec + L.w3, rec + L.s3, inter, hidden, inter * hidden / 2, inter * hidden / 32};
    v.down = {rec + L.w2, rec + L.s2, hidden, inter, inter * hidden / 2, inter * hidden / 32};
    return v;
}

}  // namespace

extern "C" {

// dee::fp4_e2m1_dequantize over one [out, in] projection.
void dee_refimpl_fp4_dequantize(const uint8_t* packed, const uint8_t* scale,
                                size_t out, size_t in, float* dst) {
    dee::fp4_e2m1_dequantize(packed, scale, out, in, dst);
}

// One routed expert for one token through ReferenceCpuExecutor (routing
// weight applied before w2, FP32).  Returns the executor's error code.
int dee_refimpl_expert(const uint8_t* record, size_t hidden, size_t inter,
                       const float* x, float routing_weight, float swiglu_limit,
                       float* out) {
    dee::ktbridge::ReferenceCpuExecutor ex;
    dee::ktbridge::ExecuteConfig cfg;
    cfg.swiglu_limit = swiglu_limit;
    const auto v = view_of(record, hidden, inter);
    return static_cast<int>(ex.execute(0, 0, v, x, hidden, routing_weight, cfg, out, hidden));
}

// A whole layer's routed experts: for every selection (t, r) run the
// executor with weight w[t, r] and sum the K results per token in rank
// order into out[t, :].  Selections are spread over `threads` host threads
// (0 = hardware concurrency).  Returns 0 or the first executor error.
int dee_refimpl_moe_layer(const uint8_t* records, size_t record_bytes,
                          size_t hidden, size_t inter, int topk,
                          const float* x, int tokens, const int32_t* ids,
                          const float* weights, float swiglu_limit, int threads,
                          float* out) {
    const size_t sel = static_cast<size_t>(tokens) * topk;
    std::vector<float> partial(sel * hidden);
    std::atomic<size_t> next{0};
    std::atomic<int> err{0};
    unsigned n = threads > 0 ? static_cast<unsigned>(threads) : std::thread::hardware_concurrency();
    if (n == 0) n = 1;
    auto worker = [&]() {
        dee::ktbridge::ReferenceCpuExecutor ex;
        dee::ktbridge::ExecuteConfig cfg;
        cfg.swiglu_limit = swiglu_limit;
        for (;;) {
            const size_t s = next.fetch_add(1);
            if (s >= sel) break;
            const size_t t = s / topk;
            const auto v = view_of(records + static_cast<size_t>(ids[s]) * record_bytes, hidden, inter);
            const auto rc = ex.execute(0, ids[s], v, x + t * hidden, hidden, weights[s], cfg,
                                       partial.data() + s * hidden, hidden);
            if (rc != dee::ktbridge::ExecuteError::kOk) err.store(static_cast<int>(rc));
        }
    };
    std::vector<std::thread> pool;
    for (unsigned i = 0; i < n; ++i) pool.emplace_back(worker);
    for (auto& th : pool) th.join();
    if (err.load() != 0) return err.load();
    for (int t = 0; t < tokens; ++t)
        for (size_t h = 0; h < hidden; ++h) {
            float acc = 0.0f;
            for (int r = 0; r < topk; ++r) acc += partial[(static_cast<size_t>(t) * topk + r) * hidden + h];
            out[static_cast<size_t>(t) * hidden + h] = acc;
        }
    return 0;
}

}  // extern "C"
