// routing.cuh -- the softmax top-k router of one token, shared by the router
// kernels (routing.cu) and the one-launch decode layer (moe_decode.cu).
#pragma once

#include "sm100.cuh"

namespace dee {

constexpr uint32_t kStatusBadRouter = 1u << 7;
constexpr int kRouteMaxPerLane = 16;  // experts <= 512

struct RouteCand {
    float p;
    int id;
};

// Probability-descending, then lower expert id: the partial_sort comparator
// of Engine::route_topk_batch (reference dee.cpp/src/engine.cpp:2755-2760).
__device__ __forceinline__ bool route_better(const RouteCand& a, const RouteCand& b) {
    if (a.p != b.p) return a.p > b.p;
    return a.id < b.id;
}

// One warp per token.  Softmax follows engine.cpp:2739-2754: the maximum
// logit, exp of (logit - max) rounded to FP32, a double-precision
// denominator summed in expert order, an FP32 inverse, FP32 probabilities.
// exp is evaluated in double and rounded once to FP32 (correctly rounded in
// practice), which the reference's libm expf matches except for rare
// last-bit cases.
//
// The expert-order double sum is reproduced exactly without running it
// serially: every term is an FP32 value in [0, 1] and E < 2^b, so when each
// term is 0 or at least 2^(b-30), every term and every partial sum is a
// multiple of 2^(b-53) below 2^b, i.e. exactly representable in double, and
// every addition is exact in any order.  A warp vote checks that; otherwise
// lane 0 sums in expert order.
//
// route_token routes one token with one warp: l is the token's logits row,
// sp a warp-private scratch of `experts` floats; rank k's id and weight go to
// ids_row[k] / weights_row[k] (lane k) and, when s_ids_row is given, also to
// s_ids_row[k].
template <int NPER>
__device__ __forceinline__ void route_token(const float* __restrict__ l, int experts, int topk, int lane,
                                            float* sp, int32_t* ids_row, float* weights_row,
                                            int32_t* s_ids_row, uint32_t* status) {
    float v[NPER];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
        const int e = lane + 32 * j;
        v[j] = e < experts ? l[e] : -INFINITY;
        if (e < experts) m = (m < v[j]) ? v[j] : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, m, o);
        m = (m < other) ? other : m;
    }
    int bits = 0;
    while ((experts >> bits) != 0) ++bits;  // E < 2^bits
    const float exact_min = __uint_as_float(static_cast<uint32_t>(127 + bits - 30) << 23);
    bool exact = true;
    double part = 0.0;
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
        const int e = lane + 32 * j;
        if (e < experts) {
            const float d = __fsub_rn(v[j], m);
            v[j] = static_cast<float>(exp(static_cast<double>(d)));
            exact = exact && (v[j] == 0.0f || v[j] >= exact_min);
            part += static_cast<double>(v[j]);
        }
    }
    double den;
    if (__all_sync(0xffffffffu, exact)) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        den = part;
    } else {
#pragma unroll
        for (int j = 0; j < NPER; ++j) {
            const int e = lane + 32 * j;
            if (e < experts) sp[e] = v[j];
        }
        __syncwarp();
        den = 0.0;
        if (lane == 0)
            for (int e = 0; e < experts; ++e) den += static_cast<double>(sp[e]);
        den = __shfl_sync(0xffffffffu, den, 0);
    }
    const bool bad = !(den > 0.0) || !isfinite(den);
    const float inv = static_cast<float>(1.0 / den);
    RouteCand mine[NPER];
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
        const int e = lane + 32 * j;
        mine[j].p = e < experts ? __fmul_rn(v[j], inv) : -INFINITY;
        mine[j].id = e < experts ? e : 0x7fffffff;
    }
    // K rounds of warp argmax over (probability descending, id ascending);
    // lane k keeps the k-th winner.  A lane offers its best remaining
    // candidate as a key ordered like the probability (p >= 0: its bits plus
    // one; 0 for none; within a lane ids ascend with j, so a strict '>'
    // keeps the lowest id), redux.sync takes the warp maximum, and a second
    // redux the lowest id among the lanes holding it.
    float my_p = 0.0f;
    int my_id = 0;
    for (int k = 0; k < topk; ++k) {
        uint32_t key = 0u;
        int id = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < NPER; ++j) {
            if (mine[j].id != 0x7fffffff) {
                const uint32_t kj = __float_as_uint(mine[j].p) + 1u;
                if (kj > key) { key = kj; id = mine[j].id; }
            }
        }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
        const int win = __reduce_min_sync(0xffffffffu, key == kmax ? id : 0x7fffffff);
        if (lane == k) { my_p = __uint_as_float(kmax - 1u); my_id = win; }
        // the owning lane retires the winner
#pragma unroll
        for (int j = 0; j < NPER; ++j)
            if (mine[j].id == win) mine[j].id = 0x7fffffff;
    }
    // sum of the selected probabilities in rank order (lane 0), then each
    // rank's weight on its own lane
    float sum = 0.0f;
    for (int k = 0; k < topk; ++k) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_p, k));
    const bool bad_sum = !(sum > 0.0f);
    if (lane == 0 && (bad || bad_sum)) atomicOr(status, kStatusBadRouter);
    if (lane < topk) {
        const bool ok = !(bad || bad_sum) && my_id >= 0 && my_id < experts;
        ids_row[lane] = ok ? my_id : 0;
        weights_row[lane] = ok ? __fdiv_rn(my_p, sum) : 0.0f;
        if (s_ids_row) s_ids_row[lane] = ok ? my_id : 0;
    }
}

}  // namespace dee
