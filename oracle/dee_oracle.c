/*
 * dee_oracle.c -- CPU restatement of the reference routed-expert MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in dee_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product path never does.
 *
 * Every function restates one piece of so-nerdyy/dee (paths relative to the
 * reference project root) in plain C:
 *
 *   dee_ref_f32_to_f16 / dee_ref_f16_to_f32   IEEE binary16 conversion with
 *       round-to-nearest-even, the rounding __float2half_rn performs in
 *       dee.cpp/src/swiglu_cuda.cu:46-59 and dee.cpp/src/cuda_convert.cu:245.
 *   dee_ref_fp4_decode_f16   fp4_e2m1_to_f16_kernel, cuda_convert.cu:212-245
 *       (16-entry table, low nibble -> column 2i, scale 2^(b-127) with the
 *       clamps of fp4_scale_value :217-223, FP16 RN output).
 *   dee_ref_fp4_dequant_f32  host decode fp4_e2m1_dequantize,
 *       dee.cpp/src/weight_mmap.cpp:84-117 (e8m0 clamp at 127).
 *   dee_ref_route_topk       Engine::route_topk_batch softmax/top-k/renorm,
 *       dee.cpp/src/engine.cpp:2739-2769 (float exp of (logit - max), double
 *       denominator, float inverse, partial_sort by probability desc then id
 *       asc, renormalise by the float sum of the selected probabilities).
 *   dee_ref_group            grouping of selections by expert in
 *       (rank, token) order, engine.cpp:812-823.
 *   dee_ref_expert_f16       the live FP16 expert chain of
 *       swiglu_expert_batch_fp16_cuda, swiglu_cuda.cu:387-431: FP16 X and
 *       FP16 weights, FP32-or-better accumulation, gate/up rounded to FP16,
 *       SiLU rounded to FP16, act = FP16(silu * up), down output FP32.
 *       Optional clamp (swiglu_limit > 0) as in :49-53.
 *   dee_ref_moe_layer        moe_forward_batch_device_impl,
 *       engine.cpp:776-1190: group, run each active expert, scatter raw FP32
 *       rows to [T, K, H] at position t*K + r (:1080-1113).
 *   dee_ref_combine_f32      live DeepSeek combine, dee.cpp/scripts/
 *       deepseek_v4_layer_candidate.py:616-629: out = 0; for r in rank order:
 *       out += w[:, r] * raw[:, r]  (FP32 multiply, FP32 add).
 *   dee_ref_combine_f16      weighted_combine_fp16_kernel,
 *       swiglu_cuda.cu:69-116: stable ascending-expert-id order, each product
 *       and each add rounded to FP16.
 *
 * Build (oracle/Makefile): gcc -O2 -pthread -ffp-contract=off -shared.
 * -ffp-contract=off keeps every multiply and add separately rounded.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* binary16 conversions                                                */
/* ------------------------------------------------------------------ */

uint16_t dee_ref_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (mant) return (uint16_t)(sign | 0x7E00u | (mant >> 13));
        return (uint16_t)(sign | 0x7C00u);
    }
    const int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        /* value = M * 2^(exp-150), M the 24-bit significand; a binary16
         * subnormal counts units of 2^-24, so drop (126 - exp) bits. */
        if (exp == 0) return (uint16_t)sign; /* float subnormal: far below 2^-25 */
        const uint32_t m = mant | 0x800000u;
        const int drop = 126 - (int)exp;
        if (drop > 24) return (uint16_t)sign;
        uint32_t r = m >> drop;
        const uint32_t rem = m & ((1u << drop) - 1u);
        const uint32_t half = 1u << (drop - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may reach inf */
    return (uint16_t)(sign | h);
}

float dee_ref_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t mant = (uint32_t)h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {
            int e = -1;
            do { ++e; mant <<= 1; } while (!(mant & 0x400u));
            mant &= 0x3FFu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7F800000u | (mant << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float f16r(float v) { return dee_ref_f16_to_f32(dee_ref_f32_to_f16(v)); }

/* ------------------------------------------------------------------ */
/* FP4 E2M1 + UE8M0 decode                                             */
/* ------------------------------------------------------------------ */

static const float kE2m1[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

const float* dee_ref_e2m1_table(void) { return kE2m1; }

/* fp4_scale_value, cuda_convert.cu:217-223: exponents >= 127 clamp to
 * FLT_MAX, <= -127 to zero. */
float dee_ref_scale_device(uint8_t b) {
    const int e = (int)b - 127;
    if (e >= 127) {
        const uint32_t bits = 0x7F7FFFFFu;
        float f; memcpy(&f, &bits, 4); return f;
    }
    if (e <= -127) return 0.0f;
    const uint32_t bits = (uint32_t)(e + 127) << 23;
    float f; memcpy(&f, &bits, 4); return f;
}

/* e8m0_to_f32, weight_mmap.cpp:88-99: exponent clamps at 127 (2^127). */
float dee_ref_scale_host(uint8_t b) {
    int e = (int)b - 127;
    if (e >= 127) e = 127;
    if (e <= -127) return 0.0f;
    const uint32_t bits = (uint32_t)(e + 127) << 23;
    float f; memcpy(&f, &bits, 4); return f;
}

void dee_ref_fp4_decode_f16(const uint8_t* packed, const uint8_t* scale,
                            uint16_t* dst, size_t out, size_t in) {
    const size_t half_in = in >> 1, sstride = in >> 5;
    for (size_t o = 0; o < out; ++o) {
        for (size_t i = 0; i < in; ++i) {
            const uint8_t byte = packed[o * half_in + (i >> 1)];
            const uint8_t nib = (i & 1) ? (byte >> 4) : (byte & 0x0F);
            const float s = dee_ref_scale_device(scale[o * sstride + (i >> 5)]);
            dst[o * in + i] = dee_ref_f32_to_f16(kE2m1[nib] * s);
        }
    }
}

void dee_ref_fp4_dequant_f32(const uint8_t* packed, const uint8_t* scale,
                             size_t out, size_t in, float* dst) {
    const size_t half_in = in >> 1, sstride = in >> 5;
    for (size_t o = 0; o < out; ++o) {
        for (size_t i = 0; i < in; ++i) {
            const uint8_t byte = packed[o * half_in + (i >> 1)];
            const uint8_t nib = (i & 1) ? (byte >> 4) : (byte & 0x0F);
            dst[o * in + i] = kE2m1[nib] * dee_ref_scale_host(scale[o * sstride + (i >> 5)]);
        }
    }
}

/* dequantize_expert_weight (dee.cpp/scripts/deepseek_v4_expert_reference.py
 * :85-99, decode_e8m0 :49-62): value * 2^(b - 127) in FP32 with no clamp,
 * so byte 0 is the subnormal 2^-127 and byte 255 overflows to infinity. */
static const float kE2m1Signed[16] = {  /* FP4_VALUES of the Python reference: code 8 is -0.0 */
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

static float scale_e8m0_exact(uint8_t b) {
    const uint32_t bits = b == 255 ? 0x7F800000u : b == 0 ? 0x00400000u : (uint32_t)b << 23;
    float f; memcpy(&f, &bits, 4); return f;
}

void dee_ref_fp4_dequant_e8m0_f32(const uint8_t* packed, const uint8_t* scale,
                                  size_t out, size_t in, float* dst) {
    const size_t half_in = in >> 1, sstride = in >> 5;
    for (size_t o = 0; o < out; ++o) {
        const uint8_t* p = packed + o * half_in;
        float* d = dst + o * in;
        for (size_t blk = 0; blk < sstride; ++blk) {
            const float s = scale_e8m0_exact(scale[o * sstride + blk]);
            for (size_t j = 0; j < 16; ++j) {
                const uint8_t byte = p[blk * 16 + j];
                d[blk * 32 + 2 * j] = kE2m1Signed[byte & 0x0F] * s;
                d[blk * 32 + 2 * j + 1] = kE2m1Signed[byte >> 4] * s;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* Router: softmax top-k with renormalisation                          */
/* ------------------------------------------------------------------ */

/* Returns 0 on success, -1 if a token's denominator or selected sum is not
 * positive and finite (the reference returns false there). */
int dee_ref_route_topk(const float* logits, int tokens, int experts, int topk,
                       int32_t* ids, float* weights) {
    if (!logits || !ids || !weights || tokens <= 0 || topk <= 0 || topk > experts) return -1;
    float* prob = (float*)malloc(sizeof(float) * (size_t)experts);
    char* taken = (char*)malloc((size_t)experts);
    if (!prob || !taken) { free(prob); free(taken); return -1; }
    int rc = 0;
    for (int t = 0; t < tokens && rc == 0; ++t) {
        const float* l = logits + (size_t)t * experts;
        float m = -INFINITY;
        for (int e = 0; e < experts; ++e) m = (m < l[e]) ? l[e] : m; /* std::max(m, l) */
        double den = 0.0;
        for (int e = 0; e < experts; ++e) {
            prob[e] = expf(l[e] - m);
            den += prob[e];
        }
        if (!(den > 0.0) || !isfinite(den)) { rc = -1; break; }
        const float inv = (float)(1.0 / den);
        for (int e = 0; e < experts; ++e) prob[e] *= inv;
        memset(taken, 0, (size_t)experts);
        float sel[64];
        int order[64];
        for (int k = 0; k < topk; ++k) {
            int best = -1;
            for (int e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best < 0 || prob[e] > prob[best]) best = e; /* ties keep lower id */
            }
            taken[best] = 1;
            order[k] = best;
            sel[k] = prob[best];
        }
        float sum = 0.0f;
        for (int k = 0; k < topk; ++k) sum += sel[k];
        if (!(sum > 0.0f)) { rc = -1; break; }
        for (int k = 0; k < topk; ++k) {
            ids[(size_t)t * topk + k] = order[k];
            weights[(size_t)t * topk + k] = sel[k] / sum;
        }
    }
    free(prob);
    free(taken);
    return rc;
}

/* ------------------------------------------------------------------ */
/* Group-by-expert                                                      */
/* ------------------------------------------------------------------ */

/* counts[E], offsets[E+1] (exclusive prefix, ascending expert id) and
 * perm[T*K]: grouped row -> position t*K + r, rows of one expert in
 * (rank, token) order.  Returns -1 on an out-of-range id. */
int dee_ref_group(const int32_t* ids, int tokens, int topk, int experts,
                  int32_t* counts, int32_t* offsets, int32_t* perm) {
    const size_t sel = (size_t)tokens * topk;
    for (size_t i = 0; i < sel; ++i)
        if (ids[i] < 0 || ids[i] >= experts) return -1;
    for (int e = 0; e < experts; ++e) counts[e] = 0;
    for (size_t i = 0; i < sel; ++i) counts[ids[i]]++;
    offsets[0] = 0;
    for (int e = 0; e < experts; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int32_t* cur = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
    if (!cur) return -1;
    for (int e = 0; e < experts; ++e) cur[e] = offsets[e];
    for (int r = 0; r < topk; ++r)
        for (int t = 0; t < tokens; ++t) {
            const int32_t p = t * topk + r;
            perm[cur[ids[p]]++] = p;
        }
    free(cur);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Record layout (DEE4): [w1][w3][w2][s1][s3][s2]                       */
/* ------------------------------------------------------------------ */

typedef struct {
    size_t w1, w3, w2, s1, s3, s2, bytes;
} dee_ref_layout;

dee_ref_layout dee_ref_record_layout(int hidden, int inter) {
    dee_ref_layout L;
    const size_t ih = (size_t)inter * (size_t)hidden;
    L.w1 = 0;
    L.w3 = ih / 2;
    L.w2 = ih;
    L.s1 = ih + ih / 2;
    L.s3 = L.s1 + ih / 32;
    L.s2 = L.s3 + ih / 32;
    L.bytes = L.s2 + ih / 32;
    return L;
}

size_t dee_ref_record_bytes(int hidden, int inter) {
    return dee_ref_record_layout(hidden, inter).bytes;
}

/* Decode one FP4 row (in elements) to FP16-valued floats, the values the
 * reference's dequant kernel writes into its FP16 scratch. */
static void decode_row(const uint8_t* packed_row, const uint8_t* scale_row, int in, float* dst) {
    for (int i = 0; i < in; ++i) {
        const uint8_t byte = packed_row[i >> 1];
        const uint8_t nib = (i & 1) ? (byte >> 4) : (byte & 0x0F);
        dst[i] = f16r(kE2m1[nib] * dee_ref_scale_device(scale_row[i >> 5]));
    }
}

/* Live FP16 chain for one expert over n rows.  x_f16: [n, H] binary16 bits.
 * y: [n, H] FP32.  Accumulation in double (the reference accumulates in
 * FP32 inside cuBLAS in an unspecified order; the exact-ish sum is the
 * order-free target). */
void dee_ref_expert_f16(const uint8_t* record, int hidden, int inter,
                        const uint16_t* x_f16, int n, float swiglu_limit, float* y) {
    const dee_ref_layout L = dee_ref_record_layout(hidden, inter);
    float* x = (float*)malloc(sizeof(float) * (size_t)n * hidden);
    float* act = (float*)malloc(sizeof(float) * (size_t)n * inter);
    float* w1 = (float*)malloc(sizeof(float) * (size_t)hidden);
    float* w3 = (float*)malloc(sizeof(float) * (size_t)hidden);
    float* w2 = (float*)malloc(sizeof(float) * (size_t)inter);
    for (size_t i = 0; i < (size_t)n * hidden; ++i) x[i] = dee_ref_f16_to_f32(x_f16[i]);
    for (int i = 0; i < inter; ++i) {
        decode_row(record + L.w1 + (size_t)i * (hidden / 2), record + L.s1 + (size_t)i * (hidden / 32), hidden, w1);
        decode_row(record + L.w3 + (size_t)i * (hidden / 2), record + L.s3 + (size_t)i * (hidden / 32), hidden, w3);
        for (int r = 0; r < n; ++r) {
            const float* xr = x + (size_t)r * hidden;
            double g = 0.0, u = 0.0;
            for (int h = 0; h < hidden; ++h) {
                g += (double)xr[h] * (double)w1[h];
                u += (double)xr[h] * (double)w3[h];
            }
            float gf = f16r((float)g);
            float uf = f16r((float)u);
            if (swiglu_limit > 0.0f) {
                gf = fminf(gf, swiglu_limit);
                uf = fminf(fmaxf(uf, -swiglu_limit), swiglu_limit);
            }
            const float silu = f16r(gf / (1.0f + expf(-gf)));
            act[(size_t)r * inter + i] = f16r(silu * uf);
        }
    }
    for (int o = 0; o < hidden; ++o) {
        decode_row(record + L.w2 + (size_t)o * (inter / 2), record + L.s2 + (size_t)o * (inter / 32), inter, w2);
        for (int r = 0; r < n; ++r) {
            const float* ar = act + (size_t)r * inter;
            double acc = 0.0;
            for (int i = 0; i < inter; ++i) acc += (double)ar[i] * (double)w2[i];
            y[(size_t)r * hidden + o] = (float)acc;
        }
    }
    free(x); free(act); free(w1); free(w3); free(w2);
}

/* Whole layer: records[e] at e * record_bytes (slot table optional, NULL
 * means identity).  raw: [T, K, H] FP32 (required).  Experts run on a small
 * pthread pool (threads <= 0: one per online CPU).  Returns -1 on bad ids. */
typedef struct {
    const uint8_t* records; size_t record_bytes; const int32_t* slot;
    int hidden, inter, topk; const uint16_t* x; float limit; float* raw;
    const int32_t* counts; const int32_t* offsets; const int32_t* perm;
    int experts; int next; pthread_mutex_t mu;
} layer_job;

static void* layer_worker(void* arg) {
    layer_job* J = (layer_job*)arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        const int e = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (e >= J->experts) break;
        const int n = J->counts[e];
        if (n == 0) continue;
        uint16_t* xe = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * J->hidden);
        float* ye = (float*)malloc(sizeof(float) * (size_t)n * J->hidden);
        for (int r = 0; r < n; ++r) {
            const int32_t p = J->perm[J->offsets[e] + r];
            memcpy(xe + (size_t)r * J->hidden, J->x + (size_t)(p / J->topk) * J->hidden,
                   sizeof(uint16_t) * J->hidden);
        }
        const int slot = J->slot ? J->slot[e] : e;
        dee_ref_expert_f16(J->records + (size_t)slot * J->record_bytes, J->hidden, J->inter,
                           xe, n, J->limit, ye);
        for (int r = 0; r < n; ++r) {
            const int32_t p = J->perm[J->offsets[e] + r];
            memcpy(J->raw + (size_t)p * J->hidden, ye + (size_t)r * J->hidden, sizeof(float) * J->hidden);
        }
        free(xe); free(ye);
    }
    return NULL;
}

int dee_ref_moe_layer(const uint8_t* records, size_t record_bytes, const int32_t* slot_of_expert,
                      int hidden, int inter, int experts, int topk,
                      const uint16_t* x_f16, int tokens, const int32_t* ids,
                      float swiglu_limit, int threads, float* raw) {
    const size_t sel = (size_t)tokens * topk;
    int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
    int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * ((size_t)experts + 1));
    int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * sel);
    if (dee_ref_group(ids, tokens, topk, experts, counts, offsets, perm) != 0) {
        free(counts); free(offsets); free(perm);
        return -1;
    }
    layer_job J;
    J.records = records; J.record_bytes = record_bytes; J.slot = slot_of_expert;
    J.hidden = hidden; J.inter = inter; J.topk = topk; J.x = x_f16; J.limit = swiglu_limit;
    J.raw = raw; J.counts = counts; J.offsets = offsets; J.perm = perm;
    J.experts = experts; J.next = 0;
    pthread_mutex_init(&J.mu, NULL);
    int n = threads > 0 ? threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 256) n = 256;
    pthread_t th[256];
    for (int i = 0; i < n; ++i) pthread_create(&th[i], NULL, layer_worker, &J);
    for (int i = 0; i < n; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&J.mu);
    free(counts); free(offsets); free(perm);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Combines                                                             */
/* ------------------------------------------------------------------ */

void dee_ref_combine_f32(const float* raw, const float* weights, int tokens, int topk,
                         int hidden, float* out) {
    for (int t = 0; t < tokens; ++t)
        for (int h = 0; h < hidden; ++h) {
            float acc = 0.0f;
            for (int r = 0; r < topk; ++r) {
                const size_t s = (size_t)t * topk + r;
                const float prod = weights[s] * raw[s * hidden + h];
                acc = acc + prod;
            }
            out[(size_t)t * hidden + h] = acc;
        }
}

/* stable_position_for_rank, swiglu_cuda.cu:69-84 */
static int stable_position(const int64_t* e, int topk, int rank) {
    for (int p = 0; p < topk; ++p) {
        int sr = 0;
        for (int o = 0; o < topk; ++o)
            if (e[o] < e[p] || (e[o] == e[p] && o < p)) ++sr;
        if (sr == rank) return p;
    }
    return -1;
}

void dee_ref_combine_f16(const float* raw, const float* weights, const int64_t* ids,
                         int tokens, int topk, int hidden, uint16_t* out) {
    for (int t = 0; t < tokens; ++t) {
        const int64_t* te = ids + (size_t)t * topk;
        for (int h = 0; h < hidden; ++h) {
            float acc = 0.0f;
            int ok = 1;
            for (int r = 0; r < topk; ++r) {
                const int p = stable_position(te, topk, r);
                if (p < 0) { ok = 0; break; }
                const size_t s = (size_t)t * topk + p;
                const float rv = f16r(raw[s * hidden + h]);
                const float wv = f16r(rv * weights[s]);
                acc = f16r(acc + wv);
            }
            if (ok) out[(size_t)t * hidden + h] = dee_ref_f32_to_f16(acc);
        }
    }
}

int dee_ref_num_threads(void) {
    return (int)sysconf(_SC_NPROCESSORS_ONLN);
}
