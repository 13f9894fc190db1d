// store.cpp -- reader of DEE4 expert stores on disk and the fills that move
// their records into pinned host memory and into HBM.
//
// Three on-disk shapes, validated the way Dee4ExpertStore validates them
// (dee.cpp/include/dee/expert_store.h:286-409, dee.cpp/src/expert_store.cpp:
// 786-1230) and as the writers emit them (dee.cpp/tools/phase3/p3_builder.py:
// 285-460 segmented, 463-578 single file, 580-625 metadata):
//   dee4-v2            one fixed-stride file, dense index (layer-start)*E+expert
//   dee4-v3-trace      one file holding only the routed (layer, expert) union,
//                      with a strictly sorted record table in metadata.json
//   dee4-v4-segmented  one file per layer bucket, each sealed by a sha256 in
//                      the segment table; identity = sha256 of the seals
// Every structural error fails closed at open() with a message; so does a
// segment whose bytes do not match its seal (unless verification is off).
//
// Reads are positional pread() straight into the caller's memory -- pinned
// host memory for the offload tier, a ring of pinned staging buffers for a
// device upload -- issued by a pool of host threads in pieces of a few MiB,
// so a store streams at the rate of the disk or page cache instead of one
// syscall at a time.  No record is mapped into the address space.
#include <cuda_runtime.h>
#include <fcntl.h>
#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#endif
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "dee_b200.h"

namespace dee {
namespace store {
namespace {

// ---------------------------------------------------------------------------
// JSON: the subset metadata.json uses (objects, arrays, strings with
// escapes, integers, floats, true/false/null).  An integer literal (no '.',
// 'e' or 'E') is an Int; everything else numeric is a Float, so "3.0" is not
// accepted where a count is required (json_min.cpp:124-135).  A repeated key
// takes its last value.
// ---------------------------------------------------------------------------
struct JVal {
    enum Type { Null, Bool, Int, Float, Str, Arr, Obj } type = Null;
    bool b = false;
    long long i = 0;
    double f = 0.0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* find(const char* key) const {
        if (type != Obj) return nullptr;
        const JVal* hit = nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) hit = &kv.second;
        return hit;
    }
};

class JParser {
public:
    explicit JParser(const std::string& text) : s_(text) {}

    bool parse(JVal* out) {
        ws();
        if (!value(out, 0)) return false;
        ws();
        return i_ == s_.size();
    }

private:
    const std::string& s_;
    size_t i_ = 0;

    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
    }
    bool word(const char* w) {
        const size_t n = std::strlen(w);
        if (s_.compare(i_, n, w) != 0) return false;
        i_ += n;
        return true;
    }
    static bool digit(char c) { return c >= '0' && c <= '9'; }

    bool value(JVal* v, int depth) {
        if (depth > 64 || i_ >= s_.size()) return false;
        const char c = s_[i_];
        if (c == '{') return object(v, depth);
        if (c == '[') return array(v, depth);
        if (c == '"') {
            v->type = JVal::Str;
            return string(&v->s);
        }
        if (word("null")) { v->type = JVal::Null; return true; }
        if (word("true")) { v->type = JVal::Bool; v->b = true; return true; }
        if (word("false")) { v->type = JVal::Bool; v->b = false; return true; }
        if (c == '-' || digit(c)) return number(v);
        return false;
    }

    bool object(JVal* v, int depth) {
        v->type = JVal::Obj;
        ++i_;  // '{'
        ws();
        if (i_ < s_.size() && s_[i_] == '}') { ++i_; return true; }
        for (;;) {
            ws();
            if (i_ >= s_.size() || s_[i_] != '"') return false;
            std::string key;
            if (!string(&key)) return false;
            ws();
            if (i_ >= s_.size() || s_[i_] != ':') return false;
            ++i_;
            ws();
            JVal item;
            if (!value(&item, depth + 1)) return false;
            v->obj.emplace_back(std::move(key), std::move(item));
            ws();
            if (i_ >= s_.size()) return false;
            if (s_[i_] == ',') { ++i_; continue; }
            if (s_[i_] == '}') { ++i_; return true; }
            return false;
        }
    }

    bool array(JVal* v, int depth) {
        v->type = JVal::Arr;
        ++i_;  // '['
        ws();
        if (i_ < s_.size() && s_[i_] == ']') { ++i_; return true; }
        for (;;) {
            ws();
            JVal item;
            if (!value(&item, depth + 1)) return false;
            v->arr.push_back(std::move(item));
            ws();
            if (i_ >= s_.size()) return false;
            if (s_[i_] == ',') { ++i_; continue; }
            if (s_[i_] == ']') { ++i_; return true; }
            return false;
        }
    }

    static void utf8(uint32_t cp, std::string* out) {
        if (cp < 0x80) {
            out->push_back(static_cast<char>(cp));
        } else if (cp < 0x800) {
            out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
            out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
            out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else {
            out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
            out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
            out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        }
    }

    bool hex4(uint32_t* out) {
        if (i_ + 4 > s_.size()) return false;
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
            else return false;
        }
        *out = v;
        return true;
    }

    bool string(std::string* out) {
        ++i_;  // opening quote
        while (i_ < s_.size()) {
            const char c = s_[i_++];
            if (c == '"') return true;
            if (static_cast<unsigned char>(c) < 0x20) return false;
            if (c != '\\') { out->push_back(c); continue; }
            if (i_ >= s_.size()) return false;
            const char e = s_[i_++];
            switch (e) {
                case '"': out->push_back('"'); break;
                case '\\': out->push_back('\\'); break;
                case '/': out->push_back('/'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'n': out->push_back('\n'); break;
                case 'r': out->push_back('\r'); break;
                case 't': out->push_back('\t'); break;
                case 'u': {
                    uint32_t cp = 0;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
                        uint32_t lo = 0;
                        if (i_ + 2 > s_.size() || s_[i_] != '\\' || s_[i_ + 1] != 'u') return false;
                        i_ += 2;
                        if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    utf8(cp, out);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }

    bool number(JVal* v) {
        const size_t start = i_;
        bool is_float = false;
        if (s_[i_] == '-') ++i_;
        if (i_ >= s_.size() || !digit(s_[i_])) return false;
        if (s_[i_] == '0') {
            ++i_;
        } else {
            while (i_ < s_.size() && digit(s_[i_])) ++i_;
        }
        if (i_ < s_.size() && s_[i_] == '.') {
            is_float = true;
            ++i_;
            if (i_ >= s_.size() || !digit(s_[i_])) return false;
            while (i_ < s_.size() && digit(s_[i_])) ++i_;
        }
        if (i_ < s_.size() && (s_[i_] == 'e' || s_[i_] == 'E')) {
            is_float = true;
            ++i_;
            if (i_ < s_.size() && (s_[i_] == '+' || s_[i_] == '-')) ++i_;
            if (i_ >= s_.size() || !digit(s_[i_])) return false;
            while (i_ < s_.size() && digit(s_[i_])) ++i_;
        }
        const std::string text = s_.substr(start, i_ - start);
        errno = 0;
        if (is_float) {
            v->type = JVal::Float;
            v->f = std::strtod(text.c_str(), nullptr);
        } else {
            v->type = JVal::Int;
            v->i = std::strtoll(text.c_str(), nullptr, 10);
        }
        return errno != ERANGE;
    }
};

// ---------------------------------------------------------------------------
// SHA-256 (FIPS 180-4, sections 4.2.2, 5.3.3 and 6.2): the segment seals and
// the segmented store's identity.  Two compressions of whole 64-byte blocks:
// the portable one, and one on the x86 SHA extensions (SHA256RNDS2 runs two
// rounds on the state held as ABEF/CDGH, SHA256MSG1/MSG2 extend the message
// schedule four words at a time), chosen once from CPUID leaf 7 (EBX bit 29).
// DEE_SHA256_PORTABLE=1 in the environment forces the portable one.
// ---------------------------------------------------------------------------

// K: the first 32 bits of the fractional parts of the cube roots of the
// first 64 primes (FIPS 180-4, 4.2.2).
alignas(16) const uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

inline uint32_t rotr32(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha256_blocks_portable(uint32_t h[8], const uint8_t* p, size_t blocks) {
    for (; blocks; --blocks, p += 64) {
        uint32_t w[64];
        for (int t = 0; t < 16; ++t)
            w[t] = (static_cast<uint32_t>(p[4 * t]) << 24) | (static_cast<uint32_t>(p[4 * t + 1]) << 16) |
                   (static_cast<uint32_t>(p[4 * t + 2]) << 8) | static_cast<uint32_t>(p[4 * t + 3]);
        for (int t = 16; t < 64; ++t) {
            const uint32_t s0 = rotr32(w[t - 15], 7) ^ rotr32(w[t - 15], 18) ^ (w[t - 15] >> 3);
            const uint32_t s1 = rotr32(w[t - 2], 17) ^ rotr32(w[t - 2], 19) ^ (w[t - 2] >> 10);
            w[t] = w[t - 16] + s0 + w[t - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int t = 0; t < 64; ++t) {
            const uint32_t t1 =
                hh + (rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25)) + ((e & f) ^ (~e & g)) + kSha256K[t] + w[t];
            const uint32_t t2 = (rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d;
        h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
}

#if defined(__x86_64__)
__attribute__((target("sha,sse4.1,ssse3"))) void sha256_blocks_shani(uint32_t h[8], const uint8_t* p,
                                                                       size_t blocks) {
    // big-endian word loads
    const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bLL, 0x0405060700010203LL);
    // state words a..h -> the ABEF / CDGH register pair the round instruction uses
    __m128i dcba = _mm_loadu_si128(reinterpret_cast<const __m128i*>(h));
    __m128i hgfe = _mm_loadu_si128(reinterpret_cast<const __m128i*>(h + 4));
    __m128i cdab = _mm_shuffle_epi32(dcba, 0xB1);
    __m128i efgh = _mm_shuffle_epi32(hgfe, 0x1B);
    __m128i abef = _mm_alignr_epi8(cdab, efgh, 8);
    __m128i cdgh = _mm_blend_epi16(efgh, cdab, 0xF0);
    for (; blocks; --blocks, p += 64) {
        const __m128i abef0 = abef, cdgh0 = cdgh;
        __m128i m[4];
        for (int g = 0; g < 16; ++g) {
            __m128i w;
            if (g < 4) {
                w = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * g)), bswap);
            } else {
                // W[t..t+3] = MSG2(MSG1(W[t-16..], W[t-12..]) + W[t-7..t-4], W[t-4..t-1])
                const __m128i x = _mm_add_epi32(_mm_sha256msg1_epu32(m[g & 3], m[(g + 1) & 3]),
                                                _mm_alignr_epi8(m[(g + 3) & 3], m[(g + 2) & 3], 4));
                w = _mm_sha256msg2_epu32(x, m[(g + 3) & 3]);
            }
            m[g & 3] = w;
            __m128i k = _mm_add_epi32(w, _mm_load_si128(reinterpret_cast<const __m128i*>(kSha256K + 4 * g)));
            cdgh = _mm_sha256rnds2_epu32(cdgh, abef, k);
            k = _mm_shuffle_epi32(k, 0x0E);
            abef = _mm_sha256rnds2_epu32(abef, cdgh, k);
        }
        abef = _mm_add_epi32(abef, abef0);
        cdgh = _mm_add_epi32(cdgh, cdgh0);
    }
    const __m128i feba = _mm_shuffle_epi32(abef, 0x1B);
    const __m128i dchg = _mm_shuffle_epi32(cdgh, 0xB1);
    _mm_storeu_si128(reinterpret_cast<__m128i*>(h), _mm_blend_epi16(feba, dchg, 0xF0));
    _mm_storeu_si128(reinterpret_cast<__m128i*>(h + 4), _mm_alignr_epi8(dchg, feba, 8));
}

bool cpu_has_sha() {
    unsigned a = 0, b = 0, c = 0, d = 0;
    if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
    unsigned a1 = 0, b1 = 0, c1 = 0, d1 = 0;
    if (!__get_cpuid(1, &a1, &b1, &c1, &d1)) return false;
    const bool sse41 = (c1 >> 19) & 1u, ssse3 = (c1 >> 9) & 1u;
    return ((b >> 29) & 1u) && sse41 && ssse3;
}
#endif

using Sha256Blocks = void (*)(uint32_t*, const uint8_t*, size_t);

Sha256Blocks sha256_blocks_impl() {
    static const Sha256Blocks impl = []() -> Sha256Blocks {
        const char* force = std::getenv("DEE_SHA256_PORTABLE");
        if (force && force[0] == '1') return sha256_blocks_portable;
#if defined(__x86_64__)
        if (cpu_has_sha()) return sha256_blocks_shani;
#endif
        return sha256_blocks_portable;
    }();
    return impl;
}

class Sha256 {
public:
    Sha256() : blocks_(sha256_blocks_impl()) { reset(); }

    void reset() {
        static const uint32_t kInit[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                          0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
        std::memcpy(h_, kInit, sizeof(h_));
        bits_ = 0;
        fill_ = 0;
    }

    void update(const void* data, size_t n) {
        const uint8_t* p = static_cast<const uint8_t*>(data);
        bits_ += static_cast<uint64_t>(n) * 8u;
        if (fill_) {
            const size_t take = std::min(n, 64 - fill_);
            std::memcpy(buf_ + fill_, p, take);
            fill_ += take;
            p += take;
            n -= take;
            if (fill_ < 64) return;
            blocks_(h_, buf_, 1);
            fill_ = 0;
        }
        if (n >= 64) {
            blocks_(h_, p, n / 64);
            p += n & ~size_t(63);
            n &= 63;
        }
        if (n) {
            std::memcpy(buf_, p, n);
            fill_ = n;
        }
    }

    std::string hex() {
        const uint64_t bits = bits_;
        uint8_t pad[72] = {0x80};
        const size_t padlen = (fill_ < 56 ? 56 : 120) - fill_;
        for (int k = 0; k < 8; ++k) pad[padlen + k] = static_cast<uint8_t>(bits >> (56 - 8 * k));
        update(pad, padlen + 8);
        static const char kHex[] = "0123456789abcdef";
        std::string out(64, '0');
        for (int w = 0; w < 8; ++w)
            for (int k = 0; k < 8; ++k) out[w * 8 + k] = kHex[(h_[w] >> (28 - 4 * k)) & 0xF];
        return out;
    }

private:
    Sha256Blocks blocks_;
    uint32_t h_[8];
    uint64_t bits_ = 0;
    uint8_t buf_[64];
    size_t fill_ = 0;
};

bool is_sha256_hex(const std::string& v) {
    if (v.size() != 64) return false;
    for (const char c : v)
        if (!((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F'))) return false;
    return true;
}

std::string lower(std::string v) {
    for (char& c : v)
        if (c >= 'A' && c <= 'Z') c = static_cast<char>(c - 'A' + 'a');
    return v;
}

bool checked_mul(size_t a, size_t b, size_t* out) {
    if (a != 0 && b > SIZE_MAX / a) return false;
    *out = a * b;
    return true;
}

bool get_string(const JVal& root, const char* key, std::string* out) {
    const JVal* v = root.find(key);
    if (!v || v->type != JVal::Str) return false;
    *out = v->s;
    return true;
}

bool get_count(const JVal& root, const char* key, size_t* out) {
    const JVal* v = root.find(key);
    if (!v || v->type != JVal::Int || v->i < 0) return false;
    *out = static_cast<size_t>(v->i);
    return true;
}

bool get_counts3(const JVal& root, const char* key, size_t out[3]) {
    const JVal* v = root.find(key);
    if (!v || v->type != JVal::Arr || v->arr.size() != 3) return false;
    for (int k = 0; k < 3; ++k) {
        if (v->arr[k].type != JVal::Int || v->arr[k].i < 0) return false;
        out[k] = static_cast<size_t>(v->arr[k].i);
    }
    return true;
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

struct ReadCounters {
    std::atomic<uint64_t> bytes{0}, calls{0}, short_reads{0};
};

// pread until n bytes arrived (EINTR retried, short reads continued).
bool pread_full(int fd, void* dst, size_t n, size_t offset, ReadCounters* rc) {
    size_t done = 0;
    while (done < n) {
        const size_t want = std::min<size_t>(n - done, size_t(1) << 30);
        const ssize_t got = ::pread(fd, static_cast<char*>(dst) + done, want, static_cast<off_t>(offset + done));
        rc->calls.fetch_add(1, std::memory_order_relaxed);
        if (got < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        if (got == 0) return false;  // file shorter than its declared size
        if (static_cast<size_t>(got) < want) rc->short_reads.fetch_add(1, std::memory_order_relaxed);
        done += static_cast<size_t>(got);
        rc->bytes.fetch_add(static_cast<uint64_t>(got), std::memory_order_relaxed);
    }
    return true;
}

// One backing file: the single data file of v2/v3, or one segment of v4.
// Records first_record .. first_record+record_count-1 sit at
// (index - first_record) * record_bytes.
struct StoreFile {
    int fd = -1;
    std::string file;
    std::string sha256;
    size_t first_record = 0;
    size_t record_count = 0;
    size_t size = 0;
};

// A contiguous byte range of one file bound for dst + dst_offset, read in
// order in pieces of `chunk` bytes.  `seal`: the range is the whole file and
// the file has a sha256 seal; the pieces are hashed as they arrive and the
// task fails on a mismatch.
struct Task {
    const StoreFile* file;
    size_t file_offset;
    size_t dst_offset;
    size_t bytes;
    size_t chunk;
    bool seal;
};

// Run fn(i) for i in [0, n) on up to `threads` host threads.
template <class Fn>
void parallel_for(size_t n, int threads, Fn fn) {
    const size_t workers = std::min<size_t>(n, static_cast<size_t>(std::max(1, threads)));
    std::atomic<size_t> next{0};
    auto body = [&]() {
        for (size_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    };
    if (workers <= 1) {
        body();
        return;
    }
    std::vector<std::thread> pool;
    pool.reserve(workers - 1);
    for (size_t k = 1; k < workers; ++k) pool.emplace_back(body);
    body();
    for (auto& t : pool) t.join();
}

// Work through `tasks` on `workers` threads.  For every piece,
// buf = acquire(w, task, offset_in_task) names where the bytes land (the
// destination itself, or worker w's staging buffer), then commit(w, buf, dst
// offset, bytes) hands them on; acquire/commit return false to stop.
// Returns the first error ("" on success).
template <class Acquire, class Commit>
std::string run_tasks(const std::vector<Task>& tasks, int workers, ReadCounters* rc, std::atomic<uint64_t>* sealed,
                      Acquire acquire, Commit commit) {
    std::atomic<size_t> next{0};
    std::atomic<bool> stop{false};
    std::mutex mu;
    std::string err;
    auto fail = [&](const std::string& m) {
        std::lock_guard<std::mutex> g(mu);
        if (err.empty()) err = m;
        stop.store(true);
    };
    auto body = [&](int w) {
        for (size_t i = next.fetch_add(1); i < tasks.size() && !stop.load(); i = next.fetch_add(1)) {
            const Task& t = tasks[i];
            Sha256 h;
            for (size_t off = 0; off < t.bytes && !stop.load(); off += t.chunk) {
                const size_t n = std::min(t.chunk, t.bytes - off);
                void* buf = acquire(w, t, off);
                if (!buf) return fail("staging buffer wait failed");
                if (!pread_full(t.file->fd, buf, n, t.file_offset + off, rc))
                    return fail("DEE4 read of " + t.file->file + " failed");
                if (t.seal) h.update(buf, n);
                if (!commit(w, buf, t.dst_offset + off, n)) return fail("device copy failed");
            }
            if (t.seal && !stop.load()) {
                if (h.hex() != t.file->sha256) return fail("DEE4 segment " + t.file->file + " sha256 mismatch");
                sealed->fetch_add(1);
            }
        }
    };
    const int n = std::max(1, std::min<int>(workers, static_cast<int>(tasks.size())));
    std::vector<std::thread> pool;
    for (int w = 1; w < n; ++w) pool.emplace_back(body, w);
    body(0);
    for (auto& t : pool) t.join();
    return err;
}

}  // namespace

class Dee4Store {
public:
    ~Dee4Store() { close(); }

    void close() {
        for (auto& f : files_)
            if (f.fd >= 0) ::close(f.fd);
        files_.clear();
        trace_.clear();
        segmented_ = trace_indexed_ = false;
        start_layer_ = num_layers_ = experts_per_layer_ = 0;
        record_bytes_ = stored_records_ = 0;
        backend_ = "dee4";
        identity_.clear();
    }

    bool fail(const std::string& msg) {
        last_error_ = msg;
        close();
        return false;
    }

    bool open(const std::string& path, bool verify, bool drop_pages, int threads);

    // Dee4ExpertStore::get (expert_store.cpp:1176-1215): the record index of
    // (layer, expert), or false outside the store (a trace store also misses
    // pairs it does not hold).
    bool lookup(int layer, int expert, size_t* record_index) {
        lookups_.fetch_add(1, std::memory_order_relaxed);
        const bool in_range = !files_.empty() && layer >= start_layer_ &&
                              layer < start_layer_ + num_layers_ && expert >= 0 && expert < experts_per_layer_;
        if (!in_range) {
            lookup_failures_.fetch_add(1, std::memory_order_relaxed);
            return false;
        }
        if (trace_indexed_) {
            const auto key = std::make_pair(layer, expert);
            const auto it = std::lower_bound(trace_.begin(), trace_.end(), key,
                                             [](const TraceRec& r, const std::pair<int, int>& k) {
                                                 return r.layer < k.first ||
                                                        (r.layer == k.first && r.expert < k.second);
                                             });
            if (it == trace_.end() || it->layer != layer || it->expert != expert) {
                lookup_failures_.fetch_add(1, std::memory_order_relaxed);
                return false;
            }
            *record_index = it->record_index;
        } else {
            *record_index = static_cast<size_t>(layer - start_layer_) * static_cast<size_t>(experts_per_layer_) +
                            static_cast<size_t>(expert);
        }
        return true;
    }

    // record index -> (file, byte offset in it); find_segment
    // (expert_store.cpp:762-784) for segmented stores.
    bool locate(size_t record_index, const StoreFile** file, size_t* offset) const {
        if (record_index >= stored_records_ || files_.empty()) return false;
        const StoreFile* f = &files_[0];
        if (segmented_) {
            const auto it = std::upper_bound(files_.begin(), files_.end(), record_index,
                                             [](size_t idx, const StoreFile& s) { return idx < s.first_record; });
            if (it == files_.begin()) return false;
            f = &*(it - 1);
        }
        if (record_index - f->first_record >= f->record_count) return false;
        const size_t off = (record_index - f->first_record) * record_bytes_;
        if (off > f->size || record_bytes_ > f->size - off) return false;
        *file = f;
        *offset = off;
        return true;
    }

    // Tasks that fill dst with experts [first_expert, first_expert+experts)
    // of layers [first_layer, first_layer+layers) as [layer][expert][record]:
    // contiguous runs of one file, each split into independent pieces of at
    // most `chunk` bytes -- or, with `verify`, kept whole (read in order and
    // hashed) when the run is an entire sealed file.  Sealed runs go first:
    // they are the longest tasks.
    bool plan_layers(int first_layer, int layers, int first_expert, int experts, size_t chunk, bool verify,
                     std::vector<Task>* tasks) {
        std::vector<Task> runs;
        size_t dst = 0;
        for (int l = first_layer; l < first_layer + layers; ++l) {
            for (int e = first_expert; e < first_expert + experts; ++e) {
                size_t idx = 0, off = 0;
                const StoreFile* f = nullptr;
                if (!lookup(l, e, &idx) || !locate(idx, &f, &off)) {
                    last_error_ = "DEE4 record (layer " + std::to_string(l) + ", expert " + std::to_string(e) +
                                  ") is not in the store";
                    return false;
                }
                if (!runs.empty() && runs.back().file == f && runs.back().file_offset + runs.back().bytes == off &&
                    runs.back().dst_offset + runs.back().bytes == dst)
                    runs.back().bytes += record_bytes_;
                else
                    runs.push_back({f, off, dst, record_bytes_, chunk, false});
                dst += record_bytes_;
            }
        }
        tasks->clear();
        for (const Task& r : runs)
            if (verify && r.file_offset == 0 && r.bytes == r.file->size && !r.file->sha256.empty())
                tasks->push_back({r.file, 0, r.dst_offset, r.bytes, chunk, true});
        for (const Task& r : runs) {
            if (verify && r.file_offset == 0 && r.bytes == r.file->size && !r.file->sha256.empty()) continue;
            for (size_t done = 0; done < r.bytes; done += chunk)
                tasks->push_back(
                    {r.file, r.file_offset + done, r.dst_offset + done, std::min(chunk, r.bytes - done), chunk, false});
        }
        return true;
    }

    size_t record_bytes() const { return record_bytes_; }
    int experts_per_layer() const { return experts_per_layer_; }
    bool valid_range(int first, int n, int first_expert, int experts) const {
        return n > 0 && first >= start_layer_ && first <= start_layer_ + num_layers_ - n && experts > 0 &&
               first_expert >= 0 && first_expert <= experts_per_layer_ - experts;
    }

    void info(dee_store_info* out) const {
        out->start_layer = start_layer_;
        out->num_layers = num_layers_;
        out->experts_per_layer = experts_per_layer_;
        out->segmented = segmented_ ? 1 : 0;
        out->trace_indexed = trace_indexed_ ? 1 : 0;
        out->record_bytes = record_bytes_;
        out->stored_records = stored_records_;
        out->file_count = files_.size();
        for (int p = 0; p < 3; ++p) {
            out->weight_offsets[p] = weight_offsets_[p];
            out->weight_nbytes[p] = weight_nbytes_[p];
            out->weight_out[p] = weight_out_[p];
            out->weight_stored_in[p] = weight_stored_in_[p];
            out->scale_offsets[p] = scale_offsets_[p];
            out->scale_nbytes[p] = scale_nbytes_[p];
            out->scale_out[p] = scale_out_[p];
            out->scale_in[p] = scale_in_[p];
        }
    }

    void stats(uint64_t out[4]) const {
        out[0] = lookups_.load();
        out[1] = lookup_failures_.load();
        out[2] = source_reads_.load();
        out[3] = bytes_read_.load();
    }

    void count_reads(uint64_t reads, uint64_t bytes) {
        source_reads_.fetch_add(reads, std::memory_order_relaxed);
        bytes_read_.fetch_add(bytes, std::memory_order_relaxed);
    }

    bool loaded() const { return !files_.empty(); }

    std::string last_error_;
    std::string backend_ = "dee4";
    std::string identity_;

private:
    struct TraceRec {
        int layer;
        int expert;
        size_t record_index;
    };

    std::vector<StoreFile> files_;
    std::vector<TraceRec> trace_;
    bool segmented_ = false;
    bool trace_indexed_ = false;
    int start_layer_ = 0, num_layers_ = 0, experts_per_layer_ = 0;
    size_t record_bytes_ = 0, stored_records_ = 0;
    size_t weight_offsets_[3] = {}, weight_nbytes_[3] = {}, weight_out_[3] = {}, weight_stored_in_[3] = {};
    size_t scale_offsets_[3] = {}, scale_nbytes_[3] = {}, scale_out_[3] = {}, scale_in_[3] = {};
    std::atomic<uint64_t> lookups_{0}, lookup_failures_{0}, source_reads_{0}, bytes_read_{0};

    bool open_file(const std::string& dir, StoreFile* f) {
        const std::string path = dir + "/" + f->file;
        f->fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (f->fd < 0) {
            last_error_ = "DEE4 data file " + f->file + " cannot be opened: " + std::strerror(errno);
            return false;
        }
        struct stat st;
        if (::fstat(f->fd, &st) != 0 || !S_ISREG(st.st_mode)) {
            last_error_ = "DEE4 data file " + f->file + " is not a regular file";
            return false;
        }
        f->size = static_cast<size_t>(st.st_size);
        return true;
    }
};

// Dee4ExpertStore::open (expert_store.cpp:790-1172): the same keys, the same
// checks in the same order, the same fail-closed outcomes.
bool Dee4Store::open(const std::string& path, bool verify, bool drop_pages, int threads) {
    close();
    last_error_.clear();
    std::string meta_path = path;
    struct stat st;
    if (::stat(path.c_str(), &st) == 0 && S_ISDIR(st.st_mode)) meta_path = path + "/metadata.json";
    if (::stat(meta_path.c_str(), &st) != 0 || !S_ISREG(st.st_mode)) return fail("DEE4 metadata.json is missing");
    const size_t slash = meta_path.find_last_of('/');
    const std::string dir = slash == std::string::npos ? "." : meta_path.substr(0, slash);

    std::string text;
    {
        FILE* fp = std::fopen(meta_path.c_str(), "rb");
        if (!fp) return fail("DEE4 metadata.json is missing");
        char buf[1 << 16];
        size_t n;
        while ((n = std::fread(buf, 1, sizeof(buf), fp)) > 0) text.append(buf, n);
        std::fclose(fp);
    }
    JVal root;
    if (!JParser(text).parse(&root) || root.type != JVal::Obj) return fail("DEE4 metadata JSON parse failed");

    std::string format, codec, data_file;
    size_t start_layer = 0, num_layers = 0, experts = 0;
    const bool known = get_string(root, "format", &format) &&
                       (format == "dee4-v2" || format == "dee4-v3-trace" || format == "dee4-v4-segmented");
    if (!known || !get_string(root, "codec", &codec) || codec != "deepseek-fp4-e2m1-e8m0" ||
        !get_count(root, "start_layer", &start_layer) || !get_count(root, "num_layers", &num_layers) ||
        !get_count(root, "experts_per_layer", &experts) || !get_count(root, "record_bytes", &record_bytes_) ||
        !get_counts3(root, "weight_offsets", weight_offsets_) || !get_counts3(root, "weight_nbytes", weight_nbytes_) ||
        !get_counts3(root, "weight_out", weight_out_) || !get_counts3(root, "weight_stored_in", weight_stored_in_) ||
        !get_counts3(root, "scale_offsets", scale_offsets_) || !get_counts3(root, "scale_nbytes", scale_nbytes_) ||
        !get_counts3(root, "scale_out", scale_out_) || !get_counts3(root, "scale_in", scale_in_))
        return fail("DEE4 metadata schema/codec/layout is invalid");
    const bool segmented = format == "dee4-v4-segmented";
    if (!segmented && (!get_string(root, "data_file", &data_file) || data_file.empty() ||
                       !get_string(root, "data_sha256", &identity_) || !is_sha256_hex(identity_)))
        return fail("DEE4 metadata schema/codec/layout is invalid");
    constexpr size_t kIntMax = 0x7fffffff;
    if (num_layers == 0 || experts == 0 || record_bytes_ == 0 || start_layer > kIntMax || num_layers > kIntMax ||
        num_layers > kIntMax - start_layer || experts > kIntMax)
        return fail("DEE4 geometry is empty or out of range");
    for (int p = 0; p < 3; ++p) {
        if (weight_nbytes_[p] == 0 || scale_nbytes_[p] == 0 || weight_offsets_[p] > record_bytes_ ||
            weight_nbytes_[p] > record_bytes_ - weight_offsets_[p] || scale_offsets_[p] > record_bytes_ ||
            scale_nbytes_[p] > record_bytes_ - scale_offsets_[p])
            return fail("DEE4 component range escapes its record");
        size_t ew = 0, es = 0;
        if (!checked_mul(weight_out_[p], weight_stored_in_[p], &ew) || !checked_mul(scale_out_[p], scale_in_[p], &es) ||
            ew != weight_nbytes_[p] || es != scale_nbytes_[p])
            return fail("DEE4 component shape/byte length mismatch");
    }

    size_t total = 0;
    if (format == "dee4-v2") {
        if (!checked_mul(num_layers, experts, &total)) return fail("DEE4 total size overflow");
    } else if (segmented) {
        const JVal* df = root.find("data_file");
        if (df && !(df->type == JVal::Null || (df->type == JVal::Str && df->s.empty())))
            return fail("DEE4 segmented metadata must not name a data_file");
        size_t declared = 0;
        const JVal* segs = root.find("segments");
        if (!get_count(root, "total_experts", &declared) || declared == 0 ||
            !checked_mul(num_layers, experts, &total) || total != declared || !segs || segs->type != JVal::Arr ||
            segs->arr.size() != num_layers)
            return fail("DEE4 segmented store metadata is invalid");
        for (const char* key : {"universe_sha256", "manifest_sha256"}) {
            const JVal* b = root.find(key);
            if (b && (b->type != JVal::Str || !is_sha256_hex(b->s)))
                return fail("DEE4 segmented universe binding is invalid");
        }
        size_t next_first = 0;
        for (size_t i = 0; i < segs->arr.size(); ++i) {
            const JVal& item = segs->arr[i];
            StoreFile f;
            size_t bucket = 0, bytes = 0;
            if (item.type != JVal::Obj || !get_string(item, "file", &f.file) || f.file.empty() ||
                !get_count(item, "bucket", &bucket) || bucket != i ||
                !get_count(item, "first_record", &f.first_record) || f.first_record != next_first ||
                !get_count(item, "record_count", &f.record_count) || f.record_count != experts ||
                !get_count(item, "bytes", &bytes) || !get_string(item, "sha256", &f.sha256) ||
                !is_sha256_hex(f.sha256))
                return fail("DEE4 segment table is invalid");
            const JVal* domain = item.find("domain");
            if (domain && domain->type != JVal::Str) return fail("DEE4 segment table is invalid");
            size_t expect = 0;
            if (!checked_mul(f.record_count, record_bytes_, &expect) || expect != bytes)
                return fail("DEE4 segment byte count is inconsistent");
            if (f.file[0] == '/' || f.file.find("..") != std::string::npos)
                return fail("DEE4 segment path escapes the store");
            f.sha256 = lower(f.sha256);
            next_first += f.record_count;
            files_.push_back(std::move(f));
        }
        if (next_first != declared) return fail("DEE4 segments do not cover the declared universe");
        Sha256 table;
        for (const auto& f : files_) table.update(f.sha256.data(), f.sha256.size());
        identity_ = table.hex();
        segmented_ = true;
        backend_ = "dee4_segmented";
    } else {
        size_t declared = 0;
        std::string journal_sha, chain_sha, selection_sha;
        const JVal* recs = root.find("records");
        if (!get_count(root, "total_experts", &declared) || declared == 0 || !recs || recs->type != JVal::Arr ||
            recs->arr.size() != declared || !get_string(root, "trace_journal_sha256", &journal_sha) ||
            !is_sha256_hex(journal_sha) || !get_string(root, "trace_final_chain_sha256", &chain_sha) ||
            !is_sha256_hex(chain_sha) || !get_string(root, "selection_sha256", &selection_sha) ||
            !is_sha256_hex(selection_sha))
            return fail("DEE4 trace index metadata is invalid");
        trace_.reserve(declared);
        for (size_t idx = 0; idx < recs->arr.size(); ++idx) {
            const JVal& item = recs->arr[idx];
            size_t layer = 0, expert = 0, record_index = 0;
            if (item.type != JVal::Obj || !get_count(item, "layer", &layer) || !get_count(item, "expert", &expert) ||
                !get_count(item, "record_index", &record_index) || layer < start_layer ||
                layer >= start_layer + num_layers || expert >= experts || record_index != idx)
                return fail("DEE4 trace record index is invalid");
            const TraceRec r{static_cast<int>(layer), static_cast<int>(expert), record_index};
            if (!trace_.empty()) {
                const TraceRec& prev = trace_.back();
                if (r.layer < prev.layer || (r.layer == prev.layer && r.expert <= prev.expert))
                    return fail("DEE4 trace records are not strictly sorted/unique");
            }
            trace_.push_back(r);
        }
        total = declared;
        trace_indexed_ = true;
        backend_ = "dee4_trace";
    }

    if (segmented_) {
        for (auto& f : files_) {
            if (!open_file(dir, &f)) {
                const std::string msg = last_error_;
                return fail(msg);
            }
            if (f.size != f.record_count * record_bytes_)
                return fail("DEE4 segment " + f.file + " size " + std::to_string(f.size) +
                            " does not match expected " + std::to_string(f.record_count * record_bytes_));
        }
        if (verify) {
            // The seal pass: every segment re-hashed from disk, segments in
            // parallel, each read sequentially in 8 MiB pieces.
            std::vector<std::string> digest(files_.size());
            std::vector<int> ok(files_.size(), 0);
            parallel_for(files_.size(), threads, [&](size_t s) {
                const StoreFile& f = files_[s];
                std::vector<uint8_t> buf(8u << 20);
                Sha256 h;
                ReadCounters rc;
                for (size_t off = 0; off < f.size; off += buf.size()) {
                    const size_t n = std::min(buf.size(), f.size - off);
                    if (!pread_full(f.fd, buf.data(), n, off, &rc)) return;
                    h.update(buf.data(), n);
                }
#ifdef POSIX_FADV_DONTNEED
                if (drop_pages) ::posix_fadvise(f.fd, 0, 0, POSIX_FADV_DONTNEED);
#endif
                digest[s] = h.hex();
                ok[s] = 1;
            });
            for (size_t s = 0; s < files_.size(); ++s) {
                if (!ok[s]) return fail("DEE4 segment " + files_[s].file + " seal read failed");
                if (digest[s] != files_[s].sha256) return fail("DEE4 segment " + files_[s].file + " sha256 mismatch");
            }
        }
    } else {
        size_t expect = 0;
        if (!checked_mul(total, record_bytes_, &expect)) return fail("DEE4 total size overflow");
        StoreFile f;
        f.file = data_file;
        f.sha256 = lower(identity_);  // data_sha256 seals the whole file
        f.first_record = 0;
        f.record_count = total;
        if (!open_file(dir, &f)) {
            if (f.fd >= 0) ::close(f.fd);
            const std::string msg = last_error_;
            return fail(msg);
        }
        files_.push_back(std::move(f));
        if (files_[0].size != expect)
            return fail("DEE4 data size " + std::to_string(files_[0].size) + " does not match expected " +
                        std::to_string(expect));
    }
    start_layer_ = static_cast<int>(start_layer);
    num_layers_ = static_cast<int>(num_layers);
    experts_per_layer_ = static_cast<int>(experts);
    stored_records_ = total;
    return true;
}

}  // namespace store
}  // namespace dee

using dee::store::Dee4Store;

struct dee_store {
    Dee4Store s;
};

namespace {

void fill_stats(dee_store_read_stats* out, const dee::store::ReadCounters& rc, uint64_t records, double seconds,
                uint64_t files_verified = 0) {
    if (!out) return;
    out->files_verified = files_verified;
    out->bytes_read = rc.bytes.load();
    out->pread_calls = rc.calls.load();
    out->short_reads = rc.short_reads.load();
    out->records = records;
    out->seconds = seconds;
}

}  // namespace

extern "C" {

DEE_API int dee_store_create(dee_store** out) {
    if (!out) return DEE_ERR_INVALID;
    *out = new (std::nothrow) dee_store();
    return *out ? DEE_OK : DEE_ERR_INVALID;
}

DEE_API void dee_store_destroy(dee_store* store) { delete store; }

DEE_API int dee_store_open(dee_store* store, const char* directory_or_metadata, int options, int threads) {
    if (!store) return DEE_ERR_INVALID;
    if (!directory_or_metadata) {
        store->s.last_error_ = "DEE4 metadata.json is missing";
        return DEE_ERR_INVALID;
    }
    return store->s.open(directory_or_metadata, (options & DEE_STORE_VERIFY_SEALS) != 0,
                         (options & DEE_STORE_SEAL_DROP_PAGES) != 0, threads)
               ? DEE_OK
               : DEE_ERR_INVALID;
}

DEE_API void dee_store_close(dee_store* store) {
    if (store) store->s.close();
}

DEE_API const char* dee_store_last_error(const dee_store* store) {
    return store ? store->s.last_error_.c_str() : "null store";
}

DEE_API const char* dee_store_backend(const dee_store* store) { return store ? store->s.backend_.c_str() : ""; }

DEE_API const char* dee_store_identity(const dee_store* store) { return store ? store->s.identity_.c_str() : ""; }

DEE_API int dee_store_get_info(const dee_store* store, dee_store_info* out) {
    if (!store || !out || !store->s.loaded()) return DEE_ERR_INVALID;
    store->s.info(out);
    return DEE_OK;
}

DEE_API int dee_store_stats(const dee_store* store, uint64_t* out4) {
    if (!store || !out4) return DEE_ERR_INVALID;
    store->s.stats(out4);
    return DEE_OK;
}

DEE_API int dee_store_lookup(dee_store* store, int layer, int expert, uint64_t* record_index) {
    if (!store || !record_index) return DEE_ERR_INVALID;
    size_t idx = 0;
    if (!store->s.lookup(layer, expert, &idx)) return DEE_ERR_RANGE;
    *record_index = idx;
    return DEE_OK;
}

DEE_API int dee_store_materialize(dee_store* store, int layer, int expert, void* dst, size_t nbytes,
                                  dee_store_read_stats* stats) {
    if (!store || !dst) return DEE_ERR_INVALID;
    Dee4Store& s = store->s;
    dee::store::ReadCounters rc;
    const auto t0 = std::chrono::steady_clock::now();
    size_t idx = 0, off = 0;
    const dee::store::StoreFile* f = nullptr;
    if (!s.lookup(layer, expert, &idx) || !s.locate(idx, &f, &off)) {
        s.last_error_ = "DEE4 record (layer " + std::to_string(layer) + ", expert " + std::to_string(expert) +
                        ") is not in the store";
        fill_stats(stats, rc, 0, 0.0);
        return DEE_ERR_RANGE;
    }
    if (nbytes != s.record_bytes()) {
        s.last_error_ = "materialize needs exactly record_bytes of destination";
        fill_stats(stats, rc, 0, 0.0);
        return DEE_ERR_INVALID;
    }
    const bool ok = dee::store::pread_full(f->fd, dst, nbytes, off, &rc);
    s.count_reads(1, rc.bytes.load());
    fill_stats(stats, rc, ok ? 1 : 0, dee::store::seconds_since(t0));
    if (!ok) {
        s.last_error_ = "DEE4 read of " + f->file + " failed";
        return DEE_ERR_INVALID;
    }
    return DEE_OK;
}

DEE_API int dee_store_read_layers(dee_store* store, int first_layer, int layers, int first_expert, int experts,
                                  void* dst, size_t dst_bytes, int threads, int verify, dee_store_read_stats* stats) {
    if (!store || !dst) return DEE_ERR_INVALID;
    Dee4Store& s = store->s;
    if (!s.loaded() || !s.valid_range(first_layer, layers, first_expert, experts)) {
        s.last_error_ = "layer or expert range outside the store";
        return DEE_ERR_RANGE;
    }
    const size_t need = static_cast<size_t>(layers) * experts * s.record_bytes();
    if (dst_bytes < need) {
        s.last_error_ = "destination smaller than the layers' records";
        return DEE_ERR_INVALID;
    }
    std::vector<dee::store::Task> tasks;
    if (!s.plan_layers(first_layer, layers, first_expert, experts, size_t(16) << 20, verify != 0, &tasks))
        return DEE_ERR_RANGE;
    dee::store::ReadCounters rc;
    std::atomic<uint64_t> sealed{0};
    const auto t0 = std::chrono::steady_clock::now();
    char* base = static_cast<char*>(dst);
    const std::string err = dee::store::run_tasks(
        tasks, std::max(1, threads), &rc, &sealed,
        [&](int, const dee::store::Task& t, size_t off) -> void* { return base + t.dst_offset + off; },
        [](int, void*, size_t, size_t) { return true; });
    const uint64_t records = static_cast<uint64_t>(layers) * experts;
    s.count_reads(records, rc.bytes.load());
    fill_stats(stats, rc, err.empty() ? records : 0, dee::store::seconds_since(t0), sealed.load());
    if (!err.empty()) {
        s.last_error_ = err;
        return DEE_ERR_INVALID;
    }
    return DEE_OK;
}

DEE_API int dee_store_upload_layers_device(dee_store* store, int first_layer, int layers, int first_expert,
                                           int experts, void* d_dst, size_t dst_bytes, size_t staging_bytes,
                                           int threads, int verify, void* stream, dee_store_read_stats* stats) {
    if (!store || !d_dst) return DEE_ERR_INVALID;
    Dee4Store& s = store->s;
    if (!s.loaded() || !s.valid_range(first_layer, layers, first_expert, experts)) {
        s.last_error_ = "layer or expert range outside the store";
        return DEE_ERR_RANGE;
    }
    const size_t need = static_cast<size_t>(layers) * experts * s.record_bytes();
    if (dst_bytes < need) {
        s.last_error_ = "device destination smaller than the layers' records";
        return DEE_ERR_INVALID;
    }
    threads = std::max(1, threads);
    // Each reader thread double-buffers: pread into one pinned half while the
    // copy engine drains the other.
    const size_t chunk = std::max<size_t>(size_t(1) << 20, (staging_bytes / (2 * threads)) & ~size_t(4095));
    std::vector<dee::store::Task> tasks;
    if (!s.plan_layers(first_layer, layers, first_expert, experts, chunk, verify != 0, &tasks)) return DEE_ERR_RANGE;
    threads = static_cast<int>(std::min<size_t>(static_cast<size_t>(threads), tasks.size()));
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        s.last_error_ = "no CUDA device";
        return DEE_ERR_CUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t nbuf = 2 * static_cast<size_t>(threads);
    std::vector<void*> bufs(nbuf, nullptr);
    std::vector<cudaEvent_t> evs(nbuf, nullptr);
    std::vector<int> used(nbuf, 0), half(threads, 0), bound(threads, 0);
    std::string cuda_err;
    std::mutex err_mu;
    auto note = [&](cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        std::lock_guard<std::mutex> g(err_mu);
        if (cuda_err.empty()) cuda_err = std::string(what) + ": " + cudaGetErrorString(e);
        return false;
    };
    bool ok = true;
    for (size_t b = 0; b < nbuf && ok; ++b)
        ok = note(cudaHostAlloc(&bufs[b], chunk, cudaHostAllocDefault), "cudaHostAlloc") &&
             note(cudaEventCreateWithFlags(&evs[b], cudaEventDisableTiming), "cudaEventCreate");
    dee::store::ReadCounters rc;
    std::atomic<uint64_t> sealed{0};
    std::string err;
    const auto t0 = std::chrono::steady_clock::now();
    if (ok) {
        err = dee::store::run_tasks(
            tasks, threads, &rc, &sealed,
            [&](int w, const dee::store::Task&, size_t) -> void* {
                if (!bound[w]) {  // a worker thread's first piece: bind it to the device
                    if (!note(cudaSetDevice(device), "cudaSetDevice")) return nullptr;
                    bound[w] = 1;
                }
                const size_t b = 2 * static_cast<size_t>(w) + half[w];
                if (used[b] && !note(cudaEventSynchronize(evs[b]), "cudaEventSynchronize")) return nullptr;
                return bufs[b];
            },
            [&](int w, void* buf, size_t dst_off, size_t n) {
                const size_t b = 2 * static_cast<size_t>(w) + half[w];
                if (!note(cudaMemcpyAsync(static_cast<char*>(d_dst) + dst_off, buf, n, cudaMemcpyHostToDevice, st),
                          "cudaMemcpyAsync") ||
                    !note(cudaEventRecord(evs[b], st), "cudaEventRecord"))
                    return false;
                used[b] = 1;
                half[w] ^= 1;
                return true;
            });
        note(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    }
    for (size_t b = 0; b < nbuf; ++b) {
        if (evs[b]) cudaEventDestroy(evs[b]);
        if (bufs[b]) cudaFreeHost(bufs[b]);
    }
    const uint64_t records = static_cast<uint64_t>(layers) * experts;
    s.count_reads(records, rc.bytes.load());
    const bool good = err.empty() && cuda_err.empty();
    fill_stats(stats, rc, good ? records : 0, dee::store::seconds_since(t0), sealed.load());
    if (!cuda_err.empty()) {
        s.last_error_ = cuda_err;
        return DEE_ERR_CUDA;
    }
    if (!err.empty()) {
        s.last_error_ = err;
        return DEE_ERR_INVALID;
    }
    return DEE_OK;
}

DEE_API int dee_sha256_hex(const void* data, size_t n, char* out65) {
    if ((!data && n) || !out65) return DEE_ERR_INVALID;
    dee::store::Sha256 h;
    if (n) h.update(data, n);
    const std::string hex = h.hex();
    std::memcpy(out65, hex.c_str(), 65);
    return DEE_OK;
}

}  // extern "C"
