// synth.cpp -- the seeded synthetic inputs of the benchmark configs, for the
// oracle side.
//
// TEST INFRASTRUCTURE ONLY (see oracle.h).  The CPU baseline and the parity
// tests need the same bytes the product's device generator writes, without
// loading the product library: this file produces them from the generator's
// specification, and a CPU test checks it byte for byte against the
// product's own host generator.
//
// Specification (counter-based, so any block can be generated alone):
//   draw(s, i)    = splitmix64 finaliser of s + (i + 1) * 0x9E3779B97F4A7C15
//   normal(s, i)  = (sum of the four 16-bit fields of draws i, i+1, i+2
//                    - 393210) / 65536       (Irwin-Hall(12), exact in fp32)
//   seed(cfg, nm) = finaliser(FNV-1a-64(nm) ^ (uint32 cfg) * 0x9E3779B97F4A7C15)
//   Q4_0 block b  : draws 5b..5b+4.  d = fp16(|normal(5b)| * 0.0025); quant
//                   bytes 0..7 and 8..15 = draws 5b+3, 5b+4, little endian.
//   Q4_K block b  : draws 24b..24b+23.  d = fp16(|normal(24b)| * 0.01),
//                   dmin = fp16(|normal(24b+3)| * 0.01); 6-bit scales and
//                   mins = bytes of draws 24b+6 / 24b+7 masked to 63, packed in
//                   GGUF's 12-byte scale layout; 128 quant bytes = draws
//                   24b+8..24b+23.
//   Q6_K block b  : draws 29b..29b+28.  ql/qh (192 bytes) = draws 29b..29b+23;
//                   the 16 int8 scales = bytes of draws 29b+24, 29b+25 masked
//                   to 63; d = fp16(|normal(29b+26)| * 0.01) at byte 208.
//   F32 element i : normal(3i), or 1 + 0.01 * normal(3i) for norm weights.
//   F16 element i : fp16(normal(3i)).
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "oracle.h"

namespace {

constexpr uint64_t kG = 0x9E3779B97F4A7C15ull;

uint64_t fin(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t draw(uint64_t s, uint64_t i) { return fin(s + (i + 1) * kG); }

uint32_t fields16(uint64_t v) {
    uint32_t t = 0;
    for (int k = 0; k < 4; k++) t += (uint32_t)((v >> (16 * k)) & 0xFFFFu);
    return t;
}

float normal(uint64_t s, uint64_t i) {
    const uint32_t sum = fields16(draw(s, i)) + fields16(draw(s, i + 1)) + fields16(draw(s, i + 2));
    return (float)((int32_t)sum - 393210) / 65536.0f;  // exact: |numerator| < 2^22
}

void le64(uint8_t* p, uint64_t v) {
    for (int k = 0; k < 8; k++) p[k] = (uint8_t)(v >> (8 * k));
}
void le16(uint8_t* p, uint16_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
}

float fabs_(float v) { return v < 0.f ? -v : v; }

void q4_0(uint64_t s, uint64_t b, uint8_t* o) {
    le16(o, or_float_to_half(fabs_(normal(s, 5 * b)) * 0.0025f));
    le64(o + 2, draw(s, 5 * b + 3));
    le64(o + 10, draw(s, 5 * b + 4));
}

void q4_k(uint64_t s, uint64_t b, uint8_t* o) {
    const uint64_t base = 24 * b;
    le16(o, or_float_to_half(fabs_(normal(s, base)) * 0.01f));
    le16(o + 2, or_float_to_half(fabs_(normal(s, base + 3)) * 0.01f));
    const uint64_t rs = draw(s, base + 6), rm = draw(s, base + 7);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)((rs >> (8 * j)) & 63u);
        mn[j] = (uint8_t)((rm >> (8 * j)) & 63u);
    }
    // the 12-byte layout GGUF (and DequantQ4K.DecodeScales) uses: sub-blocks
    // 0-3 in the low six bits of bytes 0-3 / 4-7, sub-blocks 4-7 split into a
    // low nibble in bytes 8-11 and two high bits on top of bytes 0-7
    for (int j = 0; j < 4; j++) {
        o[4 + j] = (uint8_t)(sc[j] | ((sc[4 + j] >> 4) << 6));
        o[8 + j] = (uint8_t)(mn[j] | ((mn[4 + j] >> 4) << 6));
        o[12 + j] = (uint8_t)((sc[4 + j] & 15) | ((mn[4 + j] & 15) << 4));
    }
    for (int k = 0; k < 16; k++) le64(o + 16 + 8 * k, draw(s, base + 8 + k));
}

void q6_k(uint64_t s, uint64_t b, uint8_t* o) {
    const uint64_t base = 29 * b;
    for (int k = 0; k < 24; k++) le64(o + 8 * k, draw(s, base + k));
    for (int h = 0; h < 2; h++) {
        const uint64_t r = draw(s, base + 24 + h);
        for (int j = 0; j < 8; j++) o[192 + 8 * h + j] = (uint8_t)((r >> (8 * j)) & 63u);
    }
    le16(o + 208, or_float_to_half(fabs_(normal(s, base + 26)) * 0.01f));
}

// Runs f(i) for i in [0, n) on all cores.
template <typename F>
void par(uint64_t n, F f) {
    unsigned nt = std::max(1u, std::thread::hardware_concurrency());
    if (n < 4096) nt = 1;
    std::vector<std::thread> ts;
    const uint64_t per = (n + nt - 1) / nt;
    for (unsigned t = 0; t < nt; t++) {
        const uint64_t a = t * per, e = std::min(n, a + per);
        if (a >= e) break;
        ts.emplace_back([=] {
            for (uint64_t i = a; i < e; i++) f(i);
        });
    }
    for (auto& t : ts) t.join();
}

}  // namespace

extern "C" {

uint64_t or_synth_seed(int config_id, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (const char* p = name ? name : ""; *p; p++) h = (h ^ (uint8_t)*p) * 0x100000001b3ull;
    return fin(h ^ ((uint64_t)(uint32_t)config_id * kG));
}

int or_synth_fill_rows(int type, int64_t row0, int64_t rows, int64_t cols, uint64_t seed, int norm_weight,
                       void* out, uint64_t bytes) {
    if (!out || row0 < 0 || rows < 0 || cols < 0) return -1;
    const uint64_t n = (uint64_t)rows * (uint64_t)cols, e0 = (uint64_t)row0 * (uint64_t)cols;
    if (or_byte_size(type, (uint64_t)cols) * (uint64_t)rows != bytes) return -1;
    uint8_t* o = static_cast<uint8_t*>(out);
    switch (type) {
        case OR_Q4_0:
            if (cols % 32) return -1;
            par(n / 32, [&](uint64_t b) { q4_0(seed, e0 / 32 + b, o + 18 * b); });
            return 0;
        case OR_Q4_K:
            if (cols % 256) return -1;
            par(n / 256, [&](uint64_t b) { q4_k(seed, e0 / 256 + b, o + 144 * b); });
            return 0;
        case OR_Q6_K:
            if (cols % 256) return -1;
            par(n / 256, [&](uint64_t b) { q6_k(seed, e0 / 256 + b, o + 210 * b); });
            return 0;
        case OR_F32: {
            float* f = static_cast<float*>(out);
            par(n, [&](uint64_t i) {
                const float v = normal(seed, 3 * (e0 + i));
                f[i] = norm_weight ? 1.0f + 0.01f * v : v;
            });
            return 0;
        }
        case OR_F16: {
            uint16_t* h = static_cast<uint16_t*>(out);
            par(n, [&](uint64_t i) { h[i] = or_float_to_half(normal(seed, 3 * (e0 + i))); });
            return 0;
        }
    }
    return -2;
}

int or_synth_fill(int type, int64_t rows, int64_t cols, uint64_t seed, int norm_weight, void* out,
                  uint64_t bytes) {
    return or_synth_fill_rows(type, 0, rows, cols, seed, norm_weight, out, bytes);
}

}  // extern "C"
