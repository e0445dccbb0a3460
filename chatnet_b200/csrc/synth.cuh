// synth.cuh -- seeded synthetic inputs, identical on host and device.
//
// The benchmark configs call for random GGUF blocks and N(0,1) activations.
// Every value is produced from a counter-based splitmix64 stream (the i-th
// output of the stream seeded with s is mix64(s + (i+1)*golden), so any
// block can be generated independently), and every step is integer or
// exactly-rounded fp32 arithmetic.  The host and the device therefore write
// the same bytes, which lets the benchmark generate tens of GB in HBM while
// the oracle gets the same tensors from the host generator.
//
// N(0,1) is approximated by the Irwin-Hall sum of twelve 16-bit uniforms:
// (sum - 393210) / 65536.  The sum of twelve U{0..65535} has mean 393210 and
// standard deviation sqrt(65536^2 - 1) ~= 65536, so the result has mean 0,
// variance 1 to 1e-10, support [-6, 6], and is exact in fp32.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#ifdef __CUDACC__
#define CN_HD __host__ __device__ __forceinline__
#else
#define CN_HD inline
#endif

namespace cn {
namespace synth {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

CN_HD uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

CN_HD uint64_t draw(uint64_t seed, uint64_t i) { return mix64(seed + (i + 1) * kGolden); }

CN_HD uint32_t sum4x16(uint64_t v) {
    return (uint32_t)(v & 0xFFFF) + (uint32_t)((v >> 16) & 0xFFFF) +
           (uint32_t)((v >> 32) & 0xFFFF) + (uint32_t)(v >> 48);
}

// Normal deviate from draws i, i+1, i+2.
CN_HD float normal(uint64_t seed, uint64_t i) {
    uint32_t s = sum4x16(draw(seed, i)) + sum4x16(draw(seed, i + 1)) + sum4x16(draw(seed, i + 2));
    return (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
}

// IEEE fp32 -> fp16 bits, round to nearest even.
CN_HD uint16_t f2h(float f) {
#ifdef __CUDA_ARCH__
    return __half_as_ushort(__float2half_rn(f));
#else
    uint32_t x;
    __builtin_memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        int shift = 126 - (int)e;
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = (ax - 0x38000000u) >> 13;
    uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
#endif
}

CN_HD float fmul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
CN_HD float fadd(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}

CN_HD void put64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; i++) p[i] = (uint8_t)(v >> (8 * i));
}

// Little-endian fp16 bits at a 2-byte aligned address, written as one
// 16-bit store.
CN_HD void put16(uint8_t* p, uint16_t v) { *reinterpret_cast<uint16_t*>(p) = v; }

// Q4_0 block b (18 bytes, `out` 2-byte aligned): d = fp16(|N| * 0.02/8),
// nibbles U[0,15].  Draws 5b..5b+4.
CN_HD void q4_0_block(uint64_t seed, uint64_t b, uint8_t* out) {
    uint64_t base = 5 * b;
    float n = normal(seed, base);
    float d = fmul(n < 0.f ? -n : n, 0.0025f);
    put16(out, f2h(d));
    put64(out + 2, draw(seed, base + 3));
    put64(out + 10, draw(seed, base + 4));
}

// Q4_K super-block b (144 bytes): d, dmin = fp16(|N| * 0.01); 6-bit
// scales and mins U[0,63] packed in the 12-byte layout that
// DequantQ4K.DecodeScales (DequantQ4K.cs:218-241) unpacks; 128 bytes of
// U[0,15] nibbles.  Draws 24b..24b+23.
CN_HD void q4_k_block(uint64_t seed, uint64_t b, uint8_t* out) {
    uint64_t base = 24 * b;
    float n0 = normal(seed, base), n1 = normal(seed, base + 3);
    uint16_t d = f2h(fmul(n0 < 0.f ? -n0 : n0, 0.01f));
    uint16_t dmin = f2h(fmul(n1 < 0.f ? -n1 : n1, 0.01f));
    put16(out, d);
    put16(out + 2, dmin);
    uint64_t rs = draw(seed, base + 6), rm = draw(seed, base + 7);
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)((rs >> (8 * j)) & 63);
        m[j] = (uint8_t)((rm >> (8 * j)) & 63);
    }
    uint8_t* q = out + 4;
    for (int j = 0; j < 4; j++) {
        q[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        q[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
        q[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    for (int i = 0; i < 16; i++) put64(out + 16 + 8 * i, draw(seed, base + 8 + i));
}

// Q6_K super-block b (210 bytes): ql[128], qh[64] uniform bits; int8
// scales U[0,63]; d = fp16(|N| * 0.01) at byte 208.  Draws 29b..29b+28.
CN_HD void q6_k_block(uint64_t seed, uint64_t b, uint8_t* out) {
    uint64_t base = 29 * b;
    for (int i = 0; i < 24; i++) put64(out + 8 * i, draw(seed, base + i));  // ql + qh
    uint64_t s0 = draw(seed, base + 24), s1 = draw(seed, base + 25);
    for (int j = 0; j < 8; j++) {
        out[192 + j] = (uint8_t)((s0 >> (8 * j)) & 63);
        out[200 + j] = (uint8_t)((s1 >> (8 * j)) & 63);
    }
    float n = normal(seed, base + 26);
    put16(out + 208, f2h(fmul(n < 0.f ? -n : n, 0.01f)));
}

// Element i of an F32 / F16 tensor.
CN_HD float normal_elem(uint64_t seed, uint64_t i) { return normal(seed, 3 * i); }
CN_HD float norm_weight_elem(uint64_t seed, uint64_t i) {
    return fadd(1.0f, fmul(0.01f, normal(seed, 3 * i)));
}

}  // namespace synth
}  // namespace cn
