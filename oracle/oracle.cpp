// oracle.cpp -- CPU restatement of ChatNet's quantized-weight hot path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker and timed CPU baseline for
// libchatnet_cuda.  Each function names the reference routine (file:line,
// relative to the ChatNet source tree) whose arithmetic it restates.  The
// SSE code below reproduces the reference's Vector128 lane structure so the
// rounding sequence per lane is the same as the C# SIMD path.

#include "oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

// ---------------------------------------------------------------------------
// fp16 helpers
// ---------------------------------------------------------------------------

// DequantQ4_0.HalfToFloat (DequantQ4_0.cs:190-194): (float)Half is exact.
extern "C" float or_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    float f;
    if (e == 0) {
        // zero or subnormal: m * 2^-24, exact in fp32
        f = (float)m * 5.9604644775390625e-08f;
        uint32_t bits;
        memcpy(&bits, &f, 4);
        bits |= sign;
        memcpy(&f, &bits, 4);
        return f;
    }
    uint32_t bits;
    if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    memcpy(&f, &bits, 4);
    return f;
}

// IEEE binary32 -> binary16, round to nearest even (the rounding
// BitConverter.HalfToUInt16Bits((Half)value) applies in the tests' WriteHalf,
// QuantizationTests.cs:768-773, and the rounding used for an fp16 KV cache).
extern "C" uint16_t or_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // >= 65520 -> inf
    if (ax < 0x38800000u) {                                     // below 2^-14
        if (ax < 0x33000000u) return (uint16_t)sign;            // below 2^-25
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
}

static inline float h2f(const uint8_t* p) { return or_half_to_float((uint16_t)(p[0] | (p[1] << 8))); }

// GgufTensorInfo.ByteSize (GgufTensorInfo.cs:30-114), supported types only.
extern "C" uint64_t or_byte_size(int type, uint64_t elements) {
    switch (type) {
        case OR_F32: return elements * 4;
        case OR_F16: return elements * 2;
        case OR_Q4_0: return (elements + 31) / 32 * 18;
        case OR_Q4_1: return (elements + 31) / 32 * 20;
        case OR_Q5_0: return (elements + 31) / 32 * 22;
        case OR_Q5_1: return (elements + 31) / 32 * 24;
        case OR_Q8_0: return (elements + 31) / 32 * 34;
        case OR_Q4_K: return (elements + 255) / 256 * 144;
        case OR_Q6_K: return (elements + 255) / 256 * 210;
        case OR_Q2_K: return (elements + 255) / 256 * 84;
        case OR_Q3_K: return (elements + 255) / 256 * 110;
        case OR_Q5_K: return (elements + 255) / 256 * 176;
        case OR_Q8_K: return (elements + 255) / 256 * 292;
        case OR_IQ4_NL: return (elements + 31) / 32 * 18;
        case OR_IQ4_XS: return (elements + 255) / 256 * 136;
        case OR_IQ3_S: return (elements + 255) / 256 * 110;
        case OR_IQ3_XXS: return (elements + 255) / 256 * 98;
        case OR_IQ2_XS: return (elements + 255) / 256 * 74;
        case OR_IQ2_XXS: return (elements + 255) / 256 * 66;
        case OR_IQ2_S: return (elements + 255) / 256 * 82;
        case OR_IQ1_S: return (elements + 255) / 256 * 50;
        case OR_IQ1_M: return (elements + 255) / 256 * 56;
        default: return 0;
    }
}

// ---------------------------------------------------------------------------
// Dequantize
// ---------------------------------------------------------------------------

// DequantQ4_0.Dequantize (DequantQ4_0.cs:28-58), partial last block included.
static void dequant_q4_0(const uint8_t* q, float* out, int64_t n) {
    int64_t nb = (n + 31) / 32;
    int64_t src = 0, dst = 0;
    for (int64_t b = 0; b < nb; b++) {
        float scale = h2f(q + src);
        src += 2;
        int64_t remaining = n - dst;
        int half = remaining < 16 ? (int)remaining : 16;
        for (int j = 0; j < half; j++) {
            int low = (q[src + j] & 0x0F) - 8;
            out[dst + j] = (float)low * scale;
        }
        int second = remaining < 32 ? (remaining > 16 ? (int)(remaining - 16) : 0) : 16;
        for (int j = 0; j < second; j++) {
            int high = ((q[src + j] >> 4) & 0x0F) - 8;
            out[dst + 16 + j] = (float)high * scale;
        }
        src += 16;
        dst += half + second;
    }
}

// The 32-weight codecs.  Dequantize writes `count` (or half / second-half)
// elements of a partial last block, like the Q4_0 loop above.
// DequantQ8_0.Dequantize (DequantQ8_0.cs:19-41): (sbyte)q * d.
static void dequant_q8_0(const uint8_t* q, float* out, int64_t n) {
    int64_t nb = (n + 31) / 32, src = 0, dst = 0;
    for (int64_t b = 0; b < nb; b++) {
        float scale = h2f(q + src);
        src += 2;
        int64_t remaining = n - dst;
        int count = remaining < 32 ? (int)remaining : 32;
        for (int i = 0; i < count; i++) out[dst + i] = (float)(int8_t)q[src + i] * scale;
        src += 32;
        dst += count;
    }
}

// DequantQ4_1.Dequantize (DequantQ4_1.cs:24-56): q * d + m (d@0, m@2, qs@4).
// DequantQ5_0.Dequantize (DequantQ5_0.cs:29-68): (q5 - 16) * d (d@0, qh@2, qs@6).
// DequantQ5_1.Dequantize (DequantQ5_1.cs:30-69): q5 * d + m (d@0, m@2, qh@4, qs@8).
// q5 = nibble | ((qh >> j) & 1) << 4, j the element's index in the block.
static void dequant_b32(int type, const uint8_t* q, float* out, int64_t n) {
    const int bpb = type == OR_Q4_1 ? 20 : type == OR_Q5_0 ? 22 : 24;
    const int qs_off = type == OR_Q4_1 ? 4 : type == OR_Q5_0 ? 6 : 8;
    const int qh_off = type == OR_Q5_0 ? 2 : 4;
    int64_t nb = (n + 31) / 32, dst = 0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * bpb;
        float scale = h2f(blk);
        float min = type == OR_Q5_0 ? 0.f : h2f(blk + 2);
        uint32_t qh = 0;
        if (type != OR_Q4_1)
            qh = (uint32_t)blk[qh_off] | ((uint32_t)blk[qh_off + 1] << 8) | ((uint32_t)blk[qh_off + 2] << 16) |
                 ((uint32_t)blk[qh_off + 3] << 24);
        int64_t remaining = n - dst;
        int half = remaining < 16 ? (int)remaining : 16;
        int second = remaining < 32 ? (remaining > 16 ? (int)(remaining - 16) : 0) : 16;
        for (int h = 0; h < 2; h++) {
            int cnt = h == 0 ? half : second;
            for (int j = 0; j < cnt; j++) {
                int nib = h == 0 ? (blk[qs_off + j] & 0x0F) : ((blk[qs_off + j] >> 4) & 0x0F);
                int idx = 16 * h + j;
                if (type == OR_Q4_1) {
                    out[dst + idx] = (float)nib * scale + min;
                } else {
                    int q5 = nib | (int)((qh >> idx) & 1u) << 4;
                    out[dst + idx] = type == OR_Q5_0 ? (float)(q5 - 16) * scale : (float)q5 * scale + min;
                }
            }
        }
        dst += half + second;
    }
}

// DequantQ4K.DecodeScales (DequantQ4K.cs:218-241).
static void decode_scales_q4k(const uint8_t* q, int* sc, int* m) {
    for (int j = 0; j < 4; j++) {
        sc[j] = q[j] & 63;
        m[j] = q[j + 4] & 63;
    }
    for (int j = 4; j < 8; j++) {
        sc[j] = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m[j] = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// DequantQ4K.Dequantize (DequantQ4K.cs:37-77).  Only whole super-blocks are
// written (blockCount = elementCount / 256), as in the reference.
static void dequant_q4_k(const uint8_t* q, float* out, int64_t n) {
    int64_t nb = n / 256;
    int sc[8], m[8];
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 144;
        float d = h2f(blk + 0);
        float dmin = h2f(blk + 2);
        decode_scales_q4k(blk + 4, sc, m);
        for (int sub = 0; sub < 8; sub++) {
            float dsc = d * (float)sc[sub];
            float dm = dmin * (float)m[sub];
            const uint8_t* qs = blk + 16 + sub * 16;
            float* o = out + b * 256 + sub * 32;
            for (int j = 0; j < 16; j++) {
                uint8_t byte = qs[j];
                float lo = dsc * (float)(byte & 0x0F);
                float hi = dsc * (float)((byte >> 4) & 0x0F);
                o[j] = lo - dm;
                o[j + 16] = hi - dm;
            }
        }
    }
}

// DequantQ6K.Dequantize (DequantQ6K.cs:37-88): d * sc * q, left to right.
static void dequant_q6_k(const uint8_t* q, float* out, int64_t n) {
    int64_t nb = n / 256;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = q + b * 210;
        float d = h2f(blk + 208);
        for (int half = 0; half < 2; half++) {
            const uint8_t* ql = blk + half * 64;
            const uint8_t* qh = blk + 128 + half * 32;
            const int8_t* scs = (const int8_t*)(blk + 192);
            int sc_off = half * 8;
            float* o = out + b * 256 + half * 128;
            for (int l = 0; l < 32; l++) {
                int si = sc_off + l / 16;
                int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                float t1 = d * (float)scs[si];
                float t2 = d * (float)scs[si + 2];
                float t3 = d * (float)scs[si + 4];
                float t4 = d * (float)scs[si + 6];
                o[l] = t1 * (float)q1;
                o[l + 32] = t2 * (float)q2;
                o[l + 64] = t3 * (float)q3;
                o[l + 96] = t4 * (float)q4;
            }
        }
    }
}

// ---- the other K-quants and the IQ4 codecs (generic paths on the device) ----

// DequantIQ.IQ4NL_Table (DequantIQ.cs:29-33): the 16 non-linear levels.
static const float kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// DequantQ3K.DecodeScales (DequantQ3K.cs:124-148): 16 six-bit scales, minus 32.
static void decode_scales_q3k(const uint8_t* q, int* sc) {
    for (int i = 0; i < 8; i++) {
        sc[i] = q[i] & 0x0F;
        sc[i + 8] = (q[i] >> 4) & 0x0F;
    }
    for (int i = 0; i < 4; i++) {
        const uint8_t hb = q[8 + i];
        sc[i] |= ((hb >> 0) & 3) << 4;
        sc[i + 4] |= ((hb >> 2) & 3) << 4;
        sc[i + 8] |= ((hb >> 4) & 3) << 4;
        sc[i + 12] |= ((hb >> 6) & 3) << 4;
    }
    for (int i = 0; i < 16; i++) sc[i] -= 32;
}

static inline float f32_le(const uint8_t* p) {
    const uint32_t u = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// DequantQ2K.Dequantize (DequantQ2K.cs:32-88): two groups of 128, four
// 2-bit shifts each, two 16-element halves per shift; dl * q - ml with
// dl = d * (sc & 15), ml = dmin * (sc >> 4) (d@80, dmin@82, scales@0, qs@16).
static void dequant_q2_k(const uint8_t* q, float* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 84;
        const float d = h2f(blk + 80), dmin = h2f(blk + 82);
        float* o = out + b * 256;
        int si = 0;
        for (int g = 0; g < 2; g++)
            for (int shift = 0; shift < 8; shift += 2) {
                for (int h = 0; h < 2; h++) {
                    const float dl = d * (float)(blk[si + h] & 0x0F);
                    const float ml = dmin * (float)((blk[si + h] >> 4) & 0x0F);
                    for (int l = 0; l < 16; l++) *o++ = dl * (float)((blk[16 + 32 * g + 16 * h + l] >> shift) & 3) - ml;
                }
                si += 2;
            }
    }
}

// DequantQ3K.Dequantize (DequantQ3K.cs:35-70): d * scale * (q3 - 4), q3 = the
// 2 bits of qs[i / 4] at (i % 4) * 2 | bit i % 8 of hmask[i / 8] << 2
// (hmask@0, qs@32, scales@96, d@108).
static void dequant_q3_k(const uint8_t* q, float* out, int64_t n) {
    int sc[16];
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 110;
        const float d = h2f(blk + 108);
        decode_scales_q3k(blk + 96, sc);
        for (int i = 0; i < 256; i++) {
            const int q2 = (blk[32 + i / 4] >> ((i % 4) * 2)) & 3;
            const int q3 = q2 | (((blk[i / 8] >> (i % 8)) & 1) << 2);
            out[b * 256 + i] = d * (float)sc[i / 16] * (float)(q3 - 4);
        }
    }
}

// DequantQ5K.Dequantize (DequantQ5K.cs:36-90): d * sc * q5 - dmin * m (scales
// as Q4_K), q5 = nibble | bit e % 8 of qh[e / 8] << 4 for element e
// (d@0, dmin@2, scales@4, qh@16, qs@48; sub-block s uses qs bytes 16s..16s+15).
static void dequant_q5_k(const uint8_t* q, float* out, int64_t n) {
    int sc[8], m[8];
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 176;
        const float d = h2f(blk), dmin = h2f(blk + 2);
        decode_scales_q4k(blk + 4, sc, m);
        for (int sub = 0; sub < 8; sub++) {
            const float dsc = d * (float)sc[sub], dm = dmin * (float)m[sub];
            for (int h = 0; h < 2; h++)
                for (int j = 0; j < 16; j++) {
                    const int e = sub * 32 + 16 * h + j;
                    const int nib = h == 0 ? (blk[48 + sub * 16 + j] & 0x0F) : ((blk[48 + sub * 16 + j] >> 4) & 0x0F);
                    const int q5 = nib | (((blk[16 + e / 8] >> (e % 8)) & 1) << 4);
                    out[b * 256 + e] = dsc * (float)q5 - dm;
                }
        }
    }
}

// DequantQ8K.Dequantize (DequantQ8K.cs:25-47): (sbyte)q * d, d an fp32 at 0.
static void dequant_q8_k(const uint8_t* q, float* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 292;
        const float d = f32_le(blk);
        for (int i = 0; i < 256; i++) out[b * 256 + i] = (float)(int8_t)blk[4 + i] * d;
    }
}

// DequantIQ.IQ4NL.Dequantize (DequantIQ.cs:45-76): scale * table[nibble],
// Q4_0's layout and partial last block.
static void dequant_iq4_nl(const uint8_t* q, float* out, int64_t n) {
    int64_t nb = (n + 31) / 32, src = 0, dst = 0;
    for (int64_t b = 0; b < nb; b++) {
        const float scale = h2f(q + src);
        src += 2;
        const int64_t remaining = n - dst;
        const int half = remaining < 16 ? (int)remaining : 16;
        const int second = remaining < 32 ? (remaining > 16 ? (int)(remaining - 16) : 0) : 16;
        for (int j = 0; j < half; j++) out[dst + j] = scale * kIq4nl[q[src + j] & 0x0F];
        for (int j = 0; j < second; j++) out[dst + 16 + j] = scale * kIq4nl[(q[src + j] >> 4) & 0x0F];
        src += 16;
        dst += half + second;
    }
}

// DequantIQ.IQ4XS.Dequantize (DequantIQ.cs:143-180): per 32-element sub-block
// sc = ((byte[4 + sub] & 63) | ((scales_h >> 2 sub) & 3) << 6) - 32 (scales_h
// the uint16 at 2; the scale bytes 4..11 overlap the first quant bytes, as
// in the reference), value = d * sc * table[nibble] (qs@8).
static void dequant_iq4_xs(const uint8_t* q, float* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 136;
        const float d = h2f(blk);
        const int sh = blk[2] | (blk[3] << 8);
        for (int sub = 0; sub < 8; sub++) {
            const int sc = ((blk[4 + sub] & 0x3F) | (((sh >> (2 * sub)) & 3) << 6)) - 32;
            const float dsc = d * (float)sc;
            for (int j = 0; j < 16; j++) {
                const uint8_t v = blk[8 + sub * 16 + j];
                out[b * 256 + sub * 32 + j] = dsc * kIq4nl[v & 0x0F];
                out[b * 256 + sub * 32 + j + 16] = dsc * kIq4nl[(v >> 4) & 0x0F];
            }
        }
    }
}

// ---- the importance-quantised types, as the reference decodes them ---------
//
// DequantIQ.cs restates these without codebook grids (its own simplified
// layouts).  IQ3_S reads its sign bytes at 98 + sub and its scale bytes at
// 130 + sub/4 from the block start, past the 110-byte block: inside a tensor
// those are the next block's bytes (the pointer-based DotProduct reads them
// there; the span-based Dequantize throws for the last block of its span).
// Here every such read goes through iq3s_byte, which returns the byte when
// it lies before `end` and 0 past it.
static inline uint8_t iq3s_byte(const uint8_t* blk, int k, const uint8_t* end) {
    return blk + k < end ? blk[k] : 0;
}

// DequantIQ.IQ3S.Dequantize (DequantIQ.cs:244-290).
static void dequant_iq3_s(const uint8_t* q, float* out, int64_t n, const uint8_t* end) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 110;
        const float d = h2f(blk);
        for (int sub = 0; sub < 32; sub++) {
            const int sc = ((iq3s_byte(blk, 130 + sub / 4, end) >> ((sub % 4) * 2)) & 3) + 1;
            const float dsc = d * (float)sc;
            const uint8_t sign = iq3s_byte(blk, 98 + sub, end);
            for (int j = 0; j < 8; j++) {
                const int idx = sub * 8 + j;
                const int q2 = (blk[2 + idx / 4] >> ((idx % 4) * 2)) & 3;
                const int qh = (blk[66 + idx / 8] >> (idx % 8)) & 1;
                float v = dsc * (float)(q2 | (qh << 2));
                if ((sign >> j) & 1) v = -v;
                out[b * 256 + idx] = v;
            }
        }
    }
}

// DequantIQ.IQ3XXS.Dequantize (DequantIQ.cs:364-398).
static void dequant_iq3_xxs(const uint8_t* q, float* out, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * 98;
        const float d = h2f(blk);
        for (int sub = 0; sub < 32; sub++) {
            const uint8_t* g = blk + 2 + sub * 3;
            const uint32_t packed = (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16);
            for (int j = 0; j < 8; j++) out[b * 256 + sub * 8 + j] = d * (float)((int)((packed >> (j * 3)) & 7) - 4);
        }
    }
}

// DequantIQ.IQ2XS / IQ2XXS / IQ2S.Dequantize (DequantIQ.cs:456-495, :568-597,
// :656-695): 16 sub-blocks of 16, four 2-bit quants per byte.
static void dequant_iq2(int type, const uint8_t* q, float* out, int64_t n) {
    const int bpb = type == OR_IQ2_XS ? 74 : type == OR_IQ2_XXS ? 66 : 82;
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * bpb;
        const float d = h2f(blk);
        for (int sub = 0; sub < 16; sub++) {
            float dsc = d;
            int sign = 0;
            if (type == OR_IQ2_XS) {
                const int raw = (int8_t)blk[66 + sub / 2];
                const int sc = (sub & 1) == 0 ? (raw & 0x0F) - 8 : ((raw >> 4) & 0x0F) - 8;
                dsc = d * (float)sc;
            } else if (type == OR_IQ2_S) {
                const uint8_t qh = blk[66 + sub];
                dsc = d * (float)((qh & 0x0F) + 1);
                sign = (qh >> 4) & 0x0F;
            }
            for (int j = 0; j < 4; j++) {
                const uint8_t byte = blk[2 + sub * 4 + j];
                for (int k = 0; k < 4; k++) {
                    const int qv = (byte >> (k * 2)) & 3;
                    const int e = j * 4 + k;
                    float v;
                    if (type == OR_IQ2_S) {
                        v = dsc * (float)qv;
                        if (e < 4 && ((sign >> e) & 1)) v = -v;
                    } else {
                        v = dsc * (float)(qv - 1);
                    }
                    out[b * 256 + sub * 16 + e] = v;
                }
            }
        }
    }
}

// DequantIQ.IQ1S / IQ1M.Dequantize (DequantIQ.cs:767-805, :869-912): per
// element d (or d * sc), -d (-d * sc) or 0 from a qs bit and a qh bit.
static void dequant_iq1(int type, const uint8_t* q, float* out, int64_t n) {
    const int bpb = type == OR_IQ1_S ? 50 : 56;
    for (int64_t b = 0; b < n / 256; b++) {
        const uint8_t* blk = q + b * bpb;
        const float d = h2f(blk);
        for (int sub = 0; sub < 32; sub++) {
            float sc = 1.0f;
            if (type == OR_IQ1_M && sub / 8 < 6) sc = ((blk[50 + sub / 8] >> (sub % 8)) & 1) == 1 ? 1.0f : 0.5f;
            const uint8_t qs = blk[2 + sub];
            for (int j = 0; j < 8; j++) {
                const int bit = (qs >> j) & 1;
                const int hbit = (blk[34 + sub / 2] >> ((sub % 2) * 4 + j / 2)) & 1;
                float v;
                if (type == OR_IQ1_S) v = bit ? d : hbit ? -d : 0.0f;
                else v = bit ? d * sc : hbit ? -d * sc : 0.0f;
                out[b * 256 + sub * 8 + j] = v;
            }
        }
    }
}

extern "C" int or_dequantize(int type, const uint8_t* src, float* dst, int64_t n) {
    if (n < 0) return -1;
    switch (type) {
        case OR_Q4_0: dequant_q4_0(src, dst, n); return 0;
        case OR_Q8_0: dequant_q8_0(src, dst, n); return 0;
        case OR_Q4_1:
        case OR_Q5_0:
        case OR_Q5_1: dequant_b32(type, src, dst, n); return 0;
        case OR_Q4_K: dequant_q4_k(src, dst, n); return 0;
        case OR_Q6_K: dequant_q6_k(src, dst, n); return 0;
        case OR_Q2_K: dequant_q2_k(src, dst, n); return 0;
        case OR_Q3_K: dequant_q3_k(src, dst, n); return 0;
        case OR_Q5_K: dequant_q5_k(src, dst, n); return 0;
        case OR_Q8_K: dequant_q8_k(src, dst, n); return 0;
        case OR_IQ4_NL: dequant_iq4_nl(src, dst, n); return 0;
        case OR_IQ4_XS: dequant_iq4_xs(src, dst, n); return 0;
        case OR_IQ3_S: dequant_iq3_s(src, dst, n, src + n / 256 * 110); return 0;
        case OR_IQ3_XXS: dequant_iq3_xxs(src, dst, n); return 0;
        case OR_IQ2_XS:
        case OR_IQ2_XXS:
        case OR_IQ2_S: dequant_iq2(type, src, dst, n); return 0;
        case OR_IQ1_S:
        case OR_IQ1_M: dequant_iq1(type, src, dst, n); return 0;
        case OR_F32: memcpy(dst, src, (size_t)n * 4); return 0;
        case OR_F16:
            for (int64_t i = 0; i < n; i++) dst[i] = h2f(src + 2 * i);
            return 0;
        default: return -2;
    }
}

// ---------------------------------------------------------------------------
// Fused dequant-dot products (the Vector128 paths)
// ---------------------------------------------------------------------------

static inline float sum128(__m128 v) {
    // Vector128.Sum: Sum(lower) + Sum(upper) = (v0 + v1) + (v2 + v3)
    float t[4];
    _mm_storeu_ps(t, v);
    return (t[0] + t[1]) + (t[2] + t[3]);
}

// 4 bytes starting at byte `off` of v, zero-extended to int32 lanes.
static inline __m128i widen4(__m128i v, int off) {
    switch (off) {
        case 0: return _mm_cvtepu8_epi32(v);
        case 4: return _mm_cvtepu8_epi32(_mm_srli_si128(v, 4));
        case 8: return _mm_cvtepu8_epi32(_mm_srli_si128(v, 8));
        default: return _mm_cvtepu8_epi32(_mm_srli_si128(v, 12));
    }
}

// DequantQ4_0.DotProductVec128 (DequantQ4_0.cs:80-149).
static float dot_q4_0(const uint8_t* src, const float* inp, int n) {
    int nb = n / 32;
    __m128 acc0 = _mm_setzero_ps(), acc1 = _mm_setzero_ps();
    const __m128i mask = _mm_set1_epi8(0x0F);
    const __m128i sub8 = _mm_set1_epi32(8);
    for (int b = 0; b < nb; b++) {
        float scale = h2f(src);
        src += 2;
        __m128 vs = _mm_set1_ps(scale);
        __m128i raw = _mm_loadu_si128((const __m128i*)src);
        __m128i lo = _mm_and_si128(raw, mask);
        __m128i hi = _mm_and_si128(_mm_srli_epi16(raw, 4), mask);
        __m128 b0 = _mm_setzero_ps(), b1 = _mm_setzero_ps();
        __m128 lf0 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(lo, 0), sub8));
        __m128 lf1 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(lo, 4), sub8));
        __m128 lf2 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(lo, 8), sub8));
        __m128 lf3 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(lo, 12), sub8));
        b0 = _mm_add_ps(b0, _mm_mul_ps(lf0, _mm_loadu_ps(inp + 0)));
        b1 = _mm_add_ps(b1, _mm_mul_ps(lf1, _mm_loadu_ps(inp + 4)));
        b0 = _mm_add_ps(b0, _mm_mul_ps(lf2, _mm_loadu_ps(inp + 8)));
        b1 = _mm_add_ps(b1, _mm_mul_ps(lf3, _mm_loadu_ps(inp + 12)));
        __m128 hf0 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(hi, 0), sub8));
        __m128 hf1 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(hi, 4), sub8));
        __m128 hf2 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(hi, 8), sub8));
        __m128 hf3 = _mm_cvtepi32_ps(_mm_sub_epi32(widen4(hi, 12), sub8));
        b0 = _mm_add_ps(b0, _mm_mul_ps(hf0, _mm_loadu_ps(inp + 16)));
        b1 = _mm_add_ps(b1, _mm_mul_ps(hf1, _mm_loadu_ps(inp + 20)));
        b0 = _mm_add_ps(b0, _mm_mul_ps(hf2, _mm_loadu_ps(inp + 24)));
        b1 = _mm_add_ps(b1, _mm_mul_ps(hf3, _mm_loadu_ps(inp + 28)));
        acc0 = _mm_add_ps(acc0, _mm_mul_ps(b0, vs));
        acc1 = _mm_add_ps(acc1, _mm_mul_ps(b1, vs));
        src += 16;
        inp += 32;
    }
    return sum128(_mm_add_ps(acc0, acc1));
}

// DequantQ4K.DotProductVec128 (DequantQ4K.cs:89-163).
static float dot_q4_k(const uint8_t* data, const float* input, int n) {
    int nb = n / 256;
    __m128 acc = _mm_setzero_ps();
    const __m128i mask = _mm_set1_epi8(0x0F);
    int sc[8], m[8];
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = data + (size_t)b * 144;
        float d = h2f(blk);
        float dmin = h2f(blk + 2);
        decode_scales_q4k(blk + 4, sc, m);
        __m128 bacc = _mm_setzero_ps();
        const float* in = input + (size_t)b * 256;
        for (int sub = 0; sub < 8; sub++) {
            __m128 vdsc = _mm_set1_ps(d * (float)sc[sub]);
            __m128 vdm = _mm_set1_ps(dmin * (float)m[sub]);
            __m128i raw = _mm_loadu_si128((const __m128i*)(blk + 16 + sub * 16));
            __m128i lo = _mm_and_si128(raw, mask);
            __m128i hi = _mm_and_si128(_mm_srli_epi16(raw, 4), mask);
            const float* xi = in + sub * 32;
            for (int g = 0; g < 4; g++) {
                __m128 lf = _mm_cvtepi32_ps(widen4(lo, 4 * g));
                __m128 w = _mm_sub_ps(_mm_mul_ps(lf, vdsc), vdm);
                bacc = _mm_add_ps(bacc, _mm_mul_ps(w, _mm_loadu_ps(xi + 4 * g)));
            }
            for (int g = 0; g < 4; g++) {
                __m128 hf = _mm_cvtepi32_ps(widen4(hi, 4 * g));
                __m128 w = _mm_sub_ps(_mm_mul_ps(hf, vdsc), vdm);
                bacc = _mm_add_ps(bacc, _mm_mul_ps(w, _mm_loadu_ps(xi + 16 + 4 * g)));
            }
        }
        acc = _mm_add_ps(acc, bacc);
    }
    return sum128(acc);
}

// DequantQ6K.DotProductVec128 (DequantQ6K.cs:104-188).
static float dot_q6_k(const uint8_t* data, const float* input, int n) {
    int nb = n / 256;
    __m128 acc = _mm_setzero_ps();
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = data + (size_t)b * 210;
        float d = h2f(blk + 208);
        __m128 bacc = _mm_setzero_ps();
        for (int half = 0; half < 2; half++) {
            const uint8_t* ql = blk + half * 64;
            const uint8_t* qh = blk + 128 + half * 32;
            const int8_t* scs = (const int8_t*)(blk + 192);
            int sc_off = half * 8;
            const float* in = input + (size_t)b * 256 + half * 128;
            for (int lb = 0; lb < 2; lb++) {
                int ls = lb * 16;
                int si = sc_off + lb;
                __m128 s0 = _mm_set1_ps((float)scs[si]);
                __m128 s2 = _mm_set1_ps((float)scs[si + 2]);
                __m128 s4 = _mm_set1_ps((float)scs[si + 4]);
                __m128 s6 = _mm_set1_ps((float)scs[si + 6]);
                for (int l = ls; l < ls + 16; l += 4) {
                    float a1[4], a2[4], a3[4], a4[4];
                    for (int t = 0; t < 4; t++) {
                        int i = l + t;
                        a1[t] = (float)(((ql[i] & 0xF) | (((qh[i] >> 0) & 3) << 4)) - 32);
                        a2[t] = (float)(((ql[i + 32] & 0xF) | (((qh[i] >> 2) & 3) << 4)) - 32);
                        a3[t] = (float)(((ql[i] >> 4) | (((qh[i] >> 4) & 3) << 4)) - 32);
                        a4[t] = (float)(((ql[i + 32] >> 4) | (((qh[i] >> 6) & 3) << 4)) - 32);
                    }
                    bacc = _mm_add_ps(bacc, _mm_mul_ps(_mm_mul_ps(_mm_loadu_ps(a1), s0), _mm_loadu_ps(in + l)));
                    bacc = _mm_add_ps(bacc, _mm_mul_ps(_mm_mul_ps(_mm_loadu_ps(a2), s2), _mm_loadu_ps(in + l + 32)));
                    bacc = _mm_add_ps(bacc, _mm_mul_ps(_mm_mul_ps(_mm_loadu_ps(a3), s4), _mm_loadu_ps(in + l + 64)));
                    bacc = _mm_add_ps(bacc, _mm_mul_ps(_mm_mul_ps(_mm_loadu_ps(a4), s6), _mm_loadu_ps(in + l + 96)));
                }
            }
        }
        acc = _mm_add_ps(acc, _mm_mul_ps(bacc, _mm_set1_ps(d)));
    }
    return sum128(acc);
}

// Vector<float> is 8 lanes here; VectorSum adds lanes in order
// (TensorMath.cs:750-758).
static inline float vsum8(const float* v) {
    float s = 0.f;
    for (int i = 0; i < 8; i++) s += v[i];
    return s;
}

// TensorMath.DotProductSimd (TensorMath.cs:666-702).
static float dot_f32(const float* a, const float* b, int length) {
    float sum = 0.f;
    int i = 0;
    float v0[8] = {0}, v1[8] = {0};
    int limit2 = length - 16 + 1;
    for (; i < limit2; i += 16)
        for (int k = 0; k < 8; k++) {
            v0[k] += a[i + k] * b[i + k];
            v1[k] += a[i + 8 + k] * b[i + 8 + k];
        }
    int limit1 = length - 8 + 1;
    for (; i < limit1; i += 8)
        for (int k = 0; k < 8; k++) v0[k] += a[i + k] * b[i + k];
    float t[8];
    for (int k = 0; k < 8; k++) t[k] = v0[k] + v1[k];
    sum = vsum8(t);
    for (; i < length; i++) sum += a[i] * b[i];
    return sum;
}

// DequantQ8_0.DotProductScalar (DequantQ8_0.cs:94-119): per block, sum of
// (sbyte)q * x in order, then sum += blockSum * d.
static float dot_q8_0(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    for (int b = 0; b < n / 32; b++) {
        const uint8_t* blk = row + (size_t)b * 34;
        float scale = h2f(blk), bs = 0.f;
        for (int i = 0; i < 32; i++) bs += (float)(int8_t)blk[2 + i] * x[32 * b + i];
        sum += bs * scale;
    }
    return sum;
}

// DequantQ4_1.DotProductScalar (DequantQ4_1.cs:134-171),
// DequantQ5_0.DotProductScalar (DequantQ5_0.cs:77-114),
// DequantQ5_1.DotProductScalar (DequantQ5_1.cs:78-119): per block, the low
// then the high half, sum += blockSum * d (+ inputSum * m for Q4_1 / Q5_1).
static float dot_b32(int type, const uint8_t* row, const float* x, int n) {
    const int bpb = type == OR_Q4_1 ? 20 : type == OR_Q5_0 ? 22 : 24;
    const int qs_off = type == OR_Q4_1 ? 4 : type == OR_Q5_0 ? 6 : 8;
    const int qh_off = type == OR_Q5_0 ? 2 : 4;
    float sum = 0.f;
    for (int b = 0; b < n / 32; b++) {
        const uint8_t* blk = row + (size_t)b * bpb;
        const float* xb = x + 32 * b;
        float scale = h2f(blk);
        float min = type == OR_Q5_0 ? 0.f : h2f(blk + 2);
        uint32_t qh = 0;
        if (type != OR_Q4_1)
            qh = (uint32_t)blk[qh_off] | ((uint32_t)blk[qh_off + 1] << 8) | ((uint32_t)blk[qh_off + 2] << 16) |
                 ((uint32_t)blk[qh_off + 3] << 24);
        float bs = 0.f, is = 0.f;
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++) {
                int idx = 16 * h + j;
                int nib = h == 0 ? (blk[qs_off + j] & 0x0F) : ((blk[qs_off + j] >> 4) & 0x0F);
                int q = type == OR_Q4_1 ? nib : (nib | (int)((qh >> idx) & 1u) << 4);
                if (type == OR_Q5_0) q -= 16;
                bs += (float)q * xb[idx];
                if (type != OR_Q5_0) is += xb[idx];
            }
        sum += type == OR_Q5_0 ? bs * scale : bs * scale + is * min;
    }
    return sum;
}

// LlamaModel.MatVecMulF16 row (LlamaModel.cs:570-598): scalar, in order.
static float dot_f16(const uint8_t* row, const float* x, int n) {
    float dot = 0.f;
    for (int i = 0; i < n; i++) dot += h2f(row + 2 * i) * x[i];
    return dot;
}

// DequantQ2K.DotProductScalar (DequantQ2K.cs:96-155): blockSum += (dl * q - ml) * x.
static float dot_q2_k(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 84;
        const float d = h2f(blk + 80), dmin = h2f(blk + 82);
        const float* in = x + 256 * b;
        float bs = 0.f;
        int si = 0, y = 0;
        for (int g = 0; g < 2; g++)
            for (int shift = 0; shift < 8; shift += 2) {
                for (int h = 0; h < 2; h++) {
                    const float dl = d * (float)(blk[si + h] & 0x0F);
                    const float ml = dmin * (float)((blk[si + h] >> 4) & 0x0F);
                    for (int l = 0; l < 16; l++)
                        bs += (dl * (float)((blk[16 + 32 * g + 16 * h + l] >> shift) & 3) - ml) * in[y++];
                }
                si += 2;
            }
        sum += bs;
    }
    return sum;
}

// DequantQ3K.DotProductScalar (DequantQ3K.cs:79-118): integer scale * (q3 - 4),
// times x, summed per super-block, then sum += d * blockSum.
static float dot_q3_k(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    int sc[16];
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 110;
        const float d = h2f(blk + 108);
        decode_scales_q3k(blk + 96, sc);
        float bs = 0.f;
        for (int i = 0; i < 256; i++) {
            const int q2 = (blk[32 + i / 4] >> ((i % 4) * 2)) & 3;
            const int q3 = q2 | (((blk[i / 8] >> (i % 8)) & 1) << 2);
            bs += (float)(sc[i / 16] * (q3 - 4)) * x[256 * b + i];
        }
        sum += d * bs;
    }
    return sum;
}

// DequantQ5K.DotProductScalar (DequantQ5K.cs:99-154): blockSum += (dsc * q5 - dm) * x.
static float dot_q5_k(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    int sc[8], m[8];
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 176;
        const float d = h2f(blk), dmin = h2f(blk + 2);
        decode_scales_q4k(blk + 4, sc, m);
        float bs = 0.f;
        for (int sub = 0; sub < 8; sub++) {
            const float dsc = d * (float)sc[sub], dm = dmin * (float)m[sub];
            for (int h = 0; h < 2; h++)
                for (int j = 0; j < 16; j++) {
                    const int e = sub * 32 + 16 * h + j;
                    const int nib = h == 0 ? (blk[48 + sub * 16 + j] & 0x0F) : ((blk[48 + sub * 16 + j] >> 4) & 0x0F);
                    const int q5 = nib | (((blk[16 + e / 8] >> (e % 8)) & 1) << 4);
                    bs += (dsc * (float)q5 - dm) * x[256 * b + e];
                }
        }
        sum += bs;
    }
    return sum;
}

// DequantQ8K.DotProductVec128 (DequantQ8K.cs:58-96): two 4-lane accumulators
// of (q * d) * x over the row, then Vector128.Sum(acc0 + acc1).
static float dot_q8_k(const uint8_t* row, const float* x, int n) {
    __m128 acc0 = _mm_setzero_ps(), acc1 = _mm_setzero_ps();
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 292;
        const __m128 vs = _mm_set1_ps(f32_le(blk));
        const float* in = x + 256 * b;
        for (int i = 0; i < 256; i += 8) {
            const __m128 v0 = _mm_setr_ps((float)(int8_t)blk[4 + i], (float)(int8_t)blk[5 + i],
                                          (float)(int8_t)blk[6 + i], (float)(int8_t)blk[7 + i]);
            const __m128 v1 = _mm_setr_ps((float)(int8_t)blk[8 + i], (float)(int8_t)blk[9 + i],
                                          (float)(int8_t)blk[10 + i], (float)(int8_t)blk[11 + i]);
            acc0 = _mm_add_ps(acc0, _mm_mul_ps(_mm_mul_ps(v0, vs), _mm_loadu_ps(in + i)));
            acc1 = _mm_add_ps(acc1, _mm_mul_ps(_mm_mul_ps(v1, vs), _mm_loadu_ps(in + i + 4)));
        }
    }
    return sum128(_mm_add_ps(acc0, acc1));
}

// DequantIQ.IQ4NL.DotProductScalar (DequantIQ.cs:85-118): per block, the low
// then the high nibbles' table values times x, then sum += blockSum * scale.
static float dot_iq4_nl(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    for (int b = 0; b < n / 32; b++) {
        const uint8_t* blk = row + (size_t)b * 18;
        const float scale = h2f(blk);
        float bs = 0.f;
        for (int j = 0; j < 16; j++) bs += kIq4nl[blk[2 + j] & 0x0F] * x[32 * b + j];
        for (int j = 0; j < 16; j++) bs += kIq4nl[(blk[2 + j] >> 4) & 0x0F] * x[32 * b + 16 + j];
        sum += bs * scale;
    }
    return sum;
}

// DequantIQ.IQ4XS.DotProductScalar (DequantIQ.cs:189-233): per sub-block the
// low and high nibble of each byte in turn, blockSum += dsc * subSum.
static float dot_iq4_xs(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 136;
        const float d = h2f(blk);
        const int sh = blk[2] | (blk[3] << 8);
        float bs = 0.f;
        for (int sub = 0; sub < 8; sub++) {
            const int sc = ((blk[4 + sub] & 0x3F) | (((sh >> (2 * sub)) & 3) << 6)) - 32;
            const float dsc = d * (float)sc;
            const float* in = x + 256 * b + 32 * sub;
            float ss = 0.f;
            for (int j = 0; j < 16; j++) {
                const uint8_t v = blk[8 + sub * 16 + j];
                ss += kIq4nl[v & 0x0F] * in[j];
                ss += kIq4nl[(v >> 4) & 0x0F] * in[j + 16];
            }
            bs += dsc * ss;
        }
        sum += bs;
    }
    return sum;
}

// DequantIQ.IQ3S.DotProductScalar (DequantIQ.cs:299-349): per sub-block
// subSum += (+-q3) * x, blockSum += dsc * subSum, sum += blockSum; sign and
// scale bytes past the block as in dequant_iq3_s (`end` bounds the reads).
static float dot_iq3_s(const uint8_t* row, const float* x, int n, const uint8_t* end) {
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 110;
        const float d = h2f(blk);
        float bs = 0.f;
        for (int sub = 0; sub < 32; sub++) {
            const int sc = ((iq3s_byte(blk, 130 + sub / 4, end) >> ((sub % 4) * 2)) & 3) + 1;
            const float dsc = d * (float)sc;
            const uint8_t sign = iq3s_byte(blk, 98 + sub, end);
            float ss = 0.f;
            for (int j = 0; j < 8; j++) {
                const int idx = sub * 8 + j;
                const int q3 = ((blk[2 + idx / 4] >> ((idx % 4) * 2)) & 3) | (((blk[66 + idx / 8] >> (idx % 8)) & 1) << 2);
                float v = (float)q3;
                if ((sign >> j) & 1) v = -v;
                ss += v * x[256 * b + idx];
            }
            bs += dsc * ss;
        }
        sum += bs;
    }
    return sum;
}

// DequantIQ.IQ3XXS.DotProductScalar (DequantIQ.cs:407-440): blockSum +=
// (q3 - 4) * x over the block, sum += d * blockSum.
static float dot_iq3_xxs(const uint8_t* row, const float* x, int n) {
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * 98;
        const float d = h2f(blk);
        float bs = 0.f;
        for (int sub = 0; sub < 32; sub++) {
            const uint8_t* g = blk + 2 + sub * 3;
            const uint32_t packed = (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16);
            for (int j = 0; j < 8; j++) bs += (float)((int)((packed >> (j * 3)) & 7) - 4) * x[256 * b + sub * 8 + j];
        }
        sum += d * bs;
    }
    return sum;
}

// DequantIQ.IQ2XS / IQ2S.DotProductScalar (DequantIQ.cs:505-553, :705-752):
// per sub-block subSum, blockSum += dsc * subSum; IQ2XXS (:607-640):
// blockSum += (q - 1) * x over the block, sum += d * blockSum.
static float dot_iq2(int type, const uint8_t* row, const float* x, int n) {
    const int bpb = type == OR_IQ2_XS ? 74 : type == OR_IQ2_XXS ? 66 : 82;
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * bpb;
        const float d = h2f(blk);
        float bs = 0.f;
        for (int sub = 0; sub < 16; sub++) {
            const float* in = x + 256 * b + 16 * sub;
            if (type == OR_IQ2_XXS) {
                for (int j = 0; j < 4; j++) {
                    const uint8_t byte = blk[2 + sub * 4 + j];
                    for (int k = 0; k < 4; k++) bs += (float)(((byte >> (2 * k)) & 3) - 1) * in[j * 4 + k];
                }
                continue;
            }
            float dsc;
            int sign = 0;
            if (type == OR_IQ2_XS) {
                const int raw = (int8_t)blk[66 + sub / 2];
                dsc = d * (float)((sub & 1) == 0 ? (raw & 0x0F) - 8 : ((raw >> 4) & 0x0F) - 8);
            } else {
                const uint8_t qh = blk[66 + sub];
                dsc = d * (float)((qh & 0x0F) + 1);
                sign = (qh >> 4) & 0x0F;
            }
            float ss = 0.f;
            for (int j = 0; j < 4; j++) {
                const uint8_t byte = blk[2 + sub * 4 + j];
                for (int k = 0; k < 4; k++) {
                    const int qv = (byte >> (2 * k)) & 3, e = j * 4 + k;
                    if (type == OR_IQ2_XS) {
                        ss += (float)(qv - 1) * in[e];
                    } else {
                        float v = (float)qv;
                        if (e < 4 && ((sign >> e) & 1)) v = -v;
                        ss += v * in[e];
                    }
                }
            }
            bs += dsc * ss;
        }
        sum += type == OR_IQ2_XXS ? d * bs : bs;
    }
    return sum;
}

// DequantIQ.IQ1S / IQ1M.DotProductScalar (DequantIQ.cs:814-856, :923-971):
// blockSum += weight * x (weight 1 / -1 / 0, times sc for IQ1M), sum += d * blockSum.
static float dot_iq1(int type, const uint8_t* row, const float* x, int n) {
    const int bpb = type == OR_IQ1_S ? 50 : 56;
    float sum = 0.f;
    for (int b = 0; b < n / 256; b++) {
        const uint8_t* blk = row + (size_t)b * bpb;
        const float d = h2f(blk);
        float bs = 0.f;
        for (int sub = 0; sub < 32; sub++) {
            float sc = 1.0f;
            if (type == OR_IQ1_M && sub / 8 < 6) sc = ((blk[50 + sub / 8] >> (sub % 8)) & 1) == 1 ? 1.0f : 0.5f;
            const uint8_t qs = blk[2 + sub];
            for (int j = 0; j < 8; j++) {
                const int bit = (qs >> j) & 1;
                const int hbit = (blk[34 + sub / 2] >> ((sub % 2) * 4 + j / 2)) & 1;
                const float w = bit ? sc : hbit ? -sc : 0.0f;
                bs += w * x[256 * b + sub * 8 + j];
            }
        }
        sum += d * bs;
    }
    return sum;
}

extern "C" float or_dot(int type, const uint8_t* row, const float* x, int n) {
    switch (type) {
        case OR_Q4_0: return dot_q4_0(row, x, n);
        case OR_Q8_0: return dot_q8_0(row, x, n);
        case OR_Q4_1:
        case OR_Q5_0:
        case OR_Q5_1: return dot_b32(type, row, x, n);
        case OR_Q4_K: return dot_q4_k(row, x, n);
        case OR_Q6_K: return dot_q6_k(row, x, n);
        case OR_Q2_K: return dot_q2_k(row, x, n);
        case OR_Q3_K: return dot_q3_k(row, x, n);
        case OR_Q5_K: return dot_q5_k(row, x, n);
        case OR_Q8_K: return dot_q8_k(row, x, n);
        case OR_IQ4_NL: return dot_iq4_nl(row, x, n);
        case OR_IQ4_XS: return dot_iq4_xs(row, x, n);
        case OR_IQ3_S: return dot_iq3_s(row, x, n, row + (size_t)(n / 256) * 110);
        case OR_IQ3_XXS: return dot_iq3_xxs(row, x, n);
        case OR_IQ2_XS:
        case OR_IQ2_XXS:
        case OR_IQ2_S: return dot_iq2(type, row, x, n);
        case OR_IQ1_S:
        case OR_IQ1_M: return dot_iq1(type, row, x, n);
        case OR_F32: return dot_f32((const float*)row, x, n);
        case OR_F16: return dot_f16(row, x, n);
        default: return NAN;
    }
}

// ---------------------------------------------------------------------------
// MatVecMul (TensorMath.cs:548-656) with the Parallel.For row split
// ---------------------------------------------------------------------------

static int hw_threads(int nthreads) {
    if (nthreads > 0) return nthreads;
    unsigned h = std::thread::hardware_concurrency();
    return h ? (int)h : 1;
}

template <class F>
static void parallel_rows(int rows, int nthreads, F&& body) {
    nthreads = std::min(nthreads, rows);
    if (nthreads <= 1) {
        for (int r = 0; r < rows; r++) body(r);
        return;
    }
    // dynamic row chunks, like Parallel.For's range partitioning
    std::atomic<int> next{0};
    const int chunk = 16;
    auto worker = [&]() {
        for (;;) {
            int r0 = next.fetch_add(chunk);
            if (r0 >= rows) break;
            int r1 = std::min(rows, r0 + chunk);
            for (int r = r0; r < r1; r++) body(r);
        }
    };
    std::vector<std::thread> ts;
    for (int t = 1; t < nthreads; t++) ts.emplace_back(worker);
    worker();
    for (auto& t : ts) t.join();
}

static int row_bytes(int type, int in_dim, size_t* bpr) {
    switch (type) {
        case OR_Q4_0: *bpr = (size_t)(in_dim / 32) * 18; return 0;
        case OR_Q4_1: *bpr = (size_t)(in_dim / 32) * 20; return 0;
        case OR_Q5_0: *bpr = (size_t)(in_dim / 32) * 22; return 0;
        case OR_Q5_1: *bpr = (size_t)(in_dim / 32) * 24; return 0;
        case OR_Q8_0: *bpr = (size_t)(in_dim / 32) * 34; return 0;
        case OR_Q4_K: *bpr = (size_t)(in_dim / 256) * 144; return 0;
        case OR_Q6_K: *bpr = (size_t)(in_dim / 256) * 210; return 0;
        case OR_Q2_K: *bpr = (size_t)(in_dim / 256) * 84; return 0;
        case OR_Q3_K: *bpr = (size_t)(in_dim / 256) * 110; return 0;
        case OR_Q5_K: *bpr = (size_t)(in_dim / 256) * 176; return 0;
        case OR_Q8_K: *bpr = (size_t)(in_dim / 256) * 292; return 0;
        case OR_IQ4_NL: *bpr = (size_t)(in_dim / 32) * 18; return 0;
        case OR_IQ4_XS: *bpr = (size_t)(in_dim / 256) * 136; return 0;
        case OR_IQ3_S: *bpr = (size_t)(in_dim / 256) * 110; return 0;
        case OR_IQ3_XXS: *bpr = (size_t)(in_dim / 256) * 98; return 0;
        case OR_IQ2_XS: *bpr = (size_t)(in_dim / 256) * 74; return 0;
        case OR_IQ2_XXS: *bpr = (size_t)(in_dim / 256) * 66; return 0;
        case OR_IQ2_S: *bpr = (size_t)(in_dim / 256) * 82; return 0;
        case OR_IQ1_S: *bpr = (size_t)(in_dim / 256) * 50; return 0;
        case OR_IQ1_M: *bpr = (size_t)(in_dim / 256) * 56; return 0;
        case OR_F32: *bpr = (size_t)in_dim * 4; return 0;
        case OR_F16: *bpr = (size_t)in_dim * 2; return 0;
        default: return -2;
    }
}

extern "C" int or_matvec(int type, const uint8_t* W, const float* x, float* y,
                         int out_dim, int in_dim, int nthreads) {
    size_t bpr;
    if (row_bytes(type, in_dim, &bpr)) return -2;
    // IQ3_S: the pointer-based dot reads past a row into the next one (and
    // past the matrix reads 0), see dequant_iq3_s
    const uint8_t* end = W + (size_t)out_dim * bpr;
    auto body = [&](int r) {
        y[r] = type == OR_IQ3_S ? dot_iq3_s(W + (size_t)r * bpr, x, in_dim, end)
                                : or_dot(type, W + (size_t)r * bpr, x, in_dim);
    };
    // ParallelRowThreshold = 512 (TensorMath.cs:28); MatVecMul (F32) and
    // MatVecMulF16 are sequential in the reference.
    bool par = out_dim >= 512 && type != OR_F32 && type != OR_F16;
    parallel_rows(out_dim, par ? hw_threads(nthreads) : 1, body);
    return 0;
}

extern "C" int or_matvec_batch(int type, const uint8_t* W, const float* x, float* y,
                               int out_dim, int in_dim, int batch, int nthreads) {
    for (int b = 0; b < batch; b++) {
        int rc = or_matvec(type, W, x + (size_t)b * in_dim, y + (size_t)b * out_dim,
                           out_dim, in_dim, nthreads);
        if (rc) return rc;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Elementwise ops
// ---------------------------------------------------------------------------

// TensorMath.RmsNorm (TensorMath.cs:97-165).
extern "C" void or_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
    float sumsq = 0.f;
    int i = 0;
    if (n >= 8) {
        float a0[8] = {0}, a1[8] = {0};
        int limit2 = n - 16 + 1;
        for (; i < limit2; i += 16)
            for (int k = 0; k < 8; k++) {
                a0[k] += x[i + k] * x[i + k];
                a1[k] += x[i + 8 + k] * x[i + 8 + k];
            }
        int limit1 = n - 8 + 1;
        for (; i < limit1; i += 8)
            for (int k = 0; k < 8; k++) a0[k] += x[i + k] * x[i + k];
        float t[8];
        for (int k = 0; k < 8; k++) t[k] = a0[k] + a1[k];
        sumsq = vsum8(t);
    }
    for (; i < n; i++) sumsq += x[i] * x[i];
    float rms = 1.0f / sqrtf(sumsq / (float)n + eps);
    for (i = 0; i < n; i++) y[i] = x[i] * rms * w[i];
}

// TensorMath.Softmax (TensorMath.cs:177-241).
extern "C" void or_softmax(float* data, int length) {
    float mx = -INFINITY;
    int i = 0;
    if (length >= 8) {
        float vm[8];
        for (int k = 0; k < 8; k++) vm[k] = -INFINITY;
        int limit = length - 8 + 1;
        for (; i < limit; i += 8)
            for (int k = 0; k < 8; k++) vm[k] = std::max(vm[k], data[i + k]);
        for (int k = 0; k < 8; k++)
            if (vm[k] > mx) mx = vm[k];
    }
    for (; i < length; i++)
        if (data[i] > mx) mx = data[i];
    float sum = 0.f;
    for (i = 0; i < length; i++) {
        float v = expf(data[i] - mx);
        data[i] = v;
        sum += v;
    }
    if (sum > 0.f) {
        float inv = 1.0f / sum;
        for (i = 0; i < length; i++) data[i] *= inv;
    }
}

// TensorMath.SiluElementwiseMul (TensorMath.cs:253-286).
extern "C" void or_silu_mul(float* gate, const float* up, int length) {
    for (int i = 0; i < length; i++) {
        float x = gate[i];
        float s = x / (1.0f + expf(-x));
        gate[i] = s * up[i];
    }
}

// TensorMath.ApplyRoPE (TensorMath.cs:408-458), interleaved pairs, full
// rotary dimension.
extern "C" void or_rope(float* q, float* k, int pos, int head_dim, int n_heads,
                        int n_kv_heads, float freq_base) {
    int rot = head_dim;
    float neg_log_base = -logf(freq_base);
    float dim_inv = 1.0f / (float)rot;
    for (int pass = 0; pass < 2; pass++) {
        float* base = pass == 0 ? q : k;
        int nh = pass == 0 ? n_heads : n_kv_heads;
        for (int h = 0; h < nh; h++) {
            float* v = base + (size_t)h * head_dim;
            for (int i = 0; i < rot; i += 2) {
                float theta = (float)pos * expf((float)i * dim_inv * neg_log_base);
                float c = cosf(theta), s = sinf(theta);
                float x0 = v[i], x1 = v[i + 1];
                v[i] = x0 * c - x1 * s;
                v[i + 1] = x0 * s + x1 * c;
            }
        }
    }
}

// TensorMath.ApplyRoPENeox (TensorMath.cs:475-520): split-half pairs
// (i, i + half), full rotary dimension.
extern "C" void or_rope_neox(float* q, float* k, int pos, int head_dim, int n_heads, int n_kv_heads,
                             float freq_base) {
    int half = head_dim / 2;
    float neg_log_base = -logf(freq_base);
    float dim_inv = 2.0f / (float)head_dim;
    for (int pass = 0; pass < 2; pass++) {
        float* base = pass == 0 ? q : k;
        int nh = pass == 0 ? n_heads : n_kv_heads;
        for (int h = 0; h < nh; h++) {
            float* v = base + (size_t)h * head_dim;
            for (int i = 0; i < half; i++) {
                float theta = (float)pos * expf((float)i * dim_inv * neg_log_base);
                float c = cosf(theta), s = sinf(theta);
                float x0 = v[i], x1 = v[i + half];
                v[i] = x0 * c - x1 * s;
                v[i + half] = x1 * c + x0 * s;
            }
        }
    }
}

// TensorMath.GeluElementwiseMul (TensorMath.cs:294-333), tanh approximation,
// evaluated left to right as the C# expression is.
extern "C" void or_gelu_mul(float* gate, const float* up, int length) {
    const float kSqrt2OverPi = 0.7978845608028654f, kCoeff = 0.044715f;
    for (int i = 0; i < length; i++) {
        float x = gate[i];
        float g = 0.5f * x * (1.0f + tanhf(kSqrt2OverPi * (x + kCoeff * x * x * x)));
        gate[i] = g * up[i];
    }
}

// TensorMath.RmsNormWithOffset (TensorMath.cs:335-394): the sum of squares as
// RmsNorm forms it, then input * rms * (weight + 1).
extern "C" void or_rmsnorm_offset(const float* x, const float* w, float* y, int n, float eps) {
    std::vector<float> w1(n);
    for (int i = 0; i < n; i++) w1[i] = w[i] + 1.0f;
    or_rmsnorm(x, w1.data(), y, n, eps);
}

// TensorMath.Add (TensorMath.cs:712-733).
extern "C" void or_add(float* a, const float* b, int length) {
    for (int i = 0; i < length; i++) a[i] += b[i];
}

// GreedySampler.Sample (GreedySampler.cs:13-26): first maximum wins.
extern "C" int or_argmax(const float* logits, int n) {
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > bv) {
            bv = logits[i];
            best = i;
        }
    return best;
}

// TemperatureSampler.Sample (Samplers/TemperatureSampler.cs:33-113) with the
// caller's draw r in place of _rng.NextDouble().  *margin receives the
// smallest distance of a running sum to the value it was compared with (top_p
// for the nucleus cut-off, r for the draw) up to the decision: results that
// differ by less than fp32 rounding of the probabilities can only move a
// decision whose margin is that small.
static void samp_swap(float* p, int* ix, int a, int b) {
    const float tf = p[a];
    p[a] = p[b];
    p[b] = tf;
    const int ti = ix[a];
    ix[a] = ix[b];
    ix[b] = ti;
}

// PartialSortDescending (TemperatureSampler.cs:119-162): median-of-three
// quickselect that leaves the k largest in p[0..k-1].
static void samp_partial_sort(float* p, int* ix, int left, int right, int k) {
    while (left < right) {
        const int mid = left + (right - left) / 2;
        if (p[mid] > p[left]) samp_swap(p, ix, left, mid);
        if (p[right] > p[left]) samp_swap(p, ix, left, right);
        if (p[mid] > p[right]) samp_swap(p, ix, mid, right);
        const float pivot = p[right];
        int store = left;
        for (int i = left; i < right; i++)
            if (p[i] > pivot) samp_swap(p, ix, i, store++);
        samp_swap(p, ix, store, right);
        if (store == k - 1) return;
        if (store < k - 1) left = store + 1;
        else right = store - 1;
    }
}

extern "C" int or_sample_temperature(const float* logits, int vocab, float temperature, int top_k, float top_p,
                                     float r, float* margin) {
    *margin = INFINITY;
    if (temperature <= 0.f) {
        int best = 0;
        float bv = logits[0];
        for (int i = 1; i < vocab; i++)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        return best;
    }
    std::vector<float> p(vocab);
    std::vector<int> ix(vocab);
    const float inv_temp = 1.0f / temperature;
    for (int i = 0; i < vocab; i++) {
        p[i] = logits[i] * inv_temp;
        ix[i] = i;
    }
    or_softmax(p.data(), vocab);
    const int k = top_k < vocab ? top_k : vocab;
    samp_partial_sort(p.data(), ix.data(), 0, vocab - 1, k);
    // InsertionSortDescending (TemperatureSampler.cs:168-184)
    for (int i = 1; i < k; i++) {
        const float kp = p[i];
        const int ki = ix[i];
        int j = i - 1;
        while (j >= 0 && p[j] < kp) {
            p[j + 1] = p[j];
            ix[j + 1] = ix[j];
            j--;
        }
        p[j + 1] = kp;
        ix[j + 1] = ki;
    }
    float cumulative = 0.f;
    int cutoff = k;
    for (int i = 0; i < k; i++) {
        cumulative += p[i];
        *margin = fminf(*margin, fabsf(cumulative - top_p));
        if (cumulative >= top_p) {
            cutoff = i + 1;
            break;
        }
    }
    float sum = 0.f;
    for (int i = 0; i < cutoff; i++) sum += p[i];
    const float inv_sum = 1.0f / sum;
    for (int i = 0; i < cutoff; i++) p[i] *= inv_sum;
    float acc = 0.f;
    for (int i = 0; i < cutoff; i++) {
        acc += p[i];
        *margin = fminf(*margin, fabsf(r - acc));
        if (r < acc) return ix[i];
    }
    return ix[cutoff - 1];
}

// ---------------------------------------------------------------------------
// Llama forward (LlamaModel.cs:93-238)
// ---------------------------------------------------------------------------

namespace {

struct Scratch {
    std::vector<float> xnorm, q, k, v, att, gate, up, ffn, scores, krow, vrow;
    Scratch(const or_llama_config& c) {
        int kv = c.n_kv_heads * c.head_dim;
        xnorm.resize(c.dim);
        q.resize(c.dim);
        k.resize(kv);
        v.resize(kv);
        att.resize(c.dim);
        gate.resize(c.hidden_dim);
        up.resize(c.hidden_dim);
        ffn.resize(c.dim);
        scores.resize(c.ctx_len);
        krow.resize(c.head_dim);
        vrow.resize(c.head_dim);
    }
};

inline const uint8_t* T(const void* const* t, int i) { return (const uint8_t*)t[i]; }

// Reads head `off` of cache row (layer, p) as fp32 (fp16 caches widen).
inline const float* kv_row(const or_llama_config& c, const void* cache, int layer, int p,
                           int off, float* tmp) {
    size_t kvdim = (size_t)c.n_kv_heads * c.head_dim;
    size_t idx = ((size_t)layer * c.ctx_len + p) * kvdim + off;
    if (!c.kv_f16) return (const float*)cache + idx;
    const uint16_t* h = (const uint16_t*)cache + idx;
    for (int d = 0; d < c.head_dim; d++) tmp[d] = or_half_to_float(h[d]);
    return tmp;
}

// LlamaModel.ComputeAttention (LlamaModel.cs:241-346).
void attention(const or_llama_config& c, Scratch& s, const void* kc, const void* vc, int layer,
               int pos) {
    int hd = c.head_dim;
    int kv_mul = c.n_heads / c.n_kv_heads;
    int seq = pos + 1;
    float scale = 1.0f / sqrtf((float)hd);
    std::fill(s.att.begin(), s.att.end(), 0.f);
    for (int h = 0; h < c.n_heads; h++) {
        const float* qp = s.q.data() + (size_t)h * hd;
        int kvoff = (h / kv_mul) * hd;
        for (int p = 0; p < seq; p++) {
            const float* kp = kv_row(c, kc, layer, p, kvoff, s.krow.data());
            float score = 0.f;
            int d = 0;
            if (hd >= 8) {
                float a0[8] = {0}, a1[8] = {0};
                int limit = hd - 16 + 1;
                for (; d < limit; d += 16)
                    for (int t = 0; t < 8; t++) {
                        a0[t] += qp[d + t] * kp[d + t];
                        a1[t] += qp[d + 8 + t] * kp[d + 8 + t];
                    }
                int single = hd - 8 + 1;
                for (; d < single; d += 8)
                    for (int t = 0; t < 8; t++) a0[t] += qp[d + t] * kp[d + t];
                float tt[8];
                for (int t = 0; t < 8; t++) tt[t] = a0[t] + a1[t];
                score = vsum8(tt);
            }
            for (; d < hd; d++) score += qp[d] * kp[d];
            s.scores[p] = score * scale;
        }
        or_softmax(s.scores.data(), seq);
        float* out = s.att.data() + (size_t)h * hd;
        for (int p = 0; p < seq; p++) {
            float w = s.scores[p];
            if (w == 0.f) continue;
            const float* vp = kv_row(c, vc, layer, p, kvoff, s.vrow.data());
            for (int d = 0; d < hd; d++) out[d] += vp[d] * w;
        }
    }
}

void store_kv(const or_llama_config& c, void* cache, int layer, int pos, const float* src) {
    size_t kvdim = (size_t)c.n_kv_heads * c.head_dim;
    size_t idx = ((size_t)layer * c.ctx_len + pos) * kvdim;
    if (!c.kv_f16) {
        memcpy((float*)cache + idx, src, kvdim * 4);
    } else {
        uint16_t* h = (uint16_t*)cache + idx;
        for (size_t i = 0; i < kvdim; i++) h[i] = or_float_to_half(src[i]);
    }
}

int run_layers(const or_llama_config& c, const void* const* t, const int* ty, void* kc, void* vc,
               float* x, int pos, int l0, int l1, int nth, Scratch& s) {
    int dim = c.dim, kvdim = c.n_kv_heads * c.head_dim, hid = c.hidden_dim;
    for (int l = l0; l < l1; l++) {
        int b = 3 + 9 * l;
        // the architecture variants the model config selects (Gemma: offset
        // norms and GELU; Qwen/Phi: split-half RoPE) on the Llama loop
        auto norm = c.norm_offset ? or_rmsnorm_offset : or_rmsnorm;
        norm(x, (const float*)t[b + 0], s.xnorm.data(), dim, c.eps);
        int rc = 0;
        rc |= or_matvec(ty[b + 1], T(t, b + 1), s.xnorm.data(), s.q.data(), dim, dim, nth);
        rc |= or_matvec(ty[b + 2], T(t, b + 2), s.xnorm.data(), s.k.data(), kvdim, dim, nth);
        rc |= or_matvec(ty[b + 3], T(t, b + 3), s.xnorm.data(), s.v.data(), kvdim, dim, nth);
        if (rc) return -2;
        (c.rope_neox ? or_rope_neox : or_rope)(s.q.data(), s.k.data(), pos, c.head_dim, c.n_heads, c.n_kv_heads,
                                                c.rope_base);
        store_kv(c, kc, l, pos, s.k.data());
        store_kv(c, vc, l, pos, s.v.data());
        attention(c, s, kc, vc, l, pos);
        if (or_matvec(ty[b + 4], T(t, b + 4), s.att.data(), s.ffn.data(), dim, dim, nth)) return -2;
        or_add(x, s.ffn.data(), dim);
        norm(x, (const float*)t[b + 5], s.xnorm.data(), dim, c.eps);
        rc |= or_matvec(ty[b + 6], T(t, b + 6), s.xnorm.data(), s.gate.data(), hid, dim, nth);
        rc |= or_matvec(ty[b + 7], T(t, b + 7), s.xnorm.data(), s.up.data(), hid, dim, nth);
        if (rc) return -2;
        (c.act_gelu ? or_gelu_mul : or_silu_mul)(s.gate.data(), s.up.data(), hid);
        if (or_matvec(ty[b + 8], T(t, b + 8), s.gate.data(), s.ffn.data(), dim, hid, nth)) return -2;
        or_add(x, s.ffn.data(), dim);
    }
    return 0;
}

int embed(const or_llama_config& c, const void* const* t, const int* ty, int token, float* x) {
    int type = ty[0];
    uint64_t row = or_byte_size(type, (uint64_t)c.dim);
    if (row == 0) return -2;
    if (token < 0 || token >= c.vocab) return -1;
    // LoadEmbedding (LlamaModel.cs:365-394): one row, dequantized.
    return or_dequantize(type, T(t, 0) + (size_t)token * row, x, c.dim);
}

}  // namespace

extern "C" int or_llama_layers(const or_llama_config* cfg, const void* const* tensors,
                               const int* types, void* kcache, void* vcache, float* x, int pos,
                               int l0, int l1, int nthreads) {
    Scratch s(*cfg);
    return run_layers(*cfg, tensors, types, kcache, vcache, x, pos, l0, l1, nthreads, s);
}

extern "C" int or_llama_head(const or_llama_config* cfg, const void* const* tensors,
                             const int* types, const float* x, float* logits, int nthreads) {
    std::vector<float> xn(cfg->dim);
    (cfg->norm_offset ? or_rmsnorm_offset : or_rmsnorm)(x, (const float*)tensors[2], xn.data(), cfg->dim, cfg->eps);
    return or_matvec(types[1], T(tensors, 1), xn.data(), logits, cfg->vocab, cfg->dim, nthreads);
}

extern "C" int or_llama_forward(const or_llama_config* cfg, const void* const* tensors,
                                const int* types, void* kcache, void* vcache, const int* tokens,
                                int n, int pos, float* logits, int nthreads) {
    if (n <= 0 || pos < 0 || pos + n > cfg->ctx_len) return -1;
    Scratch s(*cfg);
    std::vector<float> x(cfg->dim);
    for (int t = 0; t < n; t++) {
        int rc = embed(*cfg, tensors, types, tokens[t], x.data());
        if (rc) return rc;
        rc = run_layers(*cfg, tensors, types, kcache, vcache, x.data(), pos + t, 0,
                        cfg->n_layers, nthreads, s);
        if (rc) return rc;
        if (t == n - 1) {
            rc = or_llama_head(cfg, tensors, types, x.data(), logits, nthreads);
            if (rc) return rc;
        }
    }
    return 0;
}
