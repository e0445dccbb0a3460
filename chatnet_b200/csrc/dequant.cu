// dequant.cu -- bit-exact block dequantization and the device-side
// synthetic generator.
//
// Dequantization follows the reference's per-operation rounding order with
// explicit round-to-nearest intrinsics (no FMA contraction):
//   Q4_0: (float)(q - 8) * d                       DequantQ4_0.cs:42-53
//   Q4_K: (d*sc)*q - dmin*m, each step rounded     DequantQ4K.cs:59-71
//   Q6_K: (d*sc)*q, left to right                  DequantQ6K.cs:73-81
// fp16 -> fp32 is exact, as (float)Half is.
#include "cn_common.cuh"
#include "cn_internal.h"
#include "formats.cuh"
#include "synth.cuh"

namespace cn {

// One thread per 32-element block (partial last block handled as in
// DequantQ4_0.Dequantize: only `remaining` outputs are written).
__global__ void dequant_q4_0_kernel(const uint8_t* __restrict__ q, float* __restrict__ out,
                                    int64_t n) {
    const int64_t nb = (n + 31) / 32;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb;
         b += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = q + b * 18;
        float d = ld_half(p);
        int64_t rem = n - b * 32;
        float* o = out + b * 32;
        if (rem >= 32) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                v[j] = __fmul_rn((float)((p[2 + j] & 0x0F) - 8), d);
                v[j + 16] = __fmul_rn((float)(((p[2 + j] >> 4) & 0x0F) - 8), d);
            }
            if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                for (int j = 0; j < 32; j++) o[j] = v[j];
            }
        } else {
            int half = rem < 16 ? (int)rem : 16;
            for (int j = 0; j < half; j++) o[j] = __fmul_rn((float)((p[2 + j] & 0x0F) - 8), d);
            int second = rem > 16 ? (int)(rem - 16) : 0;
            for (int j = 0; j < second; j++)
                o[16 + j] = __fmul_rn((float)(((p[2 + j] >> 4) & 0x0F) - 8), d);
        }
    }
}

// One thread per (super-block, 32-element sub-block); only whole
// super-blocks are written (blockCount = elementCount / 256).
__global__ void dequant_q4_k_kernel(const uint8_t* __restrict__ q, float* __restrict__ out,
                                    int64_t n) {
    const int64_t subs = (n / 256) * 8;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < subs;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = i >> 3;
        int sub = (int)(i & 7);
        const uint8_t* p = q + b * 144;
        float d = ld_half(p), dmin = ld_half(p + 2);
        int sc, m;
        q4k_scale_min(p + 4, sub, sc, m);
        float dsc = __fmul_rn(d, (float)sc);
        float dm = __fmul_rn(dmin, (float)m);
        const uint8_t* qs = p + 16 + sub * 16;
        float* o = out + b * 256 + sub * 32;
        for (int j = 0; j < 16; j++) {
            uint8_t v = qs[j];
            o[j] = __fsub_rn(__fmul_rn(dsc, (float)(v & 0x0F)), dm);
            o[j + 16] = __fsub_rn(__fmul_rn(dsc, (float)((v >> 4) & 0x0F)), dm);
        }
    }
}

// One thread per (super-block, half, l) producing the four outputs l, l+32,
// l+64, l+96 of that half, as in the reference loop.
__global__ void dequant_q6_k_kernel(const uint8_t* __restrict__ q, float* __restrict__ out,
                                    int64_t n) {
    const int64_t total = (n / 256) * 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = i >> 6;
        int half = (int)((i >> 5) & 1);
        int l = (int)(i & 31);
        const uint8_t* p = q + b * 210;
        float d = ld_half(p + 208);
        const uint8_t* ql = p + half * 64;
        const uint8_t* qh = p + 128 + half * 32;
        const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192);
        int si = half * 8 + l / 16;
        int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
        int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        float* o = out + b * 256 + half * 128;
        o[l] = __fmul_rn(__fmul_rn(d, (float)sc[si]), (float)q1);
        o[l + 32] = __fmul_rn(__fmul_rn(d, (float)sc[si + 2]), (float)q2);
        o[l + 64] = __fmul_rn(__fmul_rn(d, (float)sc[si + 4]), (float)q3);
        o[l + 96] = __fmul_rn(__fmul_rn(d, (float)sc[si + 6]), (float)q4);
    }
}

// One thread per 32-element block of Q4_1 / Q5_0 / Q5_1 / Q8_0; a partial
// last block writes only its `remaining` elements, as the reference loops do.
__global__ void dequant_b32_kernel(int type, const uint8_t* __restrict__ q, float* __restrict__ out, int64_t n,
                                   int bpb) {
    const int64_t nb = (n + 31) / 32;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb;
         b += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = q + b * bpb;
        const int64_t rem = n - b * 32;
        const int cnt = rem < 32 ? (int)rem : 32;
        for (int j = 0; j < cnt; j++) out[b * 32 + j] = block32_elem(type, p, j);
    }
}

// One thread per element of the whole super-blocks of the 256-element codecs
// on the generic paths (the reference decodes n / 256 super-blocks; `end`
// bounds IQ3_S's reads past a block).
__global__ void dequant_superblock_kernel(int type, const uint8_t* __restrict__ q, float* __restrict__ out,
                                          int64_t n, int bpb, const uint8_t* end) {
    const int64_t m = n / 256 * 256;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = superblock_elem(type, q + (i >> 8) * bpb, (int)(i & 255), end);
}

__global__ void convert_f16_kernel(const uint16_t* __restrict__ h, float* __restrict__ out,
                                   int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = half_bits_to_float(h[i]);
}

static unsigned grid_for(int64_t work, int threads) {
    int64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > 148 * 32) g = 148 * 32;
    return (unsigned)g;
}

int dequant_launch(int type, const void* d_blocks, float* d_out, int64_t n, cudaStream_t s, const void* d_end) {
    CN_CHECK(n >= 0, CN_ERR_INVALID_ARG, "negative element count");
    if (n == 0) return CN_OK;
    CN_CHECK(d_blocks && d_out, CN_ERR_INVALID_ARG, "null pointer");
    const uint8_t* q = static_cast<const uint8_t*>(d_blocks);
    if (is_block32(type)) {
        dequant_b32_kernel<<<grid_for((n + 31) / 32, 256), 256, 0, s>>>(type, q, d_out, n, block32_bytes(type));
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    if (is_superblock(type)) {
        if (n / 256 == 0) return CN_OK;
        const uint8_t* end = d_end ? static_cast<const uint8_t*>(d_end) : q + (n / 256) * superblock_bytes(type);
        dequant_superblock_kernel<<<grid_for(n / 256 * 256, 256), 256, 0, s>>>(type, q, d_out, n,
                                                                                superblock_bytes(type), end);
        CN_CUDA(cudaGetLastError());
        return CN_OK;
    }
    switch (type) {
        case CN_TYPE_Q4_0:
            dequant_q4_0_kernel<<<grid_for((n + 31) / 32, 256), 256, 0, s>>>(q, d_out, n);
            break;
        case CN_TYPE_Q4_K:
            if (n / 256 == 0) return CN_OK;
            dequant_q4_k_kernel<<<grid_for((n / 256) * 8, 256), 256, 0, s>>>(q, d_out, n);
            break;
        case CN_TYPE_Q6_K:
            if (n / 256 == 0) return CN_OK;
            dequant_q6_k_kernel<<<grid_for((n / 256) * 64, 256), 256, 0, s>>>(q, d_out, n);
            break;
        case CN_TYPE_F32:
            CN_CUDA(cudaMemcpyAsync(d_out, d_blocks, (size_t)n * 4, cudaMemcpyDeviceToDevice, s));
            return CN_OK;
        case CN_TYPE_F16:
            convert_f16_kernel<<<grid_for(n, 256), 256, 0, s>>>((const uint16_t*)q, d_out, n);
            break;
        default:
            return set_error(CN_ERR_UNSUPPORTED, "Unsupported embedding type: %d", type);
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

// ---- synthetic generator (device) ----------------------------------------------

// The generators index blocks / elements of the FULL tensor (rows_full x
// cols_full), so any [row0, row0 + nrows) x [col0, col0 + ncols) slice gets
// exactly the bytes of that region of the whole tensor (tensor-parallel
// shards are generated where they live).  Local block lb of the slice is
// global block (row0 + lb / nbc) * bpr_full + cb0 + lb % nbc.
__global__ void synth_blocks_kernel(int type, uint64_t seed, int64_t bpr_full, int64_t row0, int64_t cb0,
                                    int64_t nbc, int64_t nblocks, uint8_t* out) {
    for (int64_t lb = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; lb < nblocks;
         lb += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = (row0 + lb / nbc) * bpr_full + cb0 + lb % nbc;
        if (type == CN_TYPE_Q4_0) {
            synth::q4_0_block(seed, b, out + lb * 18);
        } else if (type == CN_TYPE_Q4_K) {
            __align__(16) uint8_t tmp[144];
            synth::q4_k_block(seed, b, tmp);
            uint4* o = reinterpret_cast<uint4*>(out + lb * 144);  // 144 = 9 x 16
            const uint4* src = reinterpret_cast<const uint4*>(tmp);
            for (int i = 0; i < 9; i++) o[i] = src[i];
        } else {
            synth::q6_k_block(seed, b, out + lb * 210);
        }
    }
}

__global__ void synth_f32_kernel(uint64_t seed, int64_t cols_full, int64_t row0, int64_t col0, int64_t ncols,
                                 int64_t n, int dist, float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = (row0 + i / ncols) * cols_full + col0 + i % ncols;
        out[i] = dist == CN_DIST_NORM_W ? synth::norm_weight_elem(seed, g) : synth::normal_elem(seed, g);
    }
}

__global__ void synth_f16_kernel(uint64_t seed, int64_t cols_full, int64_t row0, int64_t col0, int64_t ncols,
                                 int64_t n, uint16_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = (row0 + i / ncols) * cols_full + col0 + i % ncols;
        out[i] = synth::f2h(synth::normal_elem(seed, g));
    }
}

int synth_slice_launch(int type, int64_t rows, int64_t cols, int64_t row0, int64_t nrows, int64_t col0,
                       int64_t ncols, uint64_t seed, int dist, void* d_out, cudaStream_t s) {
    CN_CHECK(row0 >= 0 && nrows >= 0 && row0 + nrows <= rows && col0 >= 0 && ncols >= 0 && col0 + ncols <= cols,
             CN_ERR_INVALID_ARG, "slice outside the tensor");
    const int64_t n = nrows * ncols;
    if (n == 0) return CN_OK;
    if (type == CN_TYPE_Q4_0 || type == CN_TYPE_Q4_K || type == CN_TYPE_Q6_K) {
        int want = type == CN_TYPE_Q4_0 ? CN_DIST_CFG0_Q4_0
                   : type == CN_TYPE_Q4_K ? CN_DIST_CFG2_Q4_K
                                          : CN_DIST_CFG2_Q6_K;
        CN_CHECK(dist == want, CN_ERR_INVALID_ARG, "distribution %d does not match type %d", dist,
                 type);
        int bs = type == CN_TYPE_Q4_0 ? 32 : 256;
        CN_CHECK(cols % bs == 0 && col0 % bs == 0 && ncols % bs == 0, CN_ERR_INVALID_ARG,
                 "columns not whole blocks of %d", bs);
        const int64_t nbc = ncols / bs, nb = nrows * nbc;
        synth_blocks_kernel<<<grid_for(nb, 128), 128, 0, s>>>(type, seed, cols / bs, row0, col0 / bs, nbc, nb,
                                                              (uint8_t*)d_out);
    } else if (type == CN_TYPE_F32) {
        CN_CHECK(dist == CN_DIST_NORMAL || dist == CN_DIST_NORM_W, CN_ERR_INVALID_ARG,
                 "bad F32 distribution %d", dist);
        synth_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>(seed, cols, row0, col0, ncols, n, dist, (float*)d_out);
    } else if (type == CN_TYPE_F16) {
        CN_CHECK(dist == CN_DIST_NORMAL, CN_ERR_INVALID_ARG, "bad F16 distribution %d", dist);
        synth_f16_kernel<<<grid_for(n, 256), 256, 0, s>>>(seed, cols, row0, col0, ncols, n, (uint16_t*)d_out);
    } else {
        return set_error(CN_ERR_UNSUPPORTED, "no generator for type %d", type);
    }
    CN_CUDA(cudaGetLastError());
    return CN_OK;
}

int synth_launch(int type, int64_t rows, int64_t cols, uint64_t seed, int dist, void* d_out,
                 cudaStream_t s) {
    return synth_slice_launch(type, rows, cols, 0, rows, 0, cols, seed, dist, d_out, s);
}

}  // namespace cn
