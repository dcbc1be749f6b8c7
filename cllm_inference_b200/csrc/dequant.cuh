// dequantize_block for every GGML type the reference handles (reference
// src/core/quant.cpp:28-336, dispatch :371-389): F32 :28-30, F16 :33-36,
// Q8_0 :38-50, Q4_0 :55-68, Q4_K :82-109, Q5_0 :114-131, Q6_K :134-160,
// Q4_1 :163-177, Q5_1 :181-201, Q8_1 :204-215, Q2_K :219-249, Q3_K :253-296,
// Q5_K :300-335.  One output value per call of dequant_value; the float
// expressions are the reference's (d1*q - m1, d*q + m, d*sc*(q-32), ...) with
// no multiply-add contraction, so the values are bit-exact.  (Every product of
// these formulas is exact -- an fp16-derived scale times a small integer -- so
// only the final add or subtract rounds.)
#pragma once
#include "common.cuh"

namespace cllm {

// GGML type ids without an integer dot kernel (quant.hpp:13-27)
enum : int { kF32 = 0, kF16 = 1, kQ4_1 = 3, kQ5_1 = 7, kQ8_1 = 9, kQ2_K = 10, kQ3_K = 11 };

__host__ __device__ inline bool dequant_supported(int t) {
    return t == kF32 || t == kF16 || t == kQ4_0 || t == kQ4_1 || t == kQ5_0 || t == kQ5_1 || t == kQ8_0 ||
           t == kQ8_1 || t == kQ2_K || t == kQ3_K || t == kQ4_K || t == kQ5_K || t == kQ6_K;
}

__device__ __forceinline__ uint32_t rd_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ uint32_t rd_u32(const uint8_t* p) { return rd_u16(p) | (rd_u16(p + 2) << 16); }

__device__ __forceinline__ void k4_scale_min(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Q3_K: the six-bit scale `is` (0..15) of the 12 interleaved bytes at p, minus 32
// (quant.cpp:268-275 unpacks all sixteen into four words; this takes one).
__device__ __forceinline__ int q3k_scale(const uint8_t* p, int is) {
    const uint32_t a0 = rd_u32(p), a1 = rd_u32(p + 4), t = rd_u32(p + 8);
    const uint32_t lo4 = 0x0f0f0f0fu, hi2 = 0x03030303u;
    uint32_t w;
    switch (is >> 2) {
        case 0: w = (a0 & lo4) | (((t >> 0) & hi2) << 4); break;
        case 1: w = (a1 & lo4) | (((t >> 2) & hi2) << 4); break;
        case 2: w = ((a0 >> 4) & lo4) | (((t >> 4) & hi2) << 4); break;
        default: w = ((a1 >> 4) & lo4) | (((t >> 6) & hi2) << 4); break;
    }
    return (int)(int8_t)(uint8_t)(w >> (8 * (is & 3))) - 32;
}

// Value i of a run of blocks of type t starting at src.
__device__ __forceinline__ float dequant_value(const uint8_t* __restrict__ src, int type, int64_t i) {
    switch (type) {
        case kF32:
            return __uint_as_float(rd_u32(src + 4 * i));
        case kF16:
            return h2f(rd_u16(src + 2 * i));
        case kQ8_0: {
            const uint8_t* b = src + (i >> 5) * 34;
            return __fmul_rn(h2f(rd_u16(b)), (float)(int8_t)b[2 + (i & 31)]);
        }
        case kQ8_1: {
            const uint8_t* b = src + (i >> 5) * 36;
            return __fmul_rn(h2f(rd_u16(b)), (float)(int8_t)b[4 + (i & 31)]);
        }
        case kQ4_0: {
            const uint8_t* b = src + (i >> 5) * 18;
            const int j = i & 31;
            const int q = j < 16 ? (b[2 + j] & 0xF) : (b[2 + j - 16] >> 4);
            return __fmul_rn(h2f(rd_u16(b)), (float)(q - 8));
        }
        case kQ4_1: {
            const uint8_t* b = src + (i >> 5) * 20;
            const int j = i & 31;
            const int q = j < 16 ? (b[4 + j] & 0xF) : (b[4 + j - 16] >> 4);
            return __fadd_rn(__fmul_rn(h2f(rd_u16(b)), (float)q), h2f(rd_u16(b + 2)));
        }
        case kQ5_0: {
            const uint8_t* b = src + (i >> 5) * 22;
            const int j = i & 31;
            const uint32_t qh = rd_u32(b + 2);
            const int lo = j < 16 ? (b[6 + j] & 0xF) : (b[6 + j - 16] >> 4);
            const int q = lo | (((qh >> j) & 1) << 4);
            return __fmul_rn(h2f(rd_u16(b)), (float)(q - 16));
        }
        case kQ5_1: {
            const uint8_t* b = src + (i >> 5) * 24;
            const int j = i & 31;
            const uint32_t qh = rd_u32(b + 4);
            const int lo = j < 16 ? (b[8 + j] & 0xF) : (b[8 + j - 16] >> 4);
            const int q = lo | (((qh >> j) & 1) << 4);
            return __fadd_rn(__fmul_rn(h2f(rd_u16(b)), (float)q), h2f(rd_u16(b + 2)));
        }
        case kQ2_K: {
            // [scales 16][qs 64][d][dmin]; half h of 128 values, shift pair j, lane l
            const uint8_t* b = src + (i >> 8) * 84;
            const int e = i & 255, h = e >> 7, j = (e >> 5) & 3, l = e & 31;
            const int sc = b[8 * h + 2 * j + (l >> 4)];
            const float dl = __fmul_rn(h2f(rd_u16(b + 80)), (float)(sc & 0xF));
            const float ml = __fmul_rn(h2f(rd_u16(b + 82)), (float)(sc >> 4));
            const int q = (b[16 + 32 * h + l] >> (2 * j)) & 3;
            return __fsub_rn(__fmul_rn(dl, (float)q), ml);
        }
        case kQ3_K: {
            // [hmask 32][qs 64][scales 12][d]; high-bit mask bit 4h + j of hmask[l]
            const uint8_t* b = src + (i >> 8) * 110;
            const int e = i & 255, h = e >> 7, j = (e >> 5) & 3, l = e & 31;
            const float dl = __fmul_rn(h2f(rd_u16(b + 108)), (float)q3k_scale(b + 96, 8 * h + 2 * j + (l >> 4)));
            const int q = ((b[32 + 32 * h + l] >> (2 * j)) & 3) - (((b[l] >> (4 * h + j)) & 1) ? 0 : 4);
            return __fmul_rn(dl, (float)q);
        }
        case kQ4_K:
        case kQ5_K: {
            const int ts = type == kQ4_K ? 144 : 176;
            const uint8_t* b = src + (i >> 8) * ts;
            const int e = i & 255, sub = e >> 5, l = e & 31;
            int sc, m;
            k4_scale_min(sub, b + 4, sc, m);
            const float d1 = __fmul_rn(h2f(rd_u16(b)), (float)sc);
            const float m1 = __fmul_rn(h2f(rd_u16(b + 2)), (float)m);
            const uint8_t* q = b + (type == kQ4_K ? 16 : 48) + 32 * (sub >> 1);
            int qv = (sub & 1) ? (q[l] >> 4) : (q[l] & 0xF);
            if (type == kQ5_K) qv += ((b[16 + l] >> sub) & 1) ? 16 : 0;
            return __fsub_rn(__fmul_rn(d1, (float)qv), m1);
        }
        case kQ6_K: {
            const uint8_t* b = src + (i >> 8) * 210;
            const int e = i & 255, g = e >> 7, r = e & 127, sub = r >> 5, l = r & 31;
            const uint8_t* ql = b + 64 * g + 32 * (sub & 1);
            const uint8_t* qh = b + 128 + 32 * g;
            const int lo = sub >= 2 ? (ql[l] >> 4) : (ql[l] & 0xF);
            const int q = lo | (((qh[l] >> (2 * sub)) & 3) << 4);
            const int sc = (int)(int8_t)b[192 + 8 * g + (l >> 4) + 2 * sub];
            return __fmul_rn(__fmul_rn(h2f(rd_u16(b + 208)), (float)sc), (float)(q - 32));
        }
    }
    return 0.0f;
}

__global__ void dequantize_kernel(const uint8_t* __restrict__ src, int type, int64_t n, float* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = dequant_value(src, type, i);
}

// fp32 -> fp16 bits exactly as the reference's float_to_half (quant.hpp:58-85):
// normal results keep the top 10 mantissa bits (truncation, no rounding),
// results below the normal range are rounded (the bias-plus-odd-bit step),
// magnitudes past the fp16 range become inf, NaN becomes the quiet 0x7E00.
__device__ __forceinline__ uint16_t f2h_bits(float v) {
    const uint32_t x = __float_as_uint(v);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t e8 = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (e8 == 0xFFu) return (uint16_t)(sign | (mant ? 0x7E00u : 0x7C00u));
    const int e = (int)e8 - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const uint32_t sh = (uint32_t)(14 - e);
        return (uint16_t)(sign | ((mant + ((1u << (sh - 1)) - 1u) + ((mant >> sh) & 1u)) >> sh));
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | (mant >> 13));
}

// dequantize_block_f16 (quant.cpp:391-402): F16 sources are copied, every other
// type is dequantized to float and rounded to fp16.
__global__ void dequantize_f16_kernel(const uint8_t* __restrict__ src, int type, int64_t n,
                                      uint16_t* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = type == kF16 ? (uint16_t)rd_u16(src + 2 * i) : f2h_bits(dequant_value(src, type, i));
}

}  // namespace cllm
