// dequantize_block for the six hot-path types (reference src/core/quant.cpp
// deq_q8_0 :38-50, deq_q4_0 :55-68, deq_q5_0 :114-131, deq_q4_k :82-109,
// deq_q5_k :300-335, deq_q6_k :134-160).  One thread per output value; the
// float expressions are the reference's (d1*q - m1, d*sc*(q-32), ...), with
// no multiply-add contraction so the values are bit-exact.
#pragma once
#include "common.cuh"

namespace cllm {

__device__ __forceinline__ uint32_t rd_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

__device__ __forceinline__ void k4_scale_min(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

__global__ void dequantize_kernel(const uint8_t* __restrict__ src, int type, int64_t n,
                                  float* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float v = 0.0f;
        if (type == kQ8_0) {
            const uint8_t* b = src + (i >> 5) * 34;
            v = __fmul_rn(h2f(rd_u16(b)), (float)(int8_t)b[2 + (i & 31)]);
        } else if (type == kQ4_0) {
            const uint8_t* b = src + (i >> 5) * 18;
            const int j = i & 31;
            const int q = j < 16 ? (b[2 + j] & 0xF) : (b[2 + j - 16] >> 4);
            v = __fmul_rn(h2f(rd_u16(b)), (float)(q - 8));
        } else if (type == kQ5_0) {
            const uint8_t* b = src + (i >> 5) * 22;
            const int j = i & 31;
            const uint32_t qh = rd_u16(b + 2) | (rd_u16(b + 4) << 16);
            const int lo = j < 16 ? (b[6 + j] & 0xF) : (b[6 + j - 16] >> 4);
            const int q = lo | (((qh >> j) & 1) << 4);
            v = __fmul_rn(h2f(rd_u16(b)), (float)(q - 16));
        } else if (type == kQ4_K || type == kQ5_K) {
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
            v = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
        } else if (type == kQ6_K) {
            const uint8_t* b = src + (i >> 8) * 210;
            const int e = i & 255, g = e >> 7, r = e & 127, sub = r >> 5, l = r & 31;
            const uint8_t* ql = b + 64 * g + 32 * (sub & 1);
            const uint8_t* qh = b + 128 + 32 * g;
            const int lo = sub >= 2 ? (ql[l] >> 4) : (ql[l] & 0xF);
            const int q = lo | (((qh[l] >> (2 * sub)) & 3) << 4);
            const int sc = (int)(int8_t)b[192 + 8 * g + (l >> 4) + 2 * sub];
            v = __fmul_rn(__fmul_rn(h2f(rd_u16(b + 208)), (float)sc), (float)(q - 32));
        }
        dst[i] = v;
    }
}

}  // namespace cllm
