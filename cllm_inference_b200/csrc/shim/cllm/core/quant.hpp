// Drop-in declaration of the quant API of cllm_inference, served by the B200
// library (libcllm_quant.so -> libcllm_cuda.so).
//
// Names, signatures, default arguments, the GgmlType numbering and the layout
// of QuantizedQ8_0 match the reference's include/cllm/core/quant.hpp:10-151,
// so TransformerEngine (src/core/engine.cpp) compiles and links unchanged
// against this header.  The bodies are this project's own: every compute call
// runs on the GPU through include/cllm_cuda.h; there is no CPU fallback.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

namespace cllm {

class ThreadPool;

enum class GgmlType : uint32_t {
    F32 = 0,
    F16 = 1,
    Q4_0 = 2,
    Q4_1 = 3,
    Q5_0 = 6,
    Q5_1 = 7,
    Q8_0 = 8,
    Q8_1 = 9,
    Q2_K = 10,
    Q3_K = 11,
    Q4_K = 12,
    Q5_K = 13,
    Q6_K = 14,
};

// IEEE fp16 bit pattern -> fp32, exact for every pattern (same results as the
// reference's half_to_float, quant.hpp:31-56).  Finite values: the 15 low bits
// shifted into an fp32 bit pattern equal the value times 2^-112 (also for
// subnormals, which become fp32 subnormals), so one exact multiply by 2^112
// restores them.  Inf and NaN keep their payload.
inline float half_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    const uint32_t em = h & 0x7FFFu;
    uint32_t bits;
    if (em >= 0x7C00u) {
        bits = sign | 0x7F800000u | ((em & 0x3FFu) << 13);
    } else {
        const uint32_t shifted = em << 13;
        float f;
        std::memcpy(&f, &shifted, sizeof f);
        f *= 5.192296858534828e+33f;  // 2^112
        std::memcpy(&bits, &f, sizeof bits);
        bits |= sign;
    }
    float out;
    std::memcpy(&out, &bits, sizeof out);
    return out;
}

// fp32 -> fp16 bit pattern with the reference's rounding (quant.hpp:58-87):
// normal results truncate the mantissa, subnormal results round to nearest
// even, overflow gives infinity, NaN becomes the quiet NaN 0x7E00 (signed).
inline uint16_t float_to_half(float f) {
    uint32_t x;
    std::memcpy(&x, &f, sizeof x);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t fexp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (fexp == 0xFFu) return static_cast<uint16_t>(sign | (mant ? 0x7E00u : 0x7C00u));
    const int e = static_cast<int>(fexp) - 112;  // fp16 biased exponent
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    if (e > 0) return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e) << 10) | (mant >> 13));
    if (e < -10) return static_cast<uint16_t>(sign);
    mant |= 0x800000u;
    const uint32_t shift = static_cast<uint32_t>(14 - e);
    const uint32_t half_ulp = 1u << (shift - 1);
    const uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t r = mant >> shift;
    if (rem > half_ulp || (rem == half_ulp && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
}

int block_size(GgmlType type);
size_t type_size(GgmlType type);

void dequantize_block(const void* src, float* dst, GgmlType type, int64_t n);
void dequantize_block_f16(const void* src, uint16_t* dst, GgmlType type, int64_t n);

struct QuantizedQ8_0 {
    std::vector<float> scales;
    std::vector<int8_t> qs;
    std::vector<int32_t> bsums;
    int64_t n = 0;
};

void quantize_row_q8_0(const float* x, QuantizedQ8_0& out, int64_t n);

bool has_vec_dot(GgmlType type);

float vec_dot_row(const void* w_row, GgmlType w_type, const QuantizedQ8_0& qx, int64_t n);

void matmul_quant(const float* x, const void* w, GgmlType type, const float* bias, int in_dim,
                  int out_dim, float* y, ThreadPool* pool = nullptr);

void matmul_quant_batch(const float* x, const void* w, GgmlType type, const float* bias, int in_dim,
                        int out_dim, int n_rows, float* y, ThreadPool* pool = nullptr);

}  // namespace cllm
