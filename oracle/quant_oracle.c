/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the quantized-matmul hot path.
 *
 * Only tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py
 * may load this code, and only as the checker.  The product library
 * (cllm_inference_b200/csrc) never links or calls it.
 *
 * A plain-C restatement of the cllm_inference algorithm (paths below are inside
 * the reference project).  Unlike the reference, which only returns the float
 * row sum, it also exposes the exact int32 per-block partial dot products, so
 * the GPU kernels can be checked bit-for-bit on the integer part and within a
 * tolerance on the float part.  The float accumulation follows the x86 AVX2
 * variants of vec_dot (the live code on x86 builds), statement for statement.
 *
 * Floating-point contraction: g++ 13 at the reference's flags (-std=c++20 -O3
 * -march=native, and equally -march=x86-64-v3) fuses every
 * `acc += a * b * c` / `acc -= a * b * c` of the vec_dot loops into
 * fma(a*b, c, acc) / fma(-(a*b), c, acc); nothing else changes bits (the
 * inner Q4_0/Q5_0/Q6_K terms are exact small integers).  This file writes
 * those fmaf() calls explicitly and is compiled with -ffp-contract=off so that
 * nothing else is fused; the result is bitwise equal to the reference build.
 *
 * Parity pinning: tests/test_oracle.py checks this file against
 *   - the known-answer dequant vectors of tests/quant_test.cpp:43-218,
 *   - committed golden fixtures produced by the reference build itself
 *     (tests/golden/make_golden.py, via oracle/_ref/libcllm_ref.so), and
 *   - oracle/_ref/libcllm_ref.so live, bitwise, when it is present.
 *
 * x86 conversion semantics restated on purpose:
 *   - quantize_row_q8_0 casts nearbyint(x*id) to int; on x86 a NaN (or any
 *     value outside int32) converts to INT32_MIN, which the clamp turns into
 *     -128 (quant.cpp:444-447).
 *   - The AVX2 Q8_0 and Q6_K dots use the _mm256_sign_epi8 trick
 *     (quant.cpp:517-525, :676-679): the activation byte is negated when the
 *     weight is negative, and -(-128) wraps to -128.  So for an activation of
 *     -128 (only produced by a NaN input) against a negative weight w the
 *     product is 128*w instead of -128*w.  orc_* reproduces that.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
    T_Q8_1 = 9, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14
};

/* quant.hpp:31-56 — exact fp16 bit pattern -> fp32. */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign << 31;
        } else {
            exp = 127 - 15 + 1;
            while ((mant & 0x400u) == 0) { mant <<= 1; --exp; }
            mant &= 0x3FFu;
            f = (sign << 31) | (exp << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        f = (sign << 31) | 0x7F800000u | (mant << 13);
    } else {
        f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &f, 4);
    return out;
}

/* quant.hpp:58-87 — fp32 -> fp16 bit pattern (used to build test blocks). */
uint16_t orc_float_to_half(float fv) {
    uint32_t x;
    memcpy(&x, &fv, 4);
    uint32_t sign = (x >> 16) & 0x8000u, mant = x & 0x007FFFFFu;
    int32_t exp = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    if (((x >> 23) & 0xFFu) == 0xFFu) return (uint16_t)(sign | (mant ? 0x7E00u : 0x7C00u));
    if (exp >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x00800000u;
        uint32_t t = (uint32_t)(14 - exp), a = (1u << (t - 1)) - 1u, b = (mant >> t) & 1u;
        return (uint16_t)(sign | ((mant + a + b) >> t));
    }
    return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

/* quant.cpp:340-369 */
int orc_block_size(int t) {
    switch (t) {
        case T_F32: case T_F16: return 1;
        case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: case T_Q8_1: return 32;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
    }
    return 1;
}

int64_t orc_type_size(int t) {
    switch (t) {
        case T_F32: return 4;   case T_F16: return 2;   case T_Q4_0: return 18; case T_Q4_1: return 20;
        case T_Q5_0: return 22; case T_Q5_1: return 24; case T_Q8_0: return 34; case T_Q8_1: return 36;
        case T_Q2_K: return 84; case T_Q3_K: return 110; case T_Q4_K: return 144;
        case T_Q5_K: return 176; case T_Q6_K: return 210;
    }
    return 0;
}

/* quant.cpp:1347-1357 */
int orc_has_vec_dot(int t) {
    return t == T_Q4_0 || t == T_Q5_0 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

static inline float f16at(const uint8_t* p) { return orc_half_to_float((uint16_t)(p[0] | (p[1] << 8))); }

/* quant.cpp:72-80 */
static inline void scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* x86 float->int conversion of quant.cpp:444 ((int)std::nearbyint(v)):
 * out-of-range and NaN give INT32_MIN ("integer indefinite"). */
static inline int x86_cvt(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT32_MIN;
    return (int)r;
}

/* quant.cpp:420-452 */
int orc_quantize_row_q8_0(const float* x, int64_t n, float* scales, int8_t* qs, int32_t* bsums) {
    if (n % 32 != 0) return -1;
    const int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float* xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        scales[b] = d;
        int32_t bsum = 0;
        for (int j = 0; j < 32; ++j) {
            float v = xb[j] * id;
            int q = x86_cvt(nearbyintf(v));
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            qs[b * 32 + j] = (int8_t)q;
            bsum += q;
        }
        bsums[b] = bsum;
    }
    return 0;
}

/* Product of a signed weight and an activation byte as the AVX2 sign trick
 * computes it (quant.cpp:517-525 and :676-679). */
static inline int32_t signmul(int w, int x) {
    if (w < 0 && x == -128) return 128 * w;
    return w * x;
}

/* Number of int32 partials one weight row produces: one per 32-element
 * activation block, two (one per 16-element half) for Q6_K. */
int64_t orc_partials_per_row(int t, int64_t n) {
    return t == T_Q6_K ? 2 * (n / 32) : n / 32;
}

/* Exact int32 partial dot products of one weight row against one quantized
 * activation row, in the integer semantics of the reference's live x86 path.
 * Q4_0  quant.cpp:758-777   P[b] = sum q4*qx, q4 = unsigned nibble
 * Q5_0  quant.cpp:864-893   P[b] = sum q5*qx, q5 = nibble | qh bit << 4
 * Q8_0  quant.cpp:534-547   P[b] = sum qw*qx (sign trick)
 * Q4_K  quant.cpp:549-590   P[8s+2p], P[8s+2p+1] from lo / hi nibbles of q[32p..]
 * Q5_K  quant.cpp:592-628   P[8s+k] = sum (lo4 | (qh>>k&1)<<4) * qx
 * Q6_K  quant.cpp:630-687   P[2b], P[2b+1] = halves (l<16, l>=16), q6-32 signed */
int orc_row_partials(const uint8_t* w, int t, const int8_t* qx, int64_t n, int32_t* P) {
    if (!orc_has_vec_dot(t) || n % orc_block_size(t) != 0) return -1;
    const int64_t nb = n / 32;
    switch (t) {
        case T_Q8_0:
            for (int64_t b = 0; b < nb; ++b, w += 34) {
                const int8_t* q = (const int8_t*)(w + 2);
                int32_t s = 0;
                for (int j = 0; j < 32; ++j) s += signmul(q[j], qx[b * 32 + j]);
                P[b] = s;
            }
            break;
        case T_Q4_0:
            for (int64_t b = 0; b < nb; ++b, w += 18) {
                const uint8_t* q = w + 2;
                int32_t s = 0;
                for (int j = 0; j < 16; ++j) {
                    s += (q[j] & 0xF) * qx[b * 32 + j];
                    s += (q[j] >> 4) * qx[b * 32 + j + 16];
                }
                P[b] = s;
            }
            break;
        case T_Q5_0:
            for (int64_t b = 0; b < nb; ++b, w += 22) {
                const uint32_t qh = (uint32_t)w[2] | ((uint32_t)w[3] << 8) | ((uint32_t)w[4] << 16) |
                                    ((uint32_t)w[5] << 24);
                const uint8_t* q = w + 6;
                int32_t s = 0;
                for (int j = 0; j < 16; ++j) {
                    s += (int)((q[j] & 0xF) | (((qh >> j) & 1) << 4)) * qx[b * 32 + j];
                    s += (int)((q[j] >> 4) | (((qh >> (j + 16)) & 1) << 4)) * qx[b * 32 + j + 16];
                }
                P[b] = s;
            }
            break;
        case T_Q4_K:
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 144) {
                const uint8_t* q = w + 16;
                for (int p = 0; p < 4; ++p) {
                    const int64_t b = sb * 8 + 2 * p;
                    int32_t lo = 0, hi = 0;
                    for (int l = 0; l < 32; ++l) {
                        lo += (q[32 * p + l] & 0xF) * qx[b * 32 + l];
                        hi += (q[32 * p + l] >> 4) * qx[(b + 1) * 32 + l];
                    }
                    P[b] = lo;
                    P[b + 1] = hi;
                }
            }
            break;
        case T_Q5_K:
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 176) {
                const uint8_t* qh = w + 16;
                const uint8_t* ql = w + 48;
                for (int k = 0; k < 8; ++k) {
                    const int64_t b = sb * 8 + k;
                    int32_t s = 0;
                    for (int l = 0; l < 32; ++l) {
                        int lo4 = (k & 1) ? (ql[(k / 2) * 32 + l] >> 4) : (ql[(k / 2) * 32 + l] & 0xF);
                        s += (lo4 | (((qh[l] >> k) & 1) << 4)) * qx[b * 32 + l];
                    }
                    P[b] = s;
                }
            }
            break;
        case T_Q6_K:
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 210) {
                for (int g = 0; g < 2; ++g) {
                    const uint8_t* ql = w + 64 * g;
                    const uint8_t* qh = w + 128 + 32 * g;
                    for (int sub = 0; sub < 4; ++sub) {
                        const int64_t b = sb * 8 + 4 * g + sub;
                        int32_t pa = 0, pb = 0;
                        for (int l = 0; l < 32; ++l) {
                            uint8_t raw = ql[(sub & 1) * 32 + l];
                            int lo4 = sub >= 2 ? (raw >> 4) : (raw & 0xF);
                            int q6 = (lo4 | (((qh[l] >> (2 * sub)) & 3) << 4)) - 32;
                            int32_t pr = signmul(q6, qx[b * 32 + l]);
                            if (l < 16) pa += pr; else pb += pr;
                        }
                        P[2 * b] = pa;
                        P[2 * b + 1] = pb;
                    }
                }
            }
            break;
    }
    return 0;
}

/* vec_dot_row from the partials, accumulating in the AVX2 statement order. */
static float row_from_partials(const uint8_t* w, int t, const float* dx, const int32_t* bs,
                               int64_t n, const int32_t* P) {
    const int64_t nb = n / 32;
    float acc = 0.0f;
    switch (t) {
        case T_Q8_0: /* quant.cpp:544 */
            for (int64_t b = 0; b < nb; ++b, w += 34) acc = fmaf(f16at(w) * dx[b], (float)P[b], acc);
            break;
        case T_Q4_0: /* quant.cpp:774 */
            for (int64_t b = 0; b < nb; ++b, w += 18)
                acc = fmaf(f16at(w) * dx[b], (float)P[b] - 8.0f * (float)bs[b], acc);
            break;
        case T_Q5_0: /* quant.cpp:890 */
            for (int64_t b = 0; b < nb; ++b, w += 22)
                acc = fmaf(f16at(w) * dx[b], (float)P[b] - 16.0f * (float)bs[b], acc);
            break;
        case T_Q4_K: /* quant.cpp:562-586 */
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 144) {
                const float d = f16at(w), dmin = f16at(w + 2);
                for (int p = 0; p < 4; ++p) {
                    uint8_t sc, m;
                    scale_min_k4(2 * p, w + 4, &sc, &m);
                    const float d1 = d * sc, m1 = dmin * m;
                    scale_min_k4(2 * p + 1, w + 4, &sc, &m);
                    const float d2 = d * sc, m2 = dmin * m;
                    const int64_t b = sb * 8 + 2 * p;
                    acc = fmaf(d1 * dx[b], (float)P[b], acc);
                    acc = fmaf(-(m1 * dx[b]), (float)bs[b], acc);
                    acc = fmaf(d2 * dx[b + 1], (float)P[b + 1], acc);
                    acc = fmaf(-(m2 * dx[b + 1]), (float)bs[b + 1], acc);
                }
            }
            break;
        case T_Q5_K: /* quant.cpp:609-625 */
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 176) {
                const float d = f16at(w), dmin = f16at(w + 2);
                for (int k = 0; k < 8; ++k) {
                    uint8_t sc, m;
                    scale_min_k4(k, w + 4, &sc, &m);
                    const float dk = d * sc, mk = dmin * m;
                    const int64_t b = sb * 8 + k;
                    acc = fmaf(dk * dx[b], (float)P[b], acc);
                    acc = fmaf(-(mk * dx[b]), (float)bs[b], acc);
                }
            }
            break;
        case T_Q6_K: /* quant.cpp:646-684 */
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 210) {
                const int8_t* sc = (const int8_t*)(w + 192);
                const float d = f16at(w + 208);
                for (int g = 0; g < 2; ++g)
                    for (int sub = 0; sub < 4; ++sub) {
                        const int64_t b = sb * 8 + 4 * g + sub;
                        const float sa = (float)sc[8 * g + 2 * sub], sbb = (float)sc[8 * g + 2 * sub + 1];
                        acc = fmaf(d * dx[b], sa * (float)P[2 * b] + sbb * (float)P[2 * b + 1], acc);
                    }
            }
            break;
    }
    return acc;
}

/* Sum of |term| over the float terms row_from_partials accumulates, in
 * double: the scale of the rounding error any summation order can make, used
 * by the tests as the denominator of the row tolerance. */
static double row_abs_terms(const uint8_t* w, int t, const float* dx, const int32_t* bs, int64_t n,
                            const int32_t* P) {
    const int64_t nb = n / 32;
    double s = 0.0;
    switch (t) {
        case T_Q8_0:
            for (int64_t b = 0; b < nb; ++b, w += 34) s += fabs((double)(f16at(w) * dx[b]) * P[b]);
            break;
        case T_Q4_0:
        case T_Q5_0: {
            const int ts = t == T_Q4_0 ? 18 : 22;
            const double off = t == T_Q4_0 ? 8.0 : 16.0;
            for (int64_t b = 0; b < nb; ++b, w += ts)
                s += fabs((double)(f16at(w) * dx[b]) * ((double)P[b] - off * bs[b]));
            break;
        }
        case T_Q4_K:
        case T_Q5_K: {
            const int ts = t == T_Q4_K ? 144 : 176;
            for (int64_t sb = 0; sb < n / 256; ++sb, w += ts) {
                const float d = f16at(w), dmin = f16at(w + 2);
                for (int k = 0; k < 8; ++k) {
                    uint8_t sc, m;
                    scale_min_k4(k, w + 4, &sc, &m);
                    const int64_t b = sb * 8 + k;
                    s += fabs((double)(d * sc * dx[b]) * P[b]) + fabs((double)(dmin * m * dx[b]) * bs[b]);
                }
            }
            break;
        }
        case T_Q6_K:
            for (int64_t sb = 0; sb < n / 256; ++sb, w += 210) {
                const int8_t* sc = (const int8_t*)(w + 192);
                const float d = f16at(w + 208);
                for (int g = 0; g < 2; ++g)
                    for (int sub = 0; sub < 4; ++sub) {
                        const int64_t b = sb * 8 + 4 * g + sub;
                        s += fabs((double)(d * dx[b]) *
                                  ((double)sc[8 * g + 2 * sub] * P[2 * b] + (double)sc[8 * g + 2 * sub + 1] * P[2 * b + 1]));
                    }
            }
            break;
    }
    return s;
}

/* quant.cpp:1359-1372.  Rows of up to 131072 elements (the tests use far less). */
int orc_vec_dot_row_abs(const uint8_t* w, int t, const float* dx, const int8_t* qx, const int32_t* bs,
                        int64_t n, float* out, double* abs_terms) {
    int32_t P[8192];
    if (!orc_has_vec_dot(t)) return -2;
    if (n % orc_block_size(t) != 0) return -1;
    if (orc_partials_per_row(t, n) > 8192) return -3;
    if (orc_row_partials(w, t, qx, n, P) != 0) return -1;
    *out = row_from_partials(w, t, dx, bs, n, P);
    if (abs_terms) *abs_terms = row_abs_terms(w, t, dx, bs, n, P);
    return 0;
}

int orc_vec_dot_row(const uint8_t* w, int t, const float* dx, const int8_t* qx, const int32_t* bs,
                    int64_t n, float* out) {
    return orc_vec_dot_row_abs(w, t, dx, qx, bs, n, out, 0);
}

/* quant.cpp:1433-1475 (vec_dot branch; n_rows == 1 is matmul_quant, :1374-1402).
 * Scratch: caller passes room for n_rows*(in_dim/32) floats+ints and n_rows*in_dim bytes. */
int orc_matmul_quant_batch(const float* x, const uint8_t* w, int t, const float* bias, int in_dim,
                           int out_dim, int n_rows, float* y, float* dx, int8_t* qx, int32_t* bs,
                           double* abs_terms) {
    if (n_rows <= 0) return 0;
    if (!orc_has_vec_dot(t)) return -2;
    if (in_dim % orc_block_size(t) != 0) return -1;
    const int64_t nb = in_dim / 32;
    const int64_t row_bytes = (in_dim / orc_block_size(t)) * orc_type_size(t);
    for (int r = 0; r < n_rows; ++r)
        orc_quantize_row_q8_0(x + (int64_t)r * in_dim, in_dim, dx + r * nb, qx + (int64_t)r * in_dim,
                              bs + r * nb);
    for (int j = 0; j < out_dim; ++j)
        for (int r = 0; r < n_rows; ++r) {
            float acc = 0.0f;
            double a = 0.0;
            int rc = orc_vec_dot_row_abs(w + (int64_t)j * row_bytes, t, dx + r * nb,
                                         qx + (int64_t)r * in_dim, bs + r * nb, in_dim, &acc, &a);
            if (rc != 0) return rc;
            if (bias) acc += bias[j];
            y[(int64_t)r * out_dim + j] = acc;
            if (abs_terms) abs_terms[(int64_t)r * out_dim + j] = a + (bias ? fabs((double)bias[j]) : 0.0);
        }
    return 0;
}

/* Dequantization of all thirteen types of dequantize_block (quant.cpp:371-389):
 * F32 :28-30, F16 :33-36, Q8_0 :38-50, Q4_0 :55-68, Q4_K :82-109, Q5_0 :114-131,
 * Q6_K :134-160, Q4_1 :163-177, Q5_1 :181-201, Q8_1 :204-215, Q2_K :219-249,
 * Q3_K :253-296, Q5_K :300-335.  Returns -2 for any other type. */
int orc_dequantize(const uint8_t* s, int t, int64_t n, float* dst) {
    switch (t) {
        case T_F32:
            memcpy(dst, s, (size_t)n * 4);
            return 0;
        case T_F16:
            for (int64_t i = 0; i < n; ++i) dst[i] = f16at(s + 2 * i);
            return 0;
        case T_Q4_1:
            for (int64_t i = 0; i < n; i += 32, s += 20) {
                const float d = f16at(s), m = f16at(s + 2);
                for (int j = 0; j < 16; ++j) {
                    if (i + j < n) dst[i + j] = d * (s[4 + j] & 0xF) + m;
                    if (i + j + 16 < n) dst[i + j + 16] = d * (s[4 + j] >> 4) + m;
                }
            }
            return 0;
        case T_Q5_1:
            for (int64_t i = 0; i < n; i += 32, s += 24) {
                const float d = f16at(s), m = f16at(s + 2);
                uint32_t qh = (uint32_t)s[4] | ((uint32_t)s[5] << 8) | ((uint32_t)s[6] << 16) |
                              ((uint32_t)s[7] << 24);
                for (int j = 0; j < 16; ++j) {
                    int q0 = (s[8 + j] & 0xF) | (((qh >> j) & 1) << 4);
                    int q1 = (s[8 + j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
                    if (i + j < n) dst[i + j] = d * q0 + m;
                    if (i + j + 16 < n) dst[i + j + 16] = d * q1 + m;
                }
            }
            return 0;
        case T_Q8_1:
            for (int64_t i = 0; i < n; i += 32, s += 36) {
                const float d = f16at(s);
                for (int j = 0; j < 32 && i + j < n; ++j) dst[i + j] = d * (int8_t)s[4 + j];
            }
            return 0;
        case T_Q2_K:
            for (int64_t i = 0; i < n; i += 256, s += 84) {
                const uint8_t* sc = s;
                const uint8_t* q = s + 16;
                const float d = f16at(s + 80), dmin = f16at(s + 82);
                int is = 0;
                for (int h = 0; h < 2; ++h, q += 32)
                    for (int j = 0; j < 4; ++j)
                        for (int part = 0; part < 2; ++part) {
                            const uint8_t b = sc[is++];
                            const float dl = d * (b & 0xF), ml = dmin * (b >> 4);
                            for (int l = 0; l < 16; ++l) {
                                const int64_t o = i + 128 * h + 32 * j + 16 * part + l;
                                if (o < n) dst[o] = dl * ((q[16 * part + l] >> (2 * j)) & 3) - ml;
                            }
                        }
            }
            return 0;
        case T_Q3_K:
            for (int64_t i = 0; i < n; i += 256, s += 110) {
                const uint8_t* hm = s;
                const uint8_t* q = s + 32;
                uint32_t a[4];
                memcpy(a, s + 96, 12);
                const float dall = f16at(s + 108);
                const uint32_t t2 = a[2];
                a[2] = ((a[0] >> 4) & 0x0f0f0f0fu) | (((t2 >> 4) & 0x03030303u) << 4);
                a[3] = ((a[1] >> 4) & 0x0f0f0f0fu) | (((t2 >> 6) & 0x03030303u) << 4);
                a[0] = (a[0] & 0x0f0f0f0fu) | (((t2 >> 0) & 0x03030303u) << 4);
                a[1] = (a[1] & 0x0f0f0f0fu) | (((t2 >> 2) & 0x03030303u) << 4);
                const int8_t* scl = (const int8_t*)a;
                int is = 0;
                uint8_t m = 1;
                for (int h = 0; h < 2; ++h, q += 32)
                    for (int j = 0; j < 4; ++j, m = (uint8_t)(m << 1))
                        for (int part = 0; part < 2; ++part) {
                            const float dl = dall * (scl[is++] - 32);
                            for (int l = 0; l < 16; ++l) {
                                const int idx = 16 * part + l;
                                const int64_t o = i + 128 * h + 32 * j + idx;
                                if (o < n) dst[o] = dl * (((q[idx] >> (2 * j)) & 3) - ((hm[idx] & m) ? 0 : 4));
                            }
                        }
            }
            return 0;
        case T_Q8_0:
            for (int64_t i = 0; i < n; i += 32, s += 34) {
                float d = f16at(s);
                for (int j = 0; j < 32 && i + j < n; ++j) dst[i + j] = d * (int8_t)s[2 + j];
            }
            return 0;
        case T_Q4_0:
            for (int64_t i = 0; i < n; i += 32, s += 18) {
                float d = f16at(s);
                for (int j = 0; j < 16; ++j) {
                    if (i + j < n) dst[i + j] = d * ((s[2 + j] & 0xF) - 8);
                    if (i + j + 16 < n) dst[i + j + 16] = d * ((s[2 + j] >> 4) - 8);
                }
            }
            return 0;
        case T_Q5_0:
            for (int64_t i = 0; i < n; i += 32, s += 22) {
                float d = f16at(s);
                uint32_t qh = (uint32_t)s[2] | ((uint32_t)s[3] << 8) | ((uint32_t)s[4] << 16) |
                              ((uint32_t)s[5] << 24);
                for (int j = 0; j < 16; ++j) {
                    int q0 = (s[6 + j] & 0xF) | (((qh >> j) & 1) << 4);
                    int q1 = (s[6 + j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
                    if (i + j < n) dst[i + j] = d * (q0 - 16);
                    if (i + j + 16 < n) dst[i + j + 16] = d * (q1 - 16);
                }
            }
            return 0;
        case T_Q4_K:
            for (int64_t i = 0; i < n; i += 256, s += 144) {
                const float d = f16at(s), dmin = f16at(s + 2);
                const uint8_t* q = s + 16;
                for (int p = 0; p < 4; ++p, q += 32) {
                    uint8_t sc, m;
                    scale_min_k4(2 * p, s + 4, &sc, &m);
                    const float d1 = d * sc, m1 = dmin * m;
                    scale_min_k4(2 * p + 1, s + 4, &sc, &m);
                    const float d2 = d * sc, m2 = dmin * m;
                    for (int l = 0; l < 32; ++l) {
                        if (i + 64 * p + l < n) dst[i + 64 * p + l] = d1 * (q[l] & 0xF) - m1;
                        if (i + 64 * p + 32 + l < n) dst[i + 64 * p + 32 + l] = d2 * (q[l] >> 4) - m2;
                    }
                }
            }
            return 0;
        case T_Q5_K:
            for (int64_t i = 0; i < n; i += 256, s += 176) {
                const float d = f16at(s), dmin = f16at(s + 2);
                const uint8_t* qh = s + 16;
                const uint8_t* ql = s + 48;
                for (int p = 0; p < 4; ++p, ql += 32) {
                    uint8_t sc, m;
                    scale_min_k4(2 * p, s + 4, &sc, &m);
                    const float d1 = d * sc, m1 = dmin * m;
                    scale_min_k4(2 * p + 1, s + 4, &sc, &m);
                    const float d2 = d * sc, m2 = dmin * m;
                    const uint8_t u1 = (uint8_t)(1u << (2 * p)), u2 = (uint8_t)(2u << (2 * p));
                    for (int l = 0; l < 32; ++l) {
                        if (i + 64 * p + l < n)
                            dst[i + 64 * p + l] = d1 * ((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
                        if (i + 64 * p + 32 + l < n)
                            dst[i + 64 * p + 32 + l] = d2 * ((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
                    }
                }
            }
            return 0;
        case T_Q6_K:
            for (int64_t i = 0; i < n; i += 256, s += 210) {
                const uint8_t* ql = s;
                const uint8_t* qh = s + 128;
                const int8_t* sc = (const int8_t*)(s + 192);
                const float d = f16at(s + 208);
                for (int g = 0; g < 2; ++g, ql += 64, qh += 32, sc += 8) {
                    for (int l = 0; l < 32; ++l) {
                        int is = l / 16;
                        int q1 = (ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4);
                        int q2 = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4);
                        int q3 = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                        int q4 = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
                        int64_t o = i + 128 * g + l;
                        if (o < n) dst[o] = d * sc[is + 0] * (q1 - 32);
                        if (o + 32 < n) dst[o + 32] = d * sc[is + 2] * (q2 - 32);
                        if (o + 64 < n) dst[o + 64] = d * sc[is + 4] * (q3 - 32);
                        if (o + 96 < n) dst[o + 96] = d * sc[is + 6] * (q4 - 32);
                    }
                }
            }
            return 0;
    }
    return -2;
}

/* quant.cpp:1404-1430 — matmul_quant's fallback for types without an integer
 * dot kernel: every row is dequantized in chunks of 512 values (rounded down to
 * whole blocks) and accumulated as acc = bias (or 0), then acc += x[i] * w[i]
 * in element order, the product rounded before the add (the reference build
 * does not fuse this statement; checked bitwise against it).  abs_terms (may be NULL) receives
 * |bias| + sum |x[i] * w[i]| per output (the tolerance denominator).  Rows of
 * up to 65536 values. */
int orc_matmul_fallback(const float* x, const uint8_t* w, int t, const float* bias, int in_dim, int out_dim,
                        int n_rows, float* y, double* abs_terms) {
    static float buf[65536];
    const int bsz = orc_block_size(t);
    if (orc_type_size(t) == 0) return -2;
    if (in_dim % bsz != 0) return -1;
    if (in_dim > 65536) return -3;
    const int64_t row_bytes = (in_dim / bsz) * orc_type_size(t);
    for (int j = 0; j < out_dim; ++j) {
        if (orc_dequantize(w + (int64_t)j * row_bytes, t, in_dim, buf) != 0) return -2;
        for (int r = 0; r < n_rows; ++r) {
            const float* xr = x + (int64_t)r * in_dim;
            float acc = bias ? bias[j] : 0.0f;
            double a = bias ? fabs((double)bias[j]) : 0.0;
            for (int i = 0; i < in_dim; ++i) {
                acc = acc + xr[i] * buf[i];
                a += fabs((double)xr[i] * (double)buf[i]);
            }
            y[(int64_t)r * out_dim + j] = acc;
            if (abs_terms) abs_terms[(int64_t)r * out_dim + j] = a;
        }
    }
    return 0;
}
