// Decode-path kernels: quantized-weight GEMV for M = 1..8 activation rows.
//
// Work decomposition.  A weight row is cut into "units" of 64 weights (two
// 32-value activation blocks) for the 256-value K types and of one 32-value
// block for Q4_0/Q5_0/Q8_0.  Lane l of a warp takes units l, l+32·WPR, ...
// of its row, forms the exact int32 partial of each 32-value block with
// dp4a, applies the block's float scales with the reference's per-block FMA
// (acc = fma(d_w·d_x, P, acc)), and the lanes' sums are reduced with shuffles.
//
// Reference algorithms (cllm_inference src/core/quant.cpp):
//   Q8_0 :534-547   Q4_0 :758-777   Q5_0 :864-893
//   Q4_K :549-590   Q5_K :592-628   Q6_K :630-687   matmul rows :1374-1475
//
// Two loaders share the unit code:
//   * gemv_tma_kernel — persistent CTAs stream tiles of R whole rows into a
//     shared-memory ring with 1-D bulk copies (cp.async.bulk, the TMA engine,
//     no multicast) and mbarrier transaction counts, S stages deep;
//   * gemv_direct_kernel — plain global loads, for weight rows whose base or
//     stride is not 16-byte aligned (bulk copies need 16-byte multiples).
#pragma once
#include "common.cuh"

namespace cllm {

struct GemvParams {
    const uint8_t* w;     // weight matrix, out_dim rows of row_bytes
    int64_t row_bytes;
    int K;                // in_dim
    int N;                // out_dim
    const float* x;       // FUSED only: raw fp32 activations [M][K], quantized in shared memory
    const int8_t* qx;     // quantized activations [M][K]
    const float* dx;      // per-block scales [M][K/32]
    const int32_t* bs;    // per-block sums [M][K/32]
    const uint8_t* fl;    // per-block "holds -128" flags [M][K/32]
    const float* bias;    // [N] or nullptr
    float* y;             // [M][N]
    int32_t* partials;    // EMIT only: [N][parts per row] for activation row 0
    int rows_per_tile;    // R
    int wpr;              // warps per row (R * wpr == warps per CTA)
    int num_tiles;
    int stages;
    uint32_t stage_bytes;
};

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvSmemHeader = 1024;  // mbarriers + reduction scratch, before the stage ring

template <int T> struct TypeInfo;
template <> struct TypeInfo<kQ4_0> { static constexpr int kBlock = 32, kBytes = 18, kUnitsPerBlock = 1; };
template <> struct TypeInfo<kQ5_0> { static constexpr int kBlock = 32, kBytes = 22, kUnitsPerBlock = 1; };
template <> struct TypeInfo<kQ8_0> { static constexpr int kBlock = 32, kBytes = 34, kUnitsPerBlock = 1; };
template <> struct TypeInfo<kQ4_K> { static constexpr int kBlock = 256, kBytes = 144, kUnitsPerBlock = 4; };
template <> struct TypeInfo<kQ5_K> { static constexpr int kBlock = 256, kBytes = 176, kUnitsPerBlock = 4; };
template <> struct TypeInfo<kQ6_K> { static constexpr int kBlock = 256, kBytes = 210, kUnitsPerBlock = 4; };

__host__ __device__ inline int units_per_row(int type, int K) {
    return (type == kQ4_K || type == kQ5_K || type == kQ6_K) ? K / 64 : K / 32;
}

// Sum of 256*w over the bytes where the weight byte w is negative and the
// activation byte is -128: the difference between the reference's AVX2
// sign-trick product (quant.cpp:517-525, :676-679) and the exact product.
__device__ __forceinline__ int signtrick_fix(int wq, int xq) {
    int fix = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int wb = (int)(int8_t)(wq >> (8 * k));
        const int xb = (int)(int8_t)(xq >> (8 * k));
        fix += (wb < 0 && xb == -128) ? 256 * wb : 0;
    }
    return fix;
}

// Q4_K / Q5_K 6-bit scales and mins of sub-blocks 2p and 2p+1
// (get_scale_min_k4, quant.cpp:72-80), from the 12 packed bytes as h1..h3.
__device__ __forceinline__ void kquant_scale_pair(uint32_t h1, uint32_t h2, uint32_t h3, int p,
                                                  float d, float dmin, float& d1, float& m1,
                                                  float& d2, float& m2) {
    uint32_t scw, mw;
    if (p < 2) {
        scw = h1 & 0x3F3F3F3Fu;
        mw = h2 & 0x3F3F3F3Fu;
    } else {
        scw = (h3 & 0x0F0F0F0Fu) | ((h1 >> 2) & 0x30303030u);
        mw = ((h3 >> 4) & 0x0F0F0F0Fu) | ((h2 >> 2) & 0x30303030u);
    }
    const int sh = (p & 1) * 16;
    d1 = d * (float)((scw >> sh) & 0xFFu);
    d2 = d * (float)((scw >> (sh + 8)) & 0xFFu);
    m1 = dmin * (float)((mw >> sh) & 0xFFu);
    m2 = dmin * (float)((mw >> (sh + 8)) & 0xFFu);
}

// Six-bit quant v in [0,63] per byte -> (v - 32) as int8 per byte, without
// inter-byte borrows: flip bit 5, then copy it into bits 6 and 7.
__device__ __forceinline__ int q6_to_s8(uint32_t v) {
    const uint32_t u = v ^ 0x20202020u;
    const uint32_t s = u & 0x20202020u;
    return (int)(u + 6u * s);
}

// Four bits (bits 0..3 of h) spread to bit 4 of each byte.
__device__ __forceinline__ uint32_t spread4_to_bit4(uint32_t h) {
    return (((h & 0xFu) * 0x00204081u) & 0x01010101u) << 4;
}

// Quantized activations in global memory (written by quantize_q8_0_kernel or
// passed in by the caller).
struct ActGmem {
    const int8_t* qx;
    const float* dx;
    const int32_t* bs;
    int K, nb;
    __device__ __forceinline__ void x32(int t, int b, int (&x)[8]) const { load_act32(qx + (int64_t)t * K, b, x); }
    __device__ __forceinline__ float dx1(int t, int b) const { return __ldg(dx + (int64_t)t * nb + b); }
    __device__ __forceinline__ int bs1(int t, int b) const { return __ldg(bs + (int64_t)t * nb + b); }
    __device__ __forceinline__ float2 dx2(int t, int b) const {
        return __ldg(reinterpret_cast<const float2*>(dx + (int64_t)t * nb + b));
    }
    __device__ __forceinline__ int2 bs2(int t, int b) const {
        return __ldg(reinterpret_cast<const int2*>(bs + (int64_t)t * nb + b));
    }
    // Q6_K unit: scales of blocks b and b + 2
    __device__ __forceinline__ float2 dx_q6(int t, int b) const { return make_float2(dx1(t, b), dx1(t, b + 2)); }
};

// Quantized activations in this CTA's shared memory (fused quantization).
//
// Layout, chosen so that the lane access pattern of every unit map is free of
// shared-memory bank conflicts:
//   * block order: activation block b is stored at position perm(b).  For
//     Q6_K, whose unit pairs sub-blocks p and p+2 of a 128-value group,
//     sub-blocks (0,1,2,3) of each group are stored as (0,2,1,3), so a unit's
//     two blocks are adjacent; every other type keeps b.
//   * row stride kp = K rounded up to 128 bytes;
//   * 16-byte slot swizzle inside each 128-byte line: slot ^= (slot >> 3) & 7.
// Lane u of a warp reads 64 contiguous logical bytes (or 32 for the
// 32-value types); with the swizzle the eight lanes of each quarter-warp hit
// eight different 16-byte bank groups.
template <int TYPE>
__host__ __device__ __forceinline__ int act_perm(int b) {
    if constexpr (TYPE == kQ6_K) {
        const int sub = b & 3;
        return (b & ~3) | ((sub & 1) << 1) | (sub >> 1);
    } else {
        return b;
    }
}

__host__ __device__ __forceinline__ uint32_t act_swizzle(uint32_t off) {
    const uint32_t slot = off >> 4;
    return ((slot ^ ((slot >> 3) & 7u)) << 4) | (off & 15u);
}

__host__ __device__ __forceinline__ int act_row_stride(int K) { return (K + 127) & ~127; }

__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

template <int TYPE>
struct ActSmem {
    uint32_t qx, dx, bs;  // shared addresses: [M][kp] int8 (swizzled), [M][nb] f32, [M][nb] i32
    int kp, nb;
    __device__ __forceinline__ void x32(int t, int b, int (&x)[8]) const {
        const uint32_t row = qx + (uint32_t)(t * kp);
        const uint32_t off = 32u * (uint32_t)act_perm<TYPE>(b);
        const uint4 v0 = lds128(row + act_swizzle(off)), v1 = lds128(row + act_swizzle(off + 16));
        x[0] = (int)v0.x; x[1] = (int)v0.y; x[2] = (int)v0.z; x[3] = (int)v0.w;
        x[4] = (int)v1.x; x[5] = (int)v1.y; x[6] = (int)v1.z; x[7] = (int)v1.w;
    }
    __device__ __forceinline__ float dx1(int t, int b) const {
        return __uint_as_float(lds32(dx + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b))));
    }
    __device__ __forceinline__ int bs1(int t, int b) const {
        return (int)lds32(bs + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b)));
    }
    // blocks b and its unit partner, stored adjacently (perm(b) even)
    __device__ __forceinline__ float2 dx2(int t, int b) const {
        const uint2 v = lds64(dx + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b)));
        return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    }
    __device__ __forceinline__ int2 bs2(int t, int b) const {
        const uint2 v = lds64(bs + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b)));
        return make_int2((int)v.x, (int)v.y);
    }
    // Q6_K unit: scales of blocks b and b + 2, adjacent after the permutation
    __device__ __forceinline__ float2 dx_q6(int t, int b) const { return dx2(t, b); }
};

template <int TYPE, int M, bool EMIT, int ALIGN, class Src, class Act>
__device__ __forceinline__ void gemv_unit(const Src& src, const Act& act, int u, const GemvParams& p,
                                          float (&acc)[M], int32_t* prow, uint32_t quirk) {
    if constexpr (TYPE == kQ4_K) {
        const int s = u >> 2, q = u & 3;
        const uint32_t o = 144u * (uint32_t)s;
        uint32_t h[4], w[8];
        src.template words<4, ALIGN>(o, h);
        src.template words<8, ALIGN>(o + 16 + 32 * q, w);
        float d1, m1, d2, m2;
        kquant_scale_pair(h[1], h[2], h[3], q, h2f(h[0]), h2f(h[0] >> 16), d1, m1, d2, m2);
        int lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (int)(w[i] & 0x0F0F0F0Fu);
            hi[i] = (int)((w[i] >> 4) & 0x0F0F0F0Fu);
        }
        const int b0 = 8 * s + 2 * q;
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int xa[8], xb[8];
            act.x32(t, b0, xa);
            act.x32(t, b0 + 1, xb);
            int P0 = 0, P1 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                P0 = dp4a(lo[i], xa[i], P0);
                P1 = dp4a(hi[i], xb[i], P1);
            }
            if constexpr (EMIT) { prow[b0] = P0; prow[b0 + 1] = P1; }
            const float2 dd = act.dx2(t, b0);
            const int2 ss = act.bs2(t, b0);
            acc[t] = fmaf(d1 * dd.x, i2f_exact(P0), acc[t]);
            acc[t] = fmaf(-(m1 * dd.x), i2f_exact(ss.x), acc[t]);
            acc[t] = fmaf(d2 * dd.y, i2f_exact(P1), acc[t]);
            acc[t] = fmaf(-(m2 * dd.y), i2f_exact(ss.y), acc[t]);
        }
    } else if constexpr (TYPE == kQ5_K) {
        const int s = u >> 2, q = u & 3;
        const uint32_t o = 176u * (uint32_t)s;
        uint32_t h[4], qh[8], ql[8];
        src.template words<4, ALIGN>(o, h);
        src.template words<8, ALIGN>(o + 16, qh);
        src.template words<8, ALIGN>(o + 48 + 32 * q, ql);
        float d1, m1, d2, m2;
        kquant_scale_pair(h[1], h[2], h[3], q, h2f(h[0]), h2f(h[0] >> 16), d1, m1, d2, m2);
        const int k0 = 2 * q;
        int q0[8], q1[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            q0[i] = (int)((ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> k0) & 0x01010101u) << 4));
            q1[i] = (int)(((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (k0 + 1)) & 0x01010101u) << 4));
        }
        const int b0 = 8 * s + k0;
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int xa[8], xb[8];
            act.x32(t, b0, xa);
            act.x32(t, b0 + 1, xb);
            int P0 = 0, P1 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                P0 = dp4a(q0[i], xa[i], P0);
                P1 = dp4a(q1[i], xb[i], P1);
            }
            if constexpr (EMIT) { prow[b0] = P0; prow[b0 + 1] = P1; }
            const float2 dd = act.dx2(t, b0);
            const int2 ss = act.bs2(t, b0);
            acc[t] = fmaf(d1 * dd.x, i2f_exact(P0), acc[t]);
            acc[t] = fmaf(-(m1 * dd.x), i2f_exact(ss.x), acc[t]);
            acc[t] = fmaf(d2 * dd.y, i2f_exact(P1), acc[t]);
            acc[t] = fmaf(-(m2 * dd.y), i2f_exact(ss.y), acc[t]);
        }
    } else if constexpr (TYPE == kQ6_K) {
        // unit = (super-block s, group g, pair pr): sub-blocks pr and pr+2 of group g
        const int s = u >> 2, g = (u >> 1) & 1, pr = u & 1;
        const uint32_t o = 210u * (uint32_t)s;
        uint32_t L[8], H[8], SC[2];
        src.template words<8, 2>(o + 64 * g + 32 * pr, L);
        src.template words<8, 2>(o + 128 + 32 * g, H);
        src.template words<2, 2>(o + 192 + 8 * g, SC);
        const float d = h2f(src.u16(o + 208));
        const int sha = 16 * pr;
        const float sA0 = (float)(int)(int8_t)(SC[0] >> sha), sA1 = (float)(int)(int8_t)(SC[0] >> (sha + 8));
        const float sB0 = (float)(int)(int8_t)(SC[1] >> sha), sB1 = (float)(int)(int8_t)(SC[1] >> (sha + 8));
        // six-bit quants v in [0,63] per byte; the weight is v - 32
        uint32_t va[8], vb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            va[i] = (L[i] & 0x0F0F0F0Fu) | ((H[i] << (4 - 2 * pr)) & 0x30303030u);
            vb[i] = ((L[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> (2 * pr)) & 0x30303030u);
        }
        // Few activation rows: form sum(v*x) and subtract 32*sum(x) per half
        // (four dp4a per half) instead of re-biasing every weight byte; the
        // integers are identical.  More rows: re-bias the weights once.
        constexpr bool kOffset = M <= 2;
        int qa[8], qb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qa[i] = kOffset ? (int)va[i] : q6_to_s8(va[i]);
            qb[i] = kOffset ? (int)vb[i] : q6_to_s8(vb[i]);
        }
        const int bA = 8 * s + 4 * g + pr, bB = bA + 2;
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int xa[8], xb[8];
            act.x32(t, bA, xa);
            act.x32(t, bB, xb);
            int PA0 = 0, PA1 = 0, PB0 = 0, PB1 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                PA0 = dp4a(qa[i], xa[i], PA0);
                PA1 = dp4a(qa[i + 4], xa[i + 4], PA1);
                PB0 = dp4a(qb[i], xb[i], PB0);
                PB1 = dp4a(qb[i + 4], xb[i + 4], PB1);
            }
            if constexpr (kOffset) {
                int hA0 = 0, hA1 = 0, hB0 = 0, hB1 = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    hA0 = dp4a(xa[i], 0x20202020, hA0);
                    hA1 = dp4a(xa[i + 4], 0x20202020, hA1);
                    hB0 = dp4a(xb[i], 0x20202020, hB0);
                    hB1 = dp4a(xb[i + 4], 0x20202020, hB1);
                }
                PA0 -= hA0; PA1 -= hA1; PB0 -= hB0; PB1 -= hB1;
            }
            if ((quirk >> t) & 1u) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    PA0 += signtrick_fix(q6_to_s8(va[i]), xa[i]);
                    PA1 += signtrick_fix(q6_to_s8(va[i + 4]), xa[i + 4]);
                    PB0 += signtrick_fix(q6_to_s8(vb[i]), xb[i]);
                    PB1 += signtrick_fix(q6_to_s8(vb[i + 4]), xb[i + 4]);
                }
            }
            if constexpr (EMIT) {
                prow[2 * bA] = PA0; prow[2 * bA + 1] = PA1;
                prow[2 * bB] = PB0; prow[2 * bB + 1] = PB1;
            }
            const float2 dxAB = act.dx_q6(t, bA);
            // sc*P products are exact integers below 2^24, as in the reference
            acc[t] = fmaf(d * dxAB.x, sA0 * i2f_exact(PA0) + sA1 * i2f_exact(PA1), acc[t]);
            acc[t] = fmaf(d * dxAB.y, sB0 * i2f_exact(PB0) + sB1 * i2f_exact(PB1), acc[t]);
        }
    } else if constexpr (TYPE == kQ8_0) {
        const int b = u;
        const uint32_t o = 34u * (uint32_t)b;
        uint32_t q[8];
        src.template words<8, 2>(o + 2, q);
        const float d = h2f(src.u16(o));
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int x[8];
            act.x32(t, b, x);
            int P = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) P = dp4a((int)q[i], x[i], P);
            if ((quirk >> t) & 1u) {
#pragma unroll
                for (int i = 0; i < 8; ++i) P += signtrick_fix((int)q[i], x[i]);
            }
            if constexpr (EMIT) prow[b] = P;
            acc[t] = fmaf(d * act.dx1(t, b), i2f_exact(P), acc[t]);
        }
    } else if constexpr (TYPE == kQ4_0) {
        const int b = u;
        const uint32_t o = 18u * (uint32_t)b;
        uint32_t q[4];
        src.template words<4, 2>(o + 2, q);
        const float d = h2f(src.u16(o));
        int lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (int)(q[i] & 0x0F0F0F0Fu);
            hi[i] = (int)((q[i] >> 4) & 0x0F0F0F0Fu);
        }
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int x[8];
            act.x32(t, b, x);
            int P = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) P = dp4a(hi[i], x[4 + i], dp4a(lo[i], x[i], P));
            if constexpr (EMIT) prow[b] = P;
            acc[t] = fmaf(d * act.dx1(t, b), i2f_exact(P - 8 * act.bs1(t, b)), acc[t]);
        }
    } else if constexpr (TYPE == kQ5_0) {
        const int b = u;
        const uint32_t o = 22u * (uint32_t)b;
        uint32_t qh[1], q[4];
        src.template words<1, 2>(o + 2, qh);
        src.template words<4, 2>(o + 6, q);
        const float d = h2f(src.u16(o));
        int lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (int)((q[i] & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (4 * i)));
            hi[i] = (int)(((q[i] >> 4) & 0x0F0F0F0Fu) | spread4_to_bit4(qh[0] >> (16 + 4 * i)));
        }
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int x[8];
            act.x32(t, b, x);
            int P = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) P = dp4a(hi[i], x[4 + i], dp4a(lo[i], x[i], P));
            if constexpr (EMIT) prow[b] = P;
            acc[t] = fmaf(d * act.dx1(t, b), i2f_exact(P - 16 * act.bs1(t, b)), acc[t]);
        }
    }
}

// OR of the per-block -128 flags of each activation row (bit t = row t).
// Only Q8_0 and Q6_K need it.  Must be called by all threads of the CTA.
template <int TYPE, int M>
__device__ __forceinline__ uint32_t gemv_quirk_mask(const GemvParams& p) {
    if constexpr (TYPE != kQ8_0 && TYPE != kQ6_K) {
        return 0u;
    } else {
        const int nb = p.K >> 5;
        uint32_t mask = 0;
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int any = 0;
            for (int i = threadIdx.x; i < nb; i += blockDim.x) any |= p.fl[(int64_t)t * nb + i];
            if (__syncthreads_or(any)) mask |= 1u << t;
        }
        return mask;
    }
}

// One row-slice of a tile: warp `w` covers row r = w / wpr, slice w % wpr.
template <int TYPE, int M, bool EMIT, int ALIGN, class Src, class Act>
__device__ __forceinline__ void gemv_row_slice(const Src& src, const Act& act, int row,
                                               const GemvParams& p, int slice, uint32_t quirk,
                                               float (&acc)[M]) {
    const int lane = threadIdx.x & 31;
    const int upr = units_per_row(TYPE, p.K);
    int32_t* prow = nullptr;
    if constexpr (EMIT) {
        const int ppr = (TYPE == kQ6_K) ? 2 * (p.K >> 5) : (p.K >> 5);
        prow = p.partials + (int64_t)row * ppr;
    }
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = 0.0f;
    for (int u = slice * 32 + lane; u < upr; u += 32 * p.wpr)
        gemv_unit<TYPE, M, EMIT, ALIGN>(src, act, u, p, acc, prow, quirk);
    warp_sum<M>(acc);
}

template <int M>
__device__ __forceinline__ void gemv_store_partial(float* red, int warp, const float (&acc)[M]) {
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int t = 0; t < M; ++t) red[warp * M + t] = acc[t];
    }
}

// y = sum of the wpr warp partials of each row (in warp order) + bias.
template <int M>
__device__ __forceinline__ void gemv_combine(const float* red, int row0, int rows,
                                             const GemvParams& p) {
    const int i = threadIdx.x;
    if (i < rows * M) {
        const int r = i / M, t = i - r * M;
        float s = 0.0f;
        for (int k = 0; k < p.wpr; ++k) s += red[(r * p.wpr + k) * M + t];
        const int j = row0 + r;
        if (p.bias) s += p.bias[j];
        p.y[(int64_t)t * p.N + j] = s;
    }
}

template <int M>
__device__ __forceinline__ void gemv_store_row(int j, const float (&acc)[M], const GemvParams& p) {
    if ((threadIdx.x & 31) == 0) {
        const float b = p.bias ? p.bias[j] : 0.0f;
#pragma unroll
        for (int t = 0; t < M; ++t) p.y[(int64_t)t * p.N + j] = acc[t] + b;
    }
}

// Quantize x [M][K] into this CTA's shared memory (quantize_row_q8_0,
// quant.cpp:420-452, the same IEEE steps as quantize_q8_0_kernel).  Eight
// lanes share a 32-value block, one float4 each; every thread issues the
// loads of four blocks before reducing them, so the prologue costs about one
// L2 round trip per four blocks per group.  x must be 16-byte aligned.
// Returns the per-row "holds -128" mask.  Called by all threads.
template <int M, int TYPE>
__device__ __forceinline__ uint32_t quantize_to_smem(const float* __restrict__ x, int K,
                                                     uint8_t* qs, float* dx, int* bs) {
    const int kp = act_row_stride(K);
    constexpr int kGroups = kGemvThreads / 8;  // 32 blocks in flight per pass
    constexpr int kUnroll = 4;
    const int g = threadIdx.x >> 3, sub = threadIdx.x & 7;
    const int nb = K >> 5;
    const int total = M * nb;
    uint32_t mask = 0;
    for (int base = 0; base < total; base += kGroups * kUnroll) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int blk = base + g + kGroups * u;
            if (blk < total) {
                const int t = blk / nb, b = blk - t * nb;
                v[u] = __ldg(reinterpret_cast<const float4*>(x + (int64_t)t * K + 32 * b + 4 * sub));
            } else {
                v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int blk = base + g + kGroups * u;  // uniform within each 8-lane group
            const float a0 = fabsf(v[u].x), a1 = fabsf(v[u].y), a2 = fabsf(v[u].z), a3 = fabsf(v[u].w);
            // max over non-NaN values, as `if (a > amax) amax = a` from 0
            float amax = (a0 > 0.0f) ? a0 : 0.0f;
            amax = (a1 > amax) ? a1 : amax;
            amax = (a2 > amax) ? a2 : amax;
            amax = (a3 > amax) ? a3 : amax;
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            const float d = amax / 127.0f;
            const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
            int q[4];
            const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float r = rintf(vv[e] * id);
                int qi = (r >= -2147483648.0f && r < 2147483648.0f) ? (int)r : INT32_MIN;
                q[e] = qi > 127 ? 127 : (qi < -128 ? -128 : qi);
            }
            int sum = q[0] + q[1] + q[2] + q[3];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
            if (blk < total) {
                const int t = blk / nb, b = blk - t * nb;
                const uint32_t packed = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) |
                                        ((uint32_t)(q[2] & 0xFF) << 16) | ((uint32_t)(q[3] & 0xFF) << 24);
                const int pb = act_perm<TYPE>(b);
                *reinterpret_cast<uint32_t*>(qs + t * kp + act_swizzle(32u * pb + 4u * sub)) = packed;
                if ((q[0] == -128) | (q[1] == -128) | (q[2] == -128) | (q[3] == -128)) mask |= 1u << t;
                if (sub == 0) {
                    dx[t * nb + pb] = d;
                    bs[t * nb + pb] = sum;
                }
            }
        }
    }
    uint32_t all = 0;
#pragma unroll
    for (int t = 0; t < M; ++t)
        if (__syncthreads_or((int)((mask >> t) & 1u))) all |= 1u << t;
    return all;
}

// Shared-memory bytes the fused quantization needs for M rows of K.
__host__ __device__ inline uint32_t fused_act_bytes(int M, int K) {
    const uint32_t nb = (uint32_t)K / 32u;
    return (uint32_t)(M * act_row_stride(K)) + 8u * (uint32_t)M * nb;
}

template <int TYPE, int M, bool EMIT, bool FUSED>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_tma_kernel(const GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t bar0 = sbase;                              // stages * 8 bytes
    float* red = reinterpret_cast<float*>(smem + 128);        // 2 x kGemvWarps x M floats
    int* s_abort = reinterpret_cast<int*>(smem + 64);
    const int nb = p.K >> 5;
    const uint32_t act_bytes = FUSED ? (fused_act_bytes(M, p.K) + 127u) / 128u * 128u : 0u;
    const uint32_t ring = sbase + kGemvSmemHeader + act_bytes;
    const int S = p.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    auto issue = [&](int tile, int stg) {
        const int row0 = tile * p.rows_per_tile;
        const int rows = min(p.rows_per_tile, p.N - row0);
        const uint32_t bytes = (uint32_t)(rows * p.row_bytes);
        mbar_arrive_expect_tx(bar0 + 8 * stg, bytes);
        bulk_g2s(ring + stg * p.stage_bytes, p.w + (int64_t)row0 * p.row_bytes, bytes, bar0 + 8 * stg);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            const int tile = blockIdx.x + s * gridDim.x;
            if (tile < p.num_tiles) issue(tile, s);
        }
    }

    // Programmatic dependent launch: the next kernel in the stream may start
    // its own prologue (barrier set-up, weight prefetch) while this one runs;
    // the activations, which a previous kernel may produce, are read only
    // after griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Activations: quantized here while the first weight tiles stream in, or
    // read from the global workspace.
    uint32_t quirk;
    ActSmem<TYPE> as{};
    ActGmem ag{p.qx, p.dx, p.bs, p.K, nb};
    if constexpr (FUSED) {
        uint8_t* qs = smem + kGemvSmemHeader;
        const uint32_t qbytes = (uint32_t)(M * act_row_stride(p.K));
        float* dxs = reinterpret_cast<float*>(qs + qbytes);
        int* bss = reinterpret_cast<int*>(qs + qbytes + 4u * (uint32_t)(M * nb));
        const uint32_t qm = quantize_to_smem<M, TYPE>(p.x, p.K, qs, dxs, bss);
        quirk = (TYPE == kQ8_0 || TYPE == kQ6_K) ? qm : 0u;
        as = ActSmem<TYPE>{smem_addr(qs), smem_addr(dxs), smem_addr(bss), act_row_stride(p.K), nb};
    } else {
        quirk = gemv_quirk_mask<TYPE, M>(p);
    }

    const int r = warp / p.wpr, slice = warp - r * p.wpr;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int stg = it % S;
        if (!mbar_wait_bounded(bar0 + 8 * stg, (uint32_t)(it / S) & 1u)) *s_abort = 1;
        const int row0 = tile * p.rows_per_tile;
        const int rows = min(p.rows_per_tile, p.N - row0);
        float acc[M];
        if (r < rows) {
            SmemSrc src{ring + stg * p.stage_bytes + (uint32_t)(r * p.row_bytes)};
            if constexpr (FUSED) gemv_row_slice<TYPE, M, EMIT, 16>(src, as, row0 + r, p, slice, quirk, acc);
            else gemv_row_slice<TYPE, M, EMIT, 16>(src, ag, row0 + r, p, slice, quirk, acc);
            if constexpr (!EMIT) {
                if (p.wpr == 1) gemv_store_row<M>(row0 + r, acc, p);
                else gemv_store_partial<M>(red + (it & 1) * kGemvWarps * M, warp, acc);
            }
        }
        __syncthreads();  // stage `stg` fully read; partial sums visible
        if (*s_abort) break;
        if (!EMIT && p.wpr > 1) gemv_combine<M>(red + (it & 1) * kGemvWarps * M, row0, rows, p);
        if (threadIdx.x == 0) {
            const int nt = tile + S * gridDim.x;
            if (nt < p.num_tiles) issue(nt, stg);
        }
    }
    if (*s_abort && threadIdx.x == 0) {
        // Let every copy still in flight land before the CTA exits.
        for (int k = 0; k < S; ++k) {
            const int itk = it + k;
            const int tile = blockIdx.x + itk * gridDim.x;
            if (tile < p.num_tiles) mbar_wait_bounded(bar0 + 8 * (itk % S), (uint32_t)(itk / S) & 1u);
        }
    }
}

template <int TYPE, int M, bool EMIT>
__global__ void __launch_bounds__(kGemvThreads) gemv_direct_kernel(const GemvParams p) {
    __shared__ float red[kGemvWarps * 8];
    const int warp = threadIdx.x >> 5;
    const uint32_t quirk = gemv_quirk_mask<TYPE, M>(p);
    const ActGmem ag{p.qx, p.dx, p.bs, p.K, p.K >> 5};
    const int r = warp / p.wpr, slice = warp - r * p.wpr;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        const int row0 = tile * p.rows_per_tile;
        const int rows = min(p.rows_per_tile, p.N - row0);
        float acc[M];
        if (r < rows) {
            GmemSrc src{p.w + (int64_t)(row0 + r) * p.row_bytes};
            gemv_row_slice<TYPE, M, EMIT, 1>(src, ag, row0 + r, p, slice, quirk, acc);
            if constexpr (!EMIT) {
                if (p.wpr == 1) gemv_store_row<M>(row0 + r, acc, p);
                else gemv_store_partial<M>(red, warp, acc);
            }
        }
        if (!EMIT && p.wpr > 1) {
            __syncthreads();
            gemv_combine<M>(red, row0, rows, p);
            __syncthreads();
        }
    }
}

}  // namespace cllm
