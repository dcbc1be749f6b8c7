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

constexpr int kMaxPeers = 8;  // GPUs of one node that a row-sharded call writes to
constexpr int kShardPadWords = 16;
constexpr int kShardCountSlot = kMaxPeers;

// An elementwise step applied to the fp32 activations just before their Q8_0
// quantization, so the engine step needs no separate kernel for it:
//   kPreRmsNorm  x = x * (1 / sqrt(sum(x^2) / K + eps)) * w   (rms_norm_ptr, engine.cpp:24-29)
//   kPreSiluMul  x = x / (1 + exp(-x)) * w                    (SwiGLU, engine.cpp:41, :511)
// w: the norm weight [K] (kPreRmsNorm) or the up-projection output [M][K]
// (kPreSiluMul).  Only the fused and activation-image paths apply it.
enum : int { kPreNone = 0, kPreRmsNorm = 1, kPreSiluMul = 2 };
struct PreOp {
    int op;
    const float* w;
    float eps;
};

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
    int32_t* partials;    // EMIT only: [M][N][parts per row] int32 block partials (y is not written)
    int rows_per_tile;    // R
    int wpr;              // warps per row (R * wpr == warps per CTA)
    int num_tiles;
    int stages;
    uint32_t stage_bytes;
    int sb_lanes;         // > 0: Q4_K super-block loop (q4k_row_sb), lanes per row
    int64_t ldy;          // row stride of y (0: N); set per launch
    int npeers;           // > 0: row-sharded call, y goes to every ypeers[q] instead of y
    float* ypeers[kMaxPeers];
    // row-sharded completion signalling (spads[0] == nullptr: none).  Signal
    // pads: kShardPadWords uint32 per rank, peer-mapped; slot q = the last
    // epoch rank q completed, slot kShardCountSlot = this rank's arrival count.
    uint32_t* spads[kMaxPeers];
    uint32_t* sepoch;     // this rank's epoch word (last completed round)
    int srank;
    int sarrive;          // the grid's last CTA announces the round (else a separate kernel or nobody)
    int swait;            // wait for every rank to have completed *sepoch before reading x
    // FUSED with image != nullptr: the activations were quantized by
    // act_image_kernel into `image` (row masks, then the shared-memory layout);
    // the producer copies it in instead of every CTA quantizing x itself.
    const uint8_t* image;
    uint32_t image_bytes;
    int image_ctas;
    PreOp pre;            // FUSED without image: applied by the CTA's own quantization
};

constexpr int kGemvWarps = 8;                      // warps that compute (R rows x wpr warps per row)
constexpr int kGemvThreads = kGemvWarps * 32;      // direct-load kernel, quantize kernel
constexpr int kTmaThreads = kGemvThreads + 32;     // + one producer warp that streams the weight tiles
constexpr int kGemvSmemHeader = 4096;              // barriers, flags, per-stage partial sums, before the ring

// Layout of the TMA kernel's shared-memory header.
constexpr int kHdrFull = 0;        // 8 x u64: "stage holds its tile" (tx-count barriers)
constexpr int kHdrEmpty = 64;      // 8 x u64: "every compute warp is done with the stage"
constexpr int kHdrAbort = 128;     // int: a bounded wait expired
constexpr int kHdrQuirk = 132;     // u32: per-row "activation holds -128" bits
constexpr int kHdrImage = 136;     // u64: "the activation image has landed" (tx-count barrier)
constexpr int kImageHeader = 128;  // image: u32 row masks of up to 32 quantizing CTAs, then the activations
constexpr int kImageMaxCtas = kImageHeader / 4;
constexpr int kHdrCount = 256;     // 8 stages x 8 rows of int: warps of a row that finished the tile
constexpr int kHdrRed = 512;       // 8 stages x 8 warps x 8 floats: partial row sums
constexpr int kHdrPre = 3072;      // 8 warps x 8 rows of partial sums of squares, then 8 rms factors

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

// Q6_K lane order: unit v -> (super-block, group, pair).  The units of the
// even super-blocks come first, so a warp's 32 lanes mostly share one
// super-block parity, and with it the 2-byte misalignment of a 210-byte
// super-block inside a 16-byte-aligned row.
__device__ __forceinline__ int q6k_superblock_of(int v, int se) {
    return v < 4 * se ? 2 * (v >> 2) : 2 * ((v - 4 * se) >> 2) + 1;
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
__host__ __device__ __forceinline__ int act_perm(int b, int nb) {
    if constexpr (TYPE == kQ6_K) {
        // Q6_K units are numbered in "lane order" v: the units of the even
        // super-blocks first, then those of the odd ones (see q6k_unit_of),
        // and unit v keeps its two blocks (sub-blocks pr and pr+2 of group g)
        // at positions 2v and 2v+1.
        const int sb = b >> 3, g = (b >> 2) & 1, sub = b & 3;
        const int se = ((nb >> 3) + 1) >> 1;  // number of even super-blocks
        const int vbase = (sb & 1) ? 4 * se + 4 * (sb >> 1) : 4 * (sb >> 1);
        return 2 * (vbase + 2 * g + (sub & 1)) + (sub >> 1);
    } else {
        (void)nb;
        return b;
    }
}

__host__ __device__ __forceinline__ uint32_t act_swizzle(uint32_t off) {
    const uint32_t slot = off >> 4;
    return ((slot ^ ((slot >> 3) & 7u)) << 4) | (off & 15u);
}

__host__ __device__ __forceinline__ int act_row_stride(int K) { return (K + 127) & ~127; }

// Q4_K with 16..32 super-blocks per row may run q4k_row_sb (lane =
// super-block; the plan's sb_lanes).  Its lanes read 16-byte slot c of
// super-blocks s, s+1, ... at once, so with that plan the activation writers
// swizzle the slots of a super-block with the super-block index instead
// (slot ^= (slot >> 4) & 7): eight consecutive super-blocks then hit eight
// different 16-byte bank groups.
template <int TYPE, int M>
__host__ __device__ __forceinline__ bool act_sb_layout(int K) {
    return TYPE == kQ4_K && K >= 4096 && K <= 8192;
}
__host__ __device__ __forceinline__ uint32_t act_swizzle_sb(uint32_t off) {
    const uint32_t slot = off >> 4;
    return ((slot ^ ((slot >> 4) & 7u)) << 4) | (off & 15u);
}

__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

template <int TYPE>
struct ActSmem {
    uint32_t qx, dx, bs, hs;  // shared addresses: [M][kp] int8 (swizzled), [M][nb] f32, [M][nb] i32,
                              // [M][nb] int2 = 32 x (sum of q over each 16-value half)
    int kp, nb;
    __device__ __forceinline__ void x32(int t, int b, int (&x)[8]) const {
        const uint32_t row = qx + (uint32_t)(t * kp);
        const uint32_t off = 32u * (uint32_t)act_perm<TYPE>(b, nb);
        const uint4 v0 = lds128(row + act_swizzle(off)), v1 = lds128(row + act_swizzle(off + 16));
        x[0] = (int)v0.x; x[1] = (int)v0.y; x[2] = (int)v0.z; x[3] = (int)v0.w;
        x[4] = (int)v1.x; x[5] = (int)v1.y; x[6] = (int)v1.z; x[7] = (int)v1.w;
    }
    __device__ __forceinline__ float dx1(int t, int b) const {
        return __uint_as_float(lds32(dx + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b, nb))));
    }
    __device__ __forceinline__ int bs1(int t, int b) const {
        return (int)lds32(bs + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b, nb)));
    }
    // blocks b and its unit partner, stored adjacently (perm(b) even)
    __device__ __forceinline__ float2 dx2(int t, int b) const {
        const uint2 v = lds64(dx + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b, nb)));
        return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    }
    __device__ __forceinline__ int2 bs2(int t, int b) const {
        const uint2 v = lds64(bs + 4u * (uint32_t)(t * nb + act_perm<TYPE>(b, nb)));
        return make_int2((int)v.x, (int)v.y);
    }
    // Q6_K unit: scales of blocks b and b + 2, adjacent after the permutation
    __device__ __forceinline__ float2 dx_q6(int t, int b) const { return dx2(t, b); }
};

template <int TYPE, int M, bool EMIT, int ALIGN, class Src, class Act>
__device__ __forceinline__ void gemv_unit(const Src& src, const Act& act, int u, const GemvParams& p,
                                          float (&acc)[M], int32_t* prow, int64_t pstride, uint32_t quirk) {
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
            if constexpr (EMIT) { prow[t * pstride + b0] = P0; prow[t * pstride + b0 + 1] = P1; }
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
            if constexpr (EMIT) { prow[t * pstride + b0] = P0; prow[t * pstride + b0 + 1] = P1; }
            const float2 dd = act.dx2(t, b0);
            const int2 ss = act.bs2(t, b0);
            acc[t] = fmaf(d1 * dd.x, i2f_exact(P0), acc[t]);
            acc[t] = fmaf(-(m1 * dd.x), i2f_exact(ss.x), acc[t]);
            acc[t] = fmaf(d2 * dd.y, i2f_exact(P1), acc[t]);
            acc[t] = fmaf(-(m2 * dd.y), i2f_exact(ss.y), acc[t]);
        }
    } else if constexpr (TYPE == kQ6_K) {
        // unit u in the lane order of q6k_superblock_of (even super-blocks
        // first) = (super-block s, group g, pair pr): sub-blocks pr and pr+2 of
        // group g.  Every Q6_K path assigns units to lanes this way, so a row's
        // result does not depend on M or on the path.
        const int s = q6k_superblock_of(u, ((p.K >> 8) + 1) >> 1), g = (u >> 1) & 1, pr = u & 1;
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
                int32_t* pt = prow + t * pstride;
                pt[2 * bA] = PA0; pt[2 * bA + 1] = PA1;
                pt[2 * bB] = PB0; pt[2 * bB + 1] = PB1;
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
            if constexpr (EMIT) prow[t * pstride + b] = P;
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
            if constexpr (EMIT) prow[t * pstride + b] = P;
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
            if constexpr (EMIT) prow[t * pstride + b] = P;
            acc[t] = fmaf(d * act.dx1(t, b), i2f_exact(P - 16 * act.bs1(t, b)), acc[t]);
        }
    }
}

// ---------------------------------------------------------------------------
// Specialised loops of the fused path for the two BASELINE weight types.
// Same arithmetic as gemv_unit (identical integer partials, same per-block
// FMA statements), with everything that is constant for a lane hoisted out
// of the unit loop: the unit's position inside its super-block, the
// swizzled activation offsets and the scale byte selectors.

// byte `sel` of w as an exact float: 0x4B0000bb is 2^23 + bb.
__device__ __forceinline__ float byte_as_float(uint32_t w, uint32_t sel) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | sel)) - 8388608.0f;
}

// byte `sel` of w sign-extended to int32: PRMT selector nibbles with bit 3
// set replicate the sign of the selected byte.
__device__ __forceinline__ int byte_as_int_signed(uint32_t w, uint32_t sel) {
    int r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"((sel | 8u) * 0x1110u | sel));
    return r;
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Q4_K row slice, activations and weights in shared memory (quant.cpp:549-590).
// Lane unit u = 4s + q: sub-blocks 2q, 2q+1 of super-block s.
// EMIT (parity builds): also store each block's int32 partial at
// prow[t * pstride + block].
template <int M, bool EMIT>
__device__ __forceinline__ void q4k_row_fused(uint32_t wrow, const ActSmem<kQ4_K>& act, int upr, int slice,
                                              int wpr, float (&acc)[M], int32_t* prow, int64_t pstride) {
    const int lane = threadIdx.x & 31;
    const int u0 = slice * 32 + lane;
    const int ustep = 32 * wpr;
    const int q = u0 & 3;
    const bool low = q < 2;
    const uint32_t sel0 = (uint32_t)(q & 1) * 2u, sel1 = sel0 + 1u;
    const uint32_t key = (uint32_t)(u0 >> 1) & 7u;
    // activation chunk u (64 bytes = blocks 2u, 2u+1), 16-byte pieces swizzled
    const uint32_t cb = 16u * ((4u * (uint32_t)u0) ^ (key & 4u));
    const uint32_t o0 = 16u * ((0u ^ key) & 3u), o1 = 16u * ((1u ^ key) & 3u);
    const uint32_t o2 = 16u * ((2u ^ key) & 3u), o3 = 16u * ((3u ^ key) & 3u);
    const uint32_t cstep = 64u * (uint32_t)ustep;
    uint32_t wo = 144u * (uint32_t)(u0 >> 2);
    const uint32_t wstep = 144u * (uint32_t)(ustep >> 2);
    const uint32_t qoff = 16u + 32u * (uint32_t)q;
    uint32_t ao = cb;                                // act byte offset of this lane's chunk
    uint32_t so = 8u * (uint32_t)u0;                 // byte offset of (dx, bs) pair of block 2u
    const uint32_t sstep = 8u * (uint32_t)ustep;
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = 0.0f;
    for (int u = u0; u < upr; u += ustep, wo += wstep, ao += cstep, so += sstep) {
        const uint4 h = lds128(wrow + wo);
        const uint4 wa = lds128(wrow + wo + qoff), wb = lds128(wrow + wo + qoff + 16u);
        const uint32_t scw = low ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
        const uint32_t mw = low ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
        const float d = h2f(h.x), dmin = h2f(h.x >> 16);
        const float d1 = d * byte_as_float(scw, sel0), d2 = d * byte_as_float(scw, sel1);
        const float m1 = dmin * byte_as_float(mw, sel0), m2 = dmin * byte_as_float(mw, sel1);
        const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        int lo[8];
        uint32_t hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (int)(w[i] & 0x0F0F0F0Fu);
            hi[i] = w[i] & 0xF0F0F0F0u;  // 16 x high nibble, unsigned
        }
#pragma unroll
        for (int t = 0; t < M; ++t) {
            const uint32_t row = act.qx + (uint32_t)(t * act.kp) + ao;
            const uint4 x0 = lds128(row + o0), x1 = lds128(row + o1), x2 = lds128(row + o2), x3 = lds128(row + o3);
            int P0 = dp4a(lo[0], (int)x0.x, 0);
            P0 = dp4a(lo[1], (int)x0.y, P0); P0 = dp4a(lo[2], (int)x0.z, P0); P0 = dp4a(lo[3], (int)x0.w, P0);
            P0 = dp4a(lo[4], (int)x1.x, P0); P0 = dp4a(lo[5], (int)x1.y, P0);
            P0 = dp4a(lo[6], (int)x1.z, P0); P0 = dp4a(lo[7], (int)x1.w, P0);
            int H1 = dp4a_us(hi[0], (int)x2.x, 0);
            H1 = dp4a_us(hi[1], (int)x2.y, H1); H1 = dp4a_us(hi[2], (int)x2.z, H1); H1 = dp4a_us(hi[3], (int)x2.w, H1);
            H1 = dp4a_us(hi[4], (int)x3.x, H1); H1 = dp4a_us(hi[5], (int)x3.y, H1);
            H1 = dp4a_us(hi[6], (int)x3.z, H1); H1 = dp4a_us(hi[7], (int)x3.w, H1);
            const int P1 = H1 >> 4;  // exact: every term is a multiple of 16
            if constexpr (EMIT) {
                prow[t * pstride + 2 * u] = P0;
                prow[t * pstride + 2 * u + 1] = P1;
            }
            const uint32_t sa = (uint32_t)(t * act.nb) * 4u + so;
            const uint2 dd = lds64(act.dx + sa), ss = lds64(act.bs + sa);
            const float dx0 = __uint_as_float(dd.x), dx1 = __uint_as_float(dd.y);
            acc[t] = fmaf(d1 * dx0, i2f_exact(P0), acc[t]);
            acc[t] = fmaf(-(m1 * dx0), i2f_exact((int)ss.x), acc[t]);
            acc[t] = fmaf(d2 * dx1, i2f_exact(P1), acc[t]);
            acc[t] = fmaf(-(m2 * dx1), i2f_exact((int)ss.y), acc[t]);
        }
    }
    warp_sum<M>(acc);
}


// Q4_K row with lane = super-block (quant.cpp:549-590), M <= 8 activation
// rows: the `lanes` lanes of a weight row take its super-blocks li,
// li + lanes, ...; a super-block's scales are decoded once for its 256 values,
// and each activation row arrives as 16-byte loads (layout act_swizzle_sb).
// Per 32-value block the same integer partial and the same two FMA statements
// as q4k_row_fused.  EMIT: also store each block's partial at
// prow[t * pstride + block].
template <int M, bool EMIT>
__device__ __forceinline__ void q4k_row_sb(uint32_t wrow, const ActSmem<kQ4_K>& act, int nsb, int li, int lanes,
                                           float (&acc)[M], int32_t* prow, int64_t pstride) {
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = 0.0f;
    for (int s = li; s < nsb; s += lanes) {
        const uint32_t wb = wrow + 144u * (uint32_t)s;
        const uint4 h = lds128(wb);
        const float d = h2f(h.x), dmin = h2f(h.x >> 16);
        const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
        const uint32_t key = (uint32_t)s & 7u;
        uint32_t dxw[8], bsw[8];  // M = 1: the eight blocks' (dx, bsum) in four loads
        if constexpr (M == 1) {
            const uint32_t da = act.dx + 32u * (uint32_t)s, ba = act.bs + 32u * (uint32_t)s;
            const uint4 d0 = lds128(da), d1 = lds128(da + 16u), q0 = lds128(ba), q1 = lds128(ba + 16u);
            dxw[0] = d0.x; dxw[1] = d0.y; dxw[2] = d0.z; dxw[3] = d0.w;
            dxw[4] = d1.x; dxw[5] = d1.y; dxw[6] = d1.z; dxw[7] = d1.w;
            bsw[0] = q0.x; bsw[1] = q0.y; bsw[2] = q0.z; bsw[3] = q0.w;
            bsw[4] = q1.x; bsw[5] = q1.y; bsw[6] = q1.z; bsw[7] = q1.w;
        }
#pragma unroll
        for (int pq = 0; pq < 4; ++pq) {
            // quant bytes of sub-blocks 2pq (low nibbles) and 2pq+1 (high nibbles)
            const uint4 wa = lds128(wb + 16u + 32u * pq), wc = lds128(wb + 32u + 32u * pq);
            const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wc.x, wc.y, wc.z, wc.w};
            int lo[8];
            uint32_t hi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                lo[i] = (int)(w[i] & 0x0F0F0F0Fu);
                hi[i] = w[i] & 0xF0F0F0F0u;  // 16 x high nibble, unsigned
            }
            const uint32_t scw = pq < 2 ? sc_lo : sc_hi, mw = pq < 2 ? m_lo : m_hi;
            const uint32_t sel0 = (uint32_t)(pq & 1) * 2u, sel1 = sel0 + 1u;
            const float d1 = d * byte_as_float(scw, sel0), d2 = d * byte_as_float(scw, sel1);
            const float m1 = dmin * byte_as_float(mw, sel0), m2 = dmin * byte_as_float(mw, sel1);
            const int b0 = 8 * s + 2 * pq;  // block of sub-block 2pq
#pragma unroll
            for (int t = 0; t < M; ++t) {
                const uint32_t xrow = act.qx + (uint32_t)(t * act.kp) + 256u * (uint32_t)s;
                const uint4 x0 = lds128(xrow + 16u * ((4u * pq) ^ key));
                const uint4 x1 = lds128(xrow + 16u * ((4u * pq + 1u) ^ key));
                const uint4 x2 = lds128(xrow + 16u * ((4u * pq + 2u) ^ key));
                const uint4 x3 = lds128(xrow + 16u * ((4u * pq + 3u) ^ key));
                int P0 = dp4a(lo[0], (int)x0.x, 0);
                P0 = dp4a(lo[1], (int)x0.y, P0); P0 = dp4a(lo[2], (int)x0.z, P0); P0 = dp4a(lo[3], (int)x0.w, P0);
                P0 = dp4a(lo[4], (int)x1.x, P0); P0 = dp4a(lo[5], (int)x1.y, P0);
                P0 = dp4a(lo[6], (int)x1.z, P0); P0 = dp4a(lo[7], (int)x1.w, P0);
                int H1 = dp4a_us(hi[0], (int)x2.x, 0);
                H1 = dp4a_us(hi[1], (int)x2.y, H1); H1 = dp4a_us(hi[2], (int)x2.z, H1); H1 = dp4a_us(hi[3], (int)x2.w, H1);
                H1 = dp4a_us(hi[4], (int)x3.x, H1); H1 = dp4a_us(hi[5], (int)x3.y, H1);
                H1 = dp4a_us(hi[6], (int)x3.z, H1); H1 = dp4a_us(hi[7], (int)x3.w, H1);
                const int P1 = H1 >> 4;  // exact: every term is a multiple of 16
                if constexpr (EMIT) {
                    prow[t * pstride + b0] = P0;
                    prow[t * pstride + b0 + 1] = P1;
                }
                uint2 dd, ss;
                if constexpr (M == 1) {
                    dd = make_uint2(dxw[2 * pq], dxw[2 * pq + 1]);
                    ss = make_uint2(bsw[2 * pq], bsw[2 * pq + 1]);
                } else {
                    const uint32_t sa = 4u * (uint32_t)(t * act.nb + b0);
                    dd = lds64(act.dx + sa);
                    ss = lds64(act.bs + sa);
                }
                const float dx0 = __uint_as_float(dd.x), dx1 = __uint_as_float(dd.y);
                acc[t] = fmaf(d1 * dx0, i2f_exact(P0), acc[t]);
                acc[t] = fmaf(-(m1 * dx0), i2f_exact((int)ss.x), acc[t]);
                acc[t] = fmaf(d2 * dx1, i2f_exact(P1), acc[t]);
                acc[t] = fmaf(-(m2 * dx1), i2f_exact((int)ss.y), acc[t]);
            }
        }
    }
}

// 8 words of a 32-byte field at shared address a, which is 4-byte aligned
// (odd == false) or 2 bytes past a 4-byte boundary (odd == true).
__device__ __forceinline__ void lds_field8(uint32_t a, bool odd, uint32_t (&w)[8]) {
    if (!odd) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = lds32(a + 4u * i);
    } else {
        const uint32_t al = a - 2u;
        uint32_t r[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) r[i] = lds32(al + 4u * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], 16);
    }
}

// Q6_K row slice, activations and weights in shared memory (quant.cpp:630-687).
// EMIT: also store the int32 half-block partials at prow[t * pstride + 2*block + half].
template <int M, bool EMIT>
__device__ __forceinline__ void q6k_row_fused(uint32_t wrow, const ActSmem<kQ6_K>& act, int upr, int slice,
                                              int wpr, uint32_t quirk, float (&acc)[M], int32_t* prow,
                                              int64_t pstride) {
    const int lane = threadIdx.x & 31;
    const int v0 = slice * 32 + lane;
    const int vstep = 32 * wpr;
    const int g = (v0 >> 1) & 1, pr = v0 & 1;
    const int se = ((act.nb >> 3) + 1) >> 1;
    const uint32_t key = (uint32_t)(v0 >> 1) & 7u;
    const uint32_t o0 = 16u * ((0u ^ key) & 3u), o1 = 16u * ((1u ^ key) & 3u);
    const uint32_t o2 = 16u * ((2u ^ key) & 3u), o3 = 16u * ((3u ^ key) & 3u);
    const uint32_t loff = 64u * (uint32_t)g + 32u * (uint32_t)pr, hoff = 128u + 32u * (uint32_t)g;
    const uint32_t scoff = 192u + 8u * (uint32_t)g;
    const uint32_t sel0 = 2u * (uint32_t)pr, sel1 = sel0 + 1u;
    const int hsh = 4 - 2 * pr, lsh = 2 * pr;
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = 0.0f;
    for (int v = v0; v < upr; v += vstep) {
        const int sb = q6k_superblock_of(v, se);
        const uint32_t o = 210u * (uint32_t)sb;
        const bool odd = (sb & 1) != 0;
        uint32_t L[8], H[8];
        lds_field8(wrow + o + loff, odd, L);
        lds_field8(wrow + o + hoff, odd, H);
        // 8 scale bytes of the group and d: 2-byte fields, 4-aligned when even
        const uint32_t sa = wrow + o + scoff;
        uint32_t SC0, SC1;
        if (!odd) {
            SC0 = lds32(sa);
            SC1 = lds32(sa + 4u);
        } else {
            const uint32_t r0 = lds32(sa - 2u), r1 = lds32(sa + 2u), r2 = lds32(sa + 6u);
            SC0 = __funnelshift_r(r0, r1, 16);
            SC1 = __funnelshift_r(r1, r2, 16);
        }
        const float d = h2f(lds16(wrow + o + 208u));
        const int sA0 = byte_as_int_signed(SC0, sel0), sA1 = byte_as_int_signed(SC0, sel1);
        const int sB0 = byte_as_int_signed(SC1, sel0), sB1 = byte_as_int_signed(SC1, sel1);
        // six-bit quants v in [0,63] per byte (the weight is v - 32)
        uint32_t va[8], vb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            va[i] = (L[i] & 0x0F0F0F0Fu) | ((H[i] << hsh) & 0x30303030u);
            vb[i] = ((L[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> lsh) & 0x30303030u);
        }
        const uint32_t cb = 16u * ((4u * (uint32_t)v) ^ (key & 4u));
#pragma unroll
        for (int t = 0; t < M; ++t) {
            const uint32_t row = act.qx + (uint32_t)(t * act.kp) + cb;
            const uint4 x0 = lds128(row + o0), x1 = lds128(row + o1), x2 = lds128(row + o2), x3 = lds128(row + o3);
            const int xa[8] = {(int)x0.x, (int)x0.y, (int)x0.z, (int)x0.w, (int)x1.x, (int)x1.y, (int)x1.z, (int)x1.w};
            const int xb[8] = {(int)x2.x, (int)x2.y, (int)x2.z, (int)x2.w, (int)x3.x, (int)x3.y, (int)x3.z, (int)x3.w};
            // 32 x (half sums of q) of blocks 2v and 2v+1, then subtract: sum((v-32)*x)
            const uint4 hsum = lds128(act.hs + 8u * (uint32_t)(t * act.nb + 2 * v));
            int PA0 = -(int)hsum.x, PA1 = -(int)hsum.y, PB0 = -(int)hsum.z, PB1 = -(int)hsum.w;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                PA0 = dp4a((int)va[i], xa[i], PA0);
                PA1 = dp4a((int)va[i + 4], xa[i + 4], PA1);
                PB0 = dp4a((int)vb[i], xb[i], PB0);
                PB1 = dp4a((int)vb[i + 4], xb[i + 4], PB1);
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
                const int bA = 8 * sb + 4 * g + pr, bB = bA + 2;
                int32_t* pt = prow + t * pstride;
                pt[2 * bA] = PA0; pt[2 * bA + 1] = PA1;
                pt[2 * bB] = PB0; pt[2 * bB + 1] = PB1;
            }
            const uint2 dd = lds64(act.dx + 4u * (uint32_t)(t * act.nb + 2 * v));
            // sc*P sums are exact integers (|.| <= 2^24), as the reference's float sums
            const float inA = (float)(sA0 * PA0 + sA1 * PA1), inB = (float)(sB0 * PB0 + sB1 * PB1);
            acc[t] = fmaf(d * __uint_as_float(dd.x), inA, acc[t]);
            acc[t] = fmaf(d * __uint_as_float(dd.y), inB, acc[t]);
        }
    }
    warp_sum<M>(acc);
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

// gemv_quirk_mask for the compute warps of the TMA kernel (producer excluded).
template <int TYPE, int M>
__device__ __forceinline__ uint32_t gemv_quirk_mask_compute(const GemvParams& p, uint32_t* s_quirk) {
    if constexpr (TYPE != kQ8_0 && TYPE != kQ6_K) {
        return 0u;
    } else {
        const int nb = p.K >> 5;
        uint32_t mask = 0;
#pragma unroll
        for (int t = 0; t < M; ++t) {
            int any = 0;
            for (int i = threadIdx.x; i < nb; i += kGemvThreads) any |= p.fl[(int64_t)t * nb + i];
            if (any) mask |= 1u << t;
        }
        const uint32_t wm = __reduce_or_sync(0xFFFFFFFFu, mask);
        if ((threadIdx.x & 31) == 0 && wm) atomicOr(s_quirk, wm);
        named_barrier_sync(kGemvThreads);
        return *reinterpret_cast<volatile uint32_t*>(s_quirk);
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
    int64_t pstride = 0;
    if constexpr (EMIT) {
        const int ppr = (TYPE == kQ6_K) ? 2 * (p.K >> 5) : (p.K >> 5);
        prow = p.partials + (int64_t)row * ppr;
        pstride = (int64_t)p.N * ppr;
    }
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = 0.0f;
    for (int u = slice * 32 + lane; u < upr; u += 32 * p.wpr)
        gemv_unit<TYPE, M, EMIT, ALIGN>(src, act, u, p, acc, prow, pstride, quirk);
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
// Row-sharded call, start: wait until every rank has completed the epoch in
// *sepoch (the previous round), so that x -- typically the previous call's
// all-gathered y -- is complete.  Threads 0..npeers-1 poll; bounded.
__device__ __forceinline__ void shard_wait_prev(const GemvParams& p) {
    const int q = threadIdx.x;
    if (q < p.npeers) {
        const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(p.sepoch);
        const uint32_t* slot = p.spads[p.srank] + q;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(slot) : "memory");
            if ((int32_t)(v - ep) >= 0) break;
            if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                atomicExch(&g_device_status, kStatusTimeout);
                break;
            }
        }
    }
}

// Row-sharded call, end: one arrival per CTA, by thread 0 after the CTA's
// compute threads have synchronized (gpu-scope fence: the arrival count is
// local); the grid's last CTA orders everything system-wide and announces
// the new epoch to every rank, then resets the count.
__device__ __forceinline__ void shard_arrive_cta(const GemvParams& p) {
    if (threadIdx.x != 0) return;
    __threadfence();
    uint32_t* count = p.spads[p.srank] + kShardCountSlot;
    if (atomicAdd(count, 1u) == gridDim.x - 1u) {
        __threadfence_system();
        const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(p.sepoch) + 1u;
        for (int q = 0; q < p.npeers; ++q)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.spads[q] + p.srank), "r"(ep) : "memory");
        *reinterpret_cast<volatile uint32_t*>(p.sepoch) = ep;
        *reinterpret_cast<volatile uint32_t*>(count) = 0u;
    }
}

// Store y[t][j]: locally, or (row-sharded call) into the y buffer of every GPU
// of the group over NVLink peer mappings, so the output is all-gathered as it
// is produced.
__device__ __forceinline__ void gemv_put(const GemvParams& p, int t, int j, float v) {
    const int64_t o = (int64_t)t * p.ldy + j;
    if (p.npeers == 0) {
        p.y[o] = v;
        return;
    }
    for (int q = 0; q < p.npeers; ++q) p.ypeers[q][o] = v;
}

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
        gemv_put(p, t, j, s);
    }
}

template <int M>
__device__ __forceinline__ void gemv_store_row(int j, const float (&acc)[M], const GemvParams& p) {
    if ((threadIdx.x & 31) == 0) {
        const float b = p.bias ? p.bias[j] : 0.0f;
#pragma unroll
        for (int t = 0; t < M; ++t) gemv_put(p, t, j, acc[t] + b);
    }
}

// Quantize x [M][K] into this CTA's shared memory (quantize_row_q8_0,
// quant.cpp:420-452, the same IEEE steps as quantize_q8_0_kernel).  Four
// lanes share a 32-value block, eight values (two float4) each, so the two
// divisions per block and the packing are spread over eight values per lane;
// every thread issues the loads of up to four blocks before reducing them.
// x must be 16-byte aligned.  Returns the per-row "holds -128" mask.  Called
// by all compute threads.
// kPreRmsNorm: 1 / sqrt(sum(x[t]^2) / K + eps) of each of the M rows into
// s_rms[t], computed by the kGemvThreads threads taking part (named barrier 1;
// s_part holds 8 x M floats).  Every CTA sums in the same order, so every CTA
// gets the same factors.
template <int M>
__device__ __forceinline__ void pre_rms(const float* __restrict__ x, int K, float eps, float* s_part, float* s_rms) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int t = 0; t < M; ++t) {
        float s = 0.0f;
        for (int i = tid; i < K; i += kGemvThreads) {
            const float v = x[(int64_t)t * K + i];
            s = fmaf(v, v, s);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) s_part[warp * M + t] = s;
    }
    named_barrier_sync(kGemvThreads);
    if (tid < M) {
        float sum = 0.0f;
        for (int w = 0; w < kGemvThreads / 32; ++w) sum += s_part[w * M + tid];
        s_rms[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), eps)));
    }
    named_barrier_sync(kGemvThreads);
}

// Apply the pre-quantization step to the eight values at x[t][k..k+7].
__device__ __forceinline__ void pre_apply(const PreOp& pre, const float* s_rms, int t, int K, int k, float4& a,
                                          float4& b) {
    if (pre.op == kPreRmsNorm) {
        const float r = s_rms[t];
        const float4* w = reinterpret_cast<const float4*>(pre.w + k);
        const float4 w0 = __ldg(w), w1 = __ldg(w + 1);
        a = make_float4(__fmul_rn(__fmul_rn(a.x, r), w0.x), __fmul_rn(__fmul_rn(a.y, r), w0.y),
                        __fmul_rn(__fmul_rn(a.z, r), w0.z), __fmul_rn(__fmul_rn(a.w, r), w0.w));
        b = make_float4(__fmul_rn(__fmul_rn(b.x, r), w1.x), __fmul_rn(__fmul_rn(b.y, r), w1.y),
                        __fmul_rn(__fmul_rn(b.z, r), w1.z), __fmul_rn(__fmul_rn(b.w, r), w1.w));
    } else if (pre.op == kPreSiluMul) {
        const float4* u = reinterpret_cast<const float4*>(pre.w + (int64_t)t * K + k);
        const float4 u0 = __ldg(u), u1 = __ldg(u + 1);
        auto sm = [](float v, float g) { return __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), g); };
        a = make_float4(sm(a.x, u0.x), sm(a.y, u0.y), sm(a.z, u0.z), sm(a.w, u0.w));
        b = make_float4(sm(b.x, u1.x), sm(b.y, u1.y), sm(b.z, u1.z), sm(b.w, u1.w));
    }
}

template <int M, int TYPE, bool GLOBAL>
__device__ __forceinline__ uint32_t quantize_blocks(const float* __restrict__ x, int K, uint8_t* qs, float* dx,
                                                    int* bs, int* hs, int gfirst, int gcount,
                                                    const PreOp& pre, const float* s_rms, bool sb_layout) {
    // sb_layout: the slot swizzle of the lane-per-super-block loop (act_swizzle_sb)
    // gfirst: this CTA's first group of blocks; gcount: groups per pass of all
    // CTAs taking part (one CTA: 0 and 64).  Returns this thread's row mask.
    const int kp = act_row_stride(K);
    constexpr int kGroups = kGemvThreads / 4;  // 64 blocks per pass of the group loop
    constexpr int kUnroll = 4;
    const int g = threadIdx.x >> 2, sub = threadIdx.x & 3;
    const int nb = K >> 5;
    const int total = M * nb;
    uint32_t mask = 0;
    for (int base = gfirst; base < total; base += gcount * kUnroll) {
        float4 v[kUnroll][2];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int blk = base + g + gcount * u;
            if (blk < total) {
                const int t = blk / nb, b = blk - t * nb;
                const float4* src = reinterpret_cast<const float4*>(x + (int64_t)t * K + 32 * b + 8 * sub);
                v[u][0] = __ldg(src);
                v[u][1] = __ldg(src + 1);
                if (pre.op != kPreNone) pre_apply(pre, s_rms, t, K, 32 * b + 8 * sub, v[u][0], v[u][1]);
            } else {
                v[u][0] = v[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            // stop once no group of this warp has a block left (warp-uniform)
            if (base + gcount * u + (g & ~7) >= total) break;
            const int blk = base + g + gcount * u;  // uniform within each 4-lane group
            const float vv[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                                 v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
            // max of |x| over non-NaN values, as `if (a > amax) amax = a` from 0
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(vv[e]));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            const float d = amax / 127.0f;
            const float id = (d != 0.0f) ? __frcp_rn(d) : 0.0f;  // == 1.0f / d, correctly rounded
            int q[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                // Round half to even without the conversion pipe: adding
                // 1.5 * 2^23 leaves the rounded integer in the low mantissa
                // bits for |v| < 2^22.  |v| <= 127 for every finite input;
                // larger magnitudes only arise as +-inf or NaN (1/d overflowed
                // or x was infinite), which x86 converts to INT32_MIN.
                const float f = vv[e] * id;
                const int qi = fabsf(f) < 4194304.0f ? __float_as_int(f + 12582912.0f) - 0x4B400000 : INT32_MIN;
                q[e] = qi > 127 ? 127 : (qi < -128 ? -128 : qi);
            }
            const uint32_t w0 = __byte_perm(__byte_perm((uint32_t)q[0], (uint32_t)q[1], 0x0040u),
                                            __byte_perm((uint32_t)q[2], (uint32_t)q[3], 0x0040u), 0x5410u);
            const uint32_t w1 = __byte_perm(__byte_perm((uint32_t)q[4], (uint32_t)q[5], 0x0040u),
                                            __byte_perm((uint32_t)q[6], (uint32_t)q[7], 0x0040u), 0x5410u);
            // sums: 8 values per lane, 16 per lane pair (half block), 32 per group
            const int s8 = __dp4a((int)w0, 0x01010101, __dp4a((int)w1, 0x01010101, 0));
            const int half = s8 + __shfl_xor_sync(0xFFFFFFFFu, s8, 1);
            const int sum = half + __shfl_xor_sync(0xFFFFFFFFu, half, 2);
            if (blk < total) {
                const int t = blk / nb, b = blk - t * nb;
                const int pb = act_perm<TYPE>(b, nb);
                const uint32_t lo = 32u * pb + 8u * sub;
                const uint32_t off = (uint32_t)(t * kp) + (sb_layout ? act_swizzle_sb(lo) : act_swizzle(lo));
                if constexpr (GLOBAL) {
                    *reinterpret_cast<uint2*>(qs + off) = make_uint2(w0, w1);
                } else {
                    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(smem_addr(qs) + off), "r"(w0), "r"(w1)
                                 : "memory");
                }
                // a byte equal to 0x80 (-128): zero byte of w ^ 0x80808080
                const uint32_t z0 = w0 ^ 0x80808080u, z1 = w1 ^ 0x80808080u;
                if (((z0 - 0x01010101u) & ~z0 & 0x80808080u) | ((z1 - 0x01010101u) & ~z1 & 0x80808080u))
                    mask |= 1u << t;
                if (sub == 0) {
                    dx[t * nb + pb] = d;
                    bs[t * nb + pb] = sum;
                }
                if (TYPE == kQ6_K && (sub & 1) == 0) hs[2 * (t * nb + pb) + (sub >> 1)] = 32 * half;
            }
        }
    }
    (void)kGroups;
    return mask;
}

template <int M, int TYPE>
__device__ __forceinline__ uint32_t quantize_to_smem(const float* __restrict__ x, int K,
                                                     uint8_t* qs, float* dx, int* bs, int* hs,
                                                     uint32_t* s_quirk, const PreOp& pre, float* s_pre, bool sb_layout) {
    if (pre.op == kPreRmsNorm) pre_rms<M>(x, K, pre.eps, s_pre, s_pre + 64);
    const uint32_t mask =
        quantize_blocks<M, TYPE, false>(x, K, qs, dx, bs, hs, 0, kGemvThreads / 4, pre, s_pre + 64, sb_layout);
    // OR over the compute warps (*s_quirk is zero on entry), then a barrier
    // over those warps only: the producer warp does not take part.
    const uint32_t wm = __reduce_or_sync(0xFFFFFFFFu, mask);
    if ((threadIdx.x & 31) == 0 && wm) atomicOr(s_quirk, wm);
    named_barrier_sync(kGemvThreads);
    return *reinterpret_cast<volatile uint32_t*>(s_quirk);
}

// Quantize x [M][K] once into an activation image in global memory: the
// per-CTA row masks, then exactly the shared-memory layout the fused GEMV
// builds (quantize_blocks), so each GEMV CTA copies it in with one bulk copy
// instead of re-reading and re-quantizing x.  CTA c takes every gridDim.x-th
// group of 64 blocks.  A programmatic dependent of the kernel that wrote x;
// lets the GEMV launch (and start streaming weights) at once.
template <int M, int TYPE>
__global__ void __launch_bounds__(kGemvThreads) act_image_kernel(const float* __restrict__ x, int K,
                                                                 uint8_t* __restrict__ image, const uint32_t* wait_pad,
                                                                 const uint32_t* wait_epoch, int wait_world,
                                                                 const PreOp pre, int sb_layout) {
    __shared__ uint32_t s_mask;
    __shared__ float s_pre[64 + 8];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // Row-sharded chain: x may be the previous round's all-gathered output, so
    // wait (bounded) until every rank has announced that round.
    if (wait_pad && (int)threadIdx.x < wait_world) {
        const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(wait_epoch);
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(wait_pad + threadIdx.x) : "memory");
            if ((int32_t)(v - ep) >= 0) break;
            if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
                atomicExch(&g_device_status, kStatusTimeout);
                break;
            }
        }
    }
    if (threadIdx.x == 0) s_mask = 0;
    __syncthreads();
    if (pre.op == kPreRmsNorm) pre_rms<M>(x, K, pre.eps, s_pre, s_pre + 64);
    const int nb = K >> 5;
    uint8_t* qs = image + kImageHeader;
    const uint32_t qbytes = (uint32_t)(M * act_row_stride(K));
    float* dx = reinterpret_cast<float*>(qs + qbytes);
    int* bs = reinterpret_cast<int*>(qs + qbytes + 4u * (uint32_t)(M * nb));
    int* hs = reinterpret_cast<int*>(qs + qbytes + 8u * (uint32_t)(M * nb));
    const uint32_t mask = quantize_blocks<M, TYPE, true>(x, K, qs, dx, bs, hs, (int)blockIdx.x * (kGemvThreads / 4),
                                                         (int)gridDim.x * (kGemvThreads / 4), pre, s_pre + 64,
                                                         sb_layout != 0);
    const uint32_t wm = __reduce_or_sync(0xFFFFFFFFu, mask);
    if ((threadIdx.x & 31) == 0 && wm) atomicOr(&s_mask, wm);
    __syncthreads();
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(image)[blockIdx.x] = s_mask;
}

// Shared-memory bytes the fused quantization needs for M rows of K.
__host__ __device__ inline uint32_t fused_act_bytes(int M, int K) {
    const uint32_t nb = (uint32_t)K / 32u;
    return (uint32_t)(M * act_row_stride(K)) + 16u * (uint32_t)M * nb;
}

// Warp specialisation: warps 0..7 compute, warp 8 (one lane) streams the
// weight tiles.  Stage s of the ring has a "full" barrier (one arrival plus
// the bulk copy's transaction bytes) and an "empty" barrier (one arrival per
// compute warp).  The producer refills a stage as soon as the eight compute
// warps have released it, so warps do not run in lockstep: a warp that
// finishes its row of tile i moves on to tile i+1 while others still work.
// A row split over wpr > 1 warps is summed by the last of its warps to finish
// (a shared counter per stage and row), in warp order, so the result does not
// depend on timing.
template <int TYPE, int M, bool EMIT, bool FUSED>
__global__ void __launch_bounds__(kTmaThreads, 2) gemv_tma_kernel(const GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t full0 = sbase + kHdrFull, empty0 = sbase + kHdrEmpty;
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kHdrAbort);
    uint32_t* s_quirk = reinterpret_cast<uint32_t*>(smem + kHdrQuirk);
    int* s_count = reinterpret_cast<int*>(smem + kHdrCount);
    float* s_red = reinterpret_cast<float*>(smem + kHdrRed);
    const int nb = p.K >> 5;
    const uint32_t act_bytes = FUSED ? (fused_act_bytes(M, p.K) + 127u) / 128u * 128u : 0u;
    const uint32_t ring = sbase + kGemvSmemHeader + act_bytes;
    const int S = p.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kGemvWarps);
        }
        mbar_init(sbase + kHdrImage, 1);
        *s_abort = 0;
        *s_quirk = 0;
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < 64; i += blockDim.x) s_count[i] = 0;
    __syncthreads();

    // Programmatic dependent launch: the next kernel in the stream may start
    // its own prologue (barrier set-up, weight prefetch) while this one runs.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == kGemvWarps) {
        // ---- producer: weights are static, so no wait on the previous kernel
        if (lane == 0) {
            // Image mode: two tiles of weights first (they do not depend on the
            // previous kernel), then the activation image once it is written.
            bool image_due = FUSED && p.image != nullptr;
            auto issue_image = [&]() {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                mbar_arrive_expect_tx(sbase + kHdrImage, p.image_bytes);
                bulk_g2s(sbase + kGemvSmemHeader - kImageHeader, p.image, p.image_bytes, sbase + kHdrImage);
                image_due = false;
            };
            int it = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
                if (image_due && it == 2) issue_image();
                const int stg = it % S;
                if (it >= S && !mbar_wait_or_abort(empty0 + 8 * stg, (uint32_t)((it / S) - 1) & 1u, s_abort))
                    break;
                const int row0 = tile * p.rows_per_tile;
                const int rows = min(p.rows_per_tile, p.N - row0);
                const uint32_t bytes = (uint32_t)(rows * p.row_bytes);
                mbar_arrive_expect_tx(full0 + 8 * stg, bytes);
                bulk_g2s(ring + stg * p.stage_bytes, p.w + (int64_t)row0 * p.row_bytes, bytes, full0 + 8 * stg);
            }
            if (image_due) issue_image();
            // On abort, let every copy this CTA issued land before it exits.
            if (*s_abort) {
                if (FUSED && p.image) mbar_wait_bounded(sbase + kHdrImage, 0u);
                const int issued = it;
                for (int k = issued > S ? issued - S : 0; k < issued; ++k)
                    mbar_wait_bounded(full0 + 8 * (k % S), (uint32_t)(k / S) & 1u);
            }
        }
        return;
    }

    // ---- compute warps: activations are read after the previous kernel is done
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (FUSED && p.spads[0] && p.swait) {  // (unfused: the host waits before the quantize kernel)
        shard_wait_prev(p);
        named_barrier_sync(kGemvThreads);
    }
    uint32_t quirk;
    ActSmem<TYPE> as{};
    ActGmem ag{p.qx, p.dx, p.bs, p.K, nb};
    if constexpr (FUSED) {
        uint8_t* qs = smem + kGemvSmemHeader;
        const uint32_t qbytes = (uint32_t)(M * act_row_stride(p.K));
        float* dxs = reinterpret_cast<float*>(qs + qbytes);
        int* bss = reinterpret_cast<int*>(qs + qbytes + 4u * (uint32_t)(M * nb));
        int* hss = reinterpret_cast<int*>(qs + qbytes + 8u * (uint32_t)(M * nb));
        uint32_t qm = 0;
        if (p.image) {
            // the producer copies the image in; masks sit just below the activations
            if (!mbar_wait_or_abort(sbase + kHdrImage, 0u, s_abort)) qm = 0;
            const uint32_t* masks = reinterpret_cast<const uint32_t*>(smem + kGemvSmemHeader - kImageHeader);
            for (int c = 0; c < p.image_ctas; ++c) qm |= masks[c];
        } else {
            qm = quantize_to_smem<M, TYPE>(p.x, p.K, qs, dxs, bss, hss, s_quirk, p.pre,
                                           reinterpret_cast<float*>(smem + kHdrPre), p.sb_lanes != 0);
        }
        quirk = (TYPE == kQ8_0 || TYPE == kQ6_K) ? qm : 0u;
        as = ActSmem<TYPE>{smem_addr(qs), smem_addr(dxs), smem_addr(bss), smem_addr(hss), act_row_stride(p.K), nb};
    } else {
        quirk = gemv_quirk_mask_compute<TYPE, M>(p, s_quirk);
    }

    const int r = warp / p.wpr, slice = warp - r * p.wpr;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        const int stg = it % S;
        if (!mbar_wait_or_abort(full0 + 8 * stg, (uint32_t)(it / S) & 1u, s_abort)) break;
        const int row0 = tile * p.rows_per_tile;
        const int rows = min(p.rows_per_tile, p.N - row0);
        if constexpr (FUSED && TYPE == kQ4_K) {
            if (p.sb_lanes) {  // lane = super-block: this warp takes 32 / sb_lanes rows of the tile
                const int lanes = p.sb_lanes, li = lane & (lanes - 1);
                const int rr = warp * (32 / lanes) + lane / lanes;
                float acc[M];
#pragma unroll
                for (int t = 0; t < M; ++t) acc[t] = 0.0f;
                if (rr < rows) {
                    int32_t* prow = EMIT ? p.partials + (int64_t)(row0 + rr) * nb : nullptr;
                    q4k_row_sb<M, EMIT>(ring + stg * p.stage_bytes + (uint32_t)(rr * p.row_bytes), as, p.K >> 8, li,
                                        lanes, acc, prow, (int64_t)p.N * nb);
                }
#pragma unroll
                for (int t = 0; t < M; ++t)
                    for (int o = lanes >> 1; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xFFFFFFFFu, acc[t], o);
                if (!EMIT && li == 0 && rr < rows) {
                    const int j = row0 + rr;
                    const float b = p.bias ? p.bias[j] : 0.0f;
#pragma unroll
                    for (int t = 0; t < M; ++t) gemv_put(p, t, j, acc[t] + b);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * stg);
                continue;
            }
        }
        if (r < rows) {
            float acc[M];
            SmemSrc src{ring + stg * p.stage_bytes + (uint32_t)(r * p.row_bytes)};
            int32_t* prow = nullptr;
            int64_t pstride = 0;
            if constexpr (EMIT) {
                const int ppr = (TYPE == kQ6_K) ? 2 * nb : nb;
                prow = p.partials + (int64_t)(row0 + r) * ppr;
                pstride = (int64_t)p.N * ppr;
            }
            if constexpr (FUSED && TYPE == kQ4_K)
                q4k_row_fused<M, EMIT>(src.base, as, units_per_row(TYPE, p.K), slice, p.wpr, acc, prow, pstride);
            else if constexpr (FUSED && TYPE == kQ6_K)
                q6k_row_fused<M, EMIT>(src.base, as, units_per_row(TYPE, p.K), slice, p.wpr, quirk, acc, prow,
                                       pstride);
            else if constexpr (FUSED) gemv_row_slice<TYPE, M, EMIT, 16>(src, as, row0 + r, p, slice, quirk, acc);
            else gemv_row_slice<TYPE, M, EMIT, 16>(src, ag, row0 + r, p, slice, quirk, acc);
            if constexpr (!EMIT) {
                const int j = row0 + r;
                if (p.wpr == 1) {
                    gemv_store_row<M>(j, acc, p);
                } else if (lane == 0) {
                    float* red = s_red + (stg * kGemvWarps + warp) * 8;
#pragma unroll
                    for (int t = 0; t < M; ++t) red[t] = acc[t];
                    __threadfence_block();
                    int* cnt = s_count + stg * 8 + r;
                    if (atomicAdd(cnt, 1) == p.wpr - 1) {
                        __threadfence_block();
                        *cnt = 0;
                        const float b = p.bias ? p.bias[j] : 0.0f;
#pragma unroll
                        for (int t = 0; t < M; ++t) {
                            float sum = 0.0f;
                            for (int k = 0; k < p.wpr; ++k)
                                sum += *reinterpret_cast<volatile float*>(s_red + (stg * kGemvWarps + r * p.wpr + k) * 8 + t);
                            gemv_put(p, t, j, sum + b);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * stg);
    }
    if (p.spads[0] && p.sarrive) {
        named_barrier_sync(kGemvThreads);
        shard_arrive_cta(p);
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
    if (p.spads[0]) {
        __syncthreads();
        shard_arrive_cta(p);
    }
}

}  // namespace cllm
