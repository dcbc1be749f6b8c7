// Prefill path (n_rows >= kTcMinRows): matmul_quant_batch
// (reference src/core/quant.cpp:1433-1475) as a tcgen05 tensor-core GEMM.
//
// Numerics.  The reference scales every 32-value block separately:
//     y[t][j] = sum_b dx[t][b] * dw[j][b] * P_b[t][j]  (+ the Q4_K min term)
// so block partials cannot be summed in an integer accumulator.  This kernel
// multiplies exact small integers on the tensor core with kind::f16:
//   A = activations as fp16 q_x (|q_x| <= 128, exact),
//   B = Q4_K weights dequantized in shared memory to fp16 sc*q (<= 945, exact),
// one TMEM accumulator per 32-value block.  Every product and every partial
// sum is an integer below 2^22, so each block's accumulator is the exact
// sc*P_b.  With r_b = dmin*m_b/d per weight row and sub-block, the epilogue
// keeps acc = sum_b dx_b * (sc*P_b - bsum_b * r_b) in registers (two FMAs per
// element and block; dx is constant along a TMEM lane, i.e. a token) and once
// per 256-value super-block adds y += d * acc into a TMEM-resident y.  A
// super-block with d == 0 is dequantized with sc = 0 and scaled by 1, so its
// contribution is the min term alone.
// Tile: 128 tokens (MMA M, TMEM lanes) x 128 weight rows (MMA N), K in
// chunks of 64 (one 128-byte SW128 row of fp16).  Warp roles (14 warps):
//   0      producer: TMA tiles of the fp16 activations and of the raw Q4_K
//          super-blocks (2-D tensor maps, no multicast)
//   1      TMEM allocation and the single-thread MMA issue
//   2..5   dequantization: thread i turns row i's super-block into fp16 B
//   6..13  epilogue: warp w reads TMEM lanes 32*(w%4).., columns 64*half..
// All barrier waits are bounded (kWaitLimitNs) and abort the whole CTA.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace cllm {

// From 32 activation rows the tensor-core GEMM beats the GEMV in chunks of 8
// rows (measured on the 8B shapes: at 32 rows the GEMV's four chunks take
// 1.2-3x the GEMM's time, except on the 1024-row k/v matrices, where the two tie).
constexpr int kTcMinRows = 32;
constexpr int kTcBM = 128, kTcBN = 128, kTcBK = 64;
constexpr int kTcStA = 4, kTcStB = 4, kTcStRaw = 2, kTcDBuf = 3;
constexpr int kTcWarps = 14;
constexpr int kTcThreads = kTcWarps * 32;
constexpr uint32_t kTcTileBytes = kTcBM * kTcBK * 2;  // 16 KB fp16 operand tile
constexpr uint32_t kTcRawBytes = kTcBN * 144;         // one Q4_K super-block per row
constexpr uint32_t kTcScBytes = kTcBN * 9 * 4;        // d[128], then r[8][128]
constexpr uint32_t kTcDxBytes = kTcBM * 16 * 4;       // (dx, dx*bsum) of 8 blocks x 128 tokens, block-major
// shared-memory layout (offsets from a 1024-aligned base)
constexpr uint32_t kTcOffA = 0;
constexpr uint32_t kTcOffB = kTcOffA + kTcStA * kTcTileBytes;
constexpr uint32_t kTcOffRaw = kTcOffB + kTcStB * kTcTileBytes;
constexpr uint32_t kTcOffSc = kTcOffRaw + kTcStRaw * kTcRawBytes;
constexpr uint32_t kTcOffDx = kTcOffSc + 2 * kTcScBytes;
constexpr uint32_t kTcOffBar = kTcOffDx + 2 * kTcDxBytes;
constexpr uint32_t kTcSmemBytes = kTcOffBar + 512 + 1024;  // + alignment slack
// barrier indices (8 bytes each, from kTcOffBar)
enum : int {
    kBarAFull = 0, kBarAEmpty = kBarAFull + kTcStA, kBarBFull = kBarAEmpty + kTcStA,
    kBarBEmpty = kBarBFull + kTcStB, kBarRawFull = kBarBEmpty + kTcStB,
    kBarRawEmpty = kBarRawFull + kTcStRaw, kBarScFull = kBarRawEmpty + kTcStRaw,
    kBarScEmpty = kBarScFull + 2, kBarDFull = kBarScEmpty + 2, kBarDEmpty = kBarDFull + kTcDBuf,
    kBarDxFull = kBarDEmpty + kTcDBuf, kBarDxEmpty = kBarDxFull + 2,
    kBarMmaDone = kBarDxEmpty + 2, kBarCount = kBarMmaDone + 1
};
constexpr uint32_t kTcOffTmem = kTcOffBar + 8 * kBarCount;  // u32 TMEM base address
constexpr uint32_t kTcOffAbort = kTcOffTmem + 4;
static_assert(kTcOffAbort + 4 <= kTcOffBar + 512, "barrier area");

struct TcParams {
    int M, N, K;
    const float* bias;  // [N] or nullptr
    float* y;           // [M][N]
    int tma_store;      // 1: y through map_y (N % 4 == 0, y 16-byte aligned)
};

// ---- PTX wrappers --------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// K-major, 128-byte swizzled operand tile: rows of 128 bytes, 8-row groups
// 1024 bytes apart (SBO), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, fp32 accumulate, A = B = fp16, both K-major, M = 128, N = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcBN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.ld without the wait, and the wait tied to the destination registers
// (as in/out operands) so that no use of them can move above it.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// Wait on an mbarrier phase as a whole warp: lane 0 polls, the outcome is
// broadcast, so warp-collective tcgen05 instructions that follow see every
// lane on the same path.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait_or_abort(bar, parity, abort) ? 1 : 0;
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    __syncwarp();
    return ok != 0;
}

__device__ __forceinline__ void sts128(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

// fp16 pair (sc*n0, sc*n1) from two 4-bit values in bytes b0, b1 of w: the
// pair 0x64nn is 1024 + n exactly, and fma(1024 + n, sc, -1024 sc) = sc*n is
// exact (it is an integer <= 945, rounded once).
__device__ __forceinline__ uint32_t nib_pair_scaled(uint32_t w, uint32_t sel, uint32_t sc2, uint32_t nsc2) {
    const uint32_t h = __byte_perm(w, 0x00006464u, sel);
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(h), "r"(sc2), "r"(nsc2));
    return r;
}

// Eight fp16 weights (one 16-byte chunk of B) from bytes 0..7 of (w0, w1),
// already masked to 4 bits per byte.
__device__ __forceinline__ uint4 nib8_scaled(uint32_t w0, uint32_t w1, uint32_t sc2, uint32_t nsc2) {
    uint4 o;
    o.x = nib_pair_scaled(w0, 0x5140u, sc2, nsc2);  // bytes 0,1
    o.y = nib_pair_scaled(w0, 0x5342u, sc2, nsc2);  // bytes 2,3
    o.z = nib_pair_scaled(w1, 0x5140u, sc2, nsc2);
    o.w = nib_pair_scaled(w1, 0x5342u, sc2, nsc2);
    return o;
}

__device__ __forceinline__ uint32_t half2_bits(float v) {
    const __half h = __float2half_rn(v);  // only exact small integers are passed
    const uint32_t b = __half_as_ushort(h);
    return b | (b << 16);
}

// One 16-column group G of a block in the epilogue: per element
// acc = fma(dx, D, acc), then acc = fma(-dx*bsum, r, acc).  (Packed f32x2 FMAs
// here raise register pressure past the 128-register ceiling.)
template <int G>
__device__ __forceinline__ void epi_group(float2 (&acc)[32], const uint32_t (&v)[16], uint32_t rq, float2 dx2,
                                          float2 nx2) {
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
        const float4 r = lds128f(rq + 64u * G + 16u * j4);
        float2& a0 = acc[8 * G + 2 * j4];
        float2& a1 = acc[8 * G + 2 * j4 + 1];
        a0.x = fmaf(dx2.x, __uint_as_float(v[4 * j4]), a0.x);
        a0.y = fmaf(dx2.x, __uint_as_float(v[4 * j4 + 1]), a0.y);
        a1.x = fmaf(dx2.x, __uint_as_float(v[4 * j4 + 2]), a1.x);
        a1.y = fmaf(dx2.x, __uint_as_float(v[4 * j4 + 3]), a1.y);
        a0.x = fmaf(nx2.x, r.x, a0.x);
        a0.y = fmaf(nx2.x, r.y, a0.y);
        a1.x = fmaf(nx2.x, r.z, a1.x);
        a1.y = fmaf(nx2.x, r.w, a1.y);
    }
}

// 14 warps put 4 warps on some SM sub-partitions (16384 registers each), so
// 128 registers per thread is the ceiling.
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_q4k_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                       const __grid_constant__ CUtensorMap map_dx, const __grid_constant__ CUtensorMap map_y,
                       const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tok0 = blockIdx.x * kTcBM, row0 = blockIdx.y * kTcBN;
    const int nsb = p.K >> 8;         // super-blocks
    const int nchunk = p.K / kTcBK;   // 64-value chunks
    auto bar = [&](int i) { return sb + kTcOffBar + 8u * (uint32_t)i; };
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kTcOffAbort);
    volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(smem + kTcOffTmem);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTcStA; ++i) { mbar_init(bar(kBarAFull + i), 1); mbar_init(bar(kBarAEmpty + i), 1); }
        for (int i = 0; i < kTcStB; ++i) { mbar_init(bar(kBarBFull + i), 4); mbar_init(bar(kBarBEmpty + i), 1); }
        for (int i = 0; i < kTcStRaw; ++i) { mbar_init(bar(kBarRawFull + i), 1); mbar_init(bar(kBarRawEmpty + i), 4); }
        for (int i = 0; i < 2; ++i) { mbar_init(bar(kBarScFull + i), 4); mbar_init(bar(kBarScEmpty + i), 8); }
        for (int i = 0; i < kTcDBuf; ++i) { mbar_init(bar(kBarDFull + i), 1); mbar_init(bar(kBarDEmpty + i), 8); }
        for (int i = 0; i < 2; ++i) { mbar_init(bar(kBarDxFull + i), 1); mbar_init(bar(kBarDxEmpty + i), 8); }
        mbar_init(bar(kBarMmaDone), 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {  // 512 TMEM columns: 3 block accumulators + the running y
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sb + kTcOffTmem)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            int issued_raw = 0, issued_a = 0;
            for (int s = 0; s < nsb && !*s_abort; ++s) {
                const int rs = s % kTcStRaw;
                if (s >= kTcStRaw &&
                    !mbar_wait_or_abort(bar(kBarRawEmpty + rs), (uint32_t)((s / kTcStRaw) - 1) & 1u, s_abort))
                    break;
                mbar_arrive_expect_tx(bar(kBarRawFull + rs), kTcRawBytes);
                tma_load_2d(sb + kTcOffRaw + rs * kTcRawBytes, &map_w, 144 * s, row0, bar(kBarRawFull + rs));
                ++issued_raw;
                const int xs = s & 1;
                if (s >= 2 && !mbar_wait_or_abort(bar(kBarDxEmpty + xs), (uint32_t)((s >> 1) - 1) & 1u, s_abort))
                    break;
                mbar_arrive_expect_tx(bar(kBarDxFull + xs), kTcDxBytes);
                tma_load_2d(sb + kTcOffDx + xs * kTcDxBytes, &map_dx, 2 * tok0, 8 * s, bar(kBarDxFull + xs));
                for (int q = 0; q < 4; ++q) {
                    const int c = 4 * s + q, as = c % kTcStA;
                    if (c >= kTcStA &&
                        !mbar_wait_or_abort(bar(kBarAEmpty + as), (uint32_t)((c / kTcStA) - 1) & 1u, s_abort))
                        break;
                    mbar_arrive_expect_tx(bar(kBarAFull + as), kTcTileBytes);
                    tma_load_2d(sb + kTcOffA + as * kTcTileBytes, &map_a, kTcBK * c, tok0, bar(kBarAFull + as));
                    ++issued_a;
                }
            }
            if (*s_abort) {  // let issued copies land before the CTA can exit
                for (int k = issued_raw > kTcStRaw ? issued_raw - kTcStRaw : 0; k < issued_raw; ++k)
                    mbar_wait_bounded(bar(kBarRawFull + k % kTcStRaw), (uint32_t)(k / kTcStRaw) & 1u);
                for (int k = issued_a > kTcStA ? issued_a - kTcStA : 0; k < issued_a; ++k)
                    mbar_wait_bounded(bar(kBarAFull + k % kTcStA), (uint32_t)(k / kTcStA) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (one thread)
        if (lane == 0) {
            for (int c = 0; c < nchunk; ++c) {
                const int as = c % kTcStA, bs = c % kTcStB;
                if (!mbar_wait_or_abort(bar(kBarAFull + as), (uint32_t)(c / kTcStA) & 1u, s_abort)) break;
                if (!mbar_wait_or_abort(bar(kBarBFull + bs), (uint32_t)(c / kTcStB) & 1u, s_abort)) break;
                tc_fence_after();
                const uint32_t a_base = sb + kTcOffA + as * kTcTileBytes, b_base = sb + kTcOffB + bs * kTcTileBytes;
                bool ok = true;
                for (int h = 0; h < 2; ++h) {
                    const int b = 2 * c + h, db = b % kTcDBuf;
                    if (b >= kTcDBuf &&
                        !mbar_wait_or_abort(bar(kBarDEmpty + db), (uint32_t)((b / kTcDBuf) - 1) & 1u, s_abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem + (uint32_t)(db * kTcBN);
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint32_t koff = (uint32_t)(2 * h + kk) * 32u;  // bytes: 16 fp16 per MMA
                        tc_mma(d_tmem, umma_desc_sw128(a_base + koff), umma_desc_sw128(b_base + koff), kk);
                    }
                    tc_commit(bar(kBarDFull + db));
                }
                if (!ok) break;
                tc_commit(bar(kBarAEmpty + as));
                tc_commit(bar(kBarBEmpty + bs));
            }
            tc_commit(bar(kBarMmaDone));
            mbar_wait_bounded(bar(kBarMmaDone), 0);
        }
    } else if (warp < 6) {
        // ---------------- dequantization: thread i owns weight row i of the tile
        const int i = threadIdx.x - 64;
        for (int s = 0; s < nsb; ++s) {
            const int rs = s % kTcStRaw;
            if (!mbar_wait_or_abort(bar(kBarRawFull + rs), (uint32_t)(s / kTcStRaw) & 1u, s_abort)) break;
            const uint32_t rb = sb + kTcOffRaw + rs * kTcRawBytes + 144u * (uint32_t)i;
            const uint4 hd = lds128(rb);
            // 6-bit scales and mins of the 8 sub-blocks (get_scale_min_k4, quant.cpp:72-80)
            const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
            // d == 0 zeroes the main term: B gets sc = 0 and the epilogue scale becomes 1
            const bool dz = (d == 0.0f);
            const float d_eff = dz ? 1.0f : d;
            const uint32_t sc_lo = dz ? 0u : (hd.y & 0x3F3F3F3Fu), m_lo = hd.z & 0x3F3F3F3Fu;
            const uint32_t sc_hi = dz ? 0u : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
            const uint32_t m_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
            // epilogue scales for this super-block: d, and r_k = dmin*m_k/d per sub-block, so that
            // d * sum_k dx_k (P_k - bsum_k r_k) = sum_k (d dx_k P_k - dmin m_k dx_k bsum_k)
            const int ss = s & 1;
            if (s >= 2 && !mbar_wait_or_abort(bar(kBarScEmpty + ss), (uint32_t)((s >> 1) - 1) & 1u, s_abort)) break;
            const uint32_t sco = sb + kTcOffSc + (uint32_t)ss * kTcScBytes;
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(sco + 4u * (uint32_t)i), "f"(d_eff) : "memory");
            // r as [8][128]: one sub-block's values for consecutive rows are contiguous
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t mw = k < 4 ? m_lo : m_hi;
                const float r = (dmin * (float)((mw >> (8 * (k & 3))) & 0xFFu)) / d_eff;
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(sco + 4u * (uint32_t)(kTcBN * (k + 1) + i)), "f"(r)
                             : "memory");
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarScFull + ss));
            bool ok = true;
            for (int pq = 0; pq < 4; ++pq) {
                const int c = 4 * s + pq, bs = c % kTcStB;
                if (c >= kTcStB && !mbar_wait_or_abort(bar(kBarBEmpty + bs), (uint32_t)((c / kTcStB) - 1) & 1u, s_abort)) {
                    ok = false;
                    break;
                }
                const uint32_t scw = pq < 2 ? sc_lo : sc_hi;
                const uint32_t s0 = (scw >> (16 * (pq & 1))) & 0xFFu, s1 = (scw >> (16 * (pq & 1) + 8)) & 0xFFu;
                const uint32_t sc0 = half2_bits((float)s0), sc1 = half2_bits((float)s1);
                const uint32_t nsc0 = half2_bits(-1024.0f * (float)s0), nsc1 = half2_bits(-1024.0f * (float)s1);
                // row i of B (128 bytes = 64 fp16): values 0..31 = sub-block 2pq (low nibbles of
                // q[32pq..32pq+31]), values 32..63 = sub-block 2pq+1 (high nibbles)
                const uint32_t brow = sb + kTcOffB + bs * kTcTileBytes + (uint32_t)(i >> 3) * 1024u + (uint32_t)(i & 7) * 128u;
                // the 32 quant bytes of sub-block pair pq
                const uint4 qa = lds128(rb + 16u + 32u * (uint32_t)pq), qb = lds128(rb + 32u + 32u * (uint32_t)pq);
                const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    const int w0i = 2 * (ch & 3);
                    uint32_t w0 = q[w0i], w1 = q[w0i + 1];
                    uint4 o;
                    if (ch < 4) {
                        o = nib8_scaled(w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, sc0, nsc0);
                    } else {
                        o = nib8_scaled((w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu, sc1, nsc1);
                    }
                    const uint32_t dst = brow + (uint32_t)((ch ^ (i & 7)) << 4);
                    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o.x), "r"(o.y), "r"(o.z),
                                 "r"(o.w)
                                 : "memory");
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarBFull + bs));
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarRawEmpty + rs));
        }
    } else {
        // ---------------- epilogue: thread = token, 64 columns
        const int quad = warp & 3, half = (warp - 6) >> 2;
        const int tl = 32 * quad + lane;  // token within the tile = TMEM lane
        const int t = tok0 + tl;
        const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
        const uint32_t ycol = (uint32_t)(kTcDBuf * kTcBN + 64 * half);  // running y in TMEM
        float2 acc[32];
        for (int s = 0; s < nsb; ++s) {
            const int xs = s & 1, ss = s & 1;
            if (!warp_wait(bar(kBarDxFull + xs), (uint32_t)(s >> 1) & 1u, s_abort)) break;
            if (!warp_wait(bar(kBarScFull + ss), (uint32_t)(s >> 1) & 1u, s_abort)) break;
            // (dx, dx*bsum) of blocks 8s..8s+7 for this token
            // (dx, dx*bsum) of block k for this token at dxa + 1024 k: consecutive lanes, consecutive pairs
            const uint32_t dxa = sb + kTcOffDx + (uint32_t)xs * kTcDxBytes + 8u * (uint32_t)tl;
            const uint32_t sca = sb + kTcOffSc + (uint32_t)ss * kTcScBytes;
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.0f, 0.0f);
            bool ok = true;
#pragma unroll 1
            for (int k = 0; k < 8; ++k) {
                const int b = 8 * s + k, db = b % kTcDBuf;
                if (!warp_wait(bar(kBarDFull + db), (uint32_t)(b / kTcDBuf) & 1u, s_abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tmem + lane_base + (uint32_t)(db * kTcBN + 64 * half);
                const uint32_t rq = sca + 4u * (uint32_t)(kTcBN * (k + 1) + 64 * half);
                float dxk, xmk;
                asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(dxk), "=f"(xmk) : "r"(dxa + 1024u * (uint32_t)k));
                const float2 dx2 = make_float2(dxk, dxk), nx2 = make_float2(-xmk, -xmk);
                // the TMEM load of the next 16 columns overlaps the FMAs of the current ones
                uint32_t v0[16], v1[16];
                tmem_ld16_issue(dcol, v0);
                tmem_ld_wait(v0);
                tmem_ld16_issue(dcol + 16u, v1);
                epi_group<0>(acc, v0, rq, dx2, nx2);
                tmem_ld_wait(v1);
                tmem_ld16_issue(dcol + 32u, v0);
                epi_group<1>(acc, v1, rq, dx2, nx2);
                tmem_ld_wait(v0);
                tmem_ld16_issue(dcol + 48u, v1);
                epi_group<2>(acc, v0, rq, dx2, nx2);
                tmem_ld_wait(v1);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarDEmpty + db));
                epi_group<3>(acc, v1, rq, dx2, nx2);
            }
            if (!ok) break;
            // super-block end: y += d * acc
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float yv[16];
                const uint32_t ya = tmem + lane_base + ycol + 16u * cg;
                if (s > 0) {
                    tmem_ld16(ya, yv);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) yv[j] = 0.0f;
                }
                const uint32_t dq = sca + 4u * (uint32_t)(64 * half + 16 * cg);
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 d = lds128f(dq + 16u * j4);
                    const float2 y0 = __ffma2_rn(make_float2(d.x, d.y), acc[8 * cg + 2 * j4],
                                                 make_float2(yv[4 * j4], yv[4 * j4 + 1]));
                    const float2 y1 = __ffma2_rn(make_float2(d.z, d.w), acc[8 * cg + 2 * j4 + 1],
                                                 make_float2(yv[4 * j4 + 2], yv[4 * j4 + 3]));
                    yv[4 * j4] = y0.x; yv[4 * j4 + 1] = y0.y; yv[4 * j4 + 2] = y1.x; yv[4 * j4 + 3] = y1.y;
                }
                tmem_st16(ya, yv);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(kBarScEmpty + ss));
                mbar_arrive(bar(kBarDxEmpty + xs));
            }
        }
        // write y (+ bias); tcgen05.ld is warp-collective, so every lane loads
        const int aborted = __shfl_sync(0xFFFFFFFFu, *s_abort, 0);
        if (!aborted && p.tma_store) {
            // Stage this warp's 32 tokens x 64 columns in the (now idle) A-operand
            // buffers as two 32x32 fp32 boxes in the 128-byte swizzled layout, then
            // one TMA store per box; TMA clips rows >= M and columns >= N.
            const uint32_t stage = sb + kTcOffA + (uint32_t)(warp - 6) * 8192u;
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float yv[16];
                tmem_ld16(tmem + lane_base + ycol + 16u * cg, yv);
                const int j0 = row0 + 64 * half + 16 * cg;
                if (p.bias) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) yv[j] += (j0 + j < p.N) ? p.bias[j0 + j] : 0.0f;
                }
                const uint32_t box = stage + (uint32_t)(cg >> 1) * 4096u + (uint32_t)lane * 128u;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t chunk = (uint32_t)((cg & 1) * 4 + q) ^ (uint32_t)(lane & 7);
                    sts128(box + (chunk << 4), yv[4 * q], yv[4 * q + 1], yv[4 * q + 2], yv[4 * q + 3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int bx = 0; bx < 2; ++bx)
                    tma_store_2d(&map_y, row0 + 64 * half + 32 * bx, tok0 + 32 * quad, stage + 4096u * bx);
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
            }
            __syncwarp();
        } else if (!aborted) {
#pragma unroll
            for (int cg = 0; cg < 4; ++cg) {
                float yv[16];
                tmem_ld16(tmem + lane_base + ycol + 16u * cg, yv);
                const int j0 = row0 + 64 * half + 16 * cg;
                if (t < p.M) {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (j0 + j < p.N) p.y[(int64_t)t * p.N + j0 + j] = yv[j] + (p.bias ? p.bias[j0 + j] : 0.0f);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// Prefill activation preparation: quantize_row_q8_0 per 32-value block
// (bit-exact, as quantize_q8_0_kernel), writing q_x as fp16 and, where the
// pointers are given, the pairs (dx, dx*bsum) block-major [nb][mp][2] (Q4_K),
// dx block-major [nb][mp] (Q6_K) and a flag per block that holds a -128 (Q6_K).
template <bool VEC>
__global__ void __launch_bounds__(256) prefill_prep_kernel(const float* __restrict__ x, int64_t n,
                                                           int64_t total_blocks, __half* __restrict__ a16,
                                                           float* __restrict__ dxx, float* __restrict__ dxT,
                                                           int64_t mp, uint8_t* __restrict__ flags) {
    // four lanes per 32-value block, eight values each (two float4 loads when
    // VEC: x 16-byte aligned); a warp takes eight blocks per step
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t nb = n >> 5;
    for (int64_t base = 8 * warp0; base < total_blocks; base += 8 * nwarps) {
        const int64_t blk = base + (lane >> 2);
        const bool valid = blk < total_blocks;
        const int64_t r = valid ? blk / nb : 0, b = valid ? blk - r * nb : 0;
        const int64_t e0 = r * n + b * 32 + 8 * sub;
        float v[8];
        if (valid) {
            if constexpr (VEC) {
                const float4 p0 = __ldg(reinterpret_cast<const float4*>(x + e0));
                const float4 p1 = __ldg(reinterpret_cast<const float4*>(x + e0) + 1);
                v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
                v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = __ldg(x + e0 + k);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = 0.0f;
        }
        // max of |x| over the block's non-NaN values (fmaxf keeps the number)
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
        const float d = amax / 127.0f;
        const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        int q[8], s8 = 0;
        bool has_min = false;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float vv = v[k] * id;
            int qi = fabsf(vv) < 4194304.0f ? __float_as_int(vv + 12582912.0f) - 0x4B400000 : INT32_MIN;
            qi = qi > 127 ? 127 : (qi < -128 ? -128 : qi);
            q[k] = qi;
            s8 += qi;
            has_min |= qi == -128;
        }
        int s = s8 + __shfl_xor_sync(0xFFFFFFFFu, s8, 1);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
        const unsigned neg = (__ballot_sync(0xFFFFFFFFu, has_min) >> (lane & ~3)) & 0xFu;
        if (!valid) continue;
        __half2 h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __halves2half2(__int2half_rn(q[2 * k]), __int2half_rn(q[2 * k + 1]));
        if constexpr (VEC) {
            *reinterpret_cast<uint4*>(a16 + e0) = *reinterpret_cast<const uint4*>(h);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) *reinterpret_cast<__half2*>(a16 + e0 + 2 * k) = h[k];
        }
        if (sub == 0) {
            if (dxx) {  // (dx, dx*bsum) pairs, [nb][mp][2]
                dxx[2 * (b * mp + r)] = d;
                dxx[2 * (b * mp + r) + 1] = d * (float)s;
            }
            if (dxT) dxT[b * mp + r] = d;
            if (flags) flags[r * nb + b] = neg ? 1 : 0;
        }
    }
}

}  // namespace cllm
