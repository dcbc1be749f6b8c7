// Prefill path for Q6_K weights (n_rows >= kTcMinRows): matmul_quant_batch
// (reference src/core/quant.cpp:1433-1475) over vec_dot_q6_K_q8_0
// (quant.cpp:630-687) as a tcgen05 tensor-core GEMM.
//
// Numerics.  Q6_K has one int8 scale per 16 weights, so the reference's
// per-block term is
//     d * dx_b * (sa_b * P_b,lo + sb_b * P_b,hi)
// with P the exact integer dots of the two 16-value halves.  The weights enter
// the tensor core as the exact fp16 integers q6 - 32 (|.| <= 32), the
// activations as fp16 q_x (|.| <= 128): products and 16-term sums are exact
// integers.  sc * (q6 - 32) needs 13 significant bits, more than fp16 holds,
// so the scale stays out of the operand: every 16-value half gets its own
// TMEM accumulator, one K=16 MMA each.
// The operand roles are swapped against the Q4_K kernel: MMA M = 128 weight
// rows (TMEM lanes, so a row's scales are per-thread registers in the
// epilogue), MMA N = 128 tokens (columns).  The epilogue thread for row j
// keeps, for 64 tokens,
//     acc += dx_b * ((d*sa_b) * D_lo + (d*sb_b) * D_hi)
// over the whole K in registers (d folded into the scales, which are per row),
// so no running y lives in TMEM: all 512 columns hold two blocks' pairs of
// accumulators, double-buffered.
//
// The AVX2 dot negates the activation byte where the weight is negative
// (quant.cpp:676-679); -(-128) wraps, so an activation of -128 (produced only
// by a NaN input, quant.cpp:444-447) against a weight w < 0 contributes
// 128*w.  The tensor core computes -128*w; prefill_q6k_finish_kernel adds the
// difference 256*w for the (token, block) pairs the preparation flagged.
//
// Few tiles (small M): split-K over blockIdx.z, the partial sums summed by
// prefill_q6k_finish_kernel in a fixed order.
//
// Tile: 128 weight rows x 128 tokens, K in chunks of 64.  Warp roles (14):
//   0      producer: TMA of the raw super-blocks (224-byte boxes from the
//          16-byte boundary at or below each 210-byte super-block), of dx per
//          block and token, and of the fp16 activation tiles (no multicast)
//   1      TMEM allocation and the single-thread MMA issue
//   2..5   dequantization: thread i turns row i's super-block into fp16
//          q6 - 32 and the 16 scales d*sc
//   6..13  epilogue: warp w reads TMEM lanes 32*(w%4).., tokens 64*half..
// All barrier waits are bounded (kWaitLimitNs) and abort the whole CTA.
#pragma once
#include "gemm_tc.cuh"

namespace cllm {

constexpr int kQ6StX = 4, kQ6StW = 4, kQ6StRaw = 2;
constexpr uint32_t kQ6RawRow = 224;                  // TMA box width per weight row
constexpr uint32_t kQ6RawBytes = kTcBN * kQ6RawRow;  // one super-block of 128 rows
constexpr uint32_t kQ6ScBytes = 16 * kTcBN * 4;      // d*sc as [16][128 rows]
constexpr uint32_t kQ6DxBytes = 8 * kTcBM * 4;       // dx as [8 blocks][128 tokens]
constexpr uint32_t kQ6OffX = 0;
constexpr uint32_t kQ6OffW = kQ6OffX + kQ6StX * kTcTileBytes;
constexpr uint32_t kQ6OffRaw = kQ6OffW + kQ6StW * kTcTileBytes;
constexpr uint32_t kQ6OffSc = kQ6OffRaw + kQ6StRaw * kQ6RawBytes;
constexpr uint32_t kQ6OffDx = kQ6OffSc + 2 * kQ6ScBytes;
constexpr uint32_t kQ6OffBar = kQ6OffDx + 2 * kQ6DxBytes;
constexpr uint32_t kQ6SmemBytes = kQ6OffBar + 512 + 1024;  // + alignment slack
static_assert(kQ6SmemBytes <= 227 * 1024, "Q6_K prefill shared memory");
enum : int {
    kQ6XFull = 0, kQ6XEmpty = kQ6XFull + kQ6StX, kQ6WFull = kQ6XEmpty + kQ6StX,
    kQ6WEmpty = kQ6WFull + kQ6StW, kQ6RawFull = kQ6WEmpty + kQ6StW,
    kQ6RawEmpty = kQ6RawFull + kQ6StRaw, kQ6ScFull = kQ6RawEmpty + kQ6StRaw,
    kQ6ScEmpty = kQ6ScFull + 2, kQ6DFull = kQ6ScEmpty + 2, kQ6DEmpty = kQ6DFull + 2,
    kQ6DxFull = kQ6DEmpty + 2, kQ6DxEmpty = kQ6DxFull + 2, kQ6MmaDone = kQ6DxEmpty + 2,
    kQ6BarCount = kQ6MmaDone + 1
};
constexpr uint32_t kQ6OffTmem = kQ6OffBar + 8 * kQ6BarCount;
constexpr uint32_t kQ6OffAbort = kQ6OffTmem + 4;
static_assert(kQ6OffAbort + 4 <= kQ6OffBar + 512, "Q6_K barrier area");

struct Q6Params {
    int M, N, K;
    const float* bias;  // [N] or nullptr
    float* y;           // [M][N]
    // split-K (few tiles): CTA z of `splits` takes super-blocks
    // [z*nsb/splits, (z+1)*nsb/splits) and writes its partial sums to
    // ypart[z][M][N] (no bias); prefill_q6k_finish_kernel adds them up
    int splits;
    float* ypart;
};

// tcgen05.ld of 8 consecutive columns, and its wait tied to the registers.
__device__ __forceinline__ void tmem_ld8_issue(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait2(uint32_t (&a)[8], uint32_t (&b)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])
                 :
                 : "memory");
}

// NW words of shared memory from a 2-byte aligned address.
template <int NW>
__device__ __forceinline__ void lds_words_a2(uint32_t a, uint32_t (&w)[NW]) {
    const uint32_t al = a & ~3u;
    uint32_t r[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) r[i] = lds32(al + 4u * i);
    const uint32_t sh = (a & 2u) * 8u;  // 0 or 16
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// Eight fp16 values q6 - 32 for one 16-byte chunk of a W row.
__device__ __forceinline__ uint4 q6_chunk(uint32_t q0, uint32_t q1) {
    const uint32_t one2 = 0x3C003C00u, m2 = 0xE420E420u;  // (1.0, 1.0), (-1056, -1056)
    return nib8_scaled(q0, q1, one2, m2);
}

__device__ __forceinline__ float lds32f(uint32_t a) { return __uint_as_float(lds32(a)); }


__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_q6k_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                       const __grid_constant__ CUtensorMap map_dx, const Q6Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tok0 = blockIdx.x * kTcBM, row0 = blockIdx.y * kTcBN;
    // this CTA's super-blocks [s0, s0 + nsb); loop counters below are local to it
    const int nsb_all = p.K >> 8;
    const int s0 = (int)((int64_t)blockIdx.z * nsb_all / p.splits);
    const int nsb = (int)((int64_t)(blockIdx.z + 1) * nsb_all / p.splits) - s0;
    const int nchunk = 4 * nsb;  // 64-value chunks
    auto bar = [&](int i) { return sb + kQ6OffBar + 8u * (uint32_t)i; };
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kQ6OffAbort);
    volatile uint32_t* s_tmem = reinterpret_cast<volatile uint32_t*>(smem + kQ6OffTmem);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kQ6StX; ++i) { mbar_init(bar(kQ6XFull + i), 1); mbar_init(bar(kQ6XEmpty + i), 1); }
        for (int i = 0; i < kQ6StW; ++i) { mbar_init(bar(kQ6WFull + i), 4); mbar_init(bar(kQ6WEmpty + i), 1); }
        for (int i = 0; i < kQ6StRaw; ++i) { mbar_init(bar(kQ6RawFull + i), 1); mbar_init(bar(kQ6RawEmpty + i), 4); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(kQ6ScFull + i), 4);
            mbar_init(bar(kQ6ScEmpty + i), 8);
            mbar_init(bar(kQ6DFull + i), 1);
            mbar_init(bar(kQ6DEmpty + i), 8);
            mbar_init(bar(kQ6DxFull + i), 1);
            mbar_init(bar(kQ6DxEmpty + i), 8);
        }
        mbar_init(bar(kQ6MmaDone), 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {  // 512 TMEM columns: two blocks x (low half, high half) x 128 tokens
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sb + kQ6OffTmem)
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
            int issued_raw = 0, issued_x = 0, issued_dx = 0;
            for (int s = 0; s < nsb && !*s_abort; ++s) {
                const int rs = s % kQ6StRaw;
                if (s >= kQ6StRaw &&
                    !mbar_wait_or_abort(bar(kQ6RawEmpty + rs), (uint32_t)((s / kQ6StRaw) - 1) & 1u, s_abort))
                    break;
                mbar_arrive_expect_tx(bar(kQ6RawFull + rs), kQ6RawBytes);
                // the box starts at the 16-byte boundary at or below byte 210*sg of each row
                const int sg = s0 + s;
                tma_load_2d(sb + kQ6OffRaw + rs * kQ6RawBytes, &map_w, (int)((210u * (uint32_t)sg) & ~15u), row0,
                            bar(kQ6RawFull + rs));
                ++issued_raw;
                const int xs = s & 1;
                if (s >= 2 && !mbar_wait_or_abort(bar(kQ6DxEmpty + xs), (uint32_t)((s >> 1) - 1) & 1u, s_abort))
                    break;
                mbar_arrive_expect_tx(bar(kQ6DxFull + xs), kQ6DxBytes);
                tma_load_2d(sb + kQ6OffDx + xs * kQ6DxBytes, &map_dx, tok0, 8 * sg, bar(kQ6DxFull + xs));
                ++issued_dx;
                for (int q = 0; q < 4; ++q) {
                    const int c = 4 * s + q, as = c % kQ6StX;
                    if (c >= kQ6StX &&
                        !mbar_wait_or_abort(bar(kQ6XEmpty + as), (uint32_t)((c / kQ6StX) - 1) & 1u, s_abort))
                        break;
                    mbar_arrive_expect_tx(bar(kQ6XFull + as), kTcTileBytes);
                    tma_load_2d(sb + kQ6OffX + as * kTcTileBytes, &map_x, kTcBK * (4 * sg + q), tok0,
                                bar(kQ6XFull + as));
                    ++issued_x;
                }
            }
            if (*s_abort) {  // let issued copies land before the CTA can exit
                for (int k = issued_raw > kQ6StRaw ? issued_raw - kQ6StRaw : 0; k < issued_raw; ++k)
                    mbar_wait_bounded(bar(kQ6RawFull + k % kQ6StRaw), (uint32_t)(k / kQ6StRaw) & 1u);
                for (int k = issued_x > kQ6StX ? issued_x - kQ6StX : 0; k < issued_x; ++k)
                    mbar_wait_bounded(bar(kQ6XFull + k % kQ6StX), (uint32_t)(k / kQ6StX) & 1u);
                for (int k = issued_dx > 2 ? issued_dx - 2 : 0; k < issued_dx; ++k)
                    mbar_wait_bounded(bar(kQ6DxFull + (k & 1)), (uint32_t)(k >> 1) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (one thread): per block, one K=16 MMA per half
        if (lane == 0) {
            for (int c = 0; c < nchunk; ++c) {
                const int xs = c % kQ6StX, ws = c % kQ6StW;
                if (!mbar_wait_or_abort(bar(kQ6XFull + xs), (uint32_t)(c / kQ6StX) & 1u, s_abort)) break;
                if (!mbar_wait_or_abort(bar(kQ6WFull + ws), (uint32_t)(c / kQ6StW) & 1u, s_abort)) break;
                tc_fence_after();
                const uint32_t x_base = sb + kQ6OffX + xs * kTcTileBytes, w_base = sb + kQ6OffW + ws * kTcTileBytes;
                bool ok = true;
                for (int h = 0; h < 2; ++h) {
                    const int b = 2 * c + h, db = b & 1;
                    if (b >= 2 && !mbar_wait_or_abort(bar(kQ6DEmpty + db), (uint32_t)((b >> 1) - 1) & 1u, s_abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem + (uint32_t)(db * 2 * kTcBM);
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t koff = (uint32_t)(2 * h + u) * 32u;  // bytes: 16 fp16 per MMA
                        tc_mma(d_tmem + (uint32_t)(u * kTcBM), umma_desc_sw128(w_base + koff),
                               umma_desc_sw128(x_base + koff), 0);
                    }
                    tc_commit(bar(kQ6DFull + db));
                }
                if (!ok) break;
                tc_commit(bar(kQ6XEmpty + xs));
                tc_commit(bar(kQ6WEmpty + ws));
            }
            tc_commit(bar(kQ6MmaDone));
            mbar_wait_bounded(bar(kQ6MmaDone), 0);
        }
    } else if (warp < 6) {
        // ---------------- dequantization: thread i owns weight row i of the tile
        const int i = threadIdx.x - 64;
        for (int s = 0; s < nsb; ++s) {
            const int rs = s % kQ6StRaw;
            if (!mbar_wait_or_abort(bar(kQ6RawFull + rs), (uint32_t)(s / kQ6StRaw) & 1u, s_abort)) break;
            // super-block layout (quant.cpp:630-687): ql[128], qh[64], int8 scales[16], fp16 d
            const uint32_t rb =
                sb + kQ6OffRaw + rs * kQ6RawBytes + kQ6RawRow * (uint32_t)i + ((210u * (uint32_t)(s0 + s)) & 15u);
            const float d = h2f(lds16(rb + 208u));
            uint32_t scw[4];
            lds_words_a2<4>(rb + 192u, scw);
            const int ss = s & 1;
            if (s >= 2 && !mbar_wait_or_abort(bar(kQ6ScEmpty + ss), (uint32_t)((s >> 1) - 1) & 1u, s_abort)) break;
            const uint32_t sco = sb + kQ6OffSc + (uint32_t)ss * kQ6ScBytes + 4u * (uint32_t)i;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float sc = (float)(int)(int8_t)((scw[j >> 2] >> (8 * (j & 3))) & 0xFFu);
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(sco + 4u * (uint32_t)(kTcBN * j)), "f"(d * sc)
                             : "memory");
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kQ6ScFull + ss));
            bool ok = true;
            for (int g = 0; g < 2 && ok; ++g) {
                uint32_t ql[16], qh[8];
                lds_words_a2<16>(rb + 64u * (uint32_t)g, ql);
                lds_words_a2<8>(rb + 128u + 32u * (uint32_t)g, qh);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = 4 * s + 2 * g + h, ws = c % kQ6StW;
                    if (c >= kQ6StW &&
                        !mbar_wait_or_abort(bar(kQ6WEmpty + ws), (uint32_t)((c / kQ6StW) - 1) & 1u, s_abort)) {
                        ok = false;
                        break;
                    }
                    // row i of W (128 bytes = 64 fp16): values 0..31 = sub-block 2h, 32..63 = 2h+1;
                    // value l of sub-block u: low (u < 2) or high nibble of ql[32*(u&1)+l], with
                    // bits 2u, 2u+1 of qh[l] on top
                    const uint32_t wrow =
                        sb + kQ6OffW + ws * kTcTileBytes + (uint32_t)(i >> 3) * 1024u + (uint32_t)(i & 7) * 128u;
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) {
                        const int sl = ch >> 2, l8 = ch & 3, sub = 2 * h + sl;
                        uint32_t q0 = ql[8 * sl + 2 * l8], q1 = ql[8 * sl + 2 * l8 + 1];
                        if (h) { q0 >>= 4; q1 >>= 4; }
                        q0 = (q0 & 0x0F0F0F0Fu) | (((qh[2 * l8] >> (2 * sub)) & 0x03030303u) << 4);
                        q1 = (q1 & 0x0F0F0F0Fu) | (((qh[2 * l8 + 1] >> (2 * sub)) & 0x03030303u) << 4);
                        const uint4 o = q6_chunk(q0, q1);
                        const uint32_t dst = wrow + (uint32_t)((ch ^ (i & 7)) << 4);
                        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o.x), "r"(o.y), "r"(o.z),
                                     "r"(o.w)
                                     : "memory");
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kQ6WFull + ws));
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kQ6RawEmpty + rs));
        }
    } else {
        // ---------------- epilogue: thread = weight row, 64 tokens
        const int quad = warp & 3, half = (warp - 6) >> 2;
        const int rl = 32 * quad + lane;  // weight row within the tile = TMEM lane
        const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
        float2 acc[32];  // tokens (2i, 2i+1) of this thread's 64
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.0f, 0.0f);
        for (int s = 0; s < nsb; ++s) {
            const int ss = s & 1;
            if (!warp_wait(bar(kQ6DxFull + ss), (uint32_t)(s >> 1) & 1u, s_abort)) break;
            if (!warp_wait(bar(kQ6ScFull + ss), (uint32_t)(s >> 1) & 1u, s_abort)) break;
            const uint32_t sca = sb + kQ6OffSc + (uint32_t)ss * kQ6ScBytes + 4u * (uint32_t)rl;
            const uint32_t dxa = sb + kQ6OffDx + (uint32_t)ss * kQ6DxBytes + 4u * (uint32_t)(64 * half);
            bool ok = true;
#pragma unroll 1
            for (int k = 0; k < 8; ++k) {
                const int b = 8 * s + k, db = b & 1;
                if (!warp_wait(bar(kQ6DFull + db), (uint32_t)(b >> 1) & 1u, s_abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float sa = lds32f(sca + 4u * (uint32_t)(kTcBN * (2 * k))),
                            sbh = lds32f(sca + 4u * (uint32_t)(kTcBN * (2 * k + 1)));
                const float2 sa2 = make_float2(sa, sa), sb2 = make_float2(sbh, sbh);
                const uint32_t dcol = tmem + lane_base + (uint32_t)(db * 2 * kTcBM + 64 * half);
                const uint32_t dxk = dxa + 4u * (uint32_t)(kTcBM * k);
                // groups of 8 tokens; the TMEM loads of group g+1 overlap the math of group g,
                // which runs on packed f32x2 operations (two tokens per instruction)
                uint32_t lo[2][8], hi[2][8];
                tmem_ld8_issue(dcol, lo[0]);
                tmem_ld8_issue(dcol + kTcBM, hi[0]);
                tmem_ld_wait2(lo[0], hi[0]);
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const int cur = g & 1;
                    if (g < 7) {
                        tmem_ld8_issue(dcol + 8u * (g + 1), lo[cur ^ 1]);
                        tmem_ld8_issue(dcol + kTcBM + 8u * (g + 1), hi[cur ^ 1]);
                    }
                    const float4 x0 = lds128f(dxk + 32u * g), x1 = lds128f(dxk + 32u * g + 16u);
                    const float2 dxv[4] = {make_float2(x0.x, x0.y), make_float2(x0.z, x0.w),
                                           make_float2(x1.x, x1.y), make_float2(x1.z, x1.w)};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 l = make_float2(__uint_as_float(lo[cur][2 * j]), __uint_as_float(lo[cur][2 * j + 1]));
                        const float2 h = make_float2(__uint_as_float(hi[cur][2 * j]), __uint_as_float(hi[cur][2 * j + 1]));
                        float2 u = __fmul2_rn(sa2, l);
                        u = __ffma2_rn(sb2, h, u);
                        acc[4 * g + j] = __ffma2_rn(dxv[j], u, acc[4 * g + j]);
                    }
                    if (g < 7) tmem_ld_wait2(lo[cur ^ 1], hi[cur ^ 1]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kQ6DEmpty + db));
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(kQ6ScEmpty + ss));
                mbar_arrive(bar(kQ6DxEmpty + ss));
            }
        }
        // y[t][row0 + rl] (+ bias), or this split's partial sums: the 32 lanes of a
        // warp write 128 contiguous bytes per token
        const int aborted = __shfl_sync(0xFFFFFFFFu, *s_abort, 0);
        const int j = row0 + rl;
        if (!aborted && j < p.N) {
            float* out = p.splits > 1 ? p.ypart + (int64_t)blockIdx.z * p.M * p.N : p.y;
            const float bj = (p.splits == 1 && p.bias) ? p.bias[j] : 0.0f;
#pragma unroll
            for (int tt = 0; tt < 64; ++tt) {
                const int t = tok0 + 64 * half + tt;
                const float v = (tt & 1) ? acc[tt >> 1].y : acc[tt >> 1].x;
                if (t < p.M) out[(int64_t)t * p.N + j] = v + bj;
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

// Per token t: the sum of the split-K partials plus the bias (splits > 1),
// and the AVX2 sign-trick difference for the (token, block) pairs whose q_x
// holds -128: y[t][j] += sum_b d * dx_b * (sa * dP_lo + sb * dP_hi), dP = 256 *
// the sum of the negative weights q6 - 32 where q_x == -128.  One CTA per
// token; with one split, a token without a flagged block returns at once.
__global__ void __launch_bounds__(128) prefill_q6k_finish_kernel(const uint8_t* __restrict__ w, int64_t row_bytes,
                                                                 const __half* __restrict__ a16,
                                                                 const float* __restrict__ dxT, int64_t mp,
                                                                 const uint8_t* __restrict__ flags, int K, int M,
                                                                 int N, const float* __restrict__ bias, int splits,
                                                                 const float* __restrict__ ypart,
                                                                 float* __restrict__ y) {
    const int t = blockIdx.x;
    const int nb = K >> 5;
    int any = 0;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) any |= flags[(int64_t)t * nb + b];
    any = __syncthreads_or(any);
    if (!any && splits == 1) return;
    const __half* xq = a16 + (int64_t)t * K;
    for (int j = threadIdx.x; j < N; j += blockDim.x) {
        float v;
        if (splits > 1) {
            v = 0.0f;
            for (int z = 0; z < splits; ++z) v += ypart[((int64_t)z * M + t) * N + j];
            if (bias) v += bias[j];
        } else {
            v = y[(int64_t)t * N + j];
        }
        if (any) {
            const uint8_t* row = w + (int64_t)j * row_bytes;
            float corr = 0.0f;
            for (int b = 0; b < nb; ++b) {
                if (!flags[(int64_t)t * nb + b]) continue;
                const uint8_t* sbp = row + 210 * (b >> 3);
                const int bl = b & 7, g = bl >> 2, sub = bl & 3;
                int dp[2] = {0, 0};
                for (int l = 0; l < 32; ++l) {
                    if (__half2float(xq[32 * b + l]) != -128.0f) continue;
                    const uint8_t raw = sbp[64 * g + 32 * (sub & 1) + l];
                    const int lo4 = sub >= 2 ? (raw >> 4) : (raw & 0xF);
                    const int q6 = (lo4 | (((sbp[128 + 32 * g + l] >> (2 * sub)) & 3) << 4)) - 32;
                    if (q6 < 0) dp[l >> 4] += 256 * q6;
                }
                const float d = __half2float(__ushort_as_half((unsigned short)(sbp[208] | (sbp[209] << 8))));
                const float sa = (float)(int8_t)sbp[192 + 2 * bl], sbh = (float)(int8_t)sbp[193 + 2 * bl];
                corr = fmaf(d * dxT[(int64_t)b * mp + t], sa * (float)dp[0] + sbh * (float)dp[1], corr);
            }
            v += corr;
        }
        y[(int64_t)t * N + j] = v;
    }
}

}  // namespace cllm
