// Device helpers shared by the hot-path kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cllm {

// GGML type ids (reference include/cllm/core/quant.hpp:13-27).
enum : int { kQ4_0 = 2, kQ5_0 = 6, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14 };

// Device status word: kernels whose bounded wait expires record a code here
// and return; the host reads and clears it (cllm_cuda_check_device_status).
__device__ int g_device_status;
constexpr int kStatusTimeout = 1;

// Bounded-wait limit for every spin in this library: 1 s of %globaltimer.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- fp16 ---------------------------------------------------------------
// IEEE fp16 -> fp32 is exact (cvt.f32.f16), equal bit for bit to the
// reference's half_to_float (quant.hpp:31-56) for every input pattern.
__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

// Exact int32 -> fp32 for |v| < 2^22: place v in the mantissa of 1.5*2^23
// and subtract.  Two full-rate ALU/FMA-pipe ops instead of a conversion-pipe
// I2F.  All partials of this path are below 2^20 in magnitude.
__device__ __forceinline__ float i2f_exact(int v) {
    return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// ---- shared-memory / global byte sources --------------------------------
// Unit code reads weight bytes through one of these.  Offsets are relative
// to the row's first byte.  ALIGN is the alignment (bytes) the caller can
// guarantee for base+off; anything below 4 takes the funnel-shift path,
// which accepts any byte alignment and never reads a word that holds none of
// the requested bytes.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}

struct SmemSrc {
    uint32_t base;  // shared-window address of the row
    // 16-bit field at an even offset (every fp16 field of the GGML blocks).
    __device__ __forceinline__ uint32_t u16(uint32_t off) const { return lds16(base + off); }
    template <int NW, int ALIGN>
    __device__ __forceinline__ void words(uint32_t off, uint32_t (&w)[NW]) const {
        const uint32_t a = base + off;
        if constexpr (ALIGN >= 16 && NW % 4 == 0) {
#pragma unroll
            for (int i = 0; i < NW / 4; ++i) {
                uint4 v = lds128(a + 16 * i);
                w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
            }
        } else if constexpr (ALIGN >= 4) {
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = lds32(a + 4 * i);
        } else {
            const uint32_t al = a & ~3u, sh = (a & 3u) * 8u;
            uint32_t r[NW + 1];
#pragma unroll
            for (int i = 0; i < NW; ++i) r[i] = lds32(al + 4 * i);
            r[NW] = sh ? lds32(al + 4 * NW) : 0u;
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
        }
    }
};

struct GmemSrc {
    const uint8_t* base;  // global address of the row (any alignment)
    __device__ __forceinline__ uint32_t u16(uint32_t off) const {
        return (uint32_t)__ldg(base + off) | ((uint32_t)__ldg(base + off + 1) << 8);
    }
    template <int NW, int ALIGN>
    __device__ __forceinline__ void words(uint32_t off, uint32_t (&w)[NW]) const {
        const uintptr_t a = reinterpret_cast<uintptr_t>(base) + off;
        const uint32_t* al = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
        const uint32_t sh = (uint32_t)(a & 3u) * 8u;
        uint32_t r[NW + 1];
#pragma unroll
        for (int i = 0; i < NW; ++i) r[i] = __ldg(al + i);
        r[NW] = sh ? __ldg(al + NW) : 0u;
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
    }
};

// ---- mbarrier + bulk async copy (TMA engine, no multicast) -------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

// One 1-D bulk copy global -> shared, completing `bytes` of transaction on
// `bar`.  dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, "
        "0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, for at most kWaitLimitNs.
// Returns false (and records kStatusTimeout) if the limit expired.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
            atomicExch(&g_device_status, kStatusTimeout);
            return false;
        }
    }
}

// Wait with the same bound, returning early once another thread of the CTA
// has set *abort (and setting it when this wait expires).
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
                atomicExch(&g_device_status, kStatusTimeout);
                *abort = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Barrier over the first `threads` threads of the CTA (named barrier 1).
__device__ __forceinline__ void named_barrier_sync(int threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// ---- misc -----------------------------------------------------------------
template <int M>
__device__ __forceinline__ void warp_sum(float (&v)[M]) {
#pragma unroll
    for (int t = 0; t < M; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[t] += __shfl_xor_sync(0xFFFFFFFFu, v[t], o);
    }
}

// Activation row t of the quantized workspace, block b: 32 int8 as 8 words.
__device__ __forceinline__ void load_act32(const int8_t* qx_row, int b, int (&x)[8]) {
    const int4* p = reinterpret_cast<const int4*>(qx_row + 32 * b);
    int4 a = __ldg(p), c = __ldg(p + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
}

}  // namespace cllm
