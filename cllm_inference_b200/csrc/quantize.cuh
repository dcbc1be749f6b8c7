// Online Q8_0 activation quantization (reference src/core/quant.cpp:420-452).
#pragma once
#include "common.cuh"

namespace cllm {

// x86 semantics of `(int)std::nearbyint(v)` in the reference: a NaN or a value
// outside int32 converts to INT32_MIN (the "integer indefinite" of CVTTSS2SI).
__device__ __forceinline__ int x86_cvt_rint(float v) {
    const float r = rintf(v);  // round half to even = nearbyint in the default mode
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT32_MIN;
    return (int)r;
}

// One warp per 32-value block, lane l owns element l.  Every step is the
// reference's IEEE operation (no fast-math): amax over non-NaN |x|,
// d = amax / 127, id = 1 / d (or 0), q = clamp(rint(x * id), -128, 127).
// Also writes flags[block] = 1 when the block holds a -128 (only a NaN input
// produces one); the dot kernels use it to reproduce the reference's AVX2
// sign-trick result for such blocks.
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ x, int64_t n,
                                                            int64_t total_blocks,
                                                            float* __restrict__ scales,
                                                            int8_t* __restrict__ qs,
                                                            int32_t* __restrict__ bsums,
                                                            uint8_t* __restrict__ flags) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t nb = n >> 5;
    for (int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; blk < total_blocks;
         blk += nwarps) {
        const int64_t r = blk / nb, b = blk - r * nb;
        const int64_t e = r * n + b * 32 + lane;
        const float v = x[e];
        const float a = fabsf(v);
        float amax = (a > 0.0f) ? a : 0.0f;  // a NaN never wins `a > amax`
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        const float d = amax / 127.0f;
        const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        int q = x86_cvt_rint(v * id);
        q = q > 127 ? 127 : (q < -128 ? -128 : q);
        qs[e] = (int8_t)q;
        int s = q;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        const unsigned has_min = __ballot_sync(0xFFFFFFFFu, q == -128);
        if (lane == 0) {
            const int64_t ob = r * nb + b;
            scales[ob] = d;
            bsums[ob] = s;
            if (flags) flags[ob] = has_min ? 1 : 0;
        }
    }
}

// Per-block "holds a -128" flags for activations quantized elsewhere.
__global__ void __launch_bounds__(256) q8_flags_kernel(const int8_t* __restrict__ qs,
                                                       int64_t total_blocks,
                                                       uint8_t* __restrict__ flags) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; blk < total_blocks;
         blk += nwarps) {
        const unsigned any = __ballot_sync(0xFFFFFFFFu, qs[blk * 32 + lane] == -128);
        if (lane == 0) flags[blk] = any ? 1 : 0;
    }
}

}  // namespace cllm
