// matmul_quant for weight types without an integer dot kernel (F32, F16, Q4_1,
// Q5_1, Q8_1, Q2_K, Q3_K): the reference's fallback path (src/core/quant.cpp
// :1404-1430) -- each weight row dequantized and dotted with the fp32
// activation in element order, acc = bias (or 0) then acc += x[i] * w[i] with
// the product rounded before the add -- restated on the GPU in that exact
// order, so every output is bit-identical to the reference's.
//
// One thread owns one weight row (and its M accumulators); a warp takes 32
// rows.  For each 32-value slice of K the warp's lanes dequantize the slice of
// all 32 rows cooperatively into shared memory (lane = element, one row after
// another), then every lane runs its row's sequential sum over the slice.
// These types are outside the decode hot path (no BASELINE model uses them),
// so the kernel keeps the reference's sequential order rather than a tree.
#pragma once
#include "dequant.cuh"

namespace cllm {

constexpr int kFallbackWarps = 4;

template <int M>
__global__ void __launch_bounds__(kFallbackWarps * 32) gemv_fallback_kernel(const uint8_t* __restrict__ w, int type,
                                                                           int64_t row_bytes, int K, int N,
                                                                           const float* __restrict__ x,
                                                                           const float* __restrict__ bias,
                                                                           float* __restrict__ y) {
    __shared__ float tile[kFallbackWarps][32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kFallbackWarps + warp) * 32;
    if (row0 >= N) return;  // the whole warp
    const int row = row0 + lane;
    const int rows = min(32, N - row0);
    float acc[M];
#pragma unroll
    for (int t = 0; t < M; ++t) acc[t] = (bias && row < N) ? bias[row] : 0.0f;
    for (int k0 = 0; k0 < K; k0 += 32) {
        const int kn = min(32, K - k0);
        for (int r = 0; r < rows; ++r)
            tile[warp][r][lane] = lane < kn ? dequant_value(w + (int64_t)(row0 + r) * row_bytes, type, k0 + lane) : 0.0f;
        __syncwarp();
        if (row < N) {
            for (int i = 0; i < kn; ++i) {
                const float wv = tile[warp][lane][i];
#pragma unroll
                for (int t = 0; t < M; ++t) acc[t] = __fadd_rn(acc[t], __fmul_rn(x[(int64_t)t * K + k0 + i], wv));
            }
        }
        __syncwarp();
    }
    if (row < N) {
#pragma unroll
        for (int t = 0; t < M; ++t) y[(int64_t)t * N + row] = acc[t];
    }
}

}  // namespace cllm
