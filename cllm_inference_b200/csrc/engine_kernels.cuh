// Device kernels of the engine step: everything of the reference's
// TransformerEngine::forward / prefill (src/core/engine.cpp:466-610) that is
// not a quantized matmul, so the activations stay in HBM between the
// matmul_quant calls.
//
//   rmsnorm_kernel       rms_norm_ptr        engine.cpp:24-29
//   embed_kernel         get_embedding       engine.cpp:310-322 (dequantize_block of one row)
//   rope_kv_kernel       apply_rope + KV append   engine.cpp:44-57, :495-501 (:585-596 batched)
//   attn_chunk_kernel /  attention (GQA)     engine.cpp:119-146
//   attn_combine_kernel
//   silu_mul_kernel      SwiGLU              engine.cpp:41, :511 (:604)
//   add_kernel           residual adds       engine.cpp:507, :513 (:600, :606)
//   argmax_kernel        greedy sampling     sampler.cpp:32-34 (std::max_element: first maximum)
//
// Float semantics: every elementwise formula is the reference's, with the
// products and sums rounded as written (no contraction); reductions (norms,
// dot products, softmax sums) are trees instead of the reference's loops, so
// those sums differ in the last bits.  RoPE uses a cos/sin table that the
// host fills with the reference's own float expressions (engine.cpp:50-52).
#pragma once
#include "dequant.cuh"

namespace cllm {
namespace eng {

constexpr int kNormThreads = 512;
constexpr int kAttnChunk = 128;    // KV positions per attention CTA
constexpr int kAttnThreads = 128;  // four warps
constexpr int kArgmaxThreads = 1024;

// Engine state words in device memory, read and advanced by the kernels so
// a captured decode step can be replayed without host writes.
enum : int { kStatePos = 0, kStateToken = 1, kStateCount = 2, kStateWords = 4 };

// Programmatic dependent launch: every kernel of the step first waits for its
// predecessor in the stream to complete (a no-op when launched without the
// attribute), then lets its own successor be scheduled, so a kernel's launch
// and prologue overlap the previous kernel's tail.
__device__ __forceinline__ void pdl_start() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; ++i) s += red[i];
    return s;
}

// out[r] = x[r] * (1 / sqrt(sum(x[r]^2) / n + eps)) * w, one CTA per row r.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               int n, float eps, float* __restrict__ y) {
    pdl_start();
    __shared__ float red[kNormThreads / 32];
    const float* xr = x + (int64_t)blockIdx.x * n;
    float* yr = y + (int64_t)blockIdx.x * n;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
    const float sum = block_sum(s, red);
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], rms), w[i]);
}

// Row tokens[t] of the embedding table (any GGML type) into x[t], exactly
// as dequantize_block does.  grid (ceil(n/256), T).
__global__ void embed_kernel(const uint8_t* __restrict__ table, int type, int64_t row_bytes, int n,
                             const int* __restrict__ tokens, float* __restrict__ x) {
    pdl_start();
    const int t = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[(int64_t)t * n + i] = dequant_value(table + (int64_t)tokens[t] * row_bytes, type, i);
}

// NEOX rotation of q (n_head heads) and k (n_kv heads) of T tokens at
// positions base + t (base = *pos_dev + pos0), and the append of the rotated
// k and of v to this layer's cache rows.  rope[p][i] = (cos, sin) of
// p / theta^(i/half).  grid (T, n_head + n_kv), block hd/2.
// q, k, v: token rows of ldq / ldkv floats (the separate projections, or
// the row-interleaved output of one grouped q|k|v GEMM); the rotated q goes
// to qo as dense [T][n_head * hd] rows (qo == q with ldq == q_dim: in place).
__global__ void rope_kv_kernel(const float* q, int ldq, float* qo, const float* __restrict__ k,
                               const float* __restrict__ v, int ldkv, int n_head, int n_kv, int hd,
                               const float2* __restrict__ rope, const int* __restrict__ pos_dev, int pos0,
                               float* __restrict__ kc, float* __restrict__ vc) {
    pdl_start();
    const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x, half = hd >> 1;
    const int pos = (pos_dev ? *pos_dev : 0) + pos0 + t;
    const float2 cs = rope[(int64_t)pos * half + i];
    const int q_dim = n_head * hd, kv_dim = n_kv * hd;
    if (h < n_head) {
        const float* qh = q + (int64_t)t * ldq + h * hd;
        float* qd = qo + (int64_t)t * q_dim + h * hd;
        const float x0 = qh[i], x1 = qh[i + half];
        qd[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        qd[i + half] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    } else {
        const int kh = h - n_head;
        const float* kr = k + (int64_t)t * ldkv + kh * hd;
        float* kd = kc + (int64_t)pos * kv_dim + kh * hd;
        const float x0 = kr[i], x1 = kr[i + half];
        kd[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        kd[i + half] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
        const float* vr = v + (int64_t)t * ldkv + kh * hd;
        float* vd = vc + (int64_t)pos * kv_dim + kh * hd;
        vd[i] = vr[i];
        vd[i + half] = vr[i + half];
    }
}

// Partial attention of one KV head over one chunk of kAttnChunk positions,
// for the REP query heads that share it (GQA), token t (seq = base + t + 1
// positions visible).  Scores s = (q . k) * scale go to shared memory; then
// per head the chunk maximum m, e = exp(s - m), l = sum e; then
// acc[d] = sum e * v[d].  The combine kernel merges the chunks.
// grid (n_kv, n_chunks, T), block kAttnThreads; HD = head_dim (64 or 128).
template <int HD, int REP>
__global__ void __launch_bounds__(kAttnThreads) attn_chunk_kernel(const float* __restrict__ q,
                                                                  const float* __restrict__ kc,
                                                                  const float* __restrict__ vc, int n_kv,
                                                                  const int* __restrict__ pos_dev, int pos0,
                                                                  float scale, float* __restrict__ part_ml,
                                                                  float* __restrict__ part_acc) {
    pdl_start();
    constexpr int DPL = HD / 16;  // dims per lane (16 lanes per position)
    __shared__ float qs[REP][HD];
    __shared__ float es[REP][kAttnChunk];
    const int kvh = blockIdx.x, c = blockIdx.y, t = blockIdx.z, n_chunks = gridDim.y;
    const int n_head = n_kv * REP, q_dim = n_head * HD, kv_dim = n_kv * HD;
    const int seq = (pos_dev ? *pos_dev : 0) + pos0 + t + 1;
    const int p0 = c * kAttnChunk;
    if (p0 >= seq) return;  // the combine kernel reads only chunks below seq
    const int len = min(kAttnChunk, seq - p0);
    for (int i = threadIdx.x; i < REP * HD; i += kAttnThreads)
        qs[i / HD][i % HD] = q[(int64_t)t * q_dim + (kvh * REP + i / HD) * HD + i % HD];
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane & 15, hf = lane >> 4;
    float qr[REP][DPL];
#pragma unroll
    for (int r = 0; r < REP; ++r)
#pragma unroll
        for (int j = 0; j < DPL; ++j) qr[r][j] = qs[r][sub * DPL + j];
    // The loop bound is uniform across the warp (both 16-lane halves run the
    // same trips; a half past the chunk's end computes on zeros and stores
    // nothing), so the full-warp shuffles below always have every lane.
    for (int base = 2 * warp; base < len; base += 2 * (kAttnThreads / 32)) {
        const int pp = base + hf;
        const bool valid = pp < len;
        float kv[DPL];
        if (valid) {
            const float4* kr = reinterpret_cast<const float4*>(kc + (int64_t)(p0 + pp) * kv_dim + kvh * HD + sub * DPL);
#pragma unroll
            for (int j = 0; j < DPL / 4; ++j) {
                const float4 f = __ldg(kr + j);
                kv[4 * j] = f.x; kv[4 * j + 1] = f.y; kv[4 * j + 2] = f.z; kv[4 * j + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < DPL; ++j) kv[j] = 0.0f;
        }
#pragma unroll
        for (int r = 0; r < REP; ++r) {
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) s = fmaf(qr[r][j], kv[j], s);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
            if (valid && sub == 0) es[r][pp] = __fmul_rn(s, scale);
        }
    }
    __syncthreads();
    // per head: chunk maximum, exponentials, their sum (warp w takes heads w, w+4, ...)
    for (int r = warp; r < REP; r += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int p = lane; p < len; p += 32) m = fmaxf(m, es[r][p]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        float l = 0.0f;
        for (int p = lane; p < len; p += 32) {
            const float e = expf(__fsub_rn(es[r][p], m));
            es[r][p] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
        if (lane == 0) {
            const int64_t pi = ((int64_t)t * n_head + kvh * REP + r) * n_chunks + c;
            part_ml[2 * pi] = m;
            part_ml[2 * pi + 1] = l;
        }
    }
    __syncthreads();
    // acc[r][d] = sum over the chunk of e[r][p] * v[p][d]
    for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
        float acc[REP];
#pragma unroll
        for (int r = 0; r < REP; ++r) acc[r] = 0.0f;
        const float* vp = vc + (int64_t)p0 * kv_dim + kvh * HD + d;
        for (int p = 0; p < len; ++p) {
            const float vv = __ldg(vp + (int64_t)p * kv_dim);
#pragma unroll
            for (int r = 0; r < REP; ++r) acc[r] = fmaf(es[r][p], vv, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < REP; ++r) {
            const int64_t pi = ((int64_t)t * n_head + kvh * REP + r) * n_chunks + c;
            part_acc[pi * HD + d] = acc[r];
        }
    }
}

// The decode step's whole attention in one launch (T = 1, position *pos_dev),
// split over chunks of kDecChunk cache positions per KV head:
//   * the chunk's K and V rows of this KV head are loaded into shared memory
//     at once (every thread's loads in flight together: one memory latency);
//   * each CTA rotates the REP query heads it serves (apply_rope); the CTA
//     whose chunk holds this step's position also rotates the new k, writes it
//     and v to the cache and into its tile (no other CTA reads that row);
//   * scores, chunk maximum, exponentials, their sum and the e*v sums as
//     attn_chunk_kernel;
//   * the last CTA of each KV head to finish (a counter per KV head, reset by
//     that CTA) merges the chunks as attn_combine_kernel.
constexpr int kDecChunk = 32;
constexpr int kDecMergeChunks = 256;  // chunks the merge keeps in shared memory (contexts up to 8192)
template <int HD, int REP>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const float* __restrict__ q,
                                                                   const float* __restrict__ k,
                                                                   const float* __restrict__ v, float* kc, float* vc,
                                                                   int n_kv, const float2* __restrict__ rope,
                                                                   const int* __restrict__ pos_dev, float scale,
                                                                   float* part_ml, float* part_acc, int* counters,
                                                                   float* __restrict__ out) {
    pdl_start();
    constexpr int HALF = HD / 2, RS = HD + 4;  // K/V tile row stride (floats): 16-byte rows, spread banks
    __shared__ __align__(16) float ks[kDecChunk][RS];
    __shared__ __align__(16) float vs[kDecChunk][RS];
    __shared__ float qs[REP][HD];
    __shared__ float es[REP][kDecChunk];
    __shared__ int s_last;
    const int kvh = blockIdx.x, c = blockIdx.y, n_chunks = gridDim.y;
    const int kv_dim = n_kv * HD;
    const int pos = *pos_dev, seq = pos + 1;
    const int p0 = c * kDecChunk;
    if (p0 >= seq) return;
    const int len = min(kDecChunk, seq - p0);
    const bool holds_pos = pos < p0 + kDecChunk;
    // K and V rows of the chunk (the new position's row comes from this step's k, v)
    const int rows = holds_pos ? len - 1 : len;
    constexpr int F4 = HD / 4;  // float4 per row
    for (int i = threadIdx.x; i < rows * F4; i += kAttnThreads) {
        const int r = i / F4, c4 = i - r * F4;
        const int64_t g = (int64_t)(p0 + r) * kv_dim + kvh * HD + 4 * c4;
        *reinterpret_cast<float4*>(&ks[r][4 * c4]) = *reinterpret_cast<const float4*>(kc + g);
        *reinterpret_cast<float4*>(&vs[r][4 * c4]) = *reinterpret_cast<const float4*>(vc + g);
    }
    const float2* cs = rope + (int64_t)pos * HALF;
    for (int i = threadIdx.x; i < REP * HALF; i += kAttnThreads) {
        const int r = i / HALF, j = i - r * HALF;
        const float* qh = q + (kvh * REP + r) * HD;
        const float x0 = qh[j], x1 = qh[j + HALF];
        const float2 t = cs[j];
        qs[r][j] = __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
        qs[r][j + HALF] = __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x));
    }
    if (holds_pos) {
        const int r = pos - p0;
        for (int j = threadIdx.x; j < HALF; j += kAttnThreads) {
            const float* kr = k + kvh * HD;
            const float x0 = kr[j], x1 = kr[j + HALF];
            const float2 t = cs[j];
            const float k0 = __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
            const float k1 = __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x));
            const float v0 = v[kvh * HD + j], v1 = v[kvh * HD + j + HALF];
            float* kd = kc + (int64_t)pos * kv_dim + kvh * HD;
            float* vd = vc + (int64_t)pos * kv_dim + kvh * HD;
            kd[j] = k0;
            kd[j + HALF] = k1;
            vd[j] = v0;
            vd[j + HALF] = v1;
            ks[r][j] = k0;
            ks[r][j + HALF] = k1;
            vs[r][j] = v0;
            vs[r][j + HALF] = v1;
        }
    }
    __syncthreads();
    // scores: thread (position p, head r) for p < len, REP * kDecChunk <= 4 * 128
    for (int i = threadIdx.x; i < REP * kDecChunk; i += kAttnThreads) {
        const int r = i / kDecChunk, p = i - r * kDecChunk;
        if (p < len) {
            float sc = 0.0f;
#pragma unroll 8
            for (int d4 = 0; d4 < F4; ++d4) {
                const float4 kk = *reinterpret_cast<const float4*>(&ks[p][4 * d4]);
                const float4 qq = *reinterpret_cast<const float4*>(&qs[r][4 * d4]);
                sc = fmaf(qq.x, kk.x, sc);
                sc = fmaf(qq.y, kk.y, sc);
                sc = fmaf(qq.z, kk.z, sc);
                sc = fmaf(qq.w, kk.w, sc);
            }
            es[r][p] = __fmul_rn(sc, scale);
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < REP; r += kAttnThreads / 32) {
        const float sv = lane < len ? es[r][lane] : -INFINITY;
        float m = sv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        const float e = lane < len ? expf(__fsub_rn(sv, m)) : 0.0f;
        if (lane < len) es[r][lane] = e;
        float l = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
        if (lane == 0) {
            const int64_t pi = (int64_t)(kvh * REP + r) * n_chunks + c;
            part_ml[2 * pi] = m;
            part_ml[2 * pi + 1] = l;
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
        float acc[REP];
#pragma unroll
        for (int r = 0; r < REP; ++r) acc[r] = 0.0f;
        for (int p = 0; p < len; ++p) {
            const float vv = vs[p][d];
#pragma unroll
            for (int r = 0; r < REP; ++r) acc[r] = fmaf(es[r][p], vv, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < REP; ++r) part_acc[((int64_t)(kvh * REP + r) * n_chunks + c) * HD + d] = acc[r];
    }
    // the last chunk CTA of this KV head merges every chunk's partials
    __syncthreads();
    const int nc = (seq + kDecChunk - 1) / kDecChunk;
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(&counters[kvh], 1) == nc - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (nc <= kDecMergeChunks) {
        // the chunk weights w_c = exp(m_c - M) and L = sum_c w_c l_c once per
        // head (warp r: head r), then every output element's sum over chunks
        // with its loads issued ahead of the FMAs
        __shared__ float s_w[REP][kDecMergeChunks];
        __shared__ float s_L[REP];
        for (int r = warp; r < REP; r += kAttnThreads / 32) {
            const int64_t base = (int64_t)(kvh * REP + r) * n_chunks;
            float M = -INFINITY;
            for (int cc = lane; cc < nc; cc += 32) M = fmaxf(M, __ldcg(part_ml + 2 * (base + cc)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
            float L = 0.0f;
            for (int cc = lane; cc < nc; cc += 32) {
                const float wgt = expf(__fsub_rn(__ldcg(part_ml + 2 * (base + cc)), M));
                s_w[r][cc] = wgt;
                L = fmaf(wgt, __ldcg(part_ml + 2 * (base + cc) + 1), L);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
            if (lane == 0) s_L[r] = L;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < REP * HD; i += kAttnThreads) {
            const int r = i / HD, d = i % HD;
            const float* pa = part_acc + (int64_t)(kvh * REP + r) * n_chunks * HD + d;
            float acc = 0.0f;
#pragma unroll 8
            for (int cc = 0; cc < nc; ++cc) acc = fmaf(s_w[r][cc], __ldcg(pa + (int64_t)cc * HD), acc);
            out[(int64_t)(kvh * REP + r) * HD + d] = __fdiv_rn(acc, s_L[r]);
        }
    } else {
        for (int i = threadIdx.x; i < REP * HD; i += kAttnThreads) {
            const int h = kvh * REP + i / HD, d = i % HD;
            const int64_t base = (int64_t)h * n_chunks;
            float M = -INFINITY;
            for (int cc = 0; cc < nc; ++cc) M = fmaxf(M, __ldcg(part_ml + 2 * (base + cc)));
            float L = 0.0f, acc = 0.0f;
            for (int cc = 0; cc < nc; ++cc) {
                const float wgt = expf(__fsub_rn(__ldcg(part_ml + 2 * (base + cc)), M));
                L = fmaf(wgt, __ldcg(part_ml + 2 * (base + cc) + 1), L);
                acc = fmaf(wgt, __ldcg(part_acc + (base + cc) * HD + d), acc);
            }
            out[(int64_t)h * HD + d] = __fdiv_rn(acc, L);
        }
    }
    if (threadIdx.x == 0) counters[kvh] = 0;
}

// Merge the chunks of attn_chunk_kernel: with M the largest chunk maximum and
// w_c = exp(m_c - M), out[d] = sum_c w_c acc_c[d] / sum_c w_c l_c.
// grid (n_head, T), block HD.
template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* __restrict__ part_ml,
                                                          const float* __restrict__ part_acc, int n_chunks,
                                                          const int* __restrict__ pos_dev, int pos0,
                                                          float* __restrict__ out) {
    pdl_start();
    const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x, n_head = gridDim.x;
    const int seq = (pos_dev ? *pos_dev : 0) + pos0 + t + 1;
    const int nc = (seq + kAttnChunk - 1) / kAttnChunk;
    const int64_t base = ((int64_t)t * n_head + h) * n_chunks;
    float M = -INFINITY;
    for (int c = 0; c < nc; ++c) M = fmaxf(M, part_ml[2 * (base + c)]);
    float L = 0.0f, acc = 0.0f;
    for (int c = 0; c < nc; ++c) {
        const float wgt = expf(__fsub_rn(part_ml[2 * (base + c)], M));
        L = fmaf(wgt, part_ml[2 * (base + c) + 1], L);
        acc = fmaf(wgt, part_acc[(base + c) * HD + d], acc);
    }
    out[((int64_t)t * n_head + h) * HD + d] = __fdiv_rn(acc, L);
}

// g[i] = silu(g[i]) * u[i], silu(v) = v / (1 + exp(-v)).
__global__ void silu_mul_kernel(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
    pdl_start();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        g[i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u[i]);
    }
}

// out[t][i] = silu(gu[t][i]) * gu[t][n + i] for the row-interleaved output of
// one grouped gate|up GEMM (rows of 2n); the operations of silu_mul_kernel.
__global__ void silu_mul_rows_kernel(float* __restrict__ out, const float* __restrict__ gu, int n) {
    pdl_start();
    const int64_t t = blockIdx.y;
    const float* g = gu + t * 2 * n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = g[i];
        out[t * n + i] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), g[n + i]);
    }
}

// x[i] += t[i]
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ t, int64_t n) {
    pdl_start();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], t[i]);
}

// Greedy sampling of one logit row: the first index of the maximum (as
// std::max_element), written as the next input token; also appended to gen[]
// with its margin over the runner-up, and the position advanced by `advance`.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits, int n,
                                                                int* __restrict__ state, int* __restrict__ gen,
                                                                float* __restrict__ margins, int gen_cap,
                                                                int advance) {
    pdl_start();
    __shared__ float sv1[kArgmaxThreads / 32], sv2[kArgmaxThreads / 32];
    __shared__ int si1[kArgmaxThreads / 32];
    float v1 = -INFINITY, v2 = -INFINITY;
    int i1 = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > v1) { v2 = v1; v1 = v; i1 = i; }
        else if (v > v2) v2 = v;
    }
    // (value, index) order: larger value first, then the smaller index
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov1 = __shfl_xor_sync(0xFFFFFFFFu, v1, o), ov2 = __shfl_xor_sync(0xFFFFFFFFu, v2, o);
        const int oi1 = __shfl_xor_sync(0xFFFFFFFFu, i1, o);
        const bool other = ov1 > v1 || (ov1 == v1 && oi1 < i1);
        const float lo1 = other ? v1 : ov1;  // the top value that lost
        if (other) { v1 = ov1; i1 = oi1; }
        v2 = fmaxf(fmaxf(v2, ov2), lo1);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv1[w] = v1; sv2[w] = v2; si1[w] = i1; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b1 = sv1[0], b2 = sv2[0];
        int bi = si1[0];
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
            const bool other = sv1[k] > b1 || (sv1[k] == b1 && si1[k] < bi);
            const float lo = other ? b1 : sv1[k];
            if (other) { b1 = sv1[k]; bi = si1[k]; }
            b2 = fmaxf(fmaxf(b2, sv2[k]), lo);
        }
        state[kStateToken] = bi;
        const int c = state[kStateCount];
        if (c < gen_cap) {
            gen[c] = bi;
            margins[c] = b1 - b2;
        }
        state[kStateCount] = c + 1;
        state[kStatePos] += advance;
    }
}

// Greedy sampling spread over kArgCtas CTAs: CTA b scans the b-th contiguous
// slice of the logits; the last CTA to finish merges the slices in order (so a
// tie still goes to the first index, as std::max_element) and does what
// argmax_kernel does with the result.  The counter is reset by that CTA.
constexpr int kArgCtas = 64;
__global__ void __launch_bounds__(256) argmax_multi_kernel(const float* __restrict__ logits, int n, float* part,
                                                           int* counter, int* __restrict__ state,
                                                           int* __restrict__ gen, float* __restrict__ margins,
                                                           int gen_cap, int advance) {
    pdl_start();
    __shared__ float sv1[8], sv2[8];
    __shared__ int si1[8], s_last;
    const int per = (n + kArgCtas - 1) / kArgCtas;
    const int lo = blockIdx.x * per, hi = min(n, lo + per);
    float v1 = -INFINITY, v2 = -INFINITY;
    int i1 = 0x7FFFFFFF;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = logits[i];
        if (v > v1) { v2 = v1; v1 = v; i1 = i; }
        else if (v > v2) v2 = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov1 = __shfl_xor_sync(0xFFFFFFFFu, v1, o), ov2 = __shfl_xor_sync(0xFFFFFFFFu, v2, o);
        const int oi1 = __shfl_xor_sync(0xFFFFFFFFu, i1, o);
        const bool other = ov1 > v1 || (ov1 == v1 && oi1 < i1);
        const float lost = other ? v1 : ov1;
        if (other) { v1 = ov1; i1 = oi1; }
        v2 = fmaxf(fmaxf(v2, ov2), lost);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv1[w] = v1; sv2[w] = v2; si1[w] = i1; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float b1 = sv1[0], b2 = sv2[0];
        int bi = si1[0];
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
            const bool other = sv1[k] > b1 || (sv1[k] == b1 && si1[k] < bi);
            const float lost = other ? b1 : sv1[k];
            if (other) { b1 = sv1[k]; bi = si1[k]; }
            b2 = fmaxf(fmaxf(b2, sv2[k]), lost);
        }
        part[3 * blockIdx.x] = b1;
        part[3 * blockIdx.x + 1] = b2;
        part[3 * blockIdx.x + 2] = __int_as_float(bi);
        __threadfence();
        s_last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    float b1 = __ldcg(part), b2 = __ldcg(part + 1);
    int bi = __float_as_int(__ldcg(part + 2));
    for (int k = 1; k < (int)gridDim.x; ++k) {
        const float c1 = __ldcg(part + 3 * k), c2 = __ldcg(part + 3 * k + 1);
        const int ci = __float_as_int(__ldcg(part + 3 * k + 2));
        const bool other = c1 > b1 || (c1 == b1 && ci < bi);
        const float lost = other ? b1 : c1;
        if (other) { b1 = c1; bi = ci; }
        b2 = fmaxf(fmaxf(b2, c2), lost);
    }
    state[kStateToken] = bi;
    const int cnt = state[kStateCount];
    if (cnt < gen_cap) {
        gen[cnt] = bi;
        margins[cnt] = b1 - b2;
    }
    state[kStateCount] = cnt + 1;
    state[kStatePos] += advance;
    *counter = 0;
}

}  // namespace eng
}  // namespace cllm
