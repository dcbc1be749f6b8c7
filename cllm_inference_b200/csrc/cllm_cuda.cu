// C-ABI of the B200 quantized-matmul hot path (declarations: include/cllm_cuda.h).
//
// Host-side responsibilities:
//   * argument checks and the reference's error strings (quant.cpp:423, 1379,
//     1443, 1370), mapped to status codes — nothing throws across the ABI;
//   * the weight registry: host ranges (GGUF mmap sections) uploaded once to
//     HBM in native block layout, looked up by pointer for CLLM_W_HOST;
//   * a per-device workspace for the quantized activations and host staging;
//   * kernel selection (TMA-ring GEMV vs direct-load GEMV, rows-per-tile,
//     pipeline depth) and launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <map>
#include <unordered_map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cllm_cuda.h"
#include "common.cuh"
#include "dequant.cuh"
#include "fallback.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc_q6k.cuh"
#include "gemv.cuh"
#include "shard.cuh"
#include "quantize.cuh"

namespace cllm {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define CLLM_CUDA_TRY(expr)                                                                    \
    do {                                                                                       \
        cudaError_t e_ = (expr);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(CLLM_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));        \
    } while (0)

int block_size_of(int t) {
    switch (t) {
        case 0: case 1: return 1;
        case 2: case 3: case 6: case 7: case 8: case 9: return 32;
        case 10: case 11: case 12: case 13: case 14: return 256;
    }
    return 1;
}

int64_t type_size_of(int t) {
    switch (t) {
        case 0: return 4;   case 1: return 2;   case 2: return 18;  case 3: return 20;
        case 6: return 22;  case 7: return 24;  case 8: return 34;  case 9: return 36;
        case 10: return 84; case 11: return 110; case 12: return 144; case 13: return 176;
        case 14: return 210;
    }
    return 0;
}

bool has_vec_dot_of(int t) {
    return t == kQ4_0 || t == kQ5_0 || t == kQ8_0 || t == kQ4_K || t == kQ5_K || t == kQ6_K;
}

struct DeviceInfo {
    bool ready = false;
    int sms = 0;
    size_t max_smem_optin = 0;
    // GEMV CTAs per SM of one call (1 or 2; environment CLLM_GEMV_CTAS_PER_SM).
    // With 1, a second CTA slot stays free on every SM, so the next call's
    // CTAs become resident while this one runs (programmatic dependent
    // launch) and prefetch their first weight tiles.
    int gemv_ctas_per_sm = 2;
    // Host I/O of the GEMV path through mapped pinned memory instead of copy
    // operations: bit 0 reads x in place, bit 1 writes y in place (environment
    // CLLM_HOSTIO_DIRECT, 0..3).
    int hostio_direct = 3;
    // Q4_K rows of 16..32 super-blocks on the lane-per-super-block loop
    // (environment CLLM_GEMV_SB=0: the lane-per-unit loop instead).
    int gemv_sb = 1;
    // Row-sharded calls announce their round from a separate one-warp kernel
    // after the GEMV (1) or from the GEMV's last CTA (0; environment
    // CLLM_SHARD_SIGNAL_KERNEL).
    int shard_signal_kernel = 1;
    // in_dim from which a row-sharded call quantizes x once per call
    // (act_image_kernel) rather than in every CTA (environment
    // CLLM_SHARD_IMAGE_MIN_K).
    int shard_image_min_k = 8192;
};

std::mutex g_mu;
DeviceInfo g_dev[64];

struct Workspace {
    void* ptr = nullptr;
    size_t cap = 0;
};
Workspace g_ws[64];
std::mutex g_ws_mu[64];  // one per device: held from workspace() until the call's kernels are enqueued
// Bumped whenever device memory a cached host-I/O graph may point at moves:
// the workspace is reallocated, or a weight range is registered or removed.
std::atomic<uint64_t> g_memory_gen{0};

struct WeightRange {
    size_t bytes;
    void* alloc;     // cudaMalloc'd block
    uint8_t* dev;    // device address of host_base
    int device;
};
std::map<uintptr_t, WeightRange> g_weights;  // keyed by host base address

int current_device(int* dev) {
    CLLM_CUDA_TRY(cudaGetDevice(dev));
    if (*dev < 0 || *dev >= 64) return fail(CLLM_ERR_NO_DEVICE, "device index out of range");
    return CLLM_OK;
}

int ensure_device(int* out_dev) {
    int dev;
    if (int rc = current_device(&dev)) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceInfo& di = g_dev[dev];
    if (!di.ready) {
        cudaDeviceProp prop;
        CLLM_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
        if (prop.major < 10)
            return fail(CLLM_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                        dev, prop.major, prop.minor);
        di.sms = prop.multiProcessorCount;
        di.max_smem_optin = prop.sharedMemPerBlockOptin;
        if (const char* v = std::getenv("CLLM_GEMV_CTAS_PER_SM")) di.gemv_ctas_per_sm = std::atoi(v) == 1 ? 1 : 2;
        if (const char* v = std::getenv("CLLM_HOSTIO_DIRECT")) di.hostio_direct = std::atoi(v) & 3;
        if (const char* v = std::getenv("CLLM_GEMV_SB")) di.gemv_sb = std::atoi(v) != 0;
        if (const char* v = std::getenv("CLLM_SHARD_SIGNAL_KERNEL")) di.shard_signal_kernel = std::atoi(v) != 0;
        if (const char* v = std::getenv("CLLM_SHARD_IMAGE_MIN_K")) di.shard_image_min_k = std::atoi(v);
        di.ready = true;
    }
    *out_dev = dev;
    return CLLM_OK;
}

// Device address of pinned host memory the GPU can address in place
// (cudaHostAlloc, cudaMallocHost, cudaHostRegister), else nullptr.
void* mapped_host(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// Grow the device workspace to at least `bytes` (never shrinks).  Takes the
// device's workspace lock into `lk`; the caller keeps it until every kernel
// that uses the workspace is enqueued, so another host thread cannot grow
// (free and reallocate) the buffer between this call and those launches.
// What the lock cannot order is work already enqueued on other streams:
// calls that may overlap on the GPU must be serialised by the caller.
int workspace(int dev, size_t bytes, uint8_t** out, std::unique_lock<std::mutex>& lk) {
    lk = std::unique_lock<std::mutex>(g_ws_mu[dev]);
    Workspace& ws = g_ws[dev];
    if (ws.cap < bytes) {
        if (ws.ptr) {
            CLLM_CUDA_TRY(cudaDeviceSynchronize());  // a previous call may still use it
            CLLM_CUDA_TRY(cudaFree(ws.ptr));
            ws.ptr = nullptr;
            ws.cap = 0;
        }
        const size_t cap = std::max<size_t>(bytes + (bytes >> 2), size_t(4) << 20);
        CLLM_CUDA_TRY(cudaMalloc(&ws.ptr, cap));
        ws.cap = cap;
        g_memory_gen.fetch_add(1);
    }
    *out = static_cast<uint8_t*>(ws.ptr);
    return CLLM_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int lookup(const void* host_ptr, const uint8_t** dev_ptr, size_t* avail) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uintptr_t h = reinterpret_cast<uintptr_t>(host_ptr);
    auto it = g_weights.upper_bound(h);
    if (it == g_weights.begin()) return CLLM_ERR_NOT_REGISTERED;
    --it;
    if (h >= it->first + it->second.bytes) return CLLM_ERR_NOT_REGISTERED;
    *dev_ptr = it->second.dev + (h - it->first);
    if (avail) *avail = it->first + it->second.bytes - h;
    return CLLM_OK;
}

// ---------------------------------------------------------------------------
// kernel tables
typedef void (*GemvFn)(GemvParams);

template <int T>
GemvFn gemv_fn(bool tma, bool fused, bool emit, int m) {
    // Parity builds (EMIT: partials instead of y) exist for 1 and 4 activation rows.
    if (emit && m == 1)
        return !tma ? gemv_direct_kernel<T, 1, true>
                    : (fused ? gemv_tma_kernel<T, 1, true, true> : gemv_tma_kernel<T, 1, true, false>);
    if (emit && m == 4)
        return !tma ? gemv_direct_kernel<T, 4, true>
                    : (fused ? gemv_tma_kernel<T, 4, true, true> : gemv_tma_kernel<T, 4, true, false>);
    if (emit) return nullptr;
#define CLLM_CASE(MM)                                                                     \
    case MM:                                                                              \
        return !tma ? gemv_direct_kernel<T, MM, false>                                    \
                    : (fused ? gemv_tma_kernel<T, MM, false, true> : gemv_tma_kernel<T, MM, false, false>);
    switch (m) {
        CLLM_CASE(1) CLLM_CASE(2) CLLM_CASE(3) CLLM_CASE(4)
        CLLM_CASE(5) CLLM_CASE(6) CLLM_CASE(7) CLLM_CASE(8)
    }
#undef CLLM_CASE
    return nullptr;
}

GemvFn select_gemv(int type, bool tma, bool fused, bool emit, int m) {
    switch (type) {
        case kQ4_0: return gemv_fn<kQ4_0>(tma, fused, emit, m);
        case kQ5_0: return gemv_fn<kQ5_0>(tma, fused, emit, m);
        case kQ8_0: return gemv_fn<kQ8_0>(tma, fused, emit, m);
        case kQ4_K: return gemv_fn<kQ4_K>(tma, fused, emit, m);
        case kQ5_K: return gemv_fn<kQ5_K>(tma, fused, emit, m);
        case kQ6_K: return gemv_fn<kQ6_K>(tma, fused, emit, m);
    }
    return nullptr;
}

typedef void (*ImageFn)(const float*, int, uint8_t*, const uint32_t*, const uint32_t*, int, const PreOp, int);

template <int T>
ImageFn image_fn(int m) {
    switch (m) {
        case 1: return act_image_kernel<1, T>;
        case 2: return act_image_kernel<2, T>;
        case 3: return act_image_kernel<3, T>;
        case 4: return act_image_kernel<4, T>;
        case 5: return act_image_kernel<5, T>;
        case 6: return act_image_kernel<6, T>;
        case 7: return act_image_kernel<7, T>;
        case 8: return act_image_kernel<8, T>;
    }
    return nullptr;
}

ImageFn select_image(int type, int m) {
    switch (type) {
        case kQ4_0: return image_fn<kQ4_0>(m);
        case kQ5_0: return image_fn<kQ5_0>(m);
        case kQ8_0: return image_fn<kQ8_0>(m);
        case kQ4_K: return image_fn<kQ4_K>(m);
        case kQ5_K: return image_fn<kQ5_K>(m);
        case kQ6_K: return image_fn<kQ6_K>(m);
    }
    return nullptr;
}

// Fused GEMVs with at least this many activation values per row get their
// activations quantized once (act_image_kernel) instead of in every CTA: the
// per-CTA copy of x (4 bytes per value, read by ~300 CTAs) and its
// quantization would otherwise dominate the call.
constexpr int kImageMinK = 8192;

uint32_t image_bytes(int m, int K) { return (uint32_t)kImageHeader + fused_act_bytes(m, K); }

// Launch act_image_kernel for m rows of x (programmatic dependent launch).
// wait_pad / wait_epoch / wait_world (row-sharded chains): wait for every rank's
// announcement of round *wait_epoch before reading x; nullptr: no wait.
int launch_image(int type, int m, const float* x, int K, uint8_t* img, int* ctas, cudaStream_t st,
                 const uint32_t* wait_pad = nullptr, const uint32_t* wait_epoch = nullptr, int wait_world = 0,
                 PreOp pre = PreOp{kPreNone, nullptr, 0.0f}, bool sb_layout = false) {
    ImageFn fn = select_image(type, m);
    if (!fn) return fail(CLLM_ERR_INVALID_ARG, "no activation-image kernel for type %d, %d rows", type, m);
    const int groups = (m * (K / 32) + kGemvThreads / 4 - 1) / (kGemvThreads / 4);
    const int n = std::max(1, std::min(kImageMaxCtas, groups));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, x, K, img, wait_pad, wait_epoch, wait_world, pre, sb_layout ? 1 : 0));
    *ctas = n;
    return CLLM_OK;
}

constexpr uint32_t kSmemPerCta = 110 * 1024;  // two CTAs per SM
constexpr uint32_t kTileTarget = 32 * 1024;   // bytes of weights per tile
constexpr uint32_t kFusedActMax = 48 * 1024;  // largest quantized activation kept in shared memory (M=1, K <= 32768)

struct GemvPlan {
    bool tma, fused;
    int rows_per_tile, wpr, num_tiles, stages, grid;
    int sb_lanes;  // > 0: the Q4_K super-block loop (q4k_row_sb), lanes per row
    uint32_t stage_bytes;
    size_t smem;
};

// Tile / pipeline choice.  want_fused: quantize the activations inside the
// kernel when they fit (m rows of K).
GemvPlan plan_gemv(int type, const uint8_t* w, int64_t row_bytes, int K, int N, int m, bool want_fused,
                   const DeviceInfo& di, const float* x = nullptr) {
    if (x && (reinterpret_cast<uintptr_t>(x) & 15) != 0) want_fused = false;  // fused loads are float4
    GemvPlan pl{};
    const int upr = units_per_row(type, K);
    const int max_wpr = std::max(1, std::min(kGemvWarps, upr / 32));
    int R = kGemvWarps;
    while (R > 1 && (int64_t)R * row_bytes > kTileTarget) R >>= 1;
    while (R > 1 && (N + R - 1) / R < 2 * di.sms && kGemvWarps / (R >> 1) <= max_wpr) R >>= 1;
    while (kGemvWarps / R > max_wpr) R <<= 1;  // keep every warp of a row busy
    pl.rows_per_tile = R;
    pl.wpr = kGemvWarps / R;
    pl.num_tiles = (N + R - 1) / R;
    pl.stage_bytes = (uint32_t)(((int64_t)R * row_bytes + 127) & ~int64_t(127));
    const uint32_t act = (fused_act_bytes(m, K) + 127u) / 128u * 128u;
    pl.fused = want_fused && K > 0 && act <= kFusedActMax;
    // Q4_K at M = 1 with 16..32 super-blocks per row (fused): lane =
    // super-block, every warp takes 32 / sb_lanes whole rows of the tile; the
    // fused quantization writes the matching activation layout.  (At M > 1 the
    // lane-per-unit loop is faster: its per-token scale loads are free of bank
    // conflicts.)
    pl.sb_lanes = 0;
    // Rows of 16 super-blocks pair up in 16-row tiles; with fewer tiles than SMs
    // the lane-per-unit loop's 8-row tiles spread the call wider.
    const int sb_lanes = K >= 32 * 256 ? 32 : 16;
    const bool sb_wide = sb_lanes == 32 || (N + 2 * kGemvWarps - 1) / (2 * kGemvWarps) >= di.sms;
    if (pl.fused && m == 1 && type == kQ4_K && act_sb_layout<kQ4_K, 1>(K) && di.gemv_sb && sb_wide) {
        pl.sb_lanes = sb_lanes;
        pl.rows_per_tile = kGemvWarps * (32 / pl.sb_lanes);
        pl.wpr = 1;
        pl.num_tiles = (N + pl.rows_per_tile - 1) / pl.rows_per_tile;
        pl.stage_bytes = (uint32_t)(((int64_t)pl.rows_per_tile * row_bytes + 127) & ~int64_t(127));
    }
    const size_t fixed = kGemvSmemHeader + (pl.fused ? act : 0);
    const size_t limit = di.max_smem_optin > 1024 ? di.max_smem_optin - 1024 : 0;
    pl.tma = K > 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (row_bytes & 15) == 0 &&
             fixed + 2ull * pl.stage_bytes <= limit;
    if (!pl.tma) {
        pl.fused = false;
        if (pl.sb_lanes) return plan_gemv(type, w, row_bytes, K, N, m, false, di, x);
    }
    if (pl.tma) {
        const size_t budget = std::max<size_t>(kSmemPerCta, fixed + 2ull * pl.stage_bytes);
        int S = (int)std::min<size_t>(8, (budget - fixed) / pl.stage_bytes);
        if (S < 2) S = 2;
        pl.stages = S;
        pl.smem = fixed + (size_t)S * pl.stage_bytes;
        const int per_sm = pl.smem <= kSmemPerCta ? di.gemv_ctas_per_sm : 1;
        pl.grid = std::min(pl.num_tiles, per_sm * di.sms);
        // With few tiles per CTA, as few CTAs as keep the same number of tile
        // rounds: every CTA then gets the same number of tiles (within one),
        // so none idles through the last round (gate/up 14336x4096: 296 CTAs
        // with 6 or 7 tiles -> 256 CTAs with 7, 6.6 % faster).
        // (The super-block loop's 16-row tiles are too coarse for that: it keeps
        // every CTA slot, so that no SM runs two CTAs' worth of tiles while
        // another runs one.)
        const int rounds = (pl.num_tiles + pl.grid - 1) / pl.grid;
        if (rounds <= 16 && !pl.sb_lanes) pl.grid = (pl.num_tiles + rounds - 1) / rounds;
    } else {
        pl.stages = 0;
        pl.smem = 0;
        pl.grid = std::min(pl.num_tiles, 4 * di.sms);
    }
    if (pl.grid < 1) pl.grid = 1;
    return pl;
}

// Raise a kernel's dynamic shared-memory limit to the device maximum once
// (per device); the launch's own size still decides occupancy.
int opt_in_smem(const void* fn, int dev) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, bool> done;
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_pair(fn, dev);
    if (done.count(key)) return CLLM_OK;
    CLLM_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)g_dev[dev].max_smem_optin));
    done[key] = true;
    return CLLM_OK;
}

int launch_gemv(int type, bool emit, int m, const GemvPlan& pl, const GemvParams& p_in, cudaStream_t st) {
    GemvParams p = p_in;
    if (p.ldy == 0) p.ldy = p.N;
    GemvFn fn = select_gemv(type, pl.tma, pl.fused, emit, m);
    if (!fn) return fail(CLLM_ERR_INVALID_ARG, "no kernel for type %d, %d rows", type, m);
    if (pl.smem > 48 * 1024) {
        int dev;
        CLLM_CUDA_TRY(cudaGetDevice(&dev));
        if (int rc = opt_in_smem(reinterpret_cast<const void*>(fn), dev)) return rc;
    }
    if (pl.tma) {
        // Programmatic dependent launch: the kernel may begin (barrier set-up,
        // weight prefetch) while its predecessor in the stream finishes; it
        // reads activations only after griddepcontrol.wait.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(pl.grid);
        cfg.blockDim = dim3(kTmaThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, p));
    } else {
        fn<<<pl.grid, kGemvThreads, pl.smem, st>>>(p);
    }
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

void fill_plan(GemvParams& p, const GemvPlan& pl) {
    p.sb_lanes = pl.sb_lanes;
    p.rows_per_tile = pl.rows_per_tile;
    p.wpr = pl.wpr;
    p.num_tiles = pl.num_tiles;
    p.stages = pl.stages;
    p.stage_bytes = pl.stage_bytes;
}

int launch_quantize(const float* x, int64_t n, int rows, float* sc, int8_t* qs, int32_t* bs,
                    uint8_t* fl, const DeviceInfo& di, cudaStream_t st) {
    const int64_t total = (n / 32) * rows;
    if (total == 0) return CLLM_OK;
    const int64_t warps_per_cta = kGemvThreads / 32;
    const int64_t grid = std::min<int64_t>((total + warps_per_cta - 1) / warps_per_cta, 16LL * di.sms);
    quantize_q8_0_kernel<<<(unsigned)grid, kGemvThreads, 0, st>>>(x, n, total, sc, qs, bs, fl);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// ---------------------------------------------------------------------------
// Prefill (tcgen05) path
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
    static std::mutex mu;
    static EncodeTiledFn fn = nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            return fail(CLLM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    *out = fn;
    return CLLM_OK;
}

// 2-D tiled tensor map over a row-major [rows][cols] array (row pitch in bytes,
// 0 = dense).
int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t cols,
                uint64_t rows, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz, uint64_t pitch = 0) {
    EncodeTiledFn enc;
    if (int rc = encode_fn(&enc)) return rc;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch ? pitch : cols * (uint64_t)esize};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CLLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CLLM_OK;
}

bool prefill_eligible(int type, const void* w, int64_t row_bytes, int K, int n_rows) {
    return (type == kQ4_K || type == kQ6_K) && n_rows >= kTcMinRows && K >= 256 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
           (row_bytes & 15) == 0;
}

// prefill_prep_kernel: 64 blocks per CTA and step; float4 loads when x allows.
int launch_prefill_prep(const float* x, int K, int64_t blocks, __half* a16, float* dxx, float* dxT, int64_t mp,
                        uint8_t* flags, const DeviceInfo& di, cudaStream_t st) {
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((blocks + 63) / 64, 16LL * di.sms));
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0)
        prefill_prep_kernel<true><<<(unsigned)grid, 256, 0, st>>>(x, K, blocks, a16, dxx, dxT, mp, flags);
    else
        prefill_prep_kernel<false><<<(unsigned)grid, 256, 0, st>>>(x, K, blocks, a16, dxx, dxT, mp, flags);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// Tokens per row of the block-major dx arrays of the prefill (16-byte rows for their tensor maps).
inline int64_t q6_dx_pitch(int M) { return ((int64_t)M + 3) & ~int64_t(3); }

// Split-K factor of the Q6_K prefill: with fewer 128x128 tiles than SMs, enough
// K splits to give every SM a CTA (at least four super-blocks each, at most 8).
int q6_splits(int M, int N, int K, int sms) {
    const int tiles = ((M + kTcBM - 1) / kTcBM) * ((N + kTcBN - 1) / kTcBN);
    if (tiles >= sms) return 1;
    return std::max(1, std::min({sms / tiles, (K >> 8) / 4, 8}));
}

// Workspace bytes of the prefill activations for M rows of K: fp16 q_x, then
// (dx, dx*bsum) [M][nb] for Q4_K, or dx [nb][pitch], the -128 flags [M][nb]
// and the split-K partial sums [splits][M][N] for Q6_K.
size_t prefill_bytes(int type, int M, int N, int K, int sms) {
    const size_t nb = (size_t)K / 32;
    if (type == kQ6_K) {
        const int sp = q6_splits(M, N, K, sms);
        return align256((size_t)M * K * 2) + align256(nb * (size_t)q6_dx_pitch(M) * 4) + align256((size_t)M * nb) +
               (sp > 1 ? align256((size_t)sp * M * N * 4) : 0);
    }
    return align256((size_t)M * K * 2) + align256(nb * (size_t)q6_dx_pitch(M) * 8);
}

// Q6_K: y[M][N] through prefill_q6k_kernel and the sign-trick fix-up.
int launch_prefill_q6k(const float* x, const uint8_t* w, int64_t row_bytes, const float* bias, int K, int N, int M,
                       float* y, uint8_t* ws, int dev, cudaStream_t st) {
    const DeviceInfo& di = g_dev[dev];
    const int64_t nb = K / 32, mp = q6_dx_pitch(M);
    __half* a16 = reinterpret_cast<__half*>(ws);
    float* dxT = reinterpret_cast<float*>(ws + align256((size_t)M * K * 2));
    uint8_t* flags = ws + align256((size_t)M * K * 2) + align256((size_t)(nb * mp * 4));
    const int splits = q6_splits(M, N, K, di.sms);
    float* ypart = splits > 1 ? reinterpret_cast<float*>(flags + align256((size_t)(M * nb))) : nullptr;
    const int64_t blocks = (int64_t)M * nb;
    if (int rc = launch_prefill_prep(x, K, blocks, a16, nullptr, dxT, mp, flags, di, st)) return rc;
    CLLM_CUDA_TRY(cudaGetLastError());
    CUtensorMap map_x, map_w, map_dx;
    if (int rc = make_map_2d(&map_dx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dxT, (uint64_t)M, (uint64_t)nb, kTcBM, 8,
                             CU_TENSOR_MAP_SWIZZLE_NONE, (uint64_t)mp * 4))
        return rc;
    if (int rc = make_map_2d(&map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a16, (uint64_t)K, (uint64_t)M, kTcBK, kTcBM,
                             CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if (int rc = make_map_2d(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, (uint64_t)row_bytes, (uint64_t)N, kQ6RawRow,
                             kTcBN, CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    if (int rc = opt_in_smem(reinterpret_cast<const void*>(prefill_q6k_kernel), dev)) return rc;
    const Q6Params qp{M, N, K, bias, y, splits, ypart};
    const dim3 tgrid((M + kTcBM - 1) / kTcBM, (N + kTcBN - 1) / kTcBN, splits);
    prefill_q6k_kernel<<<tgrid, kTcThreads, kQ6SmemBytes, st>>>(map_x, map_w, map_dx, qp);
    CLLM_CUDA_TRY(cudaGetLastError());
    prefill_q6k_finish_kernel<<<(unsigned)M, 128, 0, st>>>(w, row_bytes, a16, dxT, mp, flags, K, M, N, bias, splits,
                                                            ypart, y);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// y[M][N] = batch matmul through the tcgen05 kernel of the weight type; x, w,
// bias, y on the device, ws = prefill_bytes(type, M, N, K, sms) of workspace.
int launch_prefill(int type, const float* x, const uint8_t* w, int64_t row_bytes, const float* bias, int K, int N,
                   int M, float* y, uint8_t* ws, int dev, cudaStream_t st) {
    if (type == kQ6_K) return launch_prefill_q6k(x, w, row_bytes, bias, K, N, M, y, ws, dev, st);
    const DeviceInfo& di = g_dev[dev];
    const size_t nb = (size_t)K / 32;
    const size_t off_a = 0, off_dx = align256((size_t)M * K * 2);
    __half* a16 = reinterpret_cast<__half*>(ws + off_a);
    float* dxx = reinterpret_cast<float*>(ws + off_dx);  // [nb][mp][2]: (dx, dx*bsum), block-major
    const int64_t mp = q6_dx_pitch(M);
    const int64_t blocks = (int64_t)M * (K / 32);
    if (int rc = launch_prefill_prep(x, K, blocks, a16, dxx, nullptr, mp, nullptr, di, st)) return rc;
    CLLM_CUDA_TRY(cudaGetLastError());
    CUtensorMap map_a, map_w, map_dx;
    if (int rc = make_map_2d(&map_dx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dxx, (uint64_t)(2 * M), (uint64_t)nb,
                             2 * kTcBM, 8, CU_TENSOR_MAP_SWIZZLE_NONE, (uint64_t)mp * 8))
        return rc;
    if (int rc = make_map_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a16, (uint64_t)K, (uint64_t)M, kTcBK, kTcBM,
                             CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    if (int rc = make_map_2d(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, (uint64_t)row_bytes, (uint64_t)N, 144, kTcBN,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
    // y leaves through TMA stores when its rows are 16-byte multiples; else plain stores
    CUtensorMap map_y;
    std::memset(&map_y, 0, sizeof(map_y));
    const int tma_store = (N % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) ? 1 : 0;
    if (tma_store) {
        if (int rc = make_map_2d(&map_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, (uint64_t)N, (uint64_t)M, 32, 32,
                                 CU_TENSOR_MAP_SWIZZLE_128B))
            return rc;
    }
    if (int rc = opt_in_smem(reinterpret_cast<const void*>(prefill_q4k_kernel), dev)) return rc;
    TcParams tp{M, N, K, bias, y, tma_store};
    const dim3 tgrid((M + kTcBM - 1) / kTcBM, (N + kTcBN - 1) / kTcBN);
    prefill_q4k_kernel<<<tgrid, kTcThreads, kTcSmemBytes, st>>>(map_a, map_w, map_dx, map_y, tp);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// matmul_quant for a type without an integer dot kernel (quant.cpp:1404-1430):
// the dequantize-and-float-dot kernel, 8 activation rows per launch.
int launch_fallback(int type, const uint8_t* w, int64_t row_bytes, const float* x, const float* bias, int K, int N,
                    int n_rows, float* y, cudaStream_t st) {
    typedef void (*Fn)(const uint8_t*, int, int64_t, int, int, const float*, const float*, float*);
    static const Fn fns[8] = {gemv_fallback_kernel<1>, gemv_fallback_kernel<2>, gemv_fallback_kernel<3>,
                              gemv_fallback_kernel<4>, gemv_fallback_kernel<5>, gemv_fallback_kernel<6>,
                              gemv_fallback_kernel<7>, gemv_fallback_kernel<8>};
    const int rows_per_cta = kFallbackWarps * 32;
    const unsigned grid = (unsigned)((N + rows_per_cta - 1) / rows_per_cta);
    for (int t0 = 0; t0 < n_rows && grid > 0; t0 += 8) {
        const int m = std::min(8, n_rows - t0);
        fns[m - 1]<<<grid, rows_per_cta, 0, st>>>(w, type, row_bytes, K, N, x + (size_t)t0 * K, bias,
                                                  y + (size_t)t0 * N);
        CLLM_CUDA_TRY(cudaGetLastError());
    }
    return CLLM_OK;
}

// Layout of the quantized activations inside the workspace.
struct ActLayout {
    size_t qs, dx, bs, fl, end;
};
ActLayout act_layout(int m, int K, size_t at) {
    ActLayout L;
    const size_t nb = (size_t)K / 32;
    L.qs = at;
    L.dx = align256(L.qs + (size_t)m * K);
    L.bs = align256(L.dx + (size_t)m * nb * 4);
    L.fl = align256(L.bs + (size_t)m * nb * 4);
    L.end = align256(L.fl + (size_t)m * nb);
    return L;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point: a fixed scratch array for the quantized
// activations of up to CLLM_NOALLOC_MAX_ROWS rows of CLLM_NOALLOC_MAX_IN_DIM
// values, laid out as act_layout() lays out the workspace.
constexpr size_t noalloc_scratch_bytes() {
    return (size_t)CLLM_NOALLOC_MAX_ROWS * CLLM_NOALLOC_MAX_IN_DIM           // qs
           + (size_t)CLLM_NOALLOC_MAX_ROWS * (CLLM_NOALLOC_MAX_IN_DIM / 32) * 9;  // dx, bsum, flags
}
static_assert(noalloc_scratch_bytes() == CLLM_NOALLOC_SCRATCH_BYTES, "scratch size in the header");

static __device__ __align__(256) uint8_t g_noalloc_scratch[CLLM_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  In host code the array's name is only a stand-in: passing it
// to a kernel would not reach the device array.
int noalloc_scratch(int dev, uint8_t** out) {
    static std::mutex mu;
    static uint8_t* addr[64] = {};
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(CLLM_ERR_CUDA, "matmul_quant_noalloc: cudaGetSymbolAddress failed: %s",
                        cudaGetErrorString(e));
        addr[dev] = static_cast<uint8_t*>(p);
    }
    *out = addr[dev];
    return CLLM_OK;
}


// The decode-path launches of one call (device pointers): for every chunk of
// up to 8 activation rows, the activation quantization its plan asks for
// (fused into the GEMV; once per call into the activation image at img, when
// img is given and the plan is fused; or the standalone quantize kernel into
// the workspace at L) and the GEMV.  With partials != nullptr the same
// kernels run in their parity build (EMIT), which writes the int32 block
// partials [n_rows][out_dim][parts per row] instead of y, in chunks of 4 or
// 1 rows.
int run_decode(int type, const uint8_t* wd, int64_t row_bytes, const float* xd, const float* bd, int in_dim,
               int out_dim, int n_rows, float* yd, int32_t* partials, uint8_t* ws, const ActLayout& L,
               uint8_t* img, const DeviceInfo& di, cudaStream_t st, PreOp pre = PreOp{kPreNone, nullptr, 0.0f}) {
    const bool emit = partials != nullptr;
    const int64_t ppr = (type == kQ6_K ? 2 : 1) * (int64_t)(in_dim / 32);
    for (int t0 = 0; t0 < n_rows;) {
        const int left = n_rows - t0;
        const int m = emit ? (left >= 4 ? 4 : 1) : std::min(8, left);
        const GemvPlan pl = plan_gemv(type, wd, row_bytes, in_dim, out_dim, m, true, di, xd + (size_t)t0 * in_dim);
        GemvParams p{};
        p.w = wd;
        p.row_bytes = row_bytes;
        p.K = in_dim;
        p.N = out_dim;
        p.x = xd + (size_t)t0 * in_dim;
        p.qx = reinterpret_cast<int8_t*>(ws + L.qs);
        p.dx = reinterpret_cast<float*>(ws + L.dx);
        p.bs = reinterpret_cast<int32_t*>(ws + L.bs);
        p.fl = ws + L.fl;
        p.bias = bd;
        p.y = emit ? nullptr : yd + (size_t)t0 * out_dim;
        p.partials = emit ? partials + (size_t)t0 * out_dim * ppr : nullptr;
        fill_plan(p, pl);
        if (pre.op != kPreNone && (!pl.fused || !pl.tma))
            return fail(CLLM_ERR_INVALID_ARG, "matmul_quant: a pre-quantization step needs the fused GEMV");
        if (!pl.fused) {
            if (int rc = launch_quantize(p.x, in_dim, m, const_cast<float*>(p.dx), const_cast<int8_t*>(p.qx),
                                         const_cast<int32_t*>(p.bs), const_cast<uint8_t*>(p.fl), di, st))
                return rc;
        } else if (img && pl.tma) {
            if (int rc = launch_image(type, m, p.x, in_dim, img, &p.image_ctas, st, nullptr, nullptr, 0, pre,
                                      pl.sb_lanes != 0))
                return rc;
            p.image = img;
            p.image_bytes = image_bytes(m, in_dim);
        } else {
            p.pre = pre;
        }
        if (int rc = launch_gemv(type, emit, m, pl, p, st)) return rc;
        t0 += m;
    }
    return CLLM_OK;
}
// Internal flag of matmul_quant_impl: enqueue everything, but leave the final
// stream synchronization of a host-y call to the caller (graph capture).
constexpr unsigned kNoSync = 1u << 30;
// Largest y written in place to mapped host memory: the GEMV stores single
// floats, so beyond this a copy-engine transfer of y is the faster way out.
constexpr size_t kDirectYBytes = 16 * 1024;

// matmul_quant / matmul_quant_batch (quant.cpp:1374-1475) behind
// cllm_cuda_matmul_quant.  Scratch: the device workspace (scratch == nullptr),
// or a caller-owned buffer of scratch_cap bytes (the engine's decode step,
// whose captured graph must keep pointing at memory that never moves).  With
// need != nullptr only the scratch size is computed (*need) and nothing runs.
int matmul_quant_impl(const float* x, const void* w, int type, const float* bias, int in_dim, int out_dim,
                      int n_rows, float* y, unsigned flags, cudaStream_t st, uint8_t* scratch, size_t scratch_cap,
                      size_t* need, PreOp pre = PreOp{kPreNone, nullptr, 0.0f}) {
    const char* fname = n_rows > 1 ? "matmul_quant_batch" : "matmul_quant";
    if (n_rows <= 0) return CLLM_OK;  // quant.cpp:1436
    if (flags & ~(CLLM_X_HOST | CLLM_Y_HOST | CLLM_W_HOST | kNoSync))
        return fail(CLLM_ERR_INVALID_ARG, "%s: unknown flags 0x%x", fname, flags);
    if (in_dim < 0 || out_dim < 0) return fail(CLLM_ERR_INVALID_ARG, "%s: negative dimension", fname);
    const int bsz = block_size_of(type);
    if (in_dim % bsz != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "%s: in_dim not divisible by block size", fname);
    const bool fallback = !has_vec_dot_of(type);
    if (fallback && !dequant_supported(type))
        return fail(CLLM_ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize");
    if (out_dim == 0) return CLLM_OK;
    if (!need && (!y || (in_dim > 0 && (!x || !w)))) return fail(CLLM_ERR_INVALID_ARG, "%s: null pointer", fname);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const DeviceInfo& di = g_dev[dev];

    const int64_t row_bytes = (int64_t)(in_dim / bsz) * type_size_of(type);
    const uint8_t* wd = static_cast<const uint8_t*>(w);
    if (flags & CLLM_W_HOST) {
        size_t avail = 0;
        if (lookup(w, &wd, &avail) != CLLM_OK)
            return fail(CLLM_ERR_NOT_REGISTERED, "%s: weight pointer %p is not inside a registered range",
                        fname, w);
        if ((uint64_t)row_bytes * (uint64_t)out_dim > avail)
            return fail(CLLM_ERR_INVALID_ARG, "%s: weight matrix runs past its registered range", fname);
    }

    const bool use_tc = !fallback && prefill_eligible(type, wd, row_bytes, in_dim, n_rows);
    const bool gemv_path = !use_tc && !fallback;
    // GEMV host I/O without copy operations where the host buffers are pinned
    // and mapped: x is then read once, by the quantization kernel, and y is
    // written by the GEMV's own stores.
    const float* x_map = nullptr;
    float* y_map = nullptr;
    if (gemv_path) {
        if ((flags & CLLM_X_HOST) && (di.hostio_direct & 1)) x_map = static_cast<const float*>(mapped_host(x));
        if ((flags & CLLM_Y_HOST) && (di.hostio_direct & 2) && (size_t)n_rows * out_dim * 4 <= kDirectYBytes)
            y_map = static_cast<float*>(mapped_host(y));
    }
    const int mchunk = std::min(n_rows, 8);
    const ActLayout L = act_layout(use_tc || fallback ? 0 : mchunk, in_dim, 0);
    size_t off_x = L.end, off_b = L.end, off_y = L.end, total = L.end;
    if (flags & CLLM_X_HOST) {
        off_x = total;
        if (!x_map) total = align256(total + (size_t)n_rows * in_dim * 4);
        off_b = total;
        if (bias) total = align256(total + (size_t)out_dim * 4);
    }
    if ((flags & CLLM_Y_HOST) && !y_map) {
        off_y = total;
        total = align256(total + (size_t)n_rows * out_dim * 4);
    }
    const size_t off_pre = total;
    if (use_tc) total += prefill_bytes(type, n_rows, out_dim, in_dim, di.sms);
    const size_t off_img = total;
    // a mapped x goes through the activation image so that it crosses the host link once
    const bool want_image = gemv_path && (in_dim >= kImageMinK || x_map);
    if (want_image) total = align256(total + image_bytes(mchunk, in_dim));
    if (need) {
        *need = total;
        return CLLM_OK;
    }
    uint8_t* ws = scratch;
    std::unique_lock<std::mutex> ws_lock;
    if (scratch) {
        if (total > scratch_cap)
            return fail(CLLM_ERR_TOO_LARGE, "%s: %zu bytes of scratch needed, %zu given", fname, total, scratch_cap);
    } else if (int rc = workspace(dev, total, &ws, ws_lock)) {
        return rc;
    }

    const float* xd = x;
    const float* bd = bias;
    float* yd = y;
    if (flags & CLLM_X_HOST) {
        if (x_map) {
            xd = x_map;
        } else {
            xd = reinterpret_cast<float*>(ws + off_x);
            CLLM_CUDA_TRY(cudaMemcpyAsync((void*)xd, x, (size_t)n_rows * in_dim * 4, cudaMemcpyHostToDevice, st));
        }
        if (bias) {
            bd = reinterpret_cast<float*>(ws + off_b);
            CLLM_CUDA_TRY(cudaMemcpyAsync((void*)bd, bias, (size_t)out_dim * 4, cudaMemcpyHostToDevice, st));
        }
    }
    if (flags & CLLM_Y_HOST) yd = y_map ? y_map : reinterpret_cast<float*>(ws + off_y);

    if (use_tc) {
        if (int rc = launch_prefill(type, xd, wd, row_bytes, bd, in_dim, out_dim, n_rows, yd, ws + off_pre, dev, st))
            return rc;
    }
    if (pre.op != kPreNone && (use_tc || fallback || (flags & CLLM_X_HOST)))
        return fail(CLLM_ERR_INVALID_ARG, "%s: a pre-quantization step needs the fused GEMV", fname);
    if (fallback) {
        if (int rc = launch_fallback(type, wd, row_bytes, xd, bd, in_dim, out_dim, n_rows, yd, st)) return rc;
    } else if (!use_tc) {
        if (int rc = run_decode(type, wd, row_bytes, xd, bd, in_dim, out_dim, n_rows, yd, nullptr, ws, L,
                                want_image ? ws + off_img : nullptr, di, st, pre))
            return rc;
    }
    if (flags & CLLM_Y_HOST) {
        if (!y_map) CLLM_CUDA_TRY(cudaMemcpyAsync(y, yd, (size_t)n_rows * out_dim * 4, cudaMemcpyDeviceToHost, st));
        if (!(flags & kNoSync)) CLLM_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return CLLM_OK;
}

// ---------------------------------------------------------------------------
// Host-I/O calls as cached CUDA graphs.  A matmul_quant call with host x / y
// is several stream operations (copy in, quantization, GEMV, copy out) whose
// launch costs dominate a decode-sized call.  When every host buffer is
// pinned, the call's operations are captured once per argument tuple into a
// graph, and later calls with the same pointers and shape replay it: one
// launch and one synchronization.  Graphs read their buffers when they run,
// so new contents of x and of the weights are seen; a graph is rebuilt when
// device memory it points at has moved (g_memory_gen).
struct HostCallKey {
    const void *x, *w, *bias;
    void* y;
    int type, in_dim, out_dim, n_rows;
    unsigned flags;
    bool operator==(const HostCallKey& o) const {
        return x == o.x && w == o.w && bias == o.bias && y == o.y && type == o.type && in_dim == o.in_dim &&
               out_dim == o.out_dim && n_rows == o.n_rows && flags == o.flags;
    }
};
struct HostCallHash {
    size_t operator()(const HostCallKey& k) const {
        size_t h = std::hash<const void*>()(k.x);
        auto mix = [&h](size_t v) { h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2); };
        mix(std::hash<const void*>()(k.w));
        mix(std::hash<const void*>()(k.bias));
        mix(std::hash<const void*>()(k.y));
        mix((size_t)k.type * 1000003u ^ (size_t)k.in_dim);
        mix((size_t)k.out_dim * 1000033u ^ (size_t)k.n_rows ^ ((size_t)k.flags << 40));
        return h;
    }
};
struct HostCallGraph {
    cudaGraphExec_t exec = nullptr;  // nullptr: the call runs directly (prefill path, capture refused)
    uint64_t gen = 0;
    size_t total = 0;  // workspace bytes the graph uses
};
constexpr size_t kHostGraphMax = 4096;  // cached graphs per device
std::unordered_map<HostCallKey, HostCallGraph, HostCallHash> g_host_graphs[64];  // under g_ws_mu[dev]
cudaStream_t g_capture_stream[64];

void clear_host_graphs(int dev) {
    for (auto& kv : g_host_graphs[dev])
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    g_host_graphs[dev].clear();
}

// The host-I/O call through a cached graph; *handled = false when the call
// does not qualify (pageable buffers, prefill path, capture refused), in
// which case the caller runs it directly.
int host_graph_call(const float* x, const void* w, int type, const float* bias, int in_dim, int out_dim,
                    int n_rows, float* y, unsigned flags, cudaStream_t st, bool* handled) {
    *handled = false;
    if (n_rows <= 0 || out_dim <= 0 || in_dim <= 0 || !x || !w || !y) return CLLM_OK;
    if (((flags & CLLM_X_HOST) && (!mapped_host(x) || (bias && !mapped_host(bias)))) ||
        ((flags & CLLM_Y_HOST) && !mapped_host(y)))
        return CLLM_OK;
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const HostCallKey key{x, w, bias, y, type, in_dim, out_dim, n_rows, flags};
    auto& cache = g_host_graphs[dev];
    std::unique_lock<std::mutex> ws_lock(g_ws_mu[dev]);  // held until the call has finished
    auto it = cache.find(key);
    if (it != cache.end() && it->second.gen == g_memory_gen.load() && g_ws[dev].cap >= it->second.total) {
        if (!it->second.exec) return CLLM_OK;
        CLLM_CUDA_TRY(cudaGraphLaunch(it->second.exec, st));
        CLLM_CUDA_TRY(cudaStreamSynchronize(st));
        *handled = true;
        return CLLM_OK;
    }
    ws_lock.unlock();

    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        (void)cudaGetLastError();
        return CLLM_OK;  // the caller's own capture records the operations directly
    }
    if (!has_vec_dot_of(type) || in_dim % block_size_of(type) != 0) return CLLM_OK;
    const int64_t row_bytes = (int64_t)(in_dim / block_size_of(type)) * type_size_of(type);
    const uint8_t* wd = static_cast<const uint8_t*>(w);
    if ((flags & CLLM_W_HOST) && lookup(w, &wd, nullptr) != CLLM_OK) return CLLM_OK;  // reported directly
    const bool direct = prefill_eligible(type, wd, row_bytes, in_dim, n_rows);  // the tcgen05 path
    size_t total = 0;
    if (int rc = matmul_quant_impl(x, w, type, bias, in_dim, out_dim, n_rows, y, flags, st, nullptr, 0, &total))
        return rc;
    uint8_t* ws = nullptr;
    if (int rc = workspace(dev, total, &ws, ws_lock)) return rc;  // may move the workspace (new generation)
    const uint64_t gen = g_memory_gen.load();
    it = cache.find(key);
    if (it != cache.end()) {
        if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
        cache.erase(it);
    }
    if (cache.size() >= kHostGraphMax) clear_host_graphs(dev);
    if (direct) {
        cache.emplace(key, HostCallGraph{nullptr, gen, 0});
        return CLLM_OK;
    }
    if (!g_capture_stream[dev])
        CLLM_CUDA_TRY(cudaStreamCreateWithFlags(&g_capture_stream[dev], cudaStreamNonBlocking));
    cudaStream_t cap = g_capture_stream[dev];
    CLLM_CUDA_TRY(cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed));
    const int rc = matmul_quant_impl(x, w, type, bias, in_dim, out_dim, n_rows, y, flags | kNoSync, cap, ws, total,
                                     nullptr);
    cudaGraph_t g = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(cap, &g);
    cudaGraphExec_t exec = nullptr;
    if (rc == CLLM_OK && ec == cudaSuccess && g && cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) exec = nullptr;
    if (g) cudaGraphDestroy(g);
    (void)cudaGetLastError();
    cache.emplace(key, HostCallGraph{exec, gen, total});
    if (!exec) return CLLM_OK;  // not captured: the direct path runs the call (and reports its errors)
    CLLM_CUDA_TRY(cudaGraphLaunch(exec, st));
    CLLM_CUDA_TRY(cudaStreamSynchronize(st));
    *handled = true;
    return CLLM_OK;
}

}  // namespace
}  // namespace cllm

using namespace cllm;

// PDL launch of a one-warp shard kernel.
template <class... Args>
int launch_shard_kernel(void (*kern)(Args...), cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...));
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

extern "C" {

int cllm_cuda_last_error(char* buf, size_t n) {
    if (buf && n) {
        const size_t k = std::min(n - 1, g_last_error.size());
        std::memcpy(buf, g_last_error.data(), k);
        buf[k] = 0;
    }
    return (int)g_last_error.size();
}

int cllm_cuda_block_size(int type) { return block_size_of(type); }
int64_t cllm_cuda_type_size(int type) { return type_size_of(type); }
int cllm_cuda_has_vec_dot(int type) { return has_vec_dot_of(type) ? 1 : 0; }

int cllm_cuda_init(int device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return fail(CLLM_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    if (device < 0 || device >= count) return fail(CLLM_ERR_INVALID_ARG, "device %d of %d", device, count);
    CLLM_CUDA_TRY(cudaSetDevice(device));
    int dev;
    return ensure_device(&dev);
}

int cllm_cuda_register_weights(const void* host_base, size_t bytes, void** dev_base) {
    if (!host_base || bytes == 0) return fail(CLLM_ERR_INVALID_ARG, "register_weights: empty range");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const uintptr_t h = reinterpret_cast<uintptr_t>(host_base);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_weights.upper_bound(h + bytes - 1);
        if (it != g_weights.begin()) {
            --it;
            if (it->first + it->second.bytes > h)
                return fail(CLLM_ERR_INVALID_ARG, "register_weights: range overlaps a registered range");
        }
    }
    const size_t lead = h & 255;  // keep the host address's offset modulo 256
    void* alloc = nullptr;
    CLLM_CUDA_TRY(cudaMalloc(&alloc, bytes + lead));
    uint8_t* dev_ptr = static_cast<uint8_t*>(alloc) + lead;
    cudaError_t e = cudaMemcpy(dev_ptr, host_base, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(alloc);
        return fail(CLLM_ERR_CUDA, "register_weights: upload failed: %s", cudaGetErrorString(e));
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        g_weights[h] = WeightRange{bytes, alloc, dev_ptr, dev};
        g_memory_gen.fetch_add(1);
    }
    if (dev_base) *dev_base = dev_ptr;
    return CLLM_OK;
}

int cllm_cuda_unregister_weights(const void* host_base) {
    void* alloc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_weights.find(reinterpret_cast<uintptr_t>(host_base));
        if (it == g_weights.end()) return fail(CLLM_ERR_NOT_REGISTERED, "unregister_weights: unknown range");
        alloc = it->second.alloc;
        g_weights.erase(it);
        g_memory_gen.fetch_add(1);
    }
    CLLM_CUDA_TRY(cudaFree(alloc));
    return CLLM_OK;
}

int cllm_cuda_lookup_weights(const void* host_ptr, const void** dev_ptr) {
    if (!dev_ptr) return fail(CLLM_ERR_INVALID_ARG, "lookup_weights: null output");
    const uint8_t* d = nullptr;
    if (lookup(host_ptr, &d, nullptr) != CLLM_OK)
        return fail(CLLM_ERR_NOT_REGISTERED, "weight pointer %p is not inside a registered range", host_ptr);
    *dev_ptr = d;
    return CLLM_OK;
}

int cllm_cuda_quantize_q8_0(const float* x, int64_t n, int rows, float* scales, int8_t* qs,
                            int32_t* bsums, void* stream) {
    if (n < 0 || rows < 0) return fail(CLLM_ERR_INVALID_ARG, "quantize_row_q8_0: negative size");
    if (n % 32 != 0) return fail(CLLM_ERR_BLOCK_MULTIPLE, "quantize_row_q8_0: n not divisible by 32");
    if (n == 0 || rows == 0) return CLLM_OK;
    if (!x || !scales || !qs || !bsums) return fail(CLLM_ERR_INVALID_ARG, "quantize_row_q8_0: null pointer");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    return launch_quantize(x, n, rows, scales, qs, bsums, nullptr, g_dev[dev],
                           static_cast<cudaStream_t>(stream));
}

int cllm_cuda_matmul_quant(const float* x, const void* w, int type, const float* bias, int in_dim,
                           int out_dim, int n_rows, float* y, unsigned flags, void* stream) {
    if ((flags & CLLM_Y_HOST) && !(flags & ~(CLLM_X_HOST | CLLM_Y_HOST | CLLM_W_HOST))) {
        bool handled = false;
        if (int rc = host_graph_call(x, w, type, bias, in_dim, out_dim, n_rows, y, flags,
                                     static_cast<cudaStream_t>(stream), &handled))
            return rc;
        if (handled) return CLLM_OK;
    }
    return matmul_quant_impl(x, w, type, bias, in_dim, out_dim, n_rows, y, flags, static_cast<cudaStream_t>(stream),
                             nullptr, 0, nullptr);
}

int cllm_cuda_matmul_q8(const float* scales, const int8_t* qs, const int32_t* bsums, const void* w,
                        int type, const float* bias, int in_dim, int out_dim, int n_rows, float* y,
                        void* stream) {
    const char* fname = n_rows > 1 ? "matmul_quant_batch" : "matmul_quant";
    if (n_rows <= 0) return CLLM_OK;
    if (in_dim < 0 || out_dim < 0) return fail(CLLM_ERR_INVALID_ARG, "%s: negative dimension", fname);
    if (in_dim % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "%s: in_dim not divisible by block size", fname);
    if (!has_vec_dot_of(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type");
    if (out_dim == 0) return CLLM_OK;
    if (!w || !y || (in_dim > 0 && (!scales || !qs || !bsums)))
        return fail(CLLM_ERR_INVALID_ARG, "%s: null pointer", fname);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const DeviceInfo& di = g_dev[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row_bytes = (int64_t)(in_dim / block_size_of(type)) * type_size_of(type);
    const int64_t nb = in_dim / 32;
    uint8_t* ws;
    std::unique_lock<std::mutex> ws_lock;
    if (int rc = workspace(dev, align256((size_t)n_rows * nb) + 256, &ws, ws_lock)) return rc;
    const int64_t total = nb * n_rows;
    if (total > 0) {
        const int64_t grid = std::min<int64_t>((total + 7) / 8, 16LL * di.sms);
        q8_flags_kernel<<<(unsigned)grid, 256, 0, st>>>(qs, total, ws);
        CLLM_CUDA_TRY(cudaGetLastError());
    }
    for (int t0 = 0; t0 < n_rows; t0 += 8) {
        const int m = std::min(8, n_rows - t0);
        const GemvPlan pl = plan_gemv(type, static_cast<const uint8_t*>(w), row_bytes, in_dim, out_dim, m,
                                      false, di);
        GemvParams p{};
        p.w = static_cast<const uint8_t*>(w);
        p.row_bytes = row_bytes;
        p.K = in_dim;
        p.N = out_dim;
        p.qx = qs + (size_t)t0 * in_dim;
        p.dx = scales + (size_t)t0 * nb;
        p.bs = bsums + (size_t)t0 * nb;
        p.fl = ws + (size_t)t0 * nb;
        p.bias = bias;
        p.y = y + (size_t)t0 * out_dim;
        fill_plan(p, pl);
        if (int rc = launch_gemv(type, false, m, pl, p, st)) return rc;
    }
    return CLLM_OK;
}

int cllm_cuda_row_partials(const int8_t* qs, const void* w, int type, int in_dim, int out_dim,
                           int n_rows, int32_t* partials, void* stream) {
    if (in_dim < 0 || out_dim < 0 || n_rows < 0) return fail(CLLM_ERR_INVALID_ARG, "row_partials: negative size");
    if (!has_vec_dot_of(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type");
    if (in_dim % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "matmul_quant: in_dim not divisible by block size");
    if (n_rows == 0 || out_dim == 0 || in_dim == 0) return CLLM_OK;
    if (!qs || !w || !partials) return fail(CLLM_ERR_INVALID_ARG, "row_partials: null pointer");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const DeviceInfo& di = g_dev[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row_bytes = (int64_t)(in_dim / block_size_of(type)) * type_size_of(type);
    const int ppr = (type == kQ6_K ? 2 : 1) * (in_dim / 32);
    const GemvPlan pl = plan_gemv(type, static_cast<const uint8_t*>(w), row_bytes, in_dim, out_dim, 1,
                                  false, di);
    // The dot kernels also read the block scales/sums (zeros here: they do not
    // affect the integer partials) and the per-block "-128 present" flags.
    // All flags are set, so the sign-trick correction is evaluated on every
    // block; it is zero wherever no -128 activation meets a negative weight.
    const ActLayout L = act_layout(1, in_dim, 0);
    uint8_t* ws;
    std::unique_lock<std::mutex> ws_lock;
    if (int rc = workspace(dev, L.end, &ws, ws_lock)) return rc;
    CLLM_CUDA_TRY(cudaMemsetAsync(ws + L.dx, 0, L.fl - L.dx, st));
    CLLM_CUDA_TRY(cudaMemsetAsync(ws + L.fl, 1, L.end - L.fl, st));
    for (int t = 0; t < n_rows; ++t) {
        GemvParams p{};
        p.w = static_cast<const uint8_t*>(w);
        p.row_bytes = row_bytes;
        p.K = in_dim;
        p.N = out_dim;
        p.qx = qs + (size_t)t * in_dim;
        p.dx = reinterpret_cast<float*>(ws + L.dx);
        p.bs = reinterpret_cast<int32_t*>(ws + L.bs);
        p.fl = ws + L.fl;
        p.y = nullptr;
        p.partials = partials + (size_t)t * out_dim * ppr;
        fill_plan(p, pl);
        if (int rc = launch_gemv(type, true, 1, pl, p, st)) return rc;
    }
    return CLLM_OK;
}

int cllm_cuda_matmul_partials(const float* x, const void* w, int type, int in_dim, int out_dim, int n_rows,
                              int32_t* partials, void* stream) {
    if (in_dim < 0 || out_dim < 0 || n_rows < 0) return fail(CLLM_ERR_INVALID_ARG, "matmul_partials: negative size");
    if (!has_vec_dot_of(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type");
    if (in_dim % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "matmul_quant: in_dim not divisible by block size");
    if (n_rows == 0 || out_dim == 0 || in_dim == 0) return CLLM_OK;
    if (!x || !w || !partials) return fail(CLLM_ERR_INVALID_ARG, "matmul_partials: null pointer");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const int64_t row_bytes = (int64_t)(in_dim / block_size_of(type)) * type_size_of(type);
    const int mchunk = std::min(n_rows, 4);
    const ActLayout L = act_layout(mchunk, in_dim, 0);
    const bool want_image = in_dim >= kImageMinK;
    size_t total = L.end;
    const size_t off_img = total;
    if (want_image) total = align256(total + image_bytes(mchunk, in_dim));
    uint8_t* ws;
    std::unique_lock<std::mutex> ws_lock;
    if (int rc = workspace(dev, total, &ws, ws_lock)) return rc;
    return run_decode(type, static_cast<const uint8_t*>(w), row_bytes, x, nullptr, in_dim, out_dim, n_rows,
                      nullptr, partials, ws, L, want_image ? ws + off_img : nullptr, g_dev[dev],
                      static_cast<cudaStream_t>(stream));
}

int cllm_cuda_dequantize_f16(const void* src, int type, int64_t n, uint16_t* dst, void* stream) {
    if (n < 0) return fail(CLLM_ERR_INVALID_ARG, "dequantize_f16: negative size");
    if (!dequant_supported(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize");
    if (n % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "dequantize: n not divisible by block size");
    if (n == 0) return CLLM_OK;
    if (!src || !dst) return fail(CLLM_ERR_INVALID_ARG, "dequantize_f16: null pointer");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const int64_t grid = std::min<int64_t>((n + 255) / 256, 32LL * g_dev[dev].sms);
    dequantize_f16_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(src), type, n, dst);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

int cllm_cuda_dequantize(const void* src, int type, int64_t n, float* dst, void* stream) {
    if (n < 0) return fail(CLLM_ERR_INVALID_ARG, "dequantize: negative size");
    if (!dequant_supported(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize");
    if (n % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "dequantize: n not divisible by block size");
    if (n == 0) return CLLM_OK;
    if (!src || !dst) return fail(CLLM_ERR_INVALID_ARG, "dequantize: null pointer");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const int64_t grid = std::min<int64_t>((n + 255) / 256, 32LL * g_dev[dev].sms);
    dequantize_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(src), type, n, dst);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

int cllm_cuda_matmul_plan(const void* w, int type, int in_dim, int out_dim, int n_rows, int* info,
                          int n_info) {
    if (!info || n_info < 0 || in_dim < 0 || out_dim < 0)
        return fail(CLLM_ERR_INVALID_ARG, "matmul_plan: bad arguments");
    if (!has_vec_dot_of(type) && !dequant_supported(type))
        return fail(CLLM_ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize");
    if (in_dim % block_size_of(type) != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "matmul_quant: in_dim not divisible by block size");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    if (!has_vec_dot_of(type)) {  // the dequantize-and-float-dot fallback
        const int rows_per_cta = kFallbackWarps * 32;
        int vals[8] = {n_rows <= 0 ? 0 : (n_rows + 7) / 8, 3, 0, 32, 0, 0, (out_dim + rows_per_cta - 1) / rows_per_cta,
                       (int)sizeof(float) * kFallbackWarps * 32 * 33};
        for (int i = 0; i < n_info && i < 8; ++i) info[i] = vals[i];
        return CLLM_OK;
    }
    const int64_t row_bytes = (int64_t)(in_dim / block_size_of(type)) * type_size_of(type);
    const int m = std::max(1, std::min(8, n_rows));
    const GemvPlan pl = plan_gemv(type, static_cast<const uint8_t*>(w), row_bytes, in_dim, out_dim, m, true,
                                  g_dev[dev]);
    const int chunks = n_rows <= 0 ? 0 : (n_rows + 7) / 8;
    int vals[8] = {chunks * (pl.fused ? 1 : 2), pl.tma, pl.fused, pl.rows_per_tile, pl.wpr,
                   pl.stages, pl.grid, (int)pl.smem};
    if (prefill_eligible(type, w, row_bytes, in_dim, n_rows)) {
        // activation preparation + the tcgen05 GEMM (+ the Q6_K sign-trick fix-up)
        vals[0] = type == kQ6_K ? 3 : 2;
        vals[1] = 2;
        vals[2] = 0;
        vals[3] = kTcBN;
        vals[4] = 0;
        vals[5] = kTcStA;
        vals[6] = ((n_rows + kTcBM - 1) / kTcBM) * ((out_dim + kTcBN - 1) / kTcBN) *
                  (type == kQ6_K ? q6_splits(n_rows, out_dim, in_dim, g_dev[dev].sms) : 1);
        vals[7] = (int)(type == kQ6_K ? kQ6SmemBytes : kTcSmemBytes);
    }
    for (int i = 0; i < n_info && i < 8; ++i) info[i] = vals[i];
    return CLLM_OK;
}

int cllm_cuda_matmul_quant_noalloc(const float* x, const void* w, int type, const float* bias,
                                   int in_dim, int out_dim, int n_rows, float* y, void* stream) {
    const char* fname = n_rows > 1 ? "matmul_quant_batch" : "matmul_quant";
    if (n_rows <= 0) return CLLM_OK;
    if (in_dim < 0 || out_dim < 0) return fail(CLLM_ERR_INVALID_ARG, "%s: negative dimension", fname);
    const int bsz = block_size_of(type);
    if (in_dim % bsz != 0)
        return fail(CLLM_ERR_BLOCK_MULTIPLE, "%s: in_dim not divisible by block size", fname);
    if (!has_vec_dot_of(type))
        return fail(CLLM_ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type");
    if (n_rows > CLLM_NOALLOC_MAX_ROWS || in_dim > CLLM_NOALLOC_MAX_IN_DIM)
        return fail(CLLM_ERR_TOO_LARGE,
                    "matmul_quant_noalloc: at most %d rows of at most %d values (got %d x %d)",
                    CLLM_NOALLOC_MAX_ROWS, CLLM_NOALLOC_MAX_IN_DIM, n_rows, in_dim);
    if (out_dim == 0) return CLLM_OK;
    if (!y || (in_dim > 0 && (!x || !w))) return fail(CLLM_ERR_INVALID_ARG, "%s: null pointer", fname);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    uint8_t* ws;
    if (int rc = noalloc_scratch(dev, &ws)) return rc;
    const DeviceInfo& di = g_dev[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row_bytes = (int64_t)(in_dim / bsz) * type_size_of(type);
    const ActLayout L = act_layout(n_rows, in_dim, 0);
    if (L.end > CLLM_NOALLOC_SCRATCH_BYTES)  // cannot happen within the limits above; kept as a guard
        return fail(CLLM_ERR_TOO_LARGE, "matmul_quant_noalloc: %zu scratch bytes needed", L.end);
    const GemvPlan pl = plan_gemv(type, static_cast<const uint8_t*>(w), row_bytes, in_dim, out_dim, n_rows,
                                  false, di);
    GemvParams p{};
    p.w = static_cast<const uint8_t*>(w);
    p.row_bytes = row_bytes;
    p.K = in_dim;
    p.N = out_dim;
    p.x = x;
    p.qx = reinterpret_cast<int8_t*>(ws + L.qs);
    p.dx = reinterpret_cast<float*>(ws + L.dx);
    p.bs = reinterpret_cast<int32_t*>(ws + L.bs);
    p.fl = ws + L.fl;
    p.bias = bias;
    p.y = y;
    p.partials = nullptr;
    fill_plan(p, pl);
    if (int rc = launch_quantize(x, in_dim, n_rows, const_cast<float*>(p.dx), const_cast<int8_t*>(p.qx),
                                 const_cast<int32_t*>(p.bs), const_cast<uint8_t*>(p.fl), di, st))
        return rc;
    return launch_gemv(type, false, n_rows, pl, p, st);
}

int cllm_cuda_shard_rows(int out_dim, int world, int rank, int* row_begin, int* rows) {
    if (out_dim < 0 || world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !row_begin || !rows)
        return fail(CLLM_ERR_INVALID_ARG, "shard_rows: bad arguments (out_dim %d, world %d, rank %d)", out_dim,
                    world, rank);
    shard_rows(out_dim, world, rank, row_begin, rows);
    return CLLM_OK;
}

int cllm_cuda_matmul_quant_rowshard(const float* x, const void* w_shard, int type, const float* bias,
                                    int in_dim, int out_dim, int rank, int world, int n_rows,
                                    float* const* y_peers, uint32_t* const* signal_pads, uint32_t* epoch,
                                    unsigned flags, void* stream) {
    const char* fname = "matmul_quant_rowshard";
    if (n_rows <= 0) return CLLM_OK;
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !y_peers)
        return fail(CLLM_ERR_INVALID_ARG, "%s: bad group (world %d, rank %d)", fname, world, rank);
    if (flags & ~(CLLM_SHARD_WAIT_PREV | CLLM_SHARD_NO_SIGNAL))
        return fail(CLLM_ERR_INVALID_ARG, "%s: unknown flags 0x%x", fname, flags);
    const bool announce = signal_pads && !(flags & CLLM_SHARD_NO_SIGNAL);
    if (signal_pads && !epoch) return fail(CLLM_ERR_INVALID_ARG, "%s: signal pads without an epoch word", fname);
    if ((flags & CLLM_SHARD_WAIT_PREV) && !signal_pads)
        return fail(CLLM_ERR_INVALID_ARG, "%s: CLLM_SHARD_WAIT_PREV needs the signal pads", fname);
    if (n_rows > 8) return fail(CLLM_ERR_TOO_LARGE, "%s: at most 8 activation rows (got %d)", fname, n_rows);
    if (in_dim < 0 || out_dim < 0) return fail(CLLM_ERR_INVALID_ARG, "%s: negative dimension", fname);
    const int bsz = block_size_of(type);
    if (in_dim % bsz != 0) return fail(CLLM_ERR_BLOCK_MULTIPLE, "%s: in_dim not divisible by block size", fname);
    if (!has_vec_dot_of(type)) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "vec_dot_row: no kernel for this type");
    int row0, rows;
    shard_rows(out_dim, world, rank, &row0, &rows);
    for (int q = 0; q < world; ++q) {
        if (!y_peers[q]) return fail(CLLM_ERR_INVALID_ARG, "%s: null y buffer of rank %d", fname, q);
        if (signal_pads && !signal_pads[q])
            return fail(CLLM_ERR_INVALID_ARG, "%s: null signal pad of rank %d", fname, q);
    }
    if (rows == 0) {  // nothing to compute; still announce the round
        if (!announce) return CLLM_OK;
        ShardSignal sg{};
        for (int q = 0; q < world; ++q) sg.pads[q] = signal_pads[q];
        sg.epoch = epoch;
        sg.world = world;
        sg.rank = rank;
        int dev;
        if (int rc = ensure_device(&dev)) return rc;
        return launch_shard_kernel(shard_signal_kernel, static_cast<cudaStream_t>(stream), sg);
    }
    if (rows > 0 && in_dim > 0 && (!x || !w_shard)) return fail(CLLM_ERR_INVALID_ARG, "%s: null pointer", fname);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const DeviceInfo& di = g_dev[dev];
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t row_bytes = (int64_t)(in_dim / bsz) * type_size_of(type);
    const uint8_t* wd = static_cast<const uint8_t*>(w_shard);
    const ActLayout L = act_layout(n_rows, in_dim, 0);
    // The tile shape of the UNSHARDED call (it fixes how a row's units are split
    // over lanes and warps, hence the float order of the row sum), so every
    // output equals the one-GPU result bit for bit; only the tile count shrinks.
    GemvPlan pl = plan_gemv(type, wd, row_bytes, in_dim, out_dim, n_rows, true, di, x);
    pl.num_tiles = (rows + pl.rows_per_tile - 1) / pl.rows_per_tile;
    pl.grid = std::max(1, std::min(pl.grid, pl.num_tiles));
    const bool wait_prev = (flags & CLLM_SHARD_WAIT_PREV) != 0;
    // Large in_dim: quantize x once per call (act_image_kernel, which also does
    // the wait for the previous round) instead of in every CTA.
    const bool use_image = pl.fused && pl.tma && in_dim >= di.shard_image_min_k;
    if (wait_prev && !pl.fused) {  // x is read by the quantize kernel: wait before it
        if (int rc = launch_shard_kernel(shard_wait_kernel, st, (const uint32_t*)signal_pads[rank],
                                         (const uint32_t*)epoch, world))
            return rc;
    }
    uint8_t* ws = nullptr;
    std::unique_lock<std::mutex> ws_lock;
    if (!pl.fused) {
        if (int rc = workspace(dev, L.end, &ws, ws_lock)) return rc;
    } else if (use_image) {
        if (int rc = workspace(dev, image_bytes(n_rows, in_dim), &ws, ws_lock)) return rc;
    }
    GemvParams p{};
    p.w = wd;
    p.row_bytes = row_bytes;
    p.K = in_dim;
    p.N = rows;
    p.x = x;
    if (ws && !pl.fused) {
        p.qx = reinterpret_cast<int8_t*>(ws + L.qs);
        p.dx = reinterpret_cast<float*>(ws + L.dx);
        p.bs = reinterpret_cast<int32_t*>(ws + L.bs);
        p.fl = ws + L.fl;
    }
    p.bias = bias ? bias + row0 : nullptr;
    p.y = y_peers[rank] + row0;
    p.partials = nullptr;
    fill_plan(p, pl);
    p.ldy = out_dim;
    p.npeers = world;
    for (int q = 0; q < world; ++q) p.ypeers[q] = y_peers[q] + row0;
    if (signal_pads) {
        for (int q = 0; q < world; ++q) p.spads[q] = signal_pads[q];
        p.sepoch = epoch;
        p.srank = rank;
        p.swait = (wait_prev && pl.fused && !use_image) ? 1 : 0;
        p.sarrive = (announce && !di.shard_signal_kernel) ? 1 : 0;
    }
    if (use_image) {
        const bool w = wait_prev && signal_pads;
        if (int rc = launch_image(type, n_rows, x, in_dim, ws, &p.image_ctas, st, w ? signal_pads[rank] : nullptr,
                                  w ? epoch : nullptr, w ? world : 0, PreOp{kPreNone, nullptr, 0.0f}, pl.sb_lanes != 0))
            return rc;
        p.image = ws;
        p.image_bytes = image_bytes(n_rows, in_dim);
    }
    if (!pl.fused) {
        if (int rc = launch_quantize(x, in_dim, n_rows, const_cast<float*>(p.dx), const_cast<int8_t*>(p.qx),
                                     const_cast<int32_t*>(p.bs), const_cast<uint8_t*>(p.fl), di, st))
            return rc;
    }
    if (int rc = launch_gemv(type, false, n_rows, pl, p, st)) return rc;
    if (announce && di.shard_signal_kernel) {
        // A programmatic dependent of the GEMV: the kernel boundary orders the
        // GEMV's peer stores before its system-scope fence and release stores,
        // so the GEMV's CTAs end without per-CTA fences and counting.
        ShardSignal sg{};
        for (int q = 0; q < world; ++q) sg.pads[q] = signal_pads[q];
        sg.epoch = epoch;
        sg.world = world;
        sg.rank = rank;
        if (int rc = launch_shard_kernel(shard_signal_kernel, st, sg)) return rc;
    }
    return CLLM_OK;
}

int cllm_cuda_shard_wait(const uint32_t* own_pad, const uint32_t* epoch, int world, void* stream) {
    if (world < 1 || world > kMaxPeers || !own_pad || !epoch)
        return fail(CLLM_ERR_INVALID_ARG, "shard_wait: bad arguments (world %d)", world);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    return launch_shard_kernel(shard_wait_kernel, static_cast<cudaStream_t>(stream), own_pad, epoch, world);
}

int cllm_cuda_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
    if (!bytes || !dev_ptr || !handle) return fail(CLLM_ERR_INVALID_ARG, "ipc_alloc: bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == CLLM_IPC_HANDLE_BYTES, "IPC handle size");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    void* p = nullptr;
    CLLM_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(CLLM_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
    }
    std::memcpy(handle, &h, sizeof(h));
    *dev_ptr = p;
    return CLLM_OK;
}

int cllm_cuda_ipc_open(const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return fail(CLLM_ERR_INVALID_ARG, "ipc_open: bad arguments");
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    CLLM_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = p;
    return CLLM_OK;
}

int cllm_cuda_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return fail(CLLM_ERR_INVALID_ARG, "ipc_close: null pointer");
    CLLM_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
    return CLLM_OK;
}

int cllm_cuda_ipc_free(void* dev_ptr) {
    if (!dev_ptr) return fail(CLLM_ERR_INVALID_ARG, "ipc_free: null pointer");
    CLLM_CUDA_TRY(cudaFree(dev_ptr));
    return CLLM_OK;
}

int cllm_cuda_shard_barrier(uint32_t* const* signal_pads, uint32_t* epoch, int world, int rank, void* stream) {
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || !signal_pads || !epoch)
        return fail(CLLM_ERR_INVALID_ARG, "shard_barrier: bad arguments (world %d, rank %d)", world, rank);
    ShardSignal sg{};
    for (int q = 0; q < world; ++q) {
        if (!signal_pads[q]) return fail(CLLM_ERR_INVALID_ARG, "shard_barrier: null signal pad of rank %d", q);
        sg.pads[q] = signal_pads[q];
    }
    sg.epoch = epoch;
    sg.world = world;
    sg.rank = rank;
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    return launch_shard_kernel(shard_barrier_kernel, static_cast<cudaStream_t>(stream), sg);
}

int cllm_cuda_check_device_status(void) {
    CLLM_CUDA_TRY(cudaDeviceSynchronize());
    int status = 0, zero = 0;
    CLLM_CUDA_TRY(cudaMemcpyFromSymbol(&status, g_device_status, sizeof(int)));
    CLLM_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)));
    if (status == kStatusTimeout)
        return fail(CLLM_ERR_KERNEL_TIMEOUT, "a kernel's bounded wait expired (pipeline copy never landed)");
    return CLLM_OK;
}

}  // extern "C"

// The device-resident engine step (its own C ABI section of include/cllm_cuda.h).
#include "engine.cuh"
