// The quant API of cllm_inference (include/cllm/core/quant.hpp in the
// reference), implemented on the B200 library's C ABI (include/cllm_cuda.h).
//
// Every compute call runs on the GPU, for all thirteen GGML types the
// reference reads (types without an integer dot kernel take the reference's
// dequantize-and-float-dot path, on the GPU); the ThreadPool argument is
// accepted and ignored.  Errors become std::runtime_error carrying the library's message,
// which reuses the reference's strings (quant.cpp:423, :1379, :1443, :1370).
//
// Weights: the engine passes pointers into the read-only GGUF mapping
// (gguf.cpp:178, PROT_READ).  The first time a matrix inside a read-only
// mapping is seen, its byte range is uploaded once to HBM
// (cllm_cuda_register_weights, native block layout) and reused by later
// calls, unless the caller already registered an enclosing range (e.g. the
// whole data section at load time).  Weights in writable memory (heap
// buffers, as in tests) may change between calls, so they are uploaded for
// the call only.  Activations and outputs stay in host memory and are copied
// per call, as the reference's API requires.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <iterator>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

#include "cllm/core/quant.hpp"
#include "cllm/core/tensor.hpp"
#include "cllm_cuda.h"

namespace cllm {
namespace {

[[noreturn]] void raise() {
    char buf[512];
    cllm_cuda_last_error(buf, sizeof buf);
    throw std::runtime_error(buf);
}

void check(int rc) {
    if (rc != CLLM_OK) raise();
}

void ensure_init() {
    static std::once_flag once;
    static int rc = CLLM_OK;
    std::call_once(once, [] {
        const char* env = std::getenv("CLLM_CUDA_DEVICE");
        rc = cllm_cuda_init(env ? std::atoi(env) : 0);
    });
    check(rc);
}

// True when [p, p+bytes) lies inside one mapping of this process that is not
// writable (read from /proc/self/maps).
bool in_readonly_mapping(const void* p, size_t bytes) {
    FILE* f = std::fopen("/proc/self/maps", "r");
    if (!f) return false;
    const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = a + bytes;
    char line[512];
    bool ro = false;
    while (std::fgets(line, sizeof line, f)) {
        unsigned long lo = 0, hi = 0;
        char perms[8] = {0};
        if (std::sscanf(line, "%lx-%lx %7s", &lo, &hi, perms) != 3) continue;
        if (a >= lo && b <= hi) {
            ro = perms[1] != 'w';
            break;
        }
    }
    std::fclose(f);
    return ro;
}

// Ranges this shim registered itself (one per weight matrix), with a
// fingerprint of their first and last bytes.  A mapping can be unmapped and
// its addresses reused by a later one (a model closed, another loaded); such
// a stale registration is recognised when a call for the same matrix address
// finds different bytes there, or when a new range overlaps it, and is then
// dropped.  Ranges the caller registered (e.g. a whole data section) are the
// caller's to manage.
struct ShimRange {
    size_t bytes;
    uint8_t head[64], tail[64];
};
std::mutex g_ranges_mu;
std::map<uintptr_t, ShimRange> g_ranges;

size_t fp_len(size_t bytes) { return bytes < 64 ? bytes : 64; }

bool fingerprint_matches(const ShimRange& r, const uint8_t* p) {
    const size_t n = fp_len(r.bytes);
    return std::memcmp(r.head, p, n) == 0 && std::memcmp(r.tail, p + r.bytes - n, n) == 0;
}

// Drop every shim registration that overlaps [a, a + bytes).
void drop_overlapping(uintptr_t a, size_t bytes) {
    auto it = g_ranges.lower_bound(a);
    if (it != g_ranges.begin()) {
        auto prev = std::prev(it);
        if (prev->first + prev->second.bytes > a) it = prev;
    }
    while (it != g_ranges.end() && it->first < a + bytes) {
        cllm_cuda_unregister_weights(reinterpret_cast<const void*>(it->first));
        it = g_ranges.erase(it);
    }
}

// Device copy of the weight matrix [w, w + bytes) when it can stay resident
// (inside a registered range, or a read-only mapping registered now); nullptr
// when the caller's memory is writable and must be uploaded per call.
const void* resident_weights(const void* w, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_ranges_mu);
    const uintptr_t a = reinterpret_cast<uintptr_t>(w);
    const auto* p = static_cast<const uint8_t*>(w);
    auto it = g_ranges.find(a);
    if (it != g_ranges.end() && (it->second.bytes != bytes || !fingerprint_matches(it->second, p))) drop_overlapping(a, bytes);
    const void* dev = nullptr;
    if (cllm_cuda_lookup_weights(w, &dev) == CLLM_OK) {
        // a shim range that merely contains w but was made for another matrix
        // is stale (matrices never overlap): drop it and look again
        auto hit = g_ranges.upper_bound(a);
        if (hit != g_ranges.begin() && (--hit)->first + hit->second.bytes > a && hit->first != a) {
            drop_overlapping(a, bytes);
            if (cllm_cuda_lookup_weights(w, &dev) != CLLM_OK) dev = nullptr;
        }
        if (dev) return w;  // resident: callers pass the host pointer with CLLM_W_HOST
    }
    if (!in_readonly_mapping(w, bytes)) return nullptr;
    drop_overlapping(a, bytes);
    check(cllm_cuda_register_weights(w, bytes, nullptr));
    ShimRange r{bytes, {}, {}};
    const size_t n = fp_len(bytes);
    std::memcpy(r.head, p, n);
    std::memcpy(r.tail, p + bytes - n, n);
    g_ranges[a] = r;
    return w;
}

// RAII device buffer for per-call staging (the reference API is synchronous).
struct DevBuf {
    void* p = nullptr;
    explicit DevBuf(size_t n) {
        if (n && cudaMalloc(&p, n) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

void to_dev(void* d, const void* h, size_t n) {
    if (n && cudaMemcpy(d, h, n, cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("cudaMemcpy H2D failed");
}
void to_host(void* h, const void* d, size_t n) {
    if (n && cudaMemcpy(h, d, n, cudaMemcpyDeviceToHost) != cudaSuccess)
        throw std::runtime_error("cudaMemcpy D2H failed");
}

}  // namespace

int block_size(GgmlType type) { return cllm_cuda_block_size(static_cast<int>(type)); }

size_t type_size(GgmlType type) { return static_cast<size_t>(cllm_cuda_type_size(static_cast<int>(type))); }

bool has_vec_dot(GgmlType type) { return cllm_cuda_has_vec_dot(static_cast<int>(type)) != 0; }

// dequantize_block / dequantize_block_f16 for all thirteen types (quant.cpp
// :371-402) on the GPU.  n need not fill the last block: the whole block is
// uploaded and dequantized, and only n values come back.
void dequantize_block(const void* src, float* dst, GgmlType type, int64_t n) {
    const int t = static_cast<int>(type);
    if (cllm_cuda_type_size(t) == 0) throw std::runtime_error("unsupported ggml type for dequantize");
    if (n <= 0) return;
    ensure_init();
    const int bs = block_size(type);
    const size_t in_bytes = static_cast<size_t>((n + bs - 1) / bs) * type_size(type);
    const int64_t n_full = ((n + bs - 1) / bs) * bs;
    DevBuf s(in_bytes), d(static_cast<size_t>(n_full) * sizeof(float));
    to_dev(s.p, src, in_bytes);
    check(cllm_cuda_dequantize(s.p, t, n_full, d.as<float>(), nullptr));
    to_host(dst, d.p, static_cast<size_t>(n) * sizeof(float));
}

void dequantize_block_f16(const void* src, uint16_t* dst, GgmlType type, int64_t n) {
    const int t = static_cast<int>(type);
    if (cllm_cuda_type_size(t) == 0) throw std::runtime_error("unsupported ggml type for dequantize");
    if (n <= 0) return;
    ensure_init();
    const int bs = block_size(type);
    const size_t in_bytes = static_cast<size_t>((n + bs - 1) / bs) * type_size(type);
    const int64_t n_full = ((n + bs - 1) / bs) * bs;
    DevBuf s(in_bytes), d(static_cast<size_t>(n_full) * sizeof(uint16_t));
    to_dev(s.p, src, in_bytes);
    check(cllm_cuda_dequantize_f16(s.p, t, n_full, d.as<uint16_t>(), nullptr));
    to_host(dst, d.p, static_cast<size_t>(n) * sizeof(uint16_t));
}

std::vector<float> Tensor::dequantize() const {
    std::vector<float> out(numel());
    dequantize_block(data, out.data(), type, static_cast<int64_t>(numel()));
    return out;
}

std::vector<uint16_t> Tensor::dequantize_f16() const {
    std::vector<uint16_t> out(numel());
    dequantize_block_f16(data, out.data(), type, static_cast<int64_t>(numel()));
    return out;
}

void quantize_row_q8_0(const float* x, QuantizedQ8_0& out, int64_t n) {
    if (n % 32 != 0) throw std::runtime_error("quantize_row_q8_0: n not divisible by 32");
    ensure_init();
    const int64_t nb = n / 32;
    out.n = n;
    out.scales.resize(static_cast<size_t>(nb));
    out.qs.resize(static_cast<size_t>(n));
    out.bsums.resize(static_cast<size_t>(nb));
    if (n == 0) return;
    DevBuf dx(n * 4), dsc(nb * 4), dqs(n), dbs(nb * 4);
    to_dev(dx.p, x, n * 4);
    check(cllm_cuda_quantize_q8_0(dx.as<float>(), n, 1, dsc.as<float>(), dqs.as<int8_t>(),
                                  dbs.as<int32_t>(), nullptr));
    to_host(out.scales.data(), dsc.p, nb * 4);
    to_host(out.qs.data(), dqs.p, n);
    to_host(out.bsums.data(), dbs.p, nb * 4);
}

float vec_dot_row(const void* w_row, GgmlType w_type, const QuantizedQ8_0& qx, int64_t n) {
    const int t = static_cast<int>(w_type);
    if (!cllm_cuda_has_vec_dot(t)) throw std::runtime_error("vec_dot_row: no kernel for this type");
    ensure_init();
    const int64_t nb = n / 32;
    const size_t row_bytes = static_cast<size_t>(n / block_size(w_type)) * type_size(w_type);
    DevBuf dw(row_bytes), dsc(nb * 4), dqs(n), dbs(nb * 4), dy(4);
    to_dev(dw.p, w_row, row_bytes);
    to_dev(dsc.p, qx.scales.data(), nb * 4);
    to_dev(dqs.p, qx.qs.data(), n);
    to_dev(dbs.p, qx.bsums.data(), nb * 4);
    check(cllm_cuda_matmul_q8(dsc.as<float>(), dqs.as<int8_t>(), dbs.as<int32_t>(), dw.p, t, nullptr,
                              static_cast<int>(n), 1, 1, dy.as<float>(), nullptr));
    float y = 0.0f;
    to_host(&y, dy.p, 4);
    return y;
}

void matmul_quant_batch(const float* x, const void* w, GgmlType type, const float* bias, int in_dim,
                        int out_dim, int n_rows, float* y, ThreadPool* /*pool*/) {
    if (n_rows <= 0) return;
    const int t = static_cast<int>(type);
    const int bs = block_size(type);
    if (in_dim < 0 || bs <= 0 || in_dim % bs != 0)
        throw std::runtime_error(n_rows > 1 ? "matmul_quant_batch: in_dim not divisible by block size"
                                            : "matmul_quant: in_dim not divisible by block size");
    if (cllm_cuda_type_size(t) == 0) throw std::runtime_error("unsupported ggml type for dequantize");
    if (out_dim <= 0) return;
    ensure_init();
    const size_t bytes = static_cast<size_t>(in_dim / bs) * type_size(type) * static_cast<size_t>(out_dim);
    if (bytes == 0) {
        check(cllm_cuda_matmul_quant(x, w, t, bias, in_dim, out_dim, n_rows, y, CLLM_HOST_IO, nullptr));
    } else if (resident_weights(w, bytes)) {
        check(cllm_cuda_matmul_quant(x, w, t, bias, in_dim, out_dim, n_rows, y,
                                     CLLM_HOST_IO | CLLM_W_HOST, nullptr));
    } else {
        DevBuf dw(bytes);
        to_dev(dw.p, w, bytes);
        check(cllm_cuda_matmul_quant(x, dw.p, t, bias, in_dim, out_dim, n_rows, y, CLLM_HOST_IO, nullptr));
    }
}

void matmul_quant(const float* x, const void* w, GgmlType type, const float* bias, int in_dim,
                  int out_dim, float* y, ThreadPool* pool) {
    matmul_quant_batch(x, w, type, bias, in_dim, out_dim, 1, y, pool);
}

}  // namespace cllm
