// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// A C-ABI wrapper around the UNMODIFIED reference implementation of the
// quantized-matmul hot path (cllm_inference src/core/quant.cpp and
// src/core/thread_pool.cpp).  oracle/Makefile compiles this file together with
// those two reference sources, in place, into oracle/_ref/libcllm_ref.so.
//
// It exists so that Python tests, the golden-fixture generator and the CPU
// baseline leg of bench.py can call the reference's own code through ctypes.
// Every function maps reference C++ exceptions to a negative return code and
// keeps the exception text for ref_last_error().
//
// Wrapped reference entry points (paths are inside the reference project):
//   block_size / type_size          include/cllm/core/quant.hpp:90-93, src/core/quant.cpp:340-369
//   dequantize_block                quant.hpp:99,  quant.cpp:371-389
//   quantize_row_q8_0               quant.hpp:127, quant.cpp:420-452
//   has_vec_dot / vec_dot_row       quant.hpp:130-136, quant.cpp:1347-1372
//   matmul_quant                    quant.hpp:144, quant.cpp:1374-1431
//   matmul_quant_batch              quant.hpp:149, quant.cpp:1433-1475
//   ThreadPool                      include/cllm/core/thread_pool.hpp:14-36
#include "cllm/core/quant.hpp"
#include "cllm/core/thread_pool.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>

using cllm::GgmlType;

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    } catch (...) {
        g_err = "unknown exception";
        return -1;
    }
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_block_size(int type) { return cllm::block_size(static_cast<GgmlType>(type)); }

int64_t ref_type_size(int type) {
    return static_cast<int64_t>(cllm::type_size(static_cast<GgmlType>(type)));
}

int ref_has_vec_dot(int type) { return cllm::has_vec_dot(static_cast<GgmlType>(type)) ? 1 : 0; }

void* ref_pool_create(int n_threads) {
    try {
        return new cllm::ThreadPool(n_threads < 0 ? 0 : (size_t)n_threads);
    } catch (...) {
        return nullptr;
    }
}

void ref_pool_destroy(void* pool) { delete static_cast<cllm::ThreadPool*>(pool); }

int64_t ref_pool_size(void* pool) {
    return pool ? (int64_t) static_cast<cllm::ThreadPool*>(pool)->size() : 0;
}

int ref_dequantize_block(const void* src, float* dst, int type, int64_t n) {
    return guarded([&] { cllm::dequantize_block(src, dst, static_cast<GgmlType>(type), n); });
}

// Quantize one row of n floats; outputs are the three arrays of QuantizedQ8_0.
int ref_quantize_row_q8_0(const float* x, int64_t n, float* scales, int8_t* qs, int32_t* bsums) {
    return guarded([&] {
        cllm::QuantizedQ8_0 q;
        cllm::quantize_row_q8_0(x, q, n);
        std::memcpy(scales, q.scales.data(), q.scales.size() * sizeof(float));
        std::memcpy(qs, q.qs.data(), q.qs.size());
        std::memcpy(bsums, q.bsums.data(), q.bsums.size() * sizeof(int32_t));
    });
}

// vec_dot_row over an already-quantized activation row (arrays as produced above).
int ref_vec_dot_row(const void* w_row, int type, const float* scales, const int8_t* qs,
                    const int32_t* bsums, int64_t n, float* out) {
    return guarded([&] {
        cllm::QuantizedQ8_0 q;
        const int64_t nb = n / 32;
        q.n = n;
        q.scales.assign(scales, scales + nb);
        q.qs.assign(qs, qs + n);
        q.bsums.assign(bsums, bsums + nb);
        *out = cllm::vec_dot_row(w_row, static_cast<GgmlType>(type), q, n);
    });
}

int ref_matmul_quant(const float* x, const void* w, int type, const float* bias, int in_dim,
                     int out_dim, float* y, void* pool) {
    return guarded([&] {
        cllm::matmul_quant(x, w, static_cast<GgmlType>(type), bias, in_dim, out_dim, y,
                           static_cast<cllm::ThreadPool*>(pool));
    });
}

int ref_matmul_quant_batch(const float* x, const void* w, int type, const float* bias, int in_dim,
                           int out_dim, int n_rows, float* y, void* pool) {
    return guarded([&] {
        cllm::matmul_quant_batch(x, w, static_cast<GgmlType>(type), bias, in_dim, out_dim, n_rows,
                                 y, static_cast<cllm::ThreadPool*>(pool));
    });
}

}  // extern "C"
