// Test driver for the quant.hpp drop-in (libcllm_quant.so), run on a GPU by
// tests/test_shim.py.  It follows the structure of the reference's own
// tests/quant_test.cpp: known-answer dequantization of hand-built blocks
// (:58-218), matmul_quant against dequantize + double dot (:237-282), the
// bias check (:292-313) and batch == per-row (:316-361), plus the error
// strings and an exhaustive fp16 conversion check.  Prints one PASS/FAIL line
// per check and exits non-zero on any failure.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "cllm/core/quant.hpp"

using namespace cllm;

namespace {

int g_pass = 0, g_fail = 0;

void expect(bool ok, const std::string& what) {
    if (ok) {
        ++g_pass;
    } else {
        ++g_fail;
        std::printf("FAIL %s\n", what.c_str());
    }
}

void near(double got, double want, const std::string& what) {
    expect(std::fabs(got - want) <= 1e-4, what + " got " + std::to_string(got) + " want " +
                                               std::to_string(want));
}

void put_f16(uint8_t* p, uint16_t h) {
    p[0] = static_cast<uint8_t>(h & 0xFF);
    p[1] = static_cast<uint8_t>(h >> 8);
}

constexpr uint16_t kOne = 0x3C00, kZero = 0x0000;

std::vector<float> deq(GgmlType t, const std::vector<uint8_t>& b, int64_t n) {
    std::vector<float> y(n);
    dequantize_block(b.data(), y.data(), t, n);
    return y;
}

// Known-answer blocks for the six hot-path types (values of the reference's
// tests/quant_test.cpp).
void known_answers() {
    {
        std::vector<uint8_t> b(18, 0);
        put_f16(&b[0], kOne);
        b[2] = 0x9A;
        auto y = deq(GgmlType::Q4_0, b, 32);
        near(y[0], 2.0, "Q4_0[0]"); near(y[16], 1.0, "Q4_0[16]"); near(y[1], -8.0, "Q4_0[1]");
    }
    {
        std::vector<uint8_t> b(22, 0);
        put_f16(&b[0], kOne);
        b[2] = 0x01;
        b[6] = 0x21;
        auto y = deq(GgmlType::Q5_0, b, 32);
        near(y[0], 1.0, "Q5_0[0]"); near(y[16], -14.0, "Q5_0[16]");
    }
    {
        std::vector<uint8_t> b(34, 0);
        put_f16(&b[0], kOne);
        b[2] = 0xFF;
        b[3] = 0x02;
        auto y = deq(GgmlType::Q8_0, b, 32);
        near(y[0], -1.0, "Q8_0[0]"); near(y[1], 2.0, "Q8_0[1]");
    }
    {
        std::vector<uint8_t> b(144, 0);
        const uint8_t sc[12] = {1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1};
        std::memcpy(&b[4], sc, 12);
        b[16] = 0x21;
        put_f16(&b[0], kOne);
        put_f16(&b[2], kZero);
        auto y = deq(GgmlType::Q4_K, b, 256);
        near(y[0], 1.0, "Q4_K[0]"); near(y[32], 2.0, "Q4_K[32]"); near(y[1], 0.0, "Q4_K[1]");
    }
    {
        std::vector<uint8_t> b(176, 0);
        const uint8_t sc[12] = {1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1};
        std::memcpy(&b[4], sc, 12);
        b[48] = 0x21;
        put_f16(&b[0], kOne);
        put_f16(&b[2], kZero);
        auto y = deq(GgmlType::Q5_K, b, 256);
        near(y[0], 1.0, "Q5_K[0]"); near(y[32], 2.0, "Q5_K[32]");
        b[16] = 0x01;
        auto y2 = deq(GgmlType::Q5_K, b, 256);
        near(y2[0], 17.0, "Q5_K(qh)[0]");
    }
    {
        std::vector<uint8_t> b(210, 0);
        for (int i = 0; i < 16; ++i) b[192 + i] = 0x01;
        b[0] = 0x21;
        put_f16(&b[208], kOne);
        auto y = deq(GgmlType::Q6_K, b, 256);
        near(y[0], -31.0, "Q6_K[0]"); near(y[64], -30.0, "Q6_K[64]");
    }
}

std::vector<uint8_t> test_weights(GgmlType type, int in_dim, int out_dim) {
    const int bs = block_size(type);
    const size_t row_bytes = static_cast<size_t>(in_dim / bs) * type_size(type);
    std::vector<uint8_t> w(row_bytes * out_dim, 0);
    for (int j = 0; j < out_dim; ++j)
        for (int blk = 0; blk < in_dim / bs; ++blk) {
            uint8_t* p = &w[j * row_bytes + blk * type_size(type)];
            put_f16(p, kOne);
            for (size_t k = 2; k < type_size(type); ++k) p[k] = static_cast<uint8_t>((k + blk + j) % 7);
        }
    return w;
}

void matmul_vs_dequant(const char* name, GgmlType type) {
    const int bs = block_size(type);
    const int in_dim = bs <= 32 ? 64 : 256, out_dim = 40;
    const size_t row_bytes = static_cast<size_t>(in_dim / bs) * type_size(type);
    auto w = test_weights(type, in_dim, out_dim);
    std::vector<float> x(in_dim), y(out_dim);
    for (int i = 0; i < in_dim; ++i) x[i] = static_cast<float>((i % 5) - 2) * 0.5f;
    matmul_quant(x.data(), w.data(), type, nullptr, in_dim, out_dim, y.data(), nullptr);
    int bad = 0;
    for (int j = 0; j < out_dim; ++j) {
        std::vector<float> row(in_dim);
        dequantize_block(&w[j * row_bytes], row.data(), type, in_dim);
        double ref = 0;
        for (int i = 0; i < in_dim; ++i) ref += static_cast<double>(x[i]) * row[i];
        const double tol = std::max(bs <= 32 ? 1e-2 : 3e-2, (bs <= 32 ? 0.03 : 0.06) * std::fabs(ref));
        if (std::fabs(ref - y[j]) > tol) ++bad;
    }
    expect(bad == 0, std::string("matmul_quant vs dequant ") + name);
}

void bias_check() {
    const int in_dim = 64, out_dim = 40;
    const size_t row_bytes = 2 * type_size(GgmlType::Q8_0);
    std::vector<uint8_t> w(row_bytes * out_dim, 0);
    for (int j = 0; j < out_dim; ++j)
        for (int blk = 0; blk < 2; ++blk) {
            uint8_t* p = &w[j * row_bytes + blk * 34];
            put_f16(p, kOne);
            for (int i = 0; i < 32; ++i) p[2 + i] = static_cast<uint8_t>((i + j) % 7 - 3);
        }
    std::vector<float> x(in_dim), y(out_dim), y2(out_dim), bias(out_dim);
    for (int i = 0; i < in_dim; ++i) x[i] = static_cast<float>((i % 5) - 2) * 0.5f;
    for (int j = 0; j < out_dim; ++j) bias[j] = static_cast<float>(j);
    matmul_quant(x.data(), w.data(), GgmlType::Q8_0, nullptr, in_dim, out_dim, y.data(), nullptr);
    matmul_quant(x.data(), w.data(), GgmlType::Q8_0, bias.data(), in_dim, out_dim, y2.data(), nullptr);
    near(y2[3] - y[3], 3.0, "matmul_quant bias");
}

void batch_vs_rows(const char* name, GgmlType type) {
    const int bs = block_size(type);
    const int in_dim = bs <= 32 ? 64 : 256, out_dim = 40, n_rows = 3;
    auto w = test_weights(type, in_dim, out_dim);
    std::vector<float> x(n_rows * in_dim), yb(n_rows * out_dim);
    for (int t = 0; t < n_rows; ++t)
        for (int i = 0; i < in_dim; ++i) x[t * in_dim + i] = static_cast<float>(((i + t) % 5) - 2) * 0.5f;
    matmul_quant_batch(x.data(), w.data(), type, nullptr, in_dim, out_dim, n_rows, yb.data(), nullptr);
    int bad = 0;
    for (int t = 0; t < n_rows; ++t) {
        std::vector<float> y(out_dim);
        matmul_quant(x.data() + t * in_dim, w.data(), type, nullptr, in_dim, out_dim, y.data(), nullptr);
        for (int j = 0; j < out_dim; ++j)
            if (std::fabs(y[j] - yb[t * out_dim + j]) > 1e-4) ++bad;
    }
    expect(bad == 0, std::string("matmul_quant_batch == matmul_quant rows ") + name);
}

void vec_dot_row_check() {
    const int in_dim = 512;
    auto w = test_weights(GgmlType::Q4_K, in_dim, 3);
    std::vector<float> x(in_dim);
    for (int i = 0; i < in_dim; ++i) x[i] = static_cast<float>((i % 9) - 4) * 0.25f;
    QuantizedQ8_0 q;
    quantize_row_q8_0(x.data(), q, in_dim);
    std::vector<float> y(3);
    matmul_quant(x.data(), w.data(), GgmlType::Q4_K, nullptr, in_dim, 3, y.data(), nullptr);
    const size_t rb = (in_dim / 256) * 144;
    for (int j = 0; j < 3; ++j) {
        const float v = vec_dot_row(&w[j * rb], GgmlType::Q4_K, q, in_dim);
        near(v, y[j], "vec_dot_row == matmul_quant row " + std::to_string(j));
    }
    int bsum_ok = 1;
    for (int b = 0; b < in_dim / 32; ++b) {
        int s = 0;
        for (int i = 0; i < 32; ++i) s += q.qs[b * 32 + i];
        bsum_ok &= (s == q.bsums[b]);
    }
    expect(bsum_ok && q.n == in_dim, "quantize_row_q8_0 bsums");
}

template <class F>
void throws_with(F&& f, const char* msg) {
    try {
        f();
        expect(false, std::string("expected exception: ") + msg);
    } catch (const std::runtime_error& e) {
        expect(std::string(e.what()) == msg, std::string("message '") + e.what() + "' == '" + msg + "'");
    }
}

void errors() {
    std::vector<float> x(300), y(4);
    std::vector<uint8_t> w(4096);
    throws_with([&] { matmul_quant(x.data(), w.data(), GgmlType::Q4_K, nullptr, 100, 4, y.data()); },
                "matmul_quant: in_dim not divisible by block size");
    throws_with([&] { matmul_quant_batch(x.data(), w.data(), GgmlType::Q4_K, nullptr, 100, 4, 2, y.data()); },
                "matmul_quant_batch: in_dim not divisible by block size");
    QuantizedQ8_0 q;
    throws_with([&] { quantize_row_q8_0(x.data(), q, 33); }, "quantize_row_q8_0: n not divisible by 32");
    throws_with([&] { vec_dot_row(w.data(), GgmlType::Q4_1, q, 32); }, "vec_dot_row: no kernel for this type");
    // n_rows <= 0 leaves y untouched (quant.cpp:1436)
    y[0] = 7.0f;
    matmul_quant_batch(x.data(), w.data(), GgmlType::Q4_K, nullptr, 100, 4, 0, y.data());
    expect(y[0] == 7.0f, "n_rows == 0 is a no-op");
    expect(has_vec_dot(GgmlType::Q6_K) && !has_vec_dot(GgmlType::Q4_1) && !has_vec_dot(GgmlType::F16),
           "has_vec_dot");
    expect(block_size(GgmlType::Q4_K) == 256 && type_size(GgmlType::Q6_K) == 210 &&
               block_size(static_cast<GgmlType>(999)) == 1 && type_size(static_cast<GgmlType>(999)) == 0,
           "block_size / type_size");
}

// Reference-style fp16 decode written out field by field, for the exhaustive check.
float h2f_fields(uint16_t h) {
    const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
    float v;
    if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
    else if (e == 31) v = m ? std::nanf("") : INFINITY;
    else v = std::ldexp(static_cast<float>(m + 1024), e - 25);
    return s ? -v : v;
}

void fp16_conversions() {
    int bad = 0;
    for (uint32_t h = 0; h < 65536; ++h) {
        const float a = half_to_float(static_cast<uint16_t>(h)), b = h2f_fields(static_cast<uint16_t>(h));
        if (std::isnan(b)) {
            uint32_t ab;
            std::memcpy(&ab, &a, 4);
            bad += !(std::isnan(a) && ((ab >> 13) & 1023) == (h & 1023) && (ab >> 31) == (h >> 15));
        } else {
            bad += std::memcmp(&a, &b, 4) != 0;
        }
        if (!std::isnan(b)) bad += float_to_half(a) != static_cast<uint16_t>(h);
    }
    expect(bad == 0, "half_to_float / float_to_half round trip over all 65536 patterns");
    expect(float_to_half(1.0f + 0.0018765625f) == 0x3C01, "float_to_half truncates normals");
    expect(float_to_half(1e-20f) == 0 && float_to_half(-70000.0f) == 0xFC00, "float_to_half underflow/overflow");
}

}  // namespace

int main() {
    try {
        known_answers();
        matmul_vs_dequant("Q4_0", GgmlType::Q4_0);
        matmul_vs_dequant("Q5_0", GgmlType::Q5_0);
        matmul_vs_dequant("Q8_0", GgmlType::Q8_0);
        matmul_vs_dequant("Q4_K", GgmlType::Q4_K);
        matmul_vs_dequant("Q5_K", GgmlType::Q5_K);
        matmul_vs_dequant("Q6_K", GgmlType::Q6_K);
        bias_check();
        batch_vs_rows("Q8_0", GgmlType::Q8_0);
        batch_vs_rows("Q4_K", GgmlType::Q4_K);
        batch_vs_rows("Q5_K", GgmlType::Q5_K);
        batch_vs_rows("Q6_K", GgmlType::Q6_K);
        vec_dot_row_check();
        errors();
        fp16_conversions();
    } catch (const std::exception& e) {
        std::printf("FAIL uncaught exception: %s\n", e.what());
        ++g_fail;
    }
    std::printf("quant_shim_test: %d passed, %d failed\n", g_pass, g_fail);
    return g_fail == 0 ? 0 : 1;
}
