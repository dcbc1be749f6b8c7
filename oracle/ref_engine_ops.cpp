// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Exposes the reference engine's internal operators, compiled from its own
// src/core/engine.cpp (included whole into this translation unit by
// oracle/Makefile, -DREF_ENGINE_CPP="<path>"), so the GPU kernels of the
// engine step can be checked operator by operator on identical inputs:
//   rms_norm_ptr   engine.cpp:24-29
//   silu           engine.cpp:41
//   apply_rope     engine.cpp:44-57
//   attention      engine.cpp:119-146 (AVX2 dot_f32 / axpy_f32 :59-88)
#include REF_ENGINE_CPP

extern "C" {

void ref_op_rms_norm(const float* x, const float* w, int n, float eps, float* out) {
    cllm::rms_norm_ptr(x, w, n, eps, out);
}

void ref_op_silu(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = cllm::silu(x[i]);
}

void ref_op_rope(float* q, int n_head, int head_dim, int pos, float rope_theta) {
    cllm::apply_rope(q, n_head, head_dim, pos, rope_theta);
}

// q [n_head*head_dim]; kc, vc [seq][n_head_kv*head_dim]
void ref_op_attention(const float* q, const float* kc, const float* vc, int seq, int n_head, int n_head_kv,
                      int head_dim, float* out) {
    const size_t n = (size_t)seq * n_head_kv * head_dim;
    std::vector<float> k(kc, kc + n), v(vc, vc + n);
    cllm::attention(q, k, v, seq, n_head, n_head_kv, head_dim, out);
}

}  // extern "C"
