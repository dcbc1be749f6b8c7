// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// A C-ABI wrapper around the UNMODIFIED reference inference engine
// (cllm_inference src/core/engine.cpp, gguf.cpp, quant.cpp, thread_pool.cpp),
// compiled in place by oracle/Makefile into oracle/_ref/libcllm_ref_engine.so.
// The token-parity tests and the decode CPU baseline call the reference's own
// TransformerEngine through it:
//   GgufLoader::load                 include/cllm/core/gguf.hpp:78-81, src/core/gguf.cpp:120-275
//   TransformerEngine(model, pool)   include/cllm/core/engine.hpp:27-30, src/core/engine.cpp:349-409
//   forward(token, compute_logits)   engine.hpp:39, engine.cpp:466-518
//   prefill(tokens)                  engine.hpp:43, engine.cpp:520-610
//   reset_kv_cache / seq_len         engine.hpp:46-48
//   greedy sampling (temperature 0)  src/core/sampler.cpp:32-34 (argmax of the logits)
// Exceptions become a negative return code; ref_engine_last_error() keeps the text.
#include "cllm/core/engine.hpp"
#include "cllm/core/gguf.hpp"
#include "cllm/core/thread_pool.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

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
    }
}

struct RefEngine {
    cllm::GgufModel model;
    std::unique_ptr<cllm::ThreadPool> pool;
    std::unique_ptr<cllm::TransformerEngine> engine;
};

int argmax(const std::vector<float>& v) {
    return (int)(std::max_element(v.begin(), v.end()) - v.begin());
}

void emit(const std::vector<float>& logits, float* out, int* token) {
    if (out) std::memcpy(out, logits.data(), logits.size() * sizeof(float));
    if (token) *token = argmax(logits);
}
}  // namespace

extern "C" {

const char* ref_engine_last_error() { return g_err.c_str(); }

// Load a GGUF file and build the reference engine (WeightMode::Quant) on a
// ThreadPool of n_threads workers.  ctx_limit as TransformerEngine's.
int ref_engine_create(const char* path, int n_threads, int ctx_limit, void** out) {
    return guarded([&] {
        auto e = std::make_unique<RefEngine>();
        e->model = cllm::GgufLoader::load(path);
        e->pool = std::make_unique<cllm::ThreadPool>(n_threads > 0 ? (size_t)n_threads : 1);
        e->engine = std::make_unique<cllm::TransformerEngine>(e->model, *e->pool, cllm::WeightMode::Quant,
                                                               ctx_limit);
        *out = e.release();
    });
}

void ref_engine_destroy(void* h) { delete static_cast<RefEngine*>(h); }

// Model hyper-parameters: n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab, n_ctx.
int ref_engine_config(void* h, int* v) {
    const auto& c = static_cast<RefEngine*>(h)->engine->config();
    v[0] = (int)c.n_layers; v[1] = (int)c.n_embd; v[2] = (int)c.n_head; v[3] = (int)c.n_head_kv;
    v[4] = (int)c.head_dim(); v[5] = (int)c.n_ff; v[6] = (int)c.vocab_size; v[7] = (int)c.n_ctx;
    return 0;
}

// prefill(tokens) -> logits of the last token (vocab floats, may be NULL) and its argmax.
int ref_engine_prefill(void* h, const int* tokens, int n, float* logits, int* token) {
    return guarded([&] {
        std::vector<int> ids(tokens, tokens + n);
        emit(static_cast<RefEngine*>(h)->engine->prefill(ids), logits, token);
    });
}

// forward(token) -> logits (may be NULL) and the greedy next token.
int ref_engine_forward(void* h, int token, float* logits, int* next) {
    return guarded([&] { emit(static_cast<RefEngine*>(h)->engine->forward(token, true), logits, next); });
}

// Greedy generation: prefill(prompt), then `steps` forward calls, each fed the
// previous argmax.  tokens_out[steps] receives the generated ids (the first is
// the prefill's argmax); margins_out (may be NULL) the top-1 minus top-2 logit
// of each generated token, scales_out (may be NULL) the largest |logit|.
int ref_engine_greedy(void* h, const int* prompt, int n_prompt, int steps, int* tokens_out, float* margins_out,
                      float* scales_out) {
    return guarded([&] {
        auto* e = static_cast<RefEngine*>(h);
        std::vector<int> ids(prompt, prompt + n_prompt);
        std::vector<float> logits = e->engine->prefill(ids);
        for (int s = 0; s < steps; ++s) {
            const int tok = argmax(logits);
            tokens_out[s] = tok;
            if (margins_out) {
                float top1 = logits[tok], top2 = -INFINITY;
                for (size_t i = 0; i < logits.size(); ++i)
                    if ((int)i != tok && logits[i] > top2) top2 = logits[i];
                margins_out[s] = top1 - top2;
            }
            if (scales_out) {
                float m = 0.0f;
                for (float v : logits) m = std::max(m, std::fabs(v));
                scales_out[s] = m;
            }
            if (s + 1 < steps) logits = e->engine->forward(tok, true);
        }
    });
}

int ref_engine_reset(void* h) {
    return guarded([&] { static_cast<RefEngine*>(h)->engine->reset_kv_cache(); });
}

int ref_engine_seq_len(void* h) { return static_cast<RefEngine*>(h)->engine->seq_len(); }

}  // extern "C"
