// Device-resident engine step: the reference's GgufLoader::load + the
// TransformerEngine (src/core/gguf.cpp:120-275, src/core/engine.cpp:349-610),
// with the GGUF data section uploaded once to HBM in its native block layout
// and every activation kept in device memory:
// the quantized matmuls go through cllm_cuda_matmul_quant (device pointers),
// the rest through engine_kernels.cuh.  One decode step (forward) is captured
// in a CUDA graph that reads the input token and the position from device
// memory and ends with the greedy argmax, so generation replays the graph
// with no host round trip per token.  Prefill batches T tokens through
// matmul_quant_batch (the tcgen05 GEMMs for Q4_K and Q6_K weights, T >= 32).
//
// Included at the end of cllm_cuda.cu (one translation unit), after the C ABI
// it calls.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <initializer_list>
#include <memory>
#include <unordered_map>

#include "engine_kernels.cuh"

namespace cllm {
namespace eng {

// ---- GGUF parsing (gguf.cpp:120-275: header, metadata, tensor infos, data
// section at the next alignment boundary) --------------------------------
struct GgufTensor {
    int type = 0;
    std::vector<uint64_t> dims;  // innermost first, as stored
    uint64_t offset = 0;         // inside the data section
};

struct GgufMeta {
    std::unordered_map<std::string, uint32_t> u32;
    std::unordered_map<std::string, float> f32;
    std::unordered_map<std::string, std::string> str;
};

class Cursor {
   public:
    Cursor(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    bool ok() const { return ok_; }
    size_t pos() const { return at_; }
    template <class T>
    T get() {
        T v{};
        if (at_ + sizeof(T) > n_) {
            ok_ = false;
            return v;
        }
        std::memcpy(&v, p_ + at_, sizeof(T));
        at_ += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!ok_ || len > n_ - at_) {
            ok_ = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p_ + at_), len);
        at_ += len;
        return s;
    }
    void skip(uint64_t bytes) {
        if (bytes > n_ - at_) ok_ = false;
        else at_ += bytes;
    }

   private:
    const uint8_t* p_;
    size_t n_, at_ = 0;
    bool ok_ = true;
};

// GGUF metadata value types (gguf.cpp:16-19)
enum : uint32_t { kVU8, kVI8, kVU16, kVI16, kVU32, kVI32, kVF32, kVBool, kVStr, kVArr, kVU64, kVI64, kVF64 };

inline void skip_value(Cursor& c, uint32_t type, int depth = 0) {
    switch (type) {
        case kVU8: case kVI8: case kVBool: c.skip(1); break;
        case kVU16: case kVI16: c.skip(2); break;
        case kVU32: case kVI32: case kVF32: c.skip(4); break;
        case kVU64: case kVI64: case kVF64: c.skip(8); break;
        case kVStr: c.str(); break;
        case kVArr: {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (depth > 2) { c.skip(~uint64_t(0)); break; }
            if (et == kVStr || et == kVArr) {
                for (uint64_t i = 0; i < n && c.ok(); ++i) skip_value(c, et, depth + 1);
            } else {
                const uint64_t es = (et <= kVI8 || et == kVBool) ? 1 : (et <= kVI16) ? 2 : (et <= kVF32) ? 4 : 8;
                if (n > (~uint64_t(0)) / es) c.skip(~uint64_t(0));
                else c.skip(n * es);
            }
            break;
        }
        default: c.skip(~uint64_t(0)); break;  // unknown type: invalid file
    }
}

struct GgufFile {
    void* map = nullptr;
    size_t size = 0;
    size_t data_off = 0;
    GgufMeta meta;
    std::unordered_map<std::string, GgufTensor> tensors;
    ~GgufFile() {
        if (map) munmap(map, size);
    }
};

inline int parse_gguf(const char* path, GgufFile& g) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(CLLM_ERR_INVALID_ARG, "cannot open model file: %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        close(fd);
        return fail(CLLM_ERR_INVALID_ARG, "invalid GGUF magic");
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return fail(CLLM_ERR_INVALID_ARG, "mmap failed");
    g.map = m;
    g.size = (size_t)st.st_size;
    const uint8_t* p = static_cast<const uint8_t*>(m);
    if (std::memcmp(p, "GGUF", 4) != 0) return fail(CLLM_ERR_INVALID_ARG, "invalid GGUF magic");
    Cursor c(p, g.size);
    c.skip(4);
    const uint32_t version = c.get<uint32_t>();
    if (version != 2 && version != 3) return fail(CLLM_ERR_INVALID_ARG, "unsupported GGUF version: %u", version);
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    for (uint64_t i = 0; i < n_kv && c.ok(); ++i) {
        const std::string key = c.str();
        const uint32_t type = c.get<uint32_t>();
        if (type == kVU32) g.meta.u32[key] = c.get<uint32_t>();
        else if (type == kVF32) g.meta.f32[key] = c.get<float>();
        else if (type == kVStr) g.meta.str[key] = c.str();
        else skip_value(c, type);
    }
    for (uint64_t i = 0; i < n_tensors && c.ok(); ++i) {
        const std::string name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        GgufTensor t;
        for (uint32_t d = 0; d < nd && d < 8 && c.ok(); ++d) t.dims.push_back(c.get<uint64_t>());
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        g.tensors[name] = t;
    }
    if (!c.ok()) return fail(CLLM_ERR_INVALID_ARG, "truncated GGUF header: %s", path);
    uint32_t align = 32;
    if (auto it = g.meta.u32.find("general.alignment"); it != g.meta.u32.end() && it->second > 0) align = it->second;
    g.data_off = (c.pos() + align - 1) / align * align;
    if (g.data_off > g.size) return fail(CLLM_ERR_INVALID_ARG, "truncated GGUF file: %s", path);
    return CLLM_OK;
}

// ---- the engine ---------------------------------------------------------
struct Weight {
    int type = 0;
    int rows = 0, cols = 0;       // out_dim, in_dim
    const uint8_t* dev = nullptr;  // inside the uploaded data section
};

struct Layer {
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    Weight wq, wk, wv, wo, wg, wu, wd;
    // q|k|v and gate|up as one matrix each when the file stores them back to
    // back with one type (one GEMV per group; rows = the parts' rows summed)
    Weight wqkv, wgu;
};

inline uint64_t weight_bytes(const Weight& w) {
    return (uint64_t)w.rows * (uint64_t)(w.cols / block_size_of(w.type)) * (uint64_t)type_size_of(w.type);
}

// w1 | w2 | ... as one matrix when contiguous, of one type and in_dim; else rows = 0.
inline Weight group_weights(std::initializer_list<const Weight*> parts) {
    Weight g = **parts.begin();
    g.rows = 0;
    const uint8_t* next = g.dev;
    int rows = 0;
    for (const Weight* w : parts) {
        if (w->type != g.type || w->cols != g.cols || w->dev != next) return g;
        next = w->dev + weight_bytes(*w);
        rows += w->rows;
    }
    g.rows = rows;
    return g;
}

struct Config {
    int n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab, n_ctx;
    float rope_theta, norm_eps;
};

struct Engine {
    Config cfg{};
    int dev = 0;
    cudaStream_t st = nullptr;
    GgufFile file;
    uint8_t* data_dev = nullptr;  // the file's data section in HBM
    Weight tok_embd, output;
    float* out_norm = nullptr;
    std::vector<Layer> layers;
    std::vector<void*> allocs;
    // activations (decode) and caches
    float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *g = nullptr, *u = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr;  // [n_layers][n_ctx][kv_dim]
    float2* rope = nullptr;              // [n_ctx][head_dim/2]
    float *part_ml = nullptr, *part_acc = nullptr;  // prefill attention partials (grown)
    size_t part_cap = 0;                             // entries of (token, head, chunk)
    float *dpart_ml = nullptr, *dpart_acc = nullptr;  // decode attention partials (fixed: the graph uses them)
    uint8_t* scratch = nullptr;                       // decode matmul scratch (fixed: the graph uses it)
    size_t scratch_cap = 0;
    // decode fusions (every decode matmul runs the fused GEMV): RMSNorm and
    // SwiGLU inside the GEMVs' activation quantization, RoPE + KV append +
    // attention + chunk merge in one kernel, multi-CTA argmax
    bool fused = false;
    int* attn_counters = nullptr;  // [n_head_kv], zero between steps
    float* arg_part = nullptr;     // [kArgCtas][3]
    int* arg_counter = nullptr;    // zero between steps
    int* state = nullptr;
    int* gen = nullptr;
    float* margins = nullptr;
    int* tokens_dev = nullptr;
    int tokens_cap = 0;
    int* host_state = nullptr;  // pinned mirror of the state words
    // prefill buffers, grown to the largest T seen
    int pcap = 0;
    float *X = nullptr, *H = nullptr, *Q = nullptr, *K = nullptr, *V = nullptr, *A = nullptr, *TMP = nullptr;
    float *G = nullptr, *U = nullptr;
    float *QKV = nullptr, *GU = nullptr;  // row-interleaved outputs of the grouped q|k|v and gate|up GEMMs
    cudaGraphExec_t step_exec = nullptr;
    std::vector<int> cached;
    int seq_len = 0;
    uint64_t launches_per_step = 0;

    int kv_dim() const { return cfg.n_head_kv * cfg.head_dim; }
    int q_dim() const { return cfg.n_head * cfg.head_dim; }
    int n_chunks() const { return (cfg.n_ctx + kAttnChunk - 1) / kAttnChunk; }

    ~Engine() {
        if (step_exec) cudaGraphExecDestroy(step_exec);
        if (st) cudaStreamSynchronize(st);
        for (void* p : allocs) cudaFree(p);
        for (float* p : {X, H, Q, K, V, A, TMP, G, U, QKV, GU}) if (p) cudaFree(p);
        if (part_ml) cudaFree(part_ml);
        if (part_acc) cudaFree(part_acc);
        if (tokens_dev) cudaFree(tokens_dev);
        if (host_state) cudaFreeHost(host_state);
        if (st) cudaStreamDestroy(st);
    }

    template <class T>
    int alloc(T** p, size_t count) {
        void* q = nullptr;
        CLLM_CUDA_TRY(cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)));
        allocs.push_back(q);
        *p = static_cast<T*>(q);
        return CLLM_OK;
    }
};

inline uint32_t meta_u32(const GgufMeta& m, const std::string& arch, const char* suffix) {
    if (auto it = m.u32.find(arch + "." + suffix); it != m.u32.end()) return it->second;
    if (auto it = m.u32.find(std::string("llama.") + suffix); it != m.u32.end()) return it->second;
    return 0;
}
inline float meta_f32(const GgufMeta& m, const std::string& arch, const char* suffix) {
    if (auto it = m.f32.find(arch + "." + suffix); it != m.f32.end()) return it->second;
    if (auto it = m.f32.find(std::string("llama.") + suffix); it != m.f32.end()) return it->second;
    return 0.0f;
}

// A linear weight [rows][cols] (engine.cpp:180-198).
inline int find_weight(Engine& e, const std::string& name, int rows, int cols, Weight* w) {
    auto it = e.file.tensors.find(name);
    if (it == e.file.tensors.end()) return fail(CLLM_ERR_INVALID_ARG, "missing tensor: %s", name.c_str());
    const GgufTensor& t = it->second;
    const int bs = block_size_of(t.type);
    const int64_t ts = type_size_of(t.type);
    if (ts == 0) return fail(CLLM_ERR_UNSUPPORTED_TYPE, "unsupported ggml type for dequantize");
    if (cols % bs != 0) return fail(CLLM_ERR_BLOCK_MULTIPLE, "matmul_quant: in_dim not divisible by block size");
    const uint64_t bytes = (uint64_t)rows * (uint64_t)(cols / bs) * (uint64_t)ts;
    if (t.offset + bytes > e.file.size - e.file.data_off)
        return fail(CLLM_ERR_INVALID_ARG, "tensor %s runs past the end of the file", name.c_str());
    w->type = t.type;
    w->rows = rows;
    w->cols = cols;
    w->dev = e.data_dev + t.offset;
    return CLLM_OK;
}

// A 1-D tensor dequantized to fp32 in device memory (engine.cpp:201-225);
// *out = nullptr when absent and optional.
inline int load_vector(Engine& e, const std::string& name, int n, bool optional, float** out) {
    *out = nullptr;
    auto it = e.file.tensors.find(name);
    if (it == e.file.tensors.end()) {
        if (optional) return CLLM_OK;
        return fail(CLLM_ERR_INVALID_ARG, "missing tensor: %s", name.c_str());
    }
    const GgufTensor& t = it->second;
    uint64_t numel = 1;
    for (uint64_t d : t.dims) numel *= d;
    if ((int64_t)numel != n) return fail(CLLM_ERR_INVALID_ARG, "tensor %s has %llu values, expected %d", name.c_str(),
                                         (unsigned long long)numel, n);
    if (int rc = e.alloc(out, (size_t)n)) return rc;
    return cllm_cuda_dequantize(e.data_dev + t.offset, t.type, n, *out, e.st);
}

// Launch a kernel of the step with programmatic dependent launch (it starts
// with griddepcontrol.wait, engine_kernels.cuh).
template <class... KArgs, class... Args>
inline int pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CLLM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
    return CLLM_OK;
}

// A matmul of the engine: the decode step (n_rows == 1) runs on the engine's
// own fixed scratch, prefill on the library's workspace.
inline int mm(Engine& e, const float* x, const Weight& w, const float* bias, int n_rows, float* y) {
    const bool decode = n_rows == 1 && e.scratch != nullptr;
    return matmul_quant_impl(x, w.dev, w.type, bias, w.cols, w.rows, n_rows, y, 0, e.st, decode ? e.scratch : nullptr,
                             decode ? e.scratch_cap : 0, nullptr);
}

// A decode matmul with a pre-quantization step (RMSNorm or SwiGLU) applied by
// the GEMV itself.
inline int mm_pre(Engine& e, const float* x, const Weight& w, const float* bias, float* y, PreOp pre) {
    return matmul_quant_impl(x, w.dev, w.type, bias, w.cols, w.rows, 1, y, 0, e.st, e.scratch, e.scratch_cap, nullptr,
                             pre);
}

// Whether a one-row matmul with w runs the fused GEMV (so pre-steps can ride on it).
inline bool fusable(const Weight& w) {
    if (!has_vec_dot_of(w.type)) return false;
    int dev;
    if (ensure_device(&dev)) return false;
    const int64_t row_bytes = (int64_t)(w.cols / block_size_of(w.type)) * type_size_of(w.type);
    const GemvPlan pl = plan_gemv(w.type, w.dev, row_bytes, w.cols, w.rows, 1, true, g_dev[dev]);
    return pl.tma && pl.fused;
}

// Scratch bytes of a one-row matmul with w (matmul_quant_impl's size query).
inline int scratch_need(const Weight& w, size_t* need) {
    return matmul_quant_impl(nullptr, w.dev, w.type, nullptr, w.cols, w.rows, 1, nullptr, 0, nullptr, nullptr, 0, need);
}

template <int HD>
inline int launch_attention(Engine& e, const float* q, const float* kc, const float* vc, const int* pos_dev, int pos0,
                            int T, int n_chunks, float* part_ml, float* part_acc, float* out) {
    const int rep = e.cfg.n_head / e.cfg.n_head_kv;
    const float scale = 1.0f / std::sqrt((float)e.cfg.head_dim);  // engine.cpp:126
    const dim3 grid(e.cfg.n_head_kv, n_chunks, T);
#define CLLM_ATTN(R)                                                                                       \
    case R:                                                                                                \
        if (int rc_ = pdl(attn_chunk_kernel<HD, R>, grid, dim3(kAttnThreads), e.st, q, kc, vc, e.cfg.n_head_kv, \
                          pos_dev, pos0, scale, part_ml, part_acc))                                        \
            return rc_;                                                                                    \
        break;
    switch (rep) {
        CLLM_ATTN(1) CLLM_ATTN(2) CLLM_ATTN(4) CLLM_ATTN(8)
        default: return fail(CLLM_ERR_INVALID_ARG, "GQA ratio %d is not supported", rep);
    }
#undef CLLM_ATTN
    CLLM_CUDA_TRY(cudaGetLastError());
    if (int rc_ = pdl(attn_combine_kernel<HD>, dim3(dim3(e.cfg.n_head, T)), dim3(HD), e.st, part_ml, part_acc, n_chunks, pos_dev, pos0, out)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// Decode (pos_dev set, T == 1) uses the fixed decode partials; prefill the grown ones.
inline int attention(Engine& e, const float* q, const float* kc, const float* vc, const int* pos_dev, int pos0, int T,
                     int n_chunks, float* out) {
    float* ml = pos_dev ? e.dpart_ml : e.part_ml;
    float* acc = pos_dev ? e.dpart_acc : e.part_acc;
    if (e.cfg.head_dim == 128) return launch_attention<128>(e, q, kc, vc, pos_dev, pos0, T, n_chunks, ml, acc, out);
    return launch_attention<64>(e, q, kc, vc, pos_dev, pos0, T, n_chunks, ml, acc, out);
}

inline unsigned grid_for(int64_t n) { return (unsigned)std::min<int64_t>((n + 255) / 256, 1184); }

// Partial-attention buffers for T tokens over n_chunks chunks.
inline int ensure_parts(Engine& e, int T, int n_chunks) {
    const size_t need = (size_t)T * e.cfg.n_head * n_chunks;
    if (need <= e.part_cap) return CLLM_OK;
    if (e.part_ml) cudaFree(e.part_ml);
    if (e.part_acc) cudaFree(e.part_acc);
    e.part_ml = e.part_acc = nullptr;
    e.part_cap = 0;
    CLLM_CUDA_TRY(cudaMalloc(&e.part_ml, need * 2 * sizeof(float)));
    CLLM_CUDA_TRY(cudaMalloc(&e.part_acc, need * e.cfg.head_dim * sizeof(float)));
    e.part_cap = need;
    return CLLM_OK;
}

template <int HD>
inline int launch_attn_decode(Engine& e, float* kc, float* vc, const int* pos) {
    const int rep = e.cfg.n_head / e.cfg.n_head_kv;
    const float scale = 1.0f / std::sqrt((float)e.cfg.head_dim);  // engine.cpp:126
    const dim3 grid(e.cfg.n_head_kv, (e.cfg.n_ctx + kDecChunk - 1) / kDecChunk);
#define CLLM_ATTN_DEC(R)                                                                                          \
    case R:                                                                                                       \
        return pdl(attn_decode_kernel<HD, R>, grid, dim3(kAttnThreads), e.st, e.q, e.k, e.v, kc, vc,              \
                   e.cfg.n_head_kv, e.rope, pos, scale, e.dpart_ml, e.dpart_acc, e.attn_counters, e.att);
    switch (rep) {
        CLLM_ATTN_DEC(1) CLLM_ATTN_DEC(2) CLLM_ATTN_DEC(4) CLLM_ATTN_DEC(8)
    }
#undef CLLM_ATTN_DEC
    return fail(CLLM_ERR_INVALID_ARG, "GQA ratio %d is not supported", rep);
}

// The decode step with its fusions (Engine::fused): per layer the q, k and v
// GEMVs normalise x themselves, one attention kernel, the o GEMV adds into x,
// the gate and up GEMVs normalise x, the down GEMV applies SwiGLU to its input
// and adds into x; the output GEMV normalises; the argmax is spread over CTAs.
inline int enqueue_step_fused(Engine& e) {
    const Config& c = e.cfg;
    int* pos = e.state + kStatePos;
    if (int rc = pdl(embed_kernel, dim3((c.n_embd + 255) / 256, 1), dim3(256), e.st, e.tok_embd.dev, e.tok_embd.type,
                     (int64_t)(c.n_embd / block_size_of(e.tok_embd.type)) * type_size_of(e.tok_embd.type), c.n_embd,
                     (const int*)(e.state + kStateToken), e.x))
        return rc;
    const size_t kv_layer = (size_t)c.n_ctx * e.kv_dim();
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = e.layers[l];
        const PreOp n1{kPreRmsNorm, L.attn_norm, c.norm_eps}, n2{kPreRmsNorm, L.ffn_norm, c.norm_eps};
        if (L.wqkv.rows) {  // e.q, e.k, e.v are contiguous: one GEMV writes all three
            if (int rc = mm_pre(e, e.x, L.wqkv, nullptr, e.q, n1)) return rc;
        } else {
            if (int rc = mm_pre(e, e.x, L.wq, L.bq, e.q, n1)) return rc;
            if (int rc = mm_pre(e, e.x, L.wk, L.bk, e.k, n1)) return rc;
            if (int rc = mm_pre(e, e.x, L.wv, L.bv, e.v, n1)) return rc;
        }
        float* kc = e.kc + (size_t)l * kv_layer;
        float* vc = e.vc + (size_t)l * kv_layer;
        const int rc_a = c.head_dim == 128 ? launch_attn_decode<128>(e, kc, vc, pos)
                                           : launch_attn_decode<64>(e, kc, vc, pos);
        if (rc_a) return rc_a;
        if (int rc = mm(e, e.att, L.wo, e.x, 1, e.x)) return rc;  // x += W_o att
        if (L.wgu.rows) {  // e.g, e.u are contiguous
            if (int rc = mm_pre(e, e.x, L.wgu, nullptr, e.g, n2)) return rc;
        } else {
            if (int rc = mm_pre(e, e.x, L.wg, nullptr, e.g, n2)) return rc;
            if (int rc = mm_pre(e, e.x, L.wu, nullptr, e.u, n2)) return rc;
        }
        if (int rc = mm_pre(e, e.g, L.wd, e.x, e.x, PreOp{kPreSiluMul, e.u, 0.0f})) return rc;  // x += W_down swiglu
    }
    if (int rc = mm_pre(e, e.x, e.output, nullptr, e.logits, PreOp{kPreRmsNorm, e.out_norm, c.norm_eps})) return rc;
    return pdl(argmax_multi_kernel, dim3(kArgCtas), dim3(256), e.st, (const float*)e.logits, c.vocab, e.arg_part,
               e.arg_counter, e.state, e.gen, e.margins, c.n_ctx, 1);
}

// One decode step (engine.cpp:466-518) on e.st: embeds state[token] at
// position state[pos], runs every layer, the output norm and matmul, and the
// greedy argmax, which writes the next token and advances the position.
inline int enqueue_step(Engine& e) {
    if (e.fused) return enqueue_step_fused(e);
    const Config& c = e.cfg;
    int* pos = e.state + kStatePos;
    if (int rc_ = pdl(embed_kernel, dim3(dim3((c.n_embd + 255) / 256, 1)), dim3(256), e.st,
        e.tok_embd.dev, e.tok_embd.type,
        (int64_t)(c.n_embd / block_size_of(e.tok_embd.type)) * type_size_of(e.tok_embd.type), c.n_embd,
        e.state + kStateToken, e.x)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    const size_t kv_layer = (size_t)c.n_ctx * e.kv_dim();
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = e.layers[l];
        if (int rc_ = pdl(rmsnorm_kernel, dim3(1), dim3(kNormThreads), e.st, e.x, L.attn_norm, c.n_embd, c.norm_eps, e.h)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        if (int rc = mm(e, e.h, L.wq, L.bq, 1, e.q)) return rc;
        if (int rc = mm(e, e.h, L.wk, L.bk, 1, e.k)) return rc;
        if (int rc = mm(e, e.h, L.wv, L.bv, 1, e.v)) return rc;
        float* kc = e.kc + (size_t)l * kv_layer;
        float* vc = e.vc + (size_t)l * kv_layer;
        if (int rc_ = pdl(rope_kv_kernel, dim3(dim3(1, c.n_head + c.n_head_kv)), dim3(c.head_dim / 2), e.st,
            (const float*)e.q, e.q_dim(), e.q, (const float*)e.k, (const float*)e.v, e.kv_dim(), c.n_head,
            c.n_head_kv, c.head_dim, e.rope, pos, 0, kc, vc)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        if (int rc = attention(e, e.q, kc, vc, pos, 0, 1, e.n_chunks(), e.att)) return rc;
        if (int rc = mm(e, e.att, L.wo, e.x, 1, e.x)) return rc;  // x += W_o att (residual as the bias)
        if (int rc_ = pdl(rmsnorm_kernel, dim3(1), dim3(kNormThreads), e.st, e.x, L.ffn_norm, c.n_embd, c.norm_eps, e.h)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        if (int rc = mm(e, e.h, L.wg, nullptr, 1, e.g)) return rc;
        if (int rc = mm(e, e.h, L.wu, nullptr, 1, e.u)) return rc;
        if (int rc_ = pdl(silu_mul_kernel, dim3(grid_for(c.n_ff)), dim3(256), e.st, e.g, e.u, c.n_ff)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        if (int rc = mm(e, e.g, L.wd, e.x, 1, e.x)) return rc;  // x += W_down swiglu
    }
    if (int rc_ = pdl(rmsnorm_kernel, dim3(1), dim3(kNormThreads), e.st, e.x, e.out_norm, c.n_embd, c.norm_eps, e.h)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    if (int rc = mm(e, e.h, e.output, nullptr, 1, e.logits)) return rc;
    if (int rc_ = pdl(argmax_kernel, dim3(1), dim3(kArgmaxThreads), e.st, e.logits, c.vocab, e.state, e.gen, e.margins, c.n_ctx, 1)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

inline int set_state(Engine& e, int pos, int token, int count) {
    e.host_state[kStatePos] = pos;
    e.host_state[kStateToken] = token;
    e.host_state[kStateCount] = count;
    CLLM_CUDA_TRY(cudaMemcpyAsync(e.state, e.host_state, kStateWords * sizeof(int), cudaMemcpyHostToDevice, e.st));
    CLLM_CUDA_TRY(cudaStreamSynchronize(e.st));
    return CLLM_OK;
}

inline int grow_prefill(Engine& e, int T) {
    if (T <= e.pcap) return CLLM_OK;
    const Config& c = e.cfg;
    for (float** p : {&e.X, &e.H, &e.Q, &e.K, &e.V, &e.A, &e.TMP, &e.G, &e.U, &e.QKV, &e.GU}) {
        if (*p) cudaFree(*p);
        *p = nullptr;
    }
    e.pcap = 0;
    const size_t te = (size_t)T;
    CLLM_CUDA_TRY(cudaMalloc(&e.X, te * c.n_embd * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.H, te * c.n_embd * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.TMP, te * c.n_embd * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.Q, te * e.q_dim() * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.A, te * e.q_dim() * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.K, te * e.kv_dim() * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.V, te * e.kv_dim() * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.G, te * c.n_ff * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.U, te * c.n_ff * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.QKV, te * (e.q_dim() + 2 * e.kv_dim()) * 4));
    CLLM_CUDA_TRY(cudaMalloc(&e.GU, te * 2 * c.n_ff * 4));
    if ((int)te > e.tokens_cap) {
        if (e.tokens_dev) cudaFree(e.tokens_dev);
        e.tokens_dev = nullptr;
        CLLM_CUDA_TRY(cudaMalloc(&e.tokens_dev, te * sizeof(int)));
        e.tokens_cap = (int)te;
    }
    e.pcap = T;
    return CLLM_OK;
}

// The batched prefill of T tokens at positions pos0.. (engine.cpp:548-609),
// then the last token's logits and greedy argmax (state[token]); state[pos]
// becomes pos0 + T.
inline int run_prefill(Engine& e, const int* tokens, int T, int pos0) {
    const Config& c = e.cfg;
    if (int rc = grow_prefill(e, T)) return rc;
    const int chunks = (pos0 + T + kAttnChunk - 1) / kAttnChunk;
    if (int rc = ensure_parts(e, T, chunks)) return rc;
    CLLM_CUDA_TRY(cudaMemcpyAsync(e.tokens_dev, tokens, (size_t)T * sizeof(int), cudaMemcpyHostToDevice, e.st));
    if (int rc_ = pdl(embed_kernel, dim3(dim3((c.n_embd + 255) / 256, T)), dim3(256), e.st,
        e.tok_embd.dev, e.tok_embd.type,
        (int64_t)(c.n_embd / block_size_of(e.tok_embd.type)) * type_size_of(e.tok_embd.type), c.n_embd,
        e.tokens_dev, e.X)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    const size_t kv_layer = (size_t)c.n_ctx * e.kv_dim();
    const int64_t ne = (int64_t)T * c.n_embd;
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = e.layers[l];
        if (int rc_ = pdl(rmsnorm_kernel, dim3(T), dim3(kNormThreads), e.st, e.X, L.attn_norm, c.n_embd, c.norm_eps, e.H)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        // q|k|v as one GEMM where the three matrices are contiguous (rows of q_dim +
        // 2 kv_dim per token, one activation preparation, a wider grid)
        const float *qs = e.Q, *ks = e.K, *vs = e.V;
        int ldq = e.q_dim(), ldkv = e.kv_dim();
        if (L.wqkv.rows) {
            if (int rc = mm(e, e.H, L.wqkv, nullptr, T, e.QKV)) return rc;
            qs = e.QKV;
            ks = e.QKV + e.q_dim();
            vs = ks + e.kv_dim();
            ldq = ldkv = e.q_dim() + 2 * e.kv_dim();
        } else {
            if (int rc = mm(e, e.H, L.wq, L.bq, T, e.Q)) return rc;
            if (int rc = mm(e, e.H, L.wk, L.bk, T, e.K)) return rc;
            if (int rc = mm(e, e.H, L.wv, L.bv, T, e.V)) return rc;
        }
        float* kc = e.kc + (size_t)l * kv_layer;
        float* vc = e.vc + (size_t)l * kv_layer;
        if (int rc_ = pdl(rope_kv_kernel, dim3(dim3(T, c.n_head + c.n_head_kv)), dim3(c.head_dim / 2), e.st,
            qs, ldq, e.Q, ks, vs, ldkv, c.n_head, c.n_head_kv, c.head_dim, e.rope, nullptr, pos0, kc, vc)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
        if (int rc = attention(e, e.Q, kc, vc, nullptr, pos0, T, chunks, e.A)) return rc;
        if (int rc = mm(e, e.A, L.wo, nullptr, T, e.TMP)) return rc;
        if (int rc_ = pdl(add_kernel, dim3(grid_for(ne)), dim3(256), e.st, e.X, e.TMP, ne)) return rc_;
        if (int rc_ = pdl(rmsnorm_kernel, dim3(T), dim3(kNormThreads), e.st, e.X, L.ffn_norm, c.n_embd, c.norm_eps, e.H)) return rc_;
        if (L.wgu.rows) {  // gate|up as one GEMM, rows of 2 n_ff per token
            if (int rc = mm(e, e.H, L.wgu, nullptr, T, e.GU)) return rc;
            if (int rc_ = pdl(silu_mul_rows_kernel, dim3((unsigned)std::min(8, (c.n_ff + 1023) / 1024), (unsigned)T),
                              dim3(256), e.st, e.G, (const float*)e.GU, c.n_ff)) return rc_;
        } else {
            if (int rc = mm(e, e.H, L.wg, nullptr, T, e.G)) return rc;
            if (int rc = mm(e, e.H, L.wu, nullptr, T, e.U)) return rc;
            if (int rc_ = pdl(silu_mul_kernel, dim3(grid_for((int64_t)T * c.n_ff)), dim3(256), e.st, e.G, e.U, (int64_t)T * c.n_ff)) return rc_;
        }
        if (int rc = mm(e, e.G, L.wd, nullptr, T, e.TMP)) return rc;
        if (int rc_ = pdl(add_kernel, dim3(grid_for(ne)), dim3(256), e.st, e.X, e.TMP, ne)) return rc_;
        CLLM_CUDA_TRY(cudaGetLastError());
    }
    if (int rc_ = pdl(rmsnorm_kernel, dim3(1), dim3(kNormThreads), e.st, e.X + (size_t)(T - 1) * c.n_embd, e.out_norm, c.n_embd, c.norm_eps,
                                                 e.h)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    if (int rc = mm(e, e.h, e.output, nullptr, 1, e.logits)) return rc;
    if (int rc_ = pdl(argmax_kernel, dim3(1), dim3(kArgmaxThreads), e.st, e.logits, c.vocab, e.state, e.gen, e.margins, c.n_ctx, T)) return rc_;
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

// Capture one decode step into a CUDA graph (after an eager warm-up step at
// position 0, which sizes the library's workspace and sets kernel attributes
// outside the capture; the engine is then reset).
inline int build_step_graph(Engine& e) {
    if (int rc = set_state(e, 0, 0, 0)) return rc;
    if (int rc = enqueue_step(e)) return rc;
    CLLM_CUDA_TRY(cudaStreamSynchronize(e.st));
    if (int rc = cllm_cuda_check_device_status()) return rc;
    cudaGraph_t graph = nullptr;
    CLLM_CUDA_TRY(cudaStreamBeginCapture(e.st, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(e);
    const cudaError_t ce = cudaStreamEndCapture(e.st, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (ce != cudaSuccess) return fail(CLLM_ERR_CUDA, "decode-step capture failed: %s", cudaGetErrorString(ce));
    size_t nodes = 0;
    if (cudaGraphGetNodes(graph, nullptr, &nodes) == cudaSuccess) e.launches_per_step = nodes;  // all kernel nodes
    const cudaError_t ie = cudaGraphInstantiate(&e.step_exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return fail(CLLM_ERR_CUDA, "decode-step graph: %s", cudaGetErrorString(ie));
    return set_state(e, 0, 0, 0);
}

inline int create(const char* path, int ctx_limit, Engine** out) {
    auto e = std::make_unique<Engine>();
    if (int rc = ensure_device(&e->dev)) return rc;
    if (int rc = parse_gguf(path, e->file)) return rc;
    const GgufMeta& m = e->file.meta;
    auto arch_it = m.str.find("general.architecture");
    if (arch_it == m.str.end() || arch_it->second.empty())
        return fail(CLLM_ERR_INVALID_ARG, "unknown architecture (missing general.architecture)");
    const std::string arch = arch_it->second;
    Config& c = e->cfg;
    c.n_layers = (int)meta_u32(m, arch, "block_count");
    c.n_embd = (int)meta_u32(m, arch, "embedding_length");
    c.n_head = (int)meta_u32(m, arch, "attention.head_count");
    c.n_head_kv = (int)meta_u32(m, arch, "attention.head_count_kv");
    c.n_ctx = (int)meta_u32(m, arch, "context_length");
    c.n_ff = (int)meta_u32(m, arch, "feed_forward_length");
    const int hd_explicit = (int)meta_u32(m, arch, "attention.key_length");
    const float rope = meta_f32(m, arch, "rope.freq_base");
    c.rope_theta = rope > 0 ? rope : 10000.0f;
    const float eps = meta_f32(m, arch, "attention.layer_norm_rms_epsilon");
    c.norm_eps = eps > 0 ? eps : 1e-5f;
    c.vocab = (int)meta_u32(m, arch, "vocab_size");
    if (c.n_head_kv == 0) c.n_head_kv = c.n_head;
    if (c.n_head == 0 || c.n_embd == 0 || c.n_layers == 0)
        return fail(CLLM_ERR_INVALID_ARG, "incomplete model hyper-parameters in %s", path);
    c.head_dim = hd_explicit > 0 ? hd_explicit : c.n_embd / c.n_head;
    if (ctx_limit > 0 && (c.n_ctx == 0 || c.n_ctx > ctx_limit)) c.n_ctx = ctx_limit;  // engine.cpp:352-356
    if (c.n_ctx <= 0) return fail(CLLM_ERR_INVALID_ARG, "model has no context length; pass ctx_limit");
    if (c.head_dim != 128 && c.head_dim != 64)
        return fail(CLLM_ERR_INVALID_ARG, "head_dim %d is not supported (64 or 128)", c.head_dim);
    const int rep = c.n_head % c.n_head_kv == 0 ? c.n_head / c.n_head_kv : 0;
    if (rep != 1 && rep != 2 && rep != 4 && rep != 8)
        return fail(CLLM_ERR_INVALID_ARG, "GQA ratio %d/%d is not supported", c.n_head, c.n_head_kv);
    CLLM_CUDA_TRY(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));

    // upload the data section once (gguf.cpp:178-189 points every tensor into
    // it), into the engine's own allocation: tensor offsets are multiples of
    // the alignment (32), so every 16-byte-multiple row stays 16-byte aligned
    {
        const size_t bytes = e->file.size - e->file.data_off;
        if (int rc = e->alloc(&e->data_dev, bytes)) return rc;
        CLLM_CUDA_TRY(cudaMemcpy(e->data_dev, static_cast<const uint8_t*>(e->file.map) + e->file.data_off, bytes,
                                 cudaMemcpyHostToDevice));
    }

    if (c.vocab == 0) {  // gguf.cpp:270: the vocabulary size falls back to the embedding rows
        auto it = e->file.tensors.find("token_embd.weight");
        if (it != e->file.tensors.end() && it->second.dims.size() == 2) c.vocab = (int)it->second.dims[1];
    }
    const int qd = e->q_dim(), kvd = e->kv_dim();
    if (int rc = find_weight(*e, "token_embd.weight", c.vocab, c.n_embd, &e->tok_embd)) return rc;
    if (e->file.tensors.count("output.weight")) {
        if (int rc = find_weight(*e, "output.weight", c.vocab, c.n_embd, &e->output)) return rc;
    } else {
        e->output = e->tok_embd;  // tied embeddings (engine.cpp:365-369)
    }
    if (int rc = load_vector(*e, "output_norm.weight", c.n_embd, false, &e->out_norm)) return rc;
    e->layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        Layer& L = e->layers[l];
        if (e->file.tensors.count(p + "attn_q_norm.weight") || e->file.tensors.count(p + "attn_k_norm.weight"))
            return fail(CLLM_ERR_INVALID_ARG, "per-head q/k norms (%sattn_q_norm) are not supported", p.c_str());
        int rc = load_vector(*e, p + "attn_norm.weight", c.n_embd, false, &L.attn_norm);
        if (!rc) rc = find_weight(*e, p + "attn_q.weight", qd, c.n_embd, &L.wq);
        if (!rc) rc = find_weight(*e, p + "attn_k.weight", kvd, c.n_embd, &L.wk);
        if (!rc) rc = find_weight(*e, p + "attn_v.weight", kvd, c.n_embd, &L.wv);
        if (!rc) rc = load_vector(*e, p + "attn_q.bias", qd, true, &L.bq);
        if (!rc) rc = load_vector(*e, p + "attn_k.bias", kvd, true, &L.bk);
        if (!rc) rc = load_vector(*e, p + "attn_v.bias", kvd, true, &L.bv);
        if (!rc) rc = find_weight(*e, p + "attn_output.weight", c.n_embd, qd, &L.wo);
        if (!rc) rc = load_vector(*e, p + "ffn_norm.weight", c.n_embd, false, &L.ffn_norm);
        if (!rc) rc = find_weight(*e, p + "ffn_gate.weight", c.n_ff, c.n_embd, &L.wg);
        if (!rc) rc = find_weight(*e, p + "ffn_up.weight", c.n_ff, c.n_embd, &L.wu);
        if (!rc) rc = find_weight(*e, p + "ffn_down.weight", c.n_embd, c.n_ff, &L.wd);
        if (rc) return rc;
    }

    // activations, caches, the RoPE table (engine.cpp:50-52 evaluated on the host)
    Engine& E = *e;
    int rc = E.alloc(&E.x, c.n_embd);
    if (!rc) rc = E.alloc(&E.h, c.n_embd);
    if (!rc) rc = E.alloc(&E.q, (size_t)qd + 2 * kvd);  // q | k | v, one buffer
    E.k = E.q + qd;
    E.v = E.k + kvd;
    if (!rc) rc = E.alloc(&E.att, qd);
    if (!rc) rc = E.alloc(&E.g, 2 * (size_t)c.n_ff);  // gate | up, one buffer
    E.u = E.g + c.n_ff;
    if (!rc) rc = E.alloc(&E.logits, c.vocab);
    if (!rc) rc = E.alloc(&E.kc, (size_t)c.n_layers * c.n_ctx * kvd);
    if (!rc) rc = E.alloc(&E.vc, (size_t)c.n_layers * c.n_ctx * kvd);
    if (!rc) rc = E.alloc(&E.rope, (size_t)c.n_ctx * (c.head_dim / 2));
    if (!rc) rc = E.alloc(&E.state, kStateWords);
    if (!rc) rc = E.alloc(&E.gen, c.n_ctx);
    if (!rc) rc = E.alloc(&E.margins, c.n_ctx);
    if (rc) return rc;
    CLLM_CUDA_TRY(cudaMallocHost(&E.host_state, kStateWords * sizeof(int)));
    {
        const size_t parts = (size_t)c.n_head * std::max(E.n_chunks(), (c.n_ctx + kDecChunk - 1) / kDecChunk);
        if (int rc2 = E.alloc(&E.dpart_ml, parts * 2)) return rc2;
        if (int rc2 = E.alloc(&E.dpart_acc, parts * c.head_dim)) return rc2;
        size_t need = 0, n1 = 0;
        for (Layer& L : E.layers) {
            const bool no_bias = !L.bq && !L.bk && !L.bv;
            L.wqkv = no_bias ? group_weights({&L.wq, &L.wk, &L.wv}) : Weight{};
            L.wgu = group_weights({&L.wg, &L.wu});
        }
        std::vector<const Weight*> ws = {&E.output};
        for (const Layer& L : E.layers) {
            for (const Weight* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wg, &L.wu, &L.wd}) ws.push_back(w);
            if (L.wqkv.rows) ws.push_back(&L.wqkv);
            if (L.wgu.rows) ws.push_back(&L.wgu);
        }
        for (const Weight* w : ws) {
            if (int rc2 = scratch_need(*w, &n1)) return rc2;
            need = std::max(need, n1);
        }
        E.scratch_cap = std::max<size_t>(need, 256);
        if (int rc2 = E.alloc(&E.scratch, E.scratch_cap)) return rc2;
        bool fz = E.output.dev != nullptr && fusable(E.output);
        for (const Layer& L : E.layers) {
            for (const Weight* w : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wg, &L.wu, &L.wd}) fz = fz && fusable(*w);
            if (L.wqkv.rows) fz = fz && fusable(L.wqkv);
            if (L.wgu.rows) fz = fz && fusable(L.wgu);
        }
        E.fused = fz && std::getenv("CLLM_ENGINE_UNFUSED") == nullptr;
        if (int rc2 = E.alloc(&E.attn_counters, c.n_head_kv)) return rc2;
        if (int rc2 = E.alloc(&E.arg_part, 3 * kArgCtas)) return rc2;
        if (int rc2 = E.alloc(&E.arg_counter, 1)) return rc2;
        CLLM_CUDA_TRY(cudaMemset(E.attn_counters, 0, c.n_head_kv * sizeof(int)));
        CLLM_CUDA_TRY(cudaMemset(E.arg_counter, 0, sizeof(int)));
    }
    {
        const int half = c.head_dim / 2;
        std::vector<float2> table((size_t)c.n_ctx * half);
        for (int pos = 0; pos < c.n_ctx; ++pos)
            for (int i = 0; i < half; ++i) {
                const float theta = pos / std::pow(c.rope_theta, (float)i / half);
                table[(size_t)pos * half + i] = make_float2(std::cos(theta), std::sin(theta));
            }
        CLLM_CUDA_TRY(cudaMemcpy(E.rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
    if (int rc2 = build_step_graph(E)) return rc2;
    *out = e.release();
    return CLLM_OK;
}

inline int check_room(const Engine& e, int add) {
    if (e.cfg.n_ctx > 0 && e.seq_len + add > e.cfg.n_ctx)  // engine.cpp:340-344
        return fail(CLLM_ERR_TOO_LARGE, "context length exceeded");
    return CLLM_OK;
}

inline int copy_out(Engine& e, float* logits, int* next) {
    if (logits)
        CLLM_CUDA_TRY(cudaMemcpyAsync(logits, e.logits, (size_t)e.cfg.vocab * sizeof(float), cudaMemcpyDeviceToHost,
                                      e.st));
    CLLM_CUDA_TRY(cudaMemcpyAsync(e.host_state, e.state, kStateWords * sizeof(int), cudaMemcpyDeviceToHost, e.st));
    CLLM_CUDA_TRY(cudaStreamSynchronize(e.st));
    if (next) *next = e.host_state[kStateToken];
    return cllm_cuda_check_device_status();
}

inline int forward(Engine& e, int token, float* logits, int* next) {
    if (token < 0 || token >= e.cfg.vocab) return fail(CLLM_ERR_INVALID_ARG, "token %d out of range", token);
    if (int rc = check_room(e, 1)) return rc;
    if (int rc = set_state(e, e.seq_len, token, 0)) return rc;
    CLLM_CUDA_TRY(cudaGraphLaunch(e.step_exec, e.st));
    if (int rc = copy_out(e, logits, next)) return rc;
    e.cached.push_back(token);
    ++e.seq_len;
    return CLLM_OK;
}

inline void truncate_kv(Engine& e, int n) {  // engine.cpp:324-333
    if (n < 0) n = 0;
    if ((int)e.cached.size() > n) e.cached.resize(n);
    e.seq_len = n;
}

// TransformerEngine::prefill (engine.cpp:520-610) with its prefix reuse.
inline int prefill(Engine& e, const int* tokens, int n, float* logits, int* next) {
    if (n <= 0) return fail(CLLM_ERR_INVALID_ARG, "prefill: empty tokens");
    if (e.cfg.n_ctx > 0 && n > e.cfg.n_ctx) return fail(CLLM_ERR_TOO_LARGE, "context length exceeded");
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= e.cfg.vocab) return fail(CLLM_ERR_INVALID_ARG, "token %d out of range", tokens[i]);
    size_t lcp = 0;
    const size_t max_lcp = std::min((size_t)n, e.cached.size());
    while (lcp < max_lcp && tokens[lcp] == e.cached[lcp]) ++lcp;
    if (lcp == (size_t)n) {
        truncate_kv(e, (int)lcp - 1);
        return forward(e, tokens[n - 1], logits, next);
    }
    truncate_kv(e, (int)lcp);
    const int T = n - (int)lcp;
    if (T == 1) return forward(e, tokens[n - 1], logits, next);
    if (int rc = check_room(e, T)) return rc;
    if (int rc = set_state(e, (int)lcp, 0, 0)) return rc;
    if (int rc = run_prefill(e, tokens + lcp, T, (int)lcp)) return rc;
    if (int rc = copy_out(e, logits, next)) return rc;
    for (int t = 0; t < T; ++t) e.cached.push_back(tokens[lcp + t]);
    e.seq_len += T;
    return CLLM_OK;
}

// Greedy generation, device-resident: prefill(prompt), then steps - 1 replays
// of the decode-step graph, each fed the previous step's argmax on the device;
// the tokens (and margins) are read back once at the end.
inline int generate(Engine& e, const int* prompt, int n, int steps, int* tokens_out, float* margins_out) {
    if (steps <= 0) return CLLM_OK;
    if (!tokens_out) return fail(CLLM_ERR_INVALID_ARG, "generate: null output");
    if (steps > e.cfg.n_ctx) return fail(CLLM_ERR_TOO_LARGE, "context length exceeded");
    if (int rc = prefill(e, prompt, n, nullptr, nullptr)) return rc;
    if (int rc = check_room(e, steps - 1)) return rc;
    // prefill left its argmax in state[token] (count 1): decode from there
    const int first = e.host_state[kStateToken];
    if (int rc = set_state(e, e.seq_len, first, 1)) return rc;
    CLLM_CUDA_TRY(cudaMemcpyAsync(e.gen, &e.host_state[kStateToken], sizeof(int), cudaMemcpyHostToDevice, e.st));
    for (int s = 1; s < steps; ++s) CLLM_CUDA_TRY(cudaGraphLaunch(e.step_exec, e.st));
    CLLM_CUDA_TRY(cudaMemcpyAsync(tokens_out, e.gen, (size_t)steps * sizeof(int), cudaMemcpyDeviceToHost, e.st));
    if (margins_out) {
        // the prefill's margin was written at gen slot 0 by run_prefill's argmax
        CLLM_CUDA_TRY(cudaMemcpyAsync(margins_out, e.margins, (size_t)steps * sizeof(float), cudaMemcpyDeviceToHost,
                                      e.st));
    }
    CLLM_CUDA_TRY(cudaStreamSynchronize(e.st));
    if (int rc = cllm_cuda_check_device_status()) return rc;
    for (int s = 0; s + 1 < steps; ++s) e.cached.push_back(tokens_out[s]);
    e.seq_len += steps - 1;
    return CLLM_OK;
}

}  // namespace eng
}  // namespace cllm

using cllm::eng::Engine;

extern "C" {

int cllm_cuda_engine_create(const char* gguf_path, int ctx_limit, void** engine) {
    if (!gguf_path || !engine) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_create: null argument");
    Engine* e = nullptr;
    if (int rc = cllm::eng::create(gguf_path, ctx_limit, &e)) return rc;
    *engine = e;
    return CLLM_OK;
}

int cllm_cuda_engine_destroy(void* engine) {
    delete static_cast<Engine*>(engine);
    return CLLM_OK;
}

int cllm_cuda_engine_config(const void* engine, int* values, int n) {
    if (!engine || !values) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_config: null argument");
    const auto& c = static_cast<const Engine*>(engine)->cfg;
    const Engine* e = static_cast<const Engine*>(engine);
    const int v[11] = {c.n_layers, c.n_embd, c.n_head, c.n_head_kv, c.head_dim, c.n_ff, c.vocab, c.n_ctx,
                       (int)e->launches_per_step, e->seq_len, e->fused ? 1 : 0};
    for (int i = 0; i < n && i < 11; ++i) values[i] = v[i];
    return CLLM_OK;
}

int cllm_cuda_engine_forward(void* engine, int token, float* logits, int* next_token) {
    if (!engine) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_forward: null engine");
    return cllm::eng::forward(*static_cast<Engine*>(engine), token, logits, next_token);
}

int cllm_cuda_engine_prefill(void* engine, const int* tokens, int n, float* logits, int* next_token) {
    if (!engine || (n > 0 && !tokens)) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_prefill: null argument");
    return cllm::eng::prefill(*static_cast<Engine*>(engine), tokens, n, logits, next_token);
}

int cllm_cuda_engine_generate(void* engine, const int* prompt, int n_prompt, int steps, int* tokens_out,
                              float* margins_out) {
    if (!engine || (n_prompt > 0 && !prompt)) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_generate: null argument");
    return cllm::eng::generate(*static_cast<Engine*>(engine), prompt, n_prompt, steps, tokens_out, margins_out);
}

int cllm_cuda_engine_reset(void* engine) {
    if (!engine) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_reset: null engine");
    auto& e = *static_cast<Engine*>(engine);
    cllm::eng::truncate_kv(e, 0);
    return CLLM_OK;
}

int cllm_cuda_engine_seq_len(const void* engine) {
    return engine ? static_cast<const Engine*>(engine)->seq_len : 0;
}

int cllm_cuda_engine_stream(const void* engine, void** stream) {
    if (!engine || !stream) return cllm::fail(CLLM_ERR_INVALID_ARG, "engine_stream: null argument");
    *stream = static_cast<const Engine*>(engine)->st;
    return CLLM_OK;
}

}  // extern "C"

// ---- the engine's operators as standalone calls (device pointers) ---------
extern "C" {

int cllm_cuda_rms_norm(const float* x, const float* w, int n, int rows, float eps, float* y, void* stream) {
    if (n <= 0 || rows < 0 || !x || !w || !y) return cllm::fail(CLLM_ERR_INVALID_ARG, "rms_norm: bad arguments");
    if (rows == 0) return CLLM_OK;
    cllm::eng::rmsnorm_kernel<<<rows, cllm::eng::kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, w, n, eps, y);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

int cllm_cuda_silu_mul(float* g, const float* u, int64_t n, void* stream) {
    if (n < 0 || (n > 0 && (!g || !u))) return cllm::fail(CLLM_ERR_INVALID_ARG, "silu_mul: bad arguments");
    if (n == 0) return CLLM_OK;
    cllm::eng::silu_mul_kernel<<<cllm::eng::grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(g, u, n);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

int cllm_cuda_rope_table(float rope_theta, int head_dim, int n_pos, float* table) {
    if (head_dim <= 0 || head_dim % 2 || n_pos < 0 || !table) return cllm::fail(CLLM_ERR_INVALID_ARG, "rope_table: bad arguments");
    const int half = head_dim / 2;
    for (int pos = 0; pos < n_pos; ++pos)
        for (int i = 0; i < half; ++i) {
            const float theta = pos / std::pow(rope_theta, (float)i / half);  // engine.cpp:50
            table[2 * ((size_t)pos * half + i)] = std::cos(theta);
            table[2 * ((size_t)pos * half + i) + 1] = std::sin(theta);
        }
    return CLLM_OK;
}

int cllm_cuda_rope_kv(float* q, const float* k, const float* v, int n_tok, int n_head, int n_head_kv, int head_dim,
                      const float* table, int pos0, float* k_cache, float* v_cache, void* stream) {
    if (n_tok < 0 || n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 2048 || pos0 < 0 ||
        !q || !k || !v || !table || !k_cache || !v_cache)
        return cllm::fail(CLLM_ERR_INVALID_ARG, "rope_kv: bad arguments");
    if (n_tok == 0) return CLLM_OK;
    cllm::eng::rope_kv_kernel<<<dim3(n_tok, n_head + n_head_kv), head_dim / 2, 0, static_cast<cudaStream_t>(stream)>>>(
        q, n_head * head_dim, q, k, v, n_head_kv * head_dim, n_head, n_head_kv, head_dim,
        reinterpret_cast<const float2*>(table), nullptr, pos0, k_cache, v_cache);
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

int cllm_cuda_attention(const float* q, const float* k_cache, const float* v_cache, int n_tok, int pos0, int n_head,
                        int n_head_kv, int head_dim, float* out, void* stream) {
    using namespace cllm;
    if (n_tok <= 0 || pos0 < 0 || n_head <= 0 || n_head_kv <= 0 || !q || !k_cache || !v_cache || !out)
        return fail(CLLM_ERR_INVALID_ARG, "attention: bad arguments");
    if (head_dim != 64 && head_dim != 128) return fail(CLLM_ERR_INVALID_ARG, "attention: head_dim %d (64 or 128)", head_dim);
    const int rep = n_head % n_head_kv == 0 ? n_head / n_head_kv : 0;
    if (rep != 1 && rep != 2 && rep != 4 && rep != 8)
        return fail(CLLM_ERR_INVALID_ARG, "attention: GQA ratio %d/%d is not supported", n_head, n_head_kv);
    int dev;
    if (int rc = ensure_device(&dev)) return rc;
    const int chunks = (pos0 + n_tok + eng::kAttnChunk - 1) / eng::kAttnChunk;
    const size_t parts = (size_t)n_tok * n_head * chunks;
    uint8_t* ws;
    std::unique_lock<std::mutex> ws_lock;
    if (int rc = workspace(dev, align256(parts * 2 * 4) + parts * head_dim * 4, &ws, ws_lock)) return rc;
    float* ml = reinterpret_cast<float*>(ws);
    float* acc = reinterpret_cast<float*>(ws + align256(parts * 2 * 4));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const float scale = 1.0f / std::sqrt((float)head_dim);
    const dim3 grid(n_head_kv, chunks, n_tok);
#define CLLM_ATTN_OP(HD, R) eng::attn_chunk_kernel<HD, R><<<grid, eng::kAttnThreads, 0, st>>>(q, k_cache, v_cache, n_head_kv, nullptr, pos0, scale, ml, acc)
    if (head_dim == 128) {
        if (rep == 1) CLLM_ATTN_OP(128, 1); else if (rep == 2) CLLM_ATTN_OP(128, 2);
        else if (rep == 4) CLLM_ATTN_OP(128, 4); else CLLM_ATTN_OP(128, 8);
        CLLM_CUDA_TRY(cudaGetLastError());
        eng::attn_combine_kernel<128><<<dim3(n_head, n_tok), 128, 0, st>>>(ml, acc, chunks, nullptr, pos0, out);
    } else {
        if (rep == 1) CLLM_ATTN_OP(64, 1); else if (rep == 2) CLLM_ATTN_OP(64, 2);
        else if (rep == 4) CLLM_ATTN_OP(64, 4); else CLLM_ATTN_OP(64, 8);
        CLLM_CUDA_TRY(cudaGetLastError());
        eng::attn_combine_kernel<64><<<dim3(n_head, n_tok), 64, 0, st>>>(ml, acc, chunks, nullptr, pos0, out);
    }
#undef CLLM_ATTN_OP
    CLLM_CUDA_TRY(cudaGetLastError());
    return CLLM_OK;
}

}  // extern "C"
