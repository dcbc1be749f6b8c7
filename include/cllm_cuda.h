/*
 * cllm_cuda.h — C ABI of the B200 (sm_100a) quantized-matmul hot path.
 *
 * Drop-in replacement for the quant API of cllm_inference
 * (include/cllm/core/quant.hpp:90-151, src/core/quant.cpp:340-1475 in the
 * reference project).  Plain C: pointers, sizes and ints only.  Every entry
 * point returns CLLM_OK (0) or a negative CLLM_ERR_* code and never throws;
 * cllm_cuda_last_error() returns the message of the calling thread's last
 * failure, using the reference's own exception strings where it has one.
 *
 * Weight types use the GGML numbering of GgmlType (quant.hpp:13-27).  The six
 * with an integer dot kernel (quant.hpp:129-130) run the quantized-activation
 * path everywhere.  cllm_cuda_matmul_quant and cllm_cuda_dequantize also take
 * the other seven types the reference reads (F32, F16, Q4_1, Q5_1, Q8_1, Q2_K,
 * Q3_K) on the GPU, through the reference's dequantize-and-float-dot fallback
 * (quant.cpp:1404-1430) computed in its exact order; any other type id is
 * rejected with CLLM_ERR_UNSUPPORTED_TYPE — there is no CPU fallback.
 *
 * Streams are passed as `void*` (a cudaStream_t; NULL = the legacy default
 * stream).  Calls on one stream are not re-entrant: use one stream per engine.
 */
#ifndef CLLM_CUDA_H
#define CLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define CLLM_OK 0
#define CLLM_ERR_INVALID_ARG -1      /* null pointer, negative size, bad flag */
#define CLLM_ERR_UNSUPPORTED_TYPE -2 /* type without an integer dot kernel */
#define CLLM_ERR_BLOCK_MULTIPLE -3   /* in_dim not a multiple of the block size */
#define CLLM_ERR_CUDA -4             /* a CUDA runtime call failed */
#define CLLM_ERR_NOT_REGISTERED -5   /* host weight pointer outside every registered range */
#define CLLM_ERR_NO_DEVICE -6        /* no usable sm_100 device */
#define CLLM_ERR_KERNEL_TIMEOUT -7   /* a kernel's bounded wait expired (status flag set on device) */
#define CLLM_ERR_TOO_LARGE -8        /* a size beyond what an entry point supports */

/* ---- GGML type ids (quant.hpp:13-27) ----------------------------------- */
#define CLLM_TYPE_F32 0
#define CLLM_TYPE_F16 1
#define CLLM_TYPE_Q4_1 3
#define CLLM_TYPE_Q5_1 7
#define CLLM_TYPE_Q8_1 9
#define CLLM_TYPE_Q2_K 10
#define CLLM_TYPE_Q3_K 11
#define CLLM_TYPE_Q4_0 2
#define CLLM_TYPE_Q5_0 6
#define CLLM_TYPE_Q8_0 8
#define CLLM_TYPE_Q4_K 12
#define CLLM_TYPE_Q5_K 13
#define CLLM_TYPE_Q6_K 14

/* ---- cllm_cuda_matmul_quant flags -------------------------------------- */
/* Host buffers of the GEMV path (n_rows below the tensor-core prefill) that are
 * pinned and mapped (cudaHostAlloc, cudaMallocHost, cudaHostRegister) are used
 * in place: x is read once by the activation-quantization kernel and y is
 * written by the GEMV's stores, with no copy operation.  Other host buffers
 * (pageable memory, the prefill and fallback paths) are copied on the stream. */
#define CLLM_X_HOST 1u /* x and bias are host pointers (bias is always copied in) */
#define CLLM_Y_HOST 2u /* y is a host pointer; the call synchronizes the stream */
#define CLLM_W_HOST 4u /* w is a host pointer inside a range given to cllm_cuda_register_weights */
#define CLLM_HOST_IO (CLLM_X_HOST | CLLM_Y_HOST)

/* Select and initialise the device (cudaSetDevice + capability check).
 * Replaces nothing in the reference (the CPU engine has no device); the
 * quant.hpp shim calls it once on first use. */
int cllm_cuda_init(int device);

/* quant.cpp:340-352 — elements per block; 1 for F32/F16 and unknown types. */
int cllm_cuda_block_size(int type);

/* quant.cpp:354-369 — bytes per block; 0 for unknown types. */
int64_t cllm_cuda_type_size(int type);

/* quant.cpp:1347-1357 — 1 for Q4_0/Q5_0/Q8_0/Q4_K/Q5_K/Q6_K, else 0. */
int cllm_cuda_has_vec_dot(int type);

/* Upload [host_base, host_base+bytes) — e.g. a GGUF mmap'd data section
 * (gguf.cpp:171-189) — to HBM once, in its native block layout, and remember
 * the mapping so later calls can pass weight pointers into that host range
 * with CLLM_W_HOST.  The device copy keeps the host address's offset modulo
 * 256, so rows aligned on the host are aligned on the device.  *dev_base (may
 * be NULL) receives the device address of host_base.  Registering a range
 * that overlaps an existing one fails with CLLM_ERR_INVALID_ARG. */
int cllm_cuda_register_weights(const void* host_base, size_t bytes, void** dev_base);

/* Free the device copy registered for exactly host_base. */
int cllm_cuda_unregister_weights(const void* host_base);

/* Device address of host_ptr inside a registered range. */
int cllm_cuda_lookup_weights(const void* host_ptr, const void** dev_ptr);

/* quant.cpp:420-452 — quantize_row_q8_0 over `rows` rows of n floats (device
 * pointers).  Outputs, per row r: scales[r*n/32 ...] fp32, qs[r*n ...] int8,
 * bsums[r*n/32 ...] int32.  Bit-exact with the reference on x86, including
 * NaN inputs (which quantize to -128 there).  n % 32 != 0 fails with
 * CLLM_ERR_BLOCK_MULTIPLE and "quantize_row_q8_0: n not divisible by 32". */
int cllm_cuda_quantize_q8_0(const float* x, int64_t n, int rows, float* scales, int8_t* qs,
                            int32_t* bsums, void* stream);

/* quant.cpp:1374-1475 — matmul_quant (n_rows == 1) and matmul_quant_batch:
 *   y[t*out_dim + j] = vec_dot_row(W_j, quantize_row_q8_0(x_t)) (+ bias[j])
 * for t < n_rows, j < out_dim.  W is out_dim rows of (in_dim/block) blocks in
 * GGML layout.  n_rows <= 0 returns CLLM_OK without touching y
 * (quant.cpp:1436).  Error strings follow quant.cpp:1379/1443/1370.
 * By default all pointers are device pointers and the call is asynchronous on
 * `stream`; the flags above switch x/bias, y and w to host memory.  Scratch
 * for the quantized activations comes from one workspace per device that the
 * library grows on demand (cudaDeviceSynchronize, cudaFree, cudaMalloc) and
 * keeps until exit; make a first call of the largest size before capturing
 * calls into a CUDA graph.  Host threads may call concurrently (a per-device
 * lock is held until the call's kernels are enqueued), but calls whose GPU
 * work can overlap -- on different streams of one device -- share that
 * workspace and race on it: order them (one stream, or events). */
int cllm_cuda_matmul_quant(const float* x, const void* w, int type, const float* bias, int in_dim,
                           int out_dim, int n_rows, float* y, unsigned flags, void* stream);

/* matmul_quant on activations that are already quantized (the arrays of
 * QuantizedQ8_0, quant.hpp:118-124, for n_rows rows, device pointers): the
 * float path of vec_dot_row (quant.cpp:1359-1372) for every weight row.
 * Lets a caller quantize one activation once and reuse it for several
 * weight matrices (q/k/v, gate/up).  bias and y are device pointers. */
int cllm_cuda_matmul_q8(const float* scales, const int8_t* qs, const int32_t* bsums, const void* w,
                        int type, const float* bias, int in_dim, int out_dim, int n_rows, float* y,
                        void* stream);

/* Debug / parity entry: the exact int32 partial dot products of every weight
 * row against every quantized activation row, in the layout
 *   partials[(t*out_dim + j)*ppr + p],  ppr = in_dim/32 (2*in_dim/32 for Q6_K)
 * where part p is activation block p (Q6_K: block p/2, half p%2).  Inputs are
 * device pointers: the quantized activations as cllm_cuda_quantize_q8_0
 * writes them.  The reference has no counterpart (its vec_dot returns only
 * the float sum); the values are those its AVX2 kernels form internally. */
int cllm_cuda_row_partials(const int8_t* qs, const void* w, int type, int in_dim, int out_dim,
                           int n_rows, int32_t* partials, void* stream);

/* Parity entry for the production kernels: runs the launch plan that
 * cllm_cuda_matmul_quant(x, w, ...) runs with device pointers and no bias --
 * the same activation quantization (fused into the GEMV, or once per call for
 * in_dim >= 8192) and the same dot loops -- in a build whose kernels store
 * the exact int32 partials instead of y, in the layout of
 * cllm_cuda_row_partials for n_rows activation rows of x (fp32, device).
 * Rows are taken 4 or 1 at a time (both row counts of the production
 * templates' loops).  No counterpart in the reference; the values are those
 * its AVX2 kernels form internally (quant.cpp:549-687). */
int cllm_cuda_matmul_partials(const float* x, const void* w, int type, int in_dim, int out_dim, int n_rows,
                              int32_t* partials, void* stream);

/* quant.cpp:371-389 (dequantize_block) for all thirteen types the reference
 * handles: n values from the blocks at src (device) into dst (device fp32),
 * bit-exact.  n must be a multiple of the block size.  Unknown types fail with
 * "unsupported ggml type for dequantize".  Used by the engine's embedding
 * lookup (engine.cpp:310-316) and its norm weights (engine.cpp:201-225). */
int cllm_cuda_dequantize(const void* src, int type, int64_t n, float* dst, void* stream);

/* quant.cpp:391-402 (dequantize_block_f16): as cllm_cuda_dequantize, then each
 * value rounded to fp16 bits as the reference's float_to_half does
 * (quant.hpp:58-85); F16 sources are copied. */
int cllm_cuda_dequantize_f16(const void* src, int type, int64_t n, uint16_t* dst, void* stream);

/* Launch plan cllm_cuda_matmul_quant would use for these arguments (device
 * weights at w): info[0] kernels launched per call, [1] the dot kernel: 0
 * direct loads, 1 bulk-copy (TMA) ring GEMV, 2 tcgen05 tensor-core GEMM
 * (Q4_K and Q6_K batches of >= 32 rows), 3 the dequantize-and-float-dot fallback
 * (types without an integer dot kernel), [2] 1 if activation quantization is fused
 * into the dot kernel, [3] weight rows per tile, [4] warps per row, [5]
 * pipeline stages, [6] CTAs, [7] dynamic shared memory bytes.  No
 * counterpart in the reference; used by tests and the benchmark. */
int cllm_cuda_matmul_plan(const void* w, int type, int in_dim, int out_dim, int n_rows, int* info,
                          int n_info);

/* Allocation-free matmul_quant, for callers that must not allocate device
 * memory during the call: code being recorded into a CUDA graph (an
 * allocation cannot be captured), engines whose own allocator already holds
 * the device's memory, and latency-bound loops that cannot afford the device
 * synchronisation that growing the regular entry point's workspace implies.
 * No counterpart in the reference.
 *
 * Same arithmetic and results as cllm_cuda_matmul_quant with device pointers
 * (x, w, bias, y all device memory; asynchronous on `stream`).  The quantized
 * activations go to one fixed scratch array compiled into the library
 * (CLLM_NOALLOC_SCRATCH_BYTES, held by every device that loads it until the
 * process exits), so the call is limited to n_rows <= CLLM_NOALLOC_MAX_ROWS
 * and in_dim <= CLLM_NOALLOC_MAX_IN_DIM; larger calls fail with
 * CLLM_ERR_TOO_LARGE before any device work.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) and caches it
 * per device index: make that first call before any stream capture.  The
 * cached address does not survive cudaDeviceReset (or anything else that
 * recreates the device's primary context): do not call this entry point on
 * that device afterwards.  All calls share the one
 * array and every call rewrites the part it reads, so nothing needs clearing
 * between calls, but calls that can overlap on the GPU (other streams,
 * other host threads) race on it: serialise them. */
#define CLLM_NOALLOC_MAX_ROWS 8
#define CLLM_NOALLOC_MAX_IN_DIM 32768
#define CLLM_NOALLOC_SCRATCH_BYTES 335872
int cllm_cuda_matmul_quant_noalloc(const float* x, const void* w, int type, const float* bias,
                                   int in_dim, int out_dim, int n_rows, float* y, void* stream);

/* ---- Row-sharded decode across the GPUs of one node ----
 * Replaces matmul_quant (quant.cpp:1374-1431) for a weight matrix split by
 * output rows over `world` GPUs (one process per GPU): rank r holds rows
 * [row_begin, row_begin + rows) of every matrix, as cllm_cuda_shard_rows
 * assigns them.  Row sharding never splits a block, and each row's sum is
 * computed exactly as on one GPU, so the gathered y is identical to the
 * unsharded call's. */

/* The rows of an out_dim-row matrix owned by `rank` of `world` (<= 8): as
 * even as possible, the first out_dim % world ranks one row more.  Host only. */
int cllm_cuda_shard_rows(int out_dim, int world, int rank, int* row_begin, int* rows);

/* y[t][j] for this rank's rows j, written into the y buffer of EVERY rank:
 * y_peers[q] (q < world) is rank q's [n_rows][out_dim] fp32 buffer as mapped
 * into this process (NVLink peer mapping, e.g. symmetric memory), so the
 * output is all-gathered by the GEMV's own stores.  x: [n_rows][in_dim] fp32
 * on this device (the full activation, the same on every rank); w_shard:
 * this rank's rows only (rows x row_bytes, native blocks, device memory);
 * bias: the full out_dim bias or NULL.  n_rows <= 8.
 *
 * Completion.  signal_pads (NULL: none) are every rank's signal pads
 * (CLLM_SHARD_PAD_WORDS zero-initialised uint32 each, peer-mapped) and epoch
 * this rank's zero-initialised epoch word: once the GEMV has finished, the
 * call announces "this rank's slice of round epoch+1 has landed" to every
 * rank (a one-warp kernel after the GEMV) and advances *epoch.  y is complete on a rank once every rank has
 * announced the round: cllm_cuda_shard_wait waits for that, and a following
 * row-sharded call given CLLM_SHARD_WAIT_PREV waits for it before it reads
 * its x (so chained projections need no separate wait).  Without signal
 * pads, use cllm_cuda_shard_barrier.  Every rank must make the same sequence
 * of signalling calls.  A rank whose slice is empty still signals. */
#define CLLM_SHARD_PAD_WORDS 16
#define CLLM_SHARD_WAIT_PREV 1u
/* The call does not announce its round (signal pads still needed for
 * CLLM_SHARD_WAIT_PREV).  For a call whose output the next call does not wait
 * on (q and k before v, gate before up, which read the same x): the round is
 * announced by the next signalling call, whose completion implies this one's.
 * Every rank must skip the same calls. */
#define CLLM_SHARD_NO_SIGNAL 2u
int cllm_cuda_matmul_quant_rowshard(const float* x, const void* w_shard, int type, const float* bias,
                                    int in_dim, int out_dim, int rank, int world, int n_rows,
                                    float* const* y_peers, uint32_t* const* signal_pads, uint32_t* epoch,
                                    unsigned flags, void* stream);

/* Wait (on the GPU, bounded: 1 s, then the device status reports
 * CLLM_ERR_KERNEL_TIMEOUT) until every rank has announced the round in
 * *epoch into own_pad (this rank's signal pad). */
int cllm_cuda_shard_wait(const uint32_t* own_pad, const uint32_t* epoch, int world, void* stream);

/* Completion barrier of a row-sharded call: tells every rank that this
 * rank's slice has landed (a release store of the new epoch into slot `rank`
 * of signal_pads[q], q < world) and waits until every rank has reached the
 * same epoch (slot q of signal_pads[rank]), for row-sharded calls made
 * without signal pads.  signal_pads: each rank's zero-initialised pad of
 * CLLM_SHARD_PAD_WORDS uint32, peer-mapped; epoch: this
 * rank's own zero-initialised device word, advanced by one per barrier on the
 * GPU (so a CUDA graph that replays the barrier stays in step).  Every rank
 * must run the same sequence of barriers.  The wait is bounded (1 s): a
 * missing rank ends it with the device status set
 * (cllm_cuda_check_device_status then reports CLLM_ERR_KERNEL_TIMEOUT).
 * Double-buffer y across consecutive calls: a rank may start writing call
 * n+1's slice while a slower rank still reads call n's y. */
int cllm_cuda_shard_barrier(uint32_t* const* signal_pads, uint32_t* epoch, int world, int rank, void* stream);

/* Peer-mapped buffers for the row-sharded calls without any framework: each
 * rank allocates its buffer here, publishes the CLLM_IPC_HANDLE_BYTES handle
 * to the other ranks over any host transport (MPI, a TCP store, a file), and
 * maps every peer's buffer with cllm_cuda_ipc_open (CUDA IPC: plain NVLink
 * peer mappings, no multicast objects).  A rank uses its own pointer for its
 * own slot (a process cannot open its own handle).  Close peer mappings
 * before the owners free their buffers. */
#define CLLM_IPC_HANDLE_BYTES 64
/* bytes of zeroed device memory on the current device, and its handle */
int cllm_cuda_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
/* map a peer's buffer into this process */
int cllm_cuda_ipc_open(const void* handle, void** dev_ptr);
int cllm_cuda_ipc_close(void* dev_ptr);
int cllm_cuda_ipc_free(void* dev_ptr);

/* ---- Device-resident engine step ----------------------
 * The reference's GgufLoader::load + TransformerEngine (gguf.cpp:120-275,
 * engine.cpp:349-610, Llama architecture) with every activation in HBM: the
 * GGUF data section is uploaded once in its native block layout, the
 * quantized matmuls run through cllm_cuda_matmul_quant's kernels, RMSNorm,
 * NEOX RoPE, GQA attention over an fp32 KV cache, SwiGLU, the residual adds
 * and the greedy argmax (sampler.cpp:32-34) are GPU kernels, and one decode
 * step is a CUDA graph that reads its token and position from device memory.
 * The engine owns a CUDA stream; calls on one engine must not overlap (the
 * reference engine is single-threaded too, http_server.cpp:715).  Models with
 * per-head q/k norms (Qwen3), head_dim other than 64/128 or a GQA ratio other
 * than 1/2/4/8 are rejected at creation. */

/* GgufLoader::load + TransformerEngine(model, pool, Quant, ctx_limit):
 * *engine receives an opaque handle.  ctx_limit > 0 caps the context as the
 * reference does (engine.cpp:352-356). */
int cllm_cuda_engine_create(const char* gguf_path, int ctx_limit, void** engine);
int cllm_cuda_engine_destroy(void* engine);

/* values[0..10]: n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab,
 * n_ctx, kernel launches of one decode step (graph nodes), seq_len, 1 if the
 * decode step runs fused (RMSNorm and SwiGLU inside the GEMVs' activation
 * quantization, one attention kernel per layer, q|k|v and gate|up as one GEMV
 * each where the file stores them back to back; needs every decode matrix on
 * the bulk-copy GEMV, i.e. 16-byte-multiple rows). */
int cllm_cuda_engine_config(const void* engine, int* values, int n);

/* TransformerEngine::forward(token) (engine.cpp:466-518): logits (host,
 * vocab floats, may be NULL) and the greedy next token (may be NULL).
 * "context length exceeded" (CLLM_ERR_TOO_LARGE) when the cache is full. */
int cllm_cuda_engine_forward(void* engine, int token, float* logits, int* next_token);

/* TransformerEngine::prefill(tokens) (engine.cpp:520-610), including its
 * reuse of the cached prefix: the last token's logits and greedy next token. */
int cllm_cuda_engine_prefill(void* engine, const int* tokens, int n, float* logits, int* next_token);

/* Greedy generation on the device: prefill(prompt), then steps - 1 decode
 * steps, each fed the previous step's argmax without a host round trip.
 * tokens_out[steps] receives the generated tokens (the first is the
 * prefill's argmax), margins_out[steps] (may be NULL) each token's logit
 * minus the runner-up's.  Equivalent to the reference's greedy loop of
 * prefill + forward(argmax) calls. */
int cllm_cuda_engine_generate(void* engine, const int* prompt, int n_prompt, int steps, int* tokens_out,
                              float* margins_out);

/* TransformerEngine::reset_kv_cache / seq_len (engine.hpp:46-48). */
int cllm_cuda_engine_reset(void* engine);
int cllm_cuda_engine_seq_len(const void* engine);

/* The engine's CUDA stream (for callers that time or order work around it). */
int cllm_cuda_engine_stream(const void* engine, void** stream);

/* ---- The engine step's operators as standalone calls ----------------------
 * Device pointers, asynchronous on `stream`; the reference computes these on
 * the host inside TransformerEngine.  Reductions (sums of squares, dot
 * products, softmax sums) are trees, not the reference's loops. */

/* rms_norm_ptr (engine.cpp:24-29) for `rows` rows of n:
 * y = x * (1 / sqrt(sum(x^2) / n + eps)) * w. */
int cllm_cuda_rms_norm(const float* x, const float* w, int n, int rows, float eps, float* y, void* stream);

/* SwiGLU (engine.cpp:41, :511): g[i] = g[i] / (1 + exp(-g[i])) * u[i]. */
int cllm_cuda_silu_mul(float* g, const float* u, int64_t n, void* stream);

/* Host: the NEOX RoPE table of apply_rope (engine.cpp:44-57) -- (cos, sin) of
 * pos / rope_theta^(i / (head_dim/2)) with the reference's float expressions,
 * table[(pos * head_dim/2 + i) * 2 + {0,1}] for pos < n_pos. */
int cllm_cuda_rope_table(float rope_theta, int head_dim, int n_pos, float* table);

/* apply_rope on q (n_head heads) and k (n_head_kv heads) of n_tok tokens at
 * positions pos0.. (engine.cpp:493-501), with the rotated k and v appended to
 * the caches [position][n_head_kv * head_dim]; table: the device copy of
 * cllm_cuda_rope_table's output covering those positions. */
int cllm_cuda_rope_kv(float* q, const float* k, const float* v, int n_tok, int n_head, int n_head_kv, int head_dim,
                      const float* table, int pos0, float* k_cache, float* v_cache, void* stream);

/* GQA attention (engine.cpp:119-146) of n_tok query tokens at positions
 * pos0.. (token t sees cache positions 0..pos0+t) over the fp32 caches:
 * out[t][n_head * head_dim].  head_dim 64 or 128; GQA ratio 1, 2, 4 or 8.
 * Partial results go to the library's workspace (see cllm_cuda_matmul_quant). */
int cllm_cuda_attention(const float* q, const float* k_cache, const float* v_cache, int n_tok, int pos0, int n_head,
                        int n_head_kv, int head_dim, float* out, void* stream);

/* Read and clear the device-side status word that kernels set when a bounded
 * wait expires (CLLM_ERR_KERNEL_TIMEOUT); synchronizes the device. */
int cllm_cuda_check_device_status(void);

/* Copy the calling thread's last error message into buf (NUL-terminated,
 * truncated to n); returns the length of the full message. */
int cllm_cuda_last_error(char* buf, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* CLLM_CUDA_H */
