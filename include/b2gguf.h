/*
 * b2gguf — B200 (sm_100a) quantized-inference path for GGUF LLM engines.
 *
 * C ABI: plain pointers and sizes, no C++ or framework types.  Every entry
 * point returns an int status (B2_OK = 0; 1 = no KV slot; 2 = aborted; < 0 =
 * hard error, message in b2_last_error()), mirroring the llama.cpp return
 * conventions the engines already handle (Sutra/src/llm_backends.cpp:2551,
 * :2719; Milda/src/engine.cpp:920-934).  All functions are noexcept.
 *
 * Reference interfaces each group replaces are cited per declaration (paths
 * relative to the reference project root).  Device pointers are CUDA device
 * addresses on the current device; `stream` is a cudaStream_t (NULL = the
 * legacy default stream).
 */
#ifndef B2GGUF_H
#define B2GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_ABI_VERSION 1

#if defined(__GNUC__)
#define B2_API __attribute__((visibility("default")))
#else
#define B2_API
#endif

enum b2_status {
    B2_OK = 0,
    B2_NO_KV_SLOT = 1,       /* llama_decode rc 1 */
    B2_ABORTED = 2,          /* llama_decode rc 2 (abort callback) */
    B2_ERR_INVALID = -1,
    B2_ERR_CUDA = -2,
    B2_ERR_OOM = -3,
    B2_ERR_FORMAT = -4,      /* malformed / unsupported GGUF */
    B2_ERR_TIMEOUT = -5,     /* a bounded device wait gave up */
    B2_ERR_UNSUPPORTED = -6,
    B2_ERR_NCCL = -7,
    B2_ERR_IO = -8,
};

/* ggml type ids (Singularity/src/core/cortex_a5_engine.hpp:31-36,
 * Sutra/src/llm_backends.cpp:3396-3401). */
enum b2_type {
    B2_F32 = 0,
    B2_F16 = 1,
    B2_Q4_0 = 2,
    B2_Q8_0 = 8,
    B2_Q4_K = 12,
    B2_Q6_K = 14,
    B2_Q8_K = 15,
};

/* ------------------------------------------------------------------------ */
/* Library / device utilities                                                */
/* ------------------------------------------------------------------------ */

B2_API int         b2_abi_version(void);
/* Thread-local text of the last failing call on this thread. */
B2_API const char* b2_last_error(void);
B2_API int b2_device_count(int* n);
B2_API int b2_set_device(int device);
B2_API int b2_get_device(int* device);
B2_API int b2_malloc(void** dptr, size_t bytes);
B2_API int b2_free(void* dptr);
B2_API int b2_host_alloc(void** hptr, size_t bytes);     /* pinned host memory */
B2_API int b2_host_free(void* hptr);
B2_API int b2_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
B2_API int b2_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
B2_API int b2_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
B2_API int b2_memset(void* dst, int value, size_t bytes, void* stream);
B2_API int b2_stream_create(void** stream);
B2_API int b2_stream_destroy(void* stream);
B2_API int b2_stream_synchronize(void* stream);
B2_API int b2_device_synchronize(void);
B2_API int b2_event_create(void** event);
B2_API int b2_event_destroy(void* event);
B2_API int b2_event_record(void* event, void* stream);
B2_API int b2_event_elapsed_ms(void* start, void* stop, float* ms);
/* CUDA-graph capture of work issued on a (non-default) stream: everything
 * this library launches between begin and end is recorded once and replayed
 * by b2_graph_launch with one host call, as the engines' decode loop does. */
B2_API int b2_graph_capture_begin(void* stream);
B2_API int b2_graph_capture_end(void* stream, void** graph_exec);
B2_API int b2_graph_launch(void* graph_exec, void* stream);
B2_API int b2_graph_destroy(void* graph_exec);
/* Enables (1) or disables (0) programmatic dependent launch between this
 * library's kernels on the calling thread (default 1). */
B2_API int b2_set_pdl(int enabled);

/* ------------------------------------------------------------------------ */
/* Host-side format helpers (CPU only; no device needed)                     */
/* ------------------------------------------------------------------------ */

/* Bytes of one GGUF row of k values of `type` (k a multiple of the block). */
B2_API size_t b2_row_bytes(int type, int64_t k);

/* GGUF weight quantizer (the producer side of a GGUF file):
 *   Q4_0: ggml quantize_row_q4_0_ref (d = signed absmax / −8,
 *         nibble = min(15, trunc(x/d + 8.5)));
 *   Q8_0: ggml quantize_row_q8_0_ref (d = absmax/127, q = round(x/d));
 *   Q4_K / Q6_K: a valid min-max encoding of the public block layouts.
 * src fp32 [n_rows][k] -> dst GGUF bytes [n_rows][b2_row_bytes(type,k)].
 * Rows are split over n_threads host threads. */
B2_API int b2_quantize_weights(int type, const float* src, int64_t n_rows, int64_t k, void* dst, int n_threads);

/* Seeded N(mean, std) fp32 values: element i of the stream (seed) is a pure
 * function of (seed, offset+i); any slice can be generated independently. */
B2_API int b2_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float std_dev, float* out,
                    int n_threads);

/* RoPE cos/sin table, out[p*head_dim + 2i] = cos((p0+p)·θ^(−2i/head_dim)),
 * [+1] = sin(...), angles and cos/sin in double, rounded once to fp32. */
B2_API int b2_rope_table(float theta, int head_dim, int p0, int n_pos, float* out);

/* ------------------------------------------------------------------------ */
/* GGUF tensor upload — repacked device layout                               */
/* Replaces the tensor upload inside llama_model_load_from_file              */
/* (Milda/src/engine.cpp:919; Sutra/src/llm_backends.cpp:1540).              */
/* ------------------------------------------------------------------------ */

typedef struct b2_qmatrix b2_qmatrix;

/* Uploads a [n_rows x k] GGUF tensor (Q4_0, Q8_0, Q4_K, Q6_K) to the current
 * device, repacked for 16-byte aligned bulk copies; bytes stay bit-identical. */
B2_API int b2_qmatrix_upload(int type, const void* gguf_bytes, int64_t n_rows, int64_t k, b2_qmatrix** out);
B2_API int b2_qmatrix_free(b2_qmatrix* m);
/* Device bytes held by the repacked matrix. */
B2_API int b2_qmatrix_device_bytes(const b2_qmatrix* m, int64_t* bytes);
/* Dequantized weights, fp32 [n_rows][k] on the device (parity checks). */
B2_API int b2_qmatrix_dequantize(const b2_qmatrix* m, float* dst, void* stream);

/* ------------------------------------------------------------------------ */
/* Single ops (device pointers, asynchronous on `stream`)                    */
/* ------------------------------------------------------------------------ */

/* Activation quantization to GGUF-format blocks (Q8_0 or Q8_K), one row per
 * token: the reference's ref_quantize_row_q8_0
 * (Singularity/tests/test_and_bench_a5.cpp:223-245) and ggml's
 * quantize_row_q8_K.  x fp32 [n_tok][k] -> blocks [n_tok][b2_row_bytes]. */
B2_API int b2_quantize_act(int act_type, const float* x, int n_tok, int64_t k, void* blocks, void* stream);

/* Decode GEMV / skinny GEMM, the reference's matmul_quantized
 * (Singularity/src/core/cortex_a5_engine.cpp:997-1027) for n_tok in [1, 8]:
 * y[t][r] = Σ_blocks vec_dot(W row r, Q8(x[t])) with the activation
 * quantized exactly as the reference's CPU path does (Q8_0 for Q4_0/Q8_0,
 * Q8_K for Q4_K/Q6_K).  x fp32 [n_tok][k], y fp32 [n_tok][n_rows]. */
B2_API int b2_gemv(const b2_qmatrix* w, const float* x, int n_tok, float* y, void* stream);

/* Same GEMV through host buffers: uploads x, runs, reads y back, synchronous.
 * The call a host engine makes per projection when it keeps activations on
 * the host. */
B2_API int b2_gemv_host(const b2_qmatrix* w, const float* x_host, int n_tok, float* y_host);

/* Exact integer block sums of one weight row against one quantized token
 * (the int32 `sumi` of ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 per 32-block,
 * test_and_bench_a5.cpp:184-221; for Q4_K the per-super-block Σ sc_j·dot_j
 * and Σ m_j·bsum_j, for Q6_K Σ sc_g·dot_g).  x fp32 [k]; out_i, out_m
 * device int32 [blocks] (out_m only for Q4_K, may be NULL otherwise). */
B2_API int b2_block_dots(const b2_qmatrix* w, int64_t row, const float* x, int32_t* out_i, int32_t* out_m, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2GGUF_H */
