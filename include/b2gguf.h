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
/* Opens (1) or closes (0) the profiler collection range (cudaProfilerStart /
 * cudaProfilerStop): a profiler started with collection off records only
 * the work issued inside the range. */
B2_API int b2_profiler_range(int start);

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

/* Several GEMVs over one input in one launch: y[i] = W[i]·x for n_mat
 * (1..64) matrices of one type and shape, 1-2 tokens; each y[i] (device,
 * [n_tok][n_rows]) is bit-identical to b2_gemv(W[i], x, ...).  The matrices
 * stream back to back through one pipeline, with no dependency wait between
 * them: the form for independent projections of one input, as the
 * reference's q/k/v matmuls on the same quantized row
 * (Singularity/src/core/cortex_a5_engine.cpp:1129-1131).  `w` and `y` are
 * host arrays of handles and device pointers. */
B2_API int b2_gemv_multi(const b2_qmatrix* const* w, int n_mat, const float* x, int n_tok, float* const* y,
                         void* stream);

/* Mixture-of-experts FFN pieces: the MoE layers of the GGUFs Milda and Sutra
 * load, whose blk.N.ffn_{gate,up,down}_exps tensors they place with tensor
 * buffer overrides (Milda/src/engine.cpp:860-885,
 * Sutra/src/llm_backends.cpp:1716-1747), computed as llama.cpp's MoE FFN
 * does (restated; equal probabilities choose the lower expert id).
 * b2_moe_route: per token, softmax of the router logits [n_tok][n_expert]
 * (e = expf(l − max), the sum in double, p = e·(float)(1/sum)), the n_used
 * largest p (expert ids [n_tok][n_used]) and their weights, divided by
 * their sum (double, rounded to float) when norm_weights != 0.
 * n_expert <= 256, n_used <= 64.
 * b2_moe_gemv: y[t][j] = W_{ids[t][j]}·x_{t,j} over a stack of n_expert
 * expert matrices uploaded as one b2_qmatrix of n_expert·rows rows (the GGUF
 * [k, rows, n_expert] tensor in its own byte order; rows a multiple of 8),
 * each output bit-identical to b2_gemv with that expert's matrix; the ids are
 * read on the device.  x_{t,j} = x[t] ([n_tok][k], gate and up) or, with
 * x_per_expert, x[t][j] ([n_tok][n_used][k], down).  y [n_tok][n_used][rows].
 * One launch per token (per token and expert for per-expert inputs of more
 * than 8192 values).  Ids outside [0, n_expert) are clamped.
 * b2_moe_combine: out[t][i] = Σ_j y[t][j][i]·weights[t][j], each product
 * rounded and added in choice order.  All on `stream`, no host sync. */
B2_API int b2_moe_route(const float* logits, int32_t n_tok, int32_t n_expert, int32_t n_used, int32_t norm_weights,
                        int32_t* ids, float* weights, void* stream);
B2_API int b2_moe_gemv(const b2_qmatrix* experts, int32_t n_expert, const float* x, int32_t x_per_expert,
                       int32_t n_tok, const int32_t* ids, int32_t n_used, float* y, void* stream);
B2_API int b2_moe_combine(const float* y, const float* weights, int32_t n_tok, int32_t n_used, int32_t n, float* out,
                          void* stream);

/* Device scratch b2_gemm needs for n_tok tokens (the quantized activations). */
B2_API int b2_gemm_workspace_bytes(const b2_qmatrix* w, int n_tok, size_t* bytes);

/* Prefill GEMM on the tensor cores (tcgen05, fp32 accumulation in TMEM),
 * the reference's matmul_quantized (Singularity/src/core/cortex_a5_engine.cpp:997-1027)
 * for any n_tok >= 1: y[t][r] = vec_dot(W row r, Q8_K(x[t])) for Q4_K
 * weights, vec_dot(W row r, Q8_0(x[t])) for Q8_0 weights, (super-)blocks
 * added in order exactly as the CPU vec_dot adds them, so y is bit-identical
 * to the reference's per-row result.  x fp32 [n_tok][k]
 * (16-byte aligned), y fp32 [n_tok][n_rows].  `workspace` (device, 16-byte
 * aligned, b2_gemm_workspace_bytes) may be NULL: the call then allocates
 * stream-ordered scratch.  `status` (device int, may be NULL) receives a
 * nonzero code if a pipeline wait expired. */
B2_API int b2_gemm(const b2_qmatrix* w, const float* x, int n_tok, float* y, void* workspace,
                   size_t workspace_bytes, int* status, void* stream);

/* Same GEMM through host buffers (pinned for full copy bandwidth): uploads x,
 * runs, reads y back, synchronous; fails if a pipeline wait expired. */
B2_API int b2_gemm_host(const b2_qmatrix* w, const float* x_host, int n_tok, float* y_host);

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



/* Token-embedding row dequantization (Singularity/src/core/cortex_a5_engine.cpp:1066-1105):
 * out[i][:] = dequant(table row tokens[i]) for a GGUF table of `type`
 * (F32, F16, Q4_0, Q8_0, Q4_K, Q6_K) with rows of n_embd values; ids outside
 * [0, n_vocab) read row 0.  tokens device int32 [n_tok], out fp32 [n_tok][n_embd]. */
B2_API int b2_embed(int type, const void* table, int n_vocab, int n_embd, const int32_t* tokens, int n_tok,
                    float* out, void* stream);

/* Residual add + RMSNorm, one row per token (ref_rmsnorm_f32,
 * Singularity/tests/test_and_bench_a5.cpp:247-258; the residual adds of
 * Singularity/src/core/cortex_a5_engine.cpp:1259-1261, 1281-1283):
 * x += delta (delta may be NULL), out = (x·1/sqrt(mean(x²)+eps))·w.
 * x, delta, out fp32 [n_rows][n], w fp32 [n]. */
B2_API int b2_rmsnorm(float* x, const float* delta, const float* w, float* out, int n_rows, int n, float eps,
                      void* stream);

/* RoPE (adjacent pairs, ref_rope_f32 test_and_bench_a5.cpp:280-293) on the
 * q and k heads of fused qkv rows, k and v stored to an fp16 cache
 * (cortex_a5_engine.cpp:1144-1203).  qkv fp32 [n_tok][(n_head+2·n_kv)·hd];
 * rope fp32 [cap][hd] (b2_rope_table); pos, seq device int32 [n_tok];
 * q_out fp32 [n_tok][n_head][hd]; k_cache / v_cache fp16
 * [n_seq][n_kv][cap][hd], token written at [seq][·][pos].  A token whose
 * sequence id is outside [0, n_seq) or position outside [0, cap) stores
 * nothing and gets a zero q row.  Stream-ordered, no host synchronization. */
B2_API int b2_rope_kv_store(const float* qkv, int n_tok, int n_seq, int n_head, int n_kv, int head_dim,
                            const int32_t* pos, const int32_t* seq, const float* rope, float* q_out,
                            uint16_t* k_cache, uint16_t* v_cache, int cap, void* stream);

/* Decode attention over the fp16 cache (cortex_a5_engine.cpp:1205-1254) in
 * the reference's order: query i attends to positions 0..pos[i] of sequence
 * seq[i] with its n_head/n_kv grouped heads; scores, softmax (expf as the
 * host C library computes it) and the weighted V sum are the reference's
 * sequential fp32 operations, so the output is bit-identical to its CPU
 * result.  q fp32 [n_q][n_head][hd], out fp32 [n_q][n_head][hd]; caches as
 * above ([n_seq][n_kv][cap][hd]).  A query whose sequence id is outside
 * [0, n_seq) or position outside [0, cap) reads nothing and gets a zero
 * row.  Scores go to stream-ordered scratch allocated by the call; no host
 * synchronization, so the call can be captured into a CUDA graph. */
B2_API int b2_attn_decode(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                          const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv, int head_dim, int cap,
                          float* out, void* stream);

/* KV caches of any of llama.cpp's cache types (B2_F16, B2_Q8_0, B2_Q4_0;
 * Milda/src/engine.cpp:74-87).  Rows of one kv head at one slot,
 * [n_seq][n_kv][cap] rows per cache, b2_kv_row_bytes(type, head_dim) bytes
 * each: B2_F16 head_dim fp16 values; B2_Q8_0 head_dim int8 codes, B2_Q4_0
 * head_dim/2 bytes of 4-bit codes (block b's 16 bytes at 16·b, byte j: value
 * j in the low nibble, value j+16 in the high one), each followed by the
 * head_dim/32 fp16 block scales and padded to a multiple of 16 bytes.
 * Storing quantizes each 32-value block as ref_quantize_row_q8_0
 * (Singularity/tests/test_and_bench_a5.cpp:223-245) or ggml's
 * quantize_row_q4_0_ref.  Attention over a Q8_0 or Q4_0 K quantizes each
 * query head to Q8_0 (the dot type of both) and scores position t as
 * ref_vec_dot_q8_0_q8_0 (:205-221) or ref_vec_dot_q4_0_q8_0 (:184-203) of the
 * K row and the query, times 1/sqrt(hd); over a quantized V it sums
 * p_t·(dequantized value) (exact in fp32); everything else as
 * b2_attn_decode.  The shift dequantizes, rotates and re-quantizes K.
 * head_dim a multiple of 32.  b2_kv_row_bytes returns 0 for other types. */
B2_API int64_t b2_kv_row_bytes(int type, int head_dim);
B2_API int b2_rope_kv_store_typed(const float* qkv, int n_tok, int n_seq, int n_head, int n_kv, int head_dim,
                                  const int32_t* pos, const int32_t* seq, const float* rope, float* q_out,
                                  void* k_cache, int type_k, void* v_cache, int type_v, int cap, void* stream);
B2_API int b2_attn_decode_typed(const float* q, const void* k_cache, int type_k, const void* v_cache, int type_v,
                                const int32_t* pos, const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv,
                                int head_dim, int cap, float* out, void* stream);
B2_API int b2_kv_shift_k_typed(void* k_cache, int type_k, int seq, int n_kv, int head_dim, int cap, int p_begin,
                               int p_end, int delta, float theta, void* stream);

/* b2_attn_decode for callers that cannot allocate device memory while they
 * run (a host that gives the library a fixed device-memory budget at
 * start-up, or a real-time decode loop that must not pay an allocation's
 * latency or risk its failure mid-turn).  No counterpart in the reference.
 * Same arguments and results as b2_attn_decode; the scratch (scores,
 * exponentials, chunk maxima) lives in one static device array of
 * B2_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit.  Limits: n_q <= B2_NOALLOC_MAX_QUERIES and the scratch,
 * n_q·n_kv·(capS·(G + max(G, 4)) + G·nchS)·4 bytes with G = n_head/n_kv,
 * capS = cap rounded up to 4 and nchS = ceil(cap/128) rounded up to 4
 * (about 2·n_q·n_head·cap·4 for G >= 4), within the array (larger requests
 * return B2_ERR_INVALID).  The first
 * call on a device looks up the array's address (call it once before any
 * stream capture); calls outside capture look it up again, so a device reset
 * between calls is picked up, while a call under capture uses the address
 * seen last.  Calls share the array: calls that overlap on the GPU race and
 * must be serialized by the caller. */
#define B2_NOALLOC_SCRATCH_BYTES (32 * 1024 * 1024)
#define B2_NOALLOC_MAX_QUERIES 64
B2_API int b2_attn_decode_noalloc(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* pos, const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv,
                                  int head_dim, int cap, float* out, void* stream);

/* The KV shift's re-rotation (Milda/src/engine.cpp:1642-1675): K rows of
 * positions [p_begin, p_end) of sequence seq rotated in place by `delta`
 * positions (fp16 -> fp32 -> rotate -> fp16 RNE).  head_dim <= 256;
 * stream-ordered, no host synchronization. */
B2_API int b2_kv_shift_k(uint16_t* k_cache, int seq, int n_kv, int head_dim, int cap, int p_begin, int p_end,
                         int delta, float theta, void* stream);

/* The tensor-parallel exchange's bounded device wait on its own.  No
 * llama.cpp counterpart.  One device thread waits until every flag of
 * flags[0..n) (device uint64) reaches `target`, for at most 2 s of wall
 * time; on expiry it stores B2_WAIT_EXPIRED in *status (device int) and
 * returns, so the stream stays usable and the caller reads the status
 * instead of finding a hung GPU.  The same wait guards every exchange of a
 * tensor-parallel decode step (a lost peer ends the step with
 * B2_ERR_TIMEOUT). */
#define B2_WAIT_EXPIRED 3
B2_API int b2_flag_wait(const uint64_t* flags, int n, uint64_t target, int* status, void* stream);

/* ------------------------------------------------------------------------ */
/* GGUF model files                                                           */
/* ------------------------------------------------------------------------ */

/* Shape and types of a synthetic Llama-architecture GGUF (random weights). */
typedef struct b2_llama_hparams {
    int32_t  n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab, n_ctx_train;
    float    rms_eps, rope_theta;
    int32_t  wtype;       /* attention / FFN weights: Q4_0, Q8_0, Q4_K, Q6_K */
    int32_t  embd_type;   /* token_embd.weight (also F32) */
    int32_t  out_type;    /* output.weight, or -1 for a head tied to token_embd */
    uint64_t seed;        /* weights N(0, w_std) from this seed */
    float    w_std;
} b2_llama_hparams;

/* Writes a GGUF v3 file with llama metadata and tensors named as the engines
 * bind them (Singularity/src/core/cortex_a5_engine.cpp:579-654), the weights
 * quantized with b2_quantize_weights and norm weights set to 1.  This plays
 * the part of the converter / quantizer that produces the engines' model
 * files. */
B2_API int b2_gguf_write_synthetic_llama(const b2_llama_hparams* hp, const char* path, int n_threads);

/* ------------------------------------------------------------------------ */
/* Engine (the llama.cpp calls Milda and Sutra make)                          */
/* ------------------------------------------------------------------------ */

typedef struct b2_model b2_model;
typedef struct b2_context b2_context;

#define B2_NCCL_ID_BYTES 128

typedef struct b2_model_params {
    int32_t     device;     /* CUDA device of this rank, -1 = current */
    int32_t     tp_rank;    /* tensor-parallel rank of this process */
    int32_t     tp_size;    /* tensor-parallel degree (1 = whole model here) */
    const void* nccl_id;    /* B2_NCCL_ID_BYTES from b2_nccl_unique_id (rank 0),
                               the same bytes on every rank; NULL when tp_size = 1 */
    int32_t     keep_page_cache; /* 0 (default): once the weights are on the device the
                               file's mapping is dropped and its pages are evicted from
                               the page cache, as Milda evicts the ranges of tensors it
                               offloaded (Milda/src/engine.cpp:1018-1041); 1: keep them */
} b2_model_params;

/* llama_model_default_params (Milda/src/engine.cpp:897). */
B2_API void b2_model_default_params(b2_model_params* p);
B2_API int  b2_nccl_unique_id(void* out);
/* llama_model_load_from_file (Milda/src/engine.cpp:919,
 * Sutra/src/llm_backends.cpp:1540): parses the GGUF, uploads this rank's
 * shard in the repacked layout.  All ranks of a TP group call it together. */
B2_API int  b2_model_load(const char* path, const b2_model_params* params, b2_model** out);
B2_API int  b2_model_free(b2_model* m);      /* llama_model_free */
/* out[0..11]: n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab, head_dim,
 * n_ctx_train, weight type, head type, tp_rank, tp_size
 * (llama_model_n_layer / llama_vocab_n_tokens, Milda/src/engine.cpp:1150-1157). */
B2_API int  b2_model_info(const b2_model* m, int32_t* out, int32_t n);
B2_API int  b2_model_device_bytes(const b2_model* m, int64_t* bytes);

typedef struct b2_context_params {
    int32_t n_ctx;        /* KV positions per sequence (llama n_ctx) */
    int32_t n_seq_max;    /* concurrent sequences (decode batch) */
    int32_t use_graph;    /* replay each decode step as a CUDA graph */
    int32_t prefill_gemm; /* long prompts through the tensor-core GEMMs (default 1): a b2_decode
                             call of n tokens that asks no logits of its first n - 8, with
                             n - 8 >= 64, runs those first tokens through the layers in chunks
                             whose projections are tensor-core GEMMs, when every layer's
                             projections are Q4_K or Q8_0.  Under tensor parallelism each
                             rank runs its shards' GEMMs and the ranks' attention-out and
                             FFN-down partials are all-gathered (NCCL) and summed in rank
                             order, as the decode step's exchange sums them.
                             Their projections then sum in the reference's row order (the
                             CPU matmul_quantized's) instead of the decode GEMV's tile order;
                             the last 8 tokens take the decode step. */
    int32_t type_k;       /* K cache type (llama_context_params.type_k, set from Milda's
                             cache_type_k at Milda/src/engine.cpp:1195): B2_F16 (default),
                             B2_Q8_0 or B2_Q4_0 */
    int32_t type_v;       /* V cache type (type_v, :1196): B2_F16 (default), B2_Q8_0 or
                             B2_Q4_0 */
} b2_context_params;

/* llama_context_default_params / llama_init_from_model
 * (Milda/src/engine.cpp:1180-1206): fp16 KV cache by default.  A Q8_0 cache
 * (Milda's default cache_type_k / cache_type_v, Milda/include/milda/engine.hpp:85-86)
 * stores each row's 32-value blocks with the reference's Q8_0 quantizer and
 * attends as llama.cpp does over such a cache: the query quantized to Q8_0
 * and scored with the Q8_0·Q8_0 block dot, V rows dequantized (d·q), the
 * softmax and sums as for fp16 (see b2_attn_decode_typed). */
B2_API void b2_context_default_params(b2_context_params* p);
B2_API int  b2_context_create(b2_model* m, const b2_context_params* params, b2_context** out);
B2_API int  b2_context_free(b2_context* c);   /* llama_free */
/* The context's CUDA stream (for event timing by callers). */
B2_API int  b2_context_stream(b2_context* c, void** stream);

/* llama_decode over a llama_batch (Milda/src/engine.cpp:1539-1541, 2077-2081;
 * Sutra/src/llm_backends.cpp:2544, 2714): token i at position pos[i] of
 * sequence seq[i] (pos/seq NULL = next position of sequence 0).  Each token
 * must extend its sequence at its next position.  want_logits: 0 none,
 * 1 every token, 2 the last token of the call.  Returns 1 when a sequence is
 * full (no KV slot), 2 when the abort callback asked to stop.  The steps run
 * asynchronously on the context stream: a device-side failure of a step (an
 * expired tensor-parallel exchange wait: B2_ERR_TIMEOUT) is returned by the
 * next call that synchronizes (b2_get_logits, b2_get_argmax,
 * b2_synchronize_context, b2_sampler_sample). */
B2_API int b2_decode(b2_context* c, const int32_t* tokens, const int32_t* pos, const int32_t* seq,
                     int32_t n_tokens, int32_t want_logits);
/* llama_get_logits_ith (Milda/src/engine.cpp:2019, Sutra/src/llm_backends.cpp:3335):
 * fp32 logits of row i of the last decode step that computed logits. */
B2_API int b2_get_logits(b2_context* c, int32_t i, float* out, int64_t n);
/* Greedy pick on the device for every logits row of that step: token id,
 * top-1 logit and top-1 − top-2 margin (NULL outputs are skipped). */
B2_API int b2_get_argmax(b2_context* c, int32_t* ids, float* top1, float* margin, int32_t n);
/* Logits rows of that step (the rows b2_get_argmax fills; 0 when the last
 * decode computed no logits).  A call's tokens run in steps of up to 8, and a
 * long prompt's first tokens may run through the prefill GEMMs, so the last
 * step holds the call's last 1-8 tokens. */
B2_API int b2_get_last_rows(b2_context* c, int32_t* n);
/* Greedy generation with the loop on the device.  No llama.cpp counterpart:
 * it is the device-resident form of Milda's greedy turn loop, llama_decode of
 * one token → llama_get_logits_ith → pick → feed (Milda/src/engine.cpp:1962-2117),
 * for rows on greedy sampling.  Runs n_steps steps over the n (<= 8) distinct
 * sequences seq[0..n) (NULL: 0..n-1), each continuing at its next position.
 * Step 0 feeds first[i]; step t feeds row i the argmax of step t-1; the argmax
 * of step t lands in out[t*n + i].  Steps are graph replays with no host
 * synchronization between them; the logits of the last step stay readable
 * through b2_get_logits / b2_get_argmax.  Returns 1 (no KV slot) without
 * running when a sequence would pass n_ctx, 2 when the abort callback (polled
 * before each step) stopped it, with the finished steps kept. */
B2_API int b2_generate(b2_context* c, const int32_t* first, const int32_t* seq, int32_t n, int32_t n_steps,
                       int32_t* out);
B2_API int b2_synchronize_context(b2_context* c);
/* Tensor parallelism: the wall time this rank's decode steps have spent in
 * the exchange waits (each waiting kernel's first CTA adds its wait), since
 * the context was created or last reset (reset != 0 zeroes it after the
 * read).  0 without tensor parallelism.  Synchronizes the context stream. */
B2_API int b2_context_exchange_wait_ns(b2_context* c, uint64_t* ns, int32_t reset);

/* ------------------------------------------------------------------------ */
/* Sampler chain on the device                                               */
/* ------------------------------------------------------------------------ */

/* The chain Milda's rebuild_sampler builds (Milda/src/engine.cpp:1321-1384)
 * from llama.cpp's samplers, with its state (penalty window, mt19937) in
 * device memory:
 *   penalties (llama_sampler_init_penalties; when penalty_last_n > 0 and a
 *   penalty is set) over the last penalty_last_n accepted tokens: a logit
 *   l <= 0 becomes l·repeat, else l/repeat; then l − (count·freq +
 *   (count > 0)·present);
 *   temperature <= 0: greedy (the first largest logit);
 *   else top_k (k largest, in descending order; equal logits by lower id),
 *   top_p (softmax with the C library's expf, the shortest prefix whose
 *   running probability reaches p; off for p <= 0 or >= 1), min_p (logits >=
 *   the largest + logf(p); off for p <= 0), temperature (l/t) and dist
 *   (softmax, then std::discrete_distribution over the probabilities in
 *   candidate order with a std::mt19937 seeded by `seed`, as the GNU C++
 *   library draws it: u = (r1 + r2·2^32)/2^64, the first normalized running
 *   sum, in double, not below u).
 * Sampling accepts the sampled token (as llama_sampler_sample does);
 * b2_sampler_accept adds one more (Milda accepts again, :2029).
 * Device limits: penalty_last_n <= 256; with temperature > 0, 1 <= top_k <=
 * 256; vocabularies up to 131072 entries (B2_ERR_UNSUPPORTED otherwise). */
typedef struct b2_sampler b2_sampler;
typedef struct b2_sampler_params {
    int32_t  penalty_last_n;   /* 0: no penalties */
    float    penalty_repeat;   /* 1: off */
    float    penalty_freq;     /* 0: off */
    float    penalty_present;  /* 0: off */
    int32_t  top_k;
    float    top_p;
    float    min_p;
    float    temperature;      /* <= 0: greedy */
    uint32_t seed;             /* llama_sampler_init_dist */
} b2_sampler_params;
/* Milda's defaults (Milda/include/milda/engine.hpp:79-84, window 64):
 * penalty 1.08 over 64 tokens, top_k 40, top_p 0.90, min_p 0.05,
 * temperature 0.75, seed 42. */
B2_API void b2_sampler_default_params(b2_sampler_params* p);
/* llama_sampler_chain_init + _add (rebuild_sampler): a chain whose state
 * lives on the context's GPU and whose calls run on the context's stream.
 * Free a context's samplers before the context. */
B2_API int  b2_sampler_create(b2_context* c, const b2_sampler_params* p, b2_sampler** out);
B2_API int  b2_sampler_free(b2_sampler* s);                   /* llama_sampler_free   */
/* llama_sampler_reset (Milda/src/engine.cpp:1693, 1710, 1839): empty window,
 * generator re-seeded. */
B2_API int  b2_sampler_reset(b2_sampler* s);
/* llama_sampler_accept; token in [0, 131072). */
B2_API int  b2_sampler_accept(b2_sampler* s, int32_t token);
/* llama_sampler_sample(s, ctx, idx) (Milda/src/engine.cpp:1970): samples
 * logits row idx (negative: from the end) of the context's last decode on
 * the device and accepts the token; only the token comes back to the host. */
B2_API int  b2_sampler_sample(b2_sampler* s, int32_t idx, int32_t* token);
/* The same draw over a device array of n_vocab fp32 logits (any vocabulary
 * up to 131072), on the sampler's context stream. */
B2_API int  b2_sampler_sample_logits(b2_sampler* s, const float* logits, int32_t n_vocab, int32_t* token);
/* b2_generate with row i drawn by samplers[i] (distinct samplers of this
 * context) instead of the greedy argmax: the device-resident form of Milda's
 * sampled turn loop, no logits leave the device.  Row i's step-t token lands
 * in out[t*n + i]. */
B2_API int  b2_generate_sampled(b2_context* c, b2_sampler* const* samplers, const int32_t* first,
                                const int32_t* seq, int32_t n, int32_t n_steps, int32_t* out);

/* KV cache: llama_memory_clear / seq_rm / seq_add / seq_pos_max
 * (Milda/src/engine.cpp:1650-1658, 1686, 2125-2148).  seq_rm of a suffix
 * truncates; seq_rm of [p0,p1) followed by seq_add(p1, -1, -(p1-p0)) is
 * Milda's in-place shift: K rows are re-rotated by the position delta. */
B2_API int b2_kv_clear(b2_context* c);
B2_API int b2_kv_seq_rm(b2_context* c, int32_t seq, int32_t p0, int32_t p1);
B2_API int b2_kv_seq_add(b2_context* c, int32_t seq, int32_t p0, int32_t p1, int32_t delta);
B2_API int b2_kv_seq_pos_max(b2_context* c, int32_t seq, int32_t* pos);

/* llama_n_ctx (Milda/src/engine.cpp:1236): KV positions per sequence. */
B2_API int b2_n_ctx(const b2_context* c, int32_t* n_ctx);
/* llama_memory_can_shift (Milda/src/engine.cpp:1655, 2126): 1 — the cache
 * re-rotates K in place for the seq_rm + seq_add shift. */
B2_API int b2_memory_can_shift(const b2_context* c, int32_t* can_shift);

/* Sequence-state snapshot and restore: llama_state_seq_get_size /
 * get_data / set_data (Milda/src/engine.cpp:1487-1492 pins the system
 * prompt's state, :1701-1705 restores it; Sutra/src/llm_backends.cpp:2572-2580
 * caches a prefix).  The snapshot holds the sequence's positions
 * [0, pos_max] — this rank's KV heads, K and V rows per layer in position
 * order, in the cache types' storage — behind a 64-byte header naming the
 * model shape, the cache types and the rank.
 * get_size: bytes the snapshot of `seq` takes now.  get_data: writes it to
 * dst (size >= get_size) and sets *written.  set_data: replaces sequence
 * `seq` (any id of this context) with the snapshot; *read = bytes consumed.
 * A snapshot of another shape, cache type or rank is refused with
 * B2_ERR_FORMAT, one
 * longer than n_ctx with B2_NO_KV_SLOT.  Synchronous. */
B2_API int b2_state_seq_get_size(b2_context* c, int32_t seq, size_t* size);
B2_API int b2_state_seq_get_data(b2_context* c, int32_t seq, void* dst, size_t size, size_t* written);
B2_API int b2_state_seq_set_data(b2_context* c, int32_t seq, const void* src, size_t size, size_t* read);

/* Intermediate-tensor callback, the analogue of llama.cpp's cb_eval context
 * parameter: when set, decode steps run without graph replay and after each
 * op the callback receives the op name, layer (-1 outside layers), a device
 * pointer and the number of fp32 values written (rows of the step's tokens).
 * The stream is synchronized before the call.  NULL removes it. */
typedef void (*b2_eval_callback)(const char* name, int32_t layer, const float* data, int64_t n, void* user);
B2_API int b2_set_eval_callback(b2_context* c, b2_eval_callback cb, void* user);

/* llama_set_abort_callback (Sutra/src/llm_backends.cpp:3017): polled between
 * decode steps; non-zero stops the call with status 2. */
typedef int (*b2_abort_callback)(void* user);
B2_API int b2_set_abort_callback(b2_context* c, b2_abort_callback cb, void* user);

#ifdef __cplusplus
}
#endif
#endif /* B2GGUF_H */
