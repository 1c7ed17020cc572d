/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the quantized
 * decode path.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm may load it, and only as the checker or the
 * timed CPU baseline.  The product library never links or calls it.
 *
 * Sources restated (paths relative to the reference project root):
 *   Singularity/tests/test_and_bench_a5.cpp:150-293   scalar reference ops
 *   Singularity/src/core/cortex_a5_engine.cpp:429-659  GGUF parse
 *   Singularity/src/core/cortex_a5_engine.cpp:997-1293 matmul + forward order
 *   Milda/src/engine.cpp:1642-1675                     KV shift semantics
 *   ggml (llama.cpp, version unpinned, not vendored)   Q8_K quantize, K-quant
 *                                                      block layouts and dots
 *
 * Parity pins: the op-level functions are checked bit-for-bit against the
 * reference's own scalar refs compiled from its sources (oracle/_ref), and the
 * block layouts against gguf-py 0.19.0 (tests/golden).  The K-quant dot
 * products and Q8_K activation quantizer have no in-tree reference; they
 * restate ggml's published algorithm.
 *
 * Build with -ffp-contract=off: every fp32 multiply and add rounds on its own,
 * as in the reference's scalar refs.
 */
#ifndef B2_ORACLE_H
#define B2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (Singularity/src/core/cortex_a5_engine.hpp:31-36,
 * Sutra/src/llm_backends.cpp:3396-3401). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_Q8_K = 15 };

/* Block sizes in bytes. */
enum { ORC_Q4_0_BYTES = 18, ORC_Q8_0_BYTES = 34, ORC_Q4_K_BYTES = 144, ORC_Q6_K_BYTES = 210, ORC_Q8_K_BYTES = 292 };

float    orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);
void     orc_fp32_to_fp16_row(const float* x, uint16_t* y, int64_t n);
void     orc_fp16_to_fp32_row(const uint16_t* x, float* y, int64_t n);

/* Activation quantizers. */
void orc_quantize_row_q8_0(const float* x, void* y, int k);   /* Singularity formula */
void orc_quantize_row_q8_k(const float* x, void* y, int k);   /* ggml formula        */

/* Block dot products: weights x (left) · activation y (right). */
float orc_vec_dot_q4_0_q8_0(int n, const void* x, const void* y);
float orc_vec_dot_q8_0_q8_0(int n, const void* x, const void* y);
float orc_vec_dot_q4_k_q8_k(int n, const void* x, const void* y);
float orc_vec_dot_q6_k_q8_k(int n, const void* x, const void* y);
/* Exact integer block sums (one int32 per 32-weight block for Q4_0/Q8_0; per
 * 256-weight super-block the scaled sum Σ sc_j·dot_j for Q4_K/Q6_K, and the
 * min term Σ m_j·bsum_j for Q4_K in mins[]). */
void orc_block_dots_q4_0_q8_0(int n, const void* x, const void* y, int32_t* sumi);
void orc_block_dots_q8_0_q8_0(int n, const void* x, const void* y, int32_t* sumi);
void orc_block_dots_q4_k_q8_k(int n, const void* x, const void* y, int32_t* isum, int32_t* msum);
void orc_block_dots_q6_k_q8_k(int n, const void* x, const void* y, int32_t* isum);

/* Weight dequantizers (one row of k weights). */
void orc_dequantize_row(int type, const void* x, float* y, int k);

/* Elementwise ops. */
void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps);       /* Singularity ref */
void orc_rmsnorm_ggml(const float* x, const float* w, float* out, int n, float eps);  /* ggml (double sum) */
void orc_softmax(const float* x, float* out, int n);
void orc_rope_pairs(float* x, const float* cos_sin, int head_dim, int n_heads);
void orc_silu_mul(float* hb, const float* hb2, int n);

/* RoPE cos/sin table: out[p*hd + 2i] = cos(p·θ^(−2i/hd)), [+1] = sin(...),
 * p in [p0, p0+n_pos).  Angles in double, cos/sin in double, rounded once. */
void orc_rope_table(float theta, int head_dim, int p0, int n_pos, float* out);

/* Row-parallel quantized matmul: y[r] = dot(W row r, xq), rows split over
 * n_threads POSIX threads.  xq is Q8_0 for Q4_0/Q8_0 weights and Q8_K for
 * Q4_K/Q6_K weights.  row_bytes is the GGUF row size. */
void orc_matmul(int wtype, const void* w, int64_t n_rows, int k, const void* xq, float* y, int n_threads);
void orc_matmul_strided(int wtype, const void* w, int64_t n_rows, size_t row_stride, int k, const void* xq, float* y,
                        int n_threads);

/* Activation type the reference's CPU dot pairs with each weight type. */
int orc_vec_dot_type(int wtype);
size_t orc_row_bytes(int type, int k);

/* Decode attention over an fp16 cache for one token.
 * q: [n_heads*hd] fp32; kc/vc: fp16, element (t, kvh, i) at t*kv_stride + kvh*hd + i;
 * positions t in [0, n_pos).  out: [n_heads*hd] fp32. */
void orc_attn_decode(const float* q, const uint16_t* kc, const uint16_t* vc, int64_t kv_stride,
                     int n_pos, int n_heads, int n_kv_heads, int hd, float* out);

/* In-place K re-rotation for a KV shift by delta positions on n_pos cached
 * rows (fp16 → fp32 → rotate by cos/sin(delta·θ_i) → RNE fp16). */
void orc_kv_shift_k(uint16_t* kc, int64_t kv_stride, int n_pos, int n_kv_heads, int hd,
                    int delta, float theta);

/* Quantized KV cache (llama.cpp cache types; Milda's default is Q8_0 K and
 * V).  Rows hold hd values of one kv head in the type's storage: fp16, or
 * ggml Q8_0 or Q4_0 blocks.  A row is stored with the type's quantizer
 * (orc_quantize_row_q8_0, orc_quantize_row_q4_0).  Attention: with a Q8_0
 * or Q4_0 K the query head is quantized to Q8_0 (both types' dot type) and
 * scored with orc_vec_dot_q8_0_q8_0 / orc_vec_dot_q4_0_q8_0 (times 1/√hd);
 * V rows are dequantized before the weighted sum; softmax and summation
 * order as orc_attn_decode.  Row (t, kvh) at base + t*stride + kvh*row
 * bytes; strides in bytes.  The shift dequantizes, rotates as
 * orc_kv_shift_k and stores back with the type's quantizer. */
void orc_quantize_row_q4_0(const float* x, void* y, int k);   /* ggml formula */
void orc_kv_store_row(int type, const float* x, void* row, int n);
void orc_kv_store_rows(int type, const float* x, void* rows, int64_t n_rows, int n);
void orc_attn_decode_typed(const float* q, const void* kc, int ktype, size_t k_stride, const void* vc,
                           int vtype, size_t v_stride, int n_pos, int n_heads, int n_kv_heads, int hd,
                           float* out);
void orc_kv_shift_k_typed(void* kc, int ktype, size_t k_stride, int n_pos, int n_kv_heads, int hd, int delta,
                          float theta);

/* ---- Sampler chain (oracle_sampler.c) ---- */
typedef struct orc_sampler orc_sampler;
/* Milda's chain (rebuild_sampler): penalties, then greedy (temp <= 0) or
 * top_k (<= 0: all), top_p, min_p, temp, dist(seed). */
orc_sampler* orc_sampler_new(int last_n, float rep, float freq, float pres, int top_k, float top_p, float min_p,
                             float temp, uint32_t seed);
void    orc_sampler_free(orc_sampler* s);
void    orc_sampler_reset(orc_sampler* s);
void    orc_sampler_accept(orc_sampler* s, int32_t tok);
/* llama_sampler_sample over one logits row; accepts the token. */
int32_t orc_sampler_sample(orc_sampler* s, const float* logits, int n_vocab);
/* std::mt19937(seed)'s first n outputs. */
void    orc_mt19937(uint32_t seed, uint32_t* out, int n);
/* std::discrete_distribution<int>(p, p + n) drawn once with the sampler's
 * generator (GNU C++ library arithmetic). */
int     orc_discrete_draw(orc_sampler* s, const float* p, int n);

/* ---- Mixture of experts (oracle_moe.c) ---- */
/* One token: softmax of the router logits, the n_used largest probabilities
 * (ids, weights; norm: divided by their sum). */
void orc_moe_route(const float* logits, int n_expert, int n_used, int norm, int32_t* ids, float* weights);
/* out[i] = Σ_j y[j][i]·w[j] in order (y [n_used][n]). */
void orc_moe_combine(const float* y, const float* w, int n_used, int n, float* out);

/* ---- Device-order arithmetic (the GPU kernels' evaluation order) ---- */
float orc_expf_dev(float x);
void  orc_silu_mul_dev(float* hb, const float* hb2, int n);
/* Tile GEMV order (both tile kernels, any batch): units split into
 * orc_tile_splits() ranges of ceil(nu/S) units, four interleaved partial sums per
 * range combined pairwise, ranges added in order. */
int   orc_tile_splits(int wtype, int k);
float orc_tile_row_dot(int wtype, const void* wrow, int k, const void* xq);
void  orc_matmul_dev(int wtype, const void* w, int64_t n_rows, int k, const void* xq, float* y, int swiglu,
                     int n_threads);
/* As orc_matmul_dev over k columns of rows `row_stride` bytes apart (a column
 * slice of a wider matrix: the tensor-parallel shard of one rank). */
void  orc_matmul_dev_strided(int wtype, const void* w, int64_t n_rows, size_t row_stride, int k, const void* xq,
                             float* y, int swiglu, int n_threads);
void  orc_attn_decode_dev(const float* q, const uint16_t* kc, const uint16_t* vc, int64_t kv_stride, int n_pos,
                          int n_heads, int n_kv_heads, int hd, float* out);

/* ---- GGUF + Llama forward (Singularity forward_token order) ---- */
typedef struct orc_model orc_model;
orc_model* orc_model_open(const char* path);   /* mmap a GGUF file */
orc_model* orc_model_from_memory(const void* data, size_t size);
void       orc_model_free(orc_model* m);
int        orc_model_info(const orc_model* m, int32_t* out, int n_out);
/* Per-sequence KV cache of n_ctx positions (fp16 unless set otherwise). */
int  orc_model_init_cache(orc_model* m, int n_seq, int n_ctx);
/* K and V cache types (ORC_F16 or ORC_Q8_0); re-creates an existing cache
 * empty.  Returns -1 for other types. */
int  orc_model_set_kv_types(orc_model* m, int ktype, int vtype);
/* Sets every cached K and V value to the fp16 `bits` (touches the pages, so
 * timed attention reads real memory rather than never-written zero pages). */
void orc_model_cache_fill(orc_model* m, uint16_t bits);
/* Runs token `token` at position `pos` of sequence `seq`; writes logits
 * (n_vocab) when logits != NULL.  Returns 0 on success. */
int  orc_model_forward(orc_model* m, int seq, int32_t token, int pos, float* logits, int n_threads);
/* As forward, but stops after n_layers_run layers (for bounded CPU timing). */
int  orc_model_forward_layers(orc_model* m, int seq, int32_t token, int pos, float* logits,
                              int n_threads, int n_layers_run);
/* Layers [l0, l1) only, continuing from the residual the previous call left
 * (the embedding is taken when l0 == 0; logits when logits != NULL).  Timing
 * samples of single layers of a large model use it. */
int  orc_model_forward_range(orc_model* m, int seq, int32_t token, int pos, int l0, int l1, float* logits,
                             int n_threads);
/* KV shift on one sequence: drop [p0, p1), re-rotate K of [p1, n_past). */
int  orc_model_kv_shift(orc_model* m, int seq, int p0, int p1, int n_past);
/* 1: evaluate in the GPU kernels' order (orc_*_dev), 0: the reference's;
 * 2: the GPU kernels' order except the projections, which take the
 * reference's row order (orc_matmul), as the tensor-core prefill GEMMs do. */
void orc_model_set_device_order(orc_model* m, int on);
/* Emulates tp tensor-parallel ranks in device order: attention-out and
 * FFN-down become per-rank column-slice partials summed in rank order (every
 * other projection is row-sharded and needs no change).  Returns -1 when the
 * shapes do not split (heads, kv heads, FFN, vocab, 256-column shards). */
int  orc_model_set_tp(orc_model* m, int tp);
/* Per-op tap with the same names as the engine's evaluation callback. */
typedef void (*orc_tap_fn)(const char* name, int layer, const float* data, long n, void* user);
void orc_model_set_tap(orc_model* m, orc_tap_fn fn, void* user);
/* Copy of the hidden state after the last forward (n_embd floats). */
int  orc_model_hidden(const orc_model* m, float* out, int n);

#ifdef __cplusplus
}
#endif
#endif
