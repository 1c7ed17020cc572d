// Launchers for the decoder-layer kernels (b2_layers.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_internal.hpp"

namespace b2 {

int launch_embed(const int32_t* tokens, int n_tok, int n_vocab, int type, const uint8_t* table, int64_t row_bytes,
                 int n_embd, float* x, cudaStream_t s);
int launch_add_rmsnorm(float* x, const float* delta, const float* w, float* out, int n_tok, int n, float eps,
                       cudaStream_t s, const PeerIn* in = nullptr, int* status = nullptr);
// Residual add + RMSNorm fused with the next GEMV's activation quantization:
// writes the normalized rows to `out` (may be null) and their quantized image
// to `img` (n % 32 == 0, n / 8 <= 1024; n % 256 == 0 for the K-quant images).
// Returns B2_ERR_UNSUPPORTED for other shapes (callers then use the unfused
// pair).
int launch_add_rmsnorm_q(float* x, const float* delta, const float* w, float* out, int n_tok, int n, float eps,
                         const ActImage& img, cudaStream_t s, const PeerIn* in = nullptr, int* status = nullptr);
bool add_rmsnorm_q_supported(int n, int act_type);
// KV cache rows: one kv head's hd values at one slot, [n_seq][n_kv][cap]
// rows per cache.  F16: hd fp16 values.  Q8_0: hd int8 codes, then the hd/32
// fp16 block scales, padded to a multiple of 16 bytes (so every row, and
// every run of rows, starts 16-byte aligned for bulk and tensor copies).
// Q4_0: hd/2 bytes of 4-bit codes (block b at 16·b: byte j holds element j
// in its low nibble and element j+16 in its high one), then the block
// scales, padded the same way.
__host__ __device__ constexpr int64_t kv_code_bytes(int type, int hd) {
  return type == B2_Q8_0 ? hd : type == B2_Q4_0 ? hd / 2 : 2 * hd;
}
__host__ __device__ constexpr int64_t kv_row_bytes(int type, int hd) {
  return type == B2_F16 ? 2 * hd : kv_code_bytes(type, hd) + 16;
}
inline bool kv_type_ok(int type) { return type == B2_F16 || type == B2_Q8_0 || type == B2_Q4_0; }
int launch_rope_kv(const float* qkv, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                   const float* rope, float* q_out, void* kc, int kt, void* vc, int vt, const KvSeqState* st, int n_seq,
                   int cap, cudaStream_t s);
// Decode attention in the reference's order (b2_attn.cu): q fp32
// [n_tok][n_head][hd] against the caches (rows as above, types kt / vt), out
// fp32 [n_tok][n_head][hd].  `scratch` holds attn_scratch_floats floats
// (16-byte aligned) of scores, exponentials and chunk maxima; it needs no
// initialisation.  Queries whose sequence id is outside [0, n_seq) or whose
// position is outside [0, cap) read nothing and produce zero outputs.  st
// may be null (plain layout).
size_t attn_scratch_floats(int n_tok, int n_head, int n_kv, int cap);
int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const void* kc, int kt, const void* vc, int vt, const KvSeqState* st, int n_seq, int cap,
                     float* scratch, float* out, cudaStream_t s, int* status = nullptr);
// h [n_tok][ff] = silu(gate) * up over the (gate, up) row pairs of gu
// [n_tok][2 ff], with the arithmetic of the GEMV's SwiGLU epilogue.
int launch_swiglu_pairs(const float* gu, int n_tok, int ff, float* h, cudaStream_t s);
// cos/sin pairs of one position delta for every rotated pair (head_dim <= 256).
constexpr int kRotPairs = 128;
struct RotTable {
  float cs[2 * kRotPairs];
};
int launch_kv_shift(void* kc, int kt, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int p_begin, int p_end,
                    const RotTable& cs, cudaStream_t s);
int launch_kv_compact(void* kc, int kt, void* vc, int vt, int n_kv, int hd, int seq, const KvSeqState& st, int cap,
                      int dst0, int src0, int n, const RotTable& cs, cudaStream_t s);
// out = the n_parts partials [n_parts][n] summed in part order.
int launch_rank_sum(const float* parts, int n_parts, int64_t n, float* out, cudaStream_t s);
// Mixture-of-experts routing and combination (b2_moe.cu).
int launch_moe_route(const float* logits, int n_tok, int n_expert, int n_used, int norm, int32_t* ids, float* weights,
                     cudaStream_t s);
int launch_moe_combine(const float* y, const float* w, int n_tok, int n_used, int n, float* out, cudaStream_t s);
// Device-side greedy loop: argmax ids become the next step's tokens.
struct GreedyFeed {
  int32_t* tok = nullptr;    // [n_tok] next step's tokens (null: no feed)
  int32_t* pos = nullptr;    // [n_tok] positions, advanced by one
  int32_t* out = nullptr;    // [cap][n_tok] generated ids
  int32_t* count = nullptr;  // [n_tok] ids appended so far
  int cap = 0;
};
// Greedy top-1 (lowest index on ties) and top-1 − top-2 margin per token.
// `scratch` (argmax_scratch_words() words, zero before the first launch and
// left zero by every launch) lets each token's scan spread over many CTAs.
constexpr int kArgmaxParts = 64, kArgmaxTok = 8;
constexpr size_t argmax_scratch_words() { return (size_t)kArgmaxTok * kArgmaxParts * 3 + kArgmaxTok; }
int launch_argmax(const float* logits, int n_tok, int n_vocab, int v_local, int32_t* ids, float* top, cudaStream_t s,
                  const GreedyFeed& feed = GreedyFeed{}, const PeerIn* in = nullptr, int* status = nullptr,
                  uint32_t* scratch = nullptr);

}  // namespace b2
