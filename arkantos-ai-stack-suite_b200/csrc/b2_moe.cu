// Mixture-of-experts FFN pieces.  Milda and Sutra load MoE GGUFs whose
// expert tensors blk.N.ffn_{gate,up,down}_exps they place with tensor buffer
// overrides (Milda/src/engine.cpp:860-885, Sutra/src/llm_backends.cpp:1716-1747);
// llama.cpp (not in the reference tree, version not pinned) computes the
// layer as ggml's MoE FFN, restated here from its published source (the
// scalar path of each op):
//   router logits [n_expert] -> soft_max (max; e = expf(l − max) with the sum
//   kept in double; p = e·(float)(1/sum)) -> top_k (the n_used largest p;
//   equal p by lower expert id, which ggml's sort leaves open) -> weights =
//   the chosen p, optionally divided by their sum (summed in double, rounded
//   to float) -> per chosen expert j: gate_j, up_j (expert GEMVs),
//   silu(gate)·up, down_j -> out = Σ_j down_j·w_j, the products rounded and
//   added in the order of the choice.
// The expert GEMVs are this library's decode GEMV over a stack of expert
// matrices, grouped: the token's n_used experts are the launch's matrices,
// their ids read on the device (launch_gemv with mat_ids), so a routed layer
// runs without a host round trip and can be captured into a graph.
#include <float.h>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kMoeMaxExperts = 256;
constexpr int kMoeMaxUsed = 64;

__device__ __forceinline__ unsigned long long prob_key(float p, int e) {
  uint32_t u = __float_as_uint(p);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)e);
}

// One CTA per token: softmax of the router logits, the n_used largest
// probabilities (bitonic sort of (p, id) keys) and their weights.
__global__ void __launch_bounds__(256) moe_route_kernel(const float* __restrict__ logits, int n_expert, int n_used,
                                                        int norm, int32_t* __restrict__ ids,
                                                        float* __restrict__ weights) {
  __shared__ float e[kMoeMaxExperts];
  __shared__ unsigned long long key[kMoeMaxExperts];
  __shared__ unsigned long long tab[32];
  __shared__ float red[8];
  __shared__ float s_scale;
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  exp_table_to_smem(tab, tid, blockDim.x);
  const float* l = logits + (int64_t)b * n_expert;
  float mx = -FLT_MAX;
  for (int i = tid; i < n_expert; i += blockDim.x) mx = fmaxf(mx, l[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  for (int i = tid; i < n_expert; i += blockDim.x) e[i] = b2_expf_ref(__fsub_rn(l[i], mx), tab);
  __syncthreads();
  if (tid == 0) {
    double sum = 0.0;
    for (int i = 0; i < n_expert; ++i) sum = __dadd_rn(sum, (double)e[i]);
    s_scale = __double2float_rn(__ddiv_rn(1.0, sum));
  }
  __syncthreads();
  int n2 = 1;
  while (n2 < n_expert) n2 <<= 1;
  for (int i = tid; i < n2; i += blockDim.x) key[i] = i < n_expert ? prob_key(__fmul_rn(e[i], s_scale), i) : 0ull;
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = key[i], y = key[ixj];
          if (((i & k) == 0) ? (x < y) : (x > y)) {
            key[i] = y;
            key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  if (tid != 0) return;
  float wsel[kMoeMaxUsed];
  double sum = 0.0;
  for (int j = 0; j < n_used; ++j) {
    const int ex = (int)(0xFFFFFFFFu - (uint32_t)key[j]);
    ids[(int64_t)b * n_used + j] = ex;
    wsel[j] = __fmul_rn(e[ex], s_scale);
    sum = __dadd_rn(sum, (double)wsel[j]);
  }
  const float s = __double2float_rn(sum);
  for (int j = 0; j < n_used; ++j) weights[(int64_t)b * n_used + j] = norm ? __fdiv_rn(wsel[j], s) : wsel[j];
}

// out[t][i] = Σ_j y[t][j][i]·w[t][j]: each product rounded, added in order.
__global__ void moe_combine_kernel(const float* __restrict__ y, const float* __restrict__ w, int n_used, int n,
                                   float* __restrict__ out) {
  pdl_wait();
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* yt = y + (int64_t)t * n_used * n;
  const float* wt = w + (int64_t)t * n_used;
  float acc = __fmul_rn(yt[i], wt[0]);
  for (int j = 1; j < n_used; ++j) acc = __fadd_rn(acc, __fmul_rn(yt[(int64_t)j * n + i], wt[j]));
  out[(int64_t)t * n + i] = acc;
}

}  // namespace

int launch_moe_route(const float* logits, int n_tok, int n_expert, int n_used, int norm, int32_t* ids, float* weights,
                     cudaStream_t s) {
  B2_CHECK_ARG(logits && ids && weights && n_tok > 0, "moe_route arguments");
  B2_CHECK_ARG(n_expert >= 1 && n_expert <= kMoeMaxExperts && n_used >= 1 && n_used <= n_expert &&
                   n_used <= kMoeMaxUsed,
               "moe_route: 1 <= n_used <= n_expert <= 256, n_used <= 64");
  return launch_pdl(moe_route_kernel, dim3(n_tok), dim3(256), 0, s, logits, n_expert, n_used, norm, ids, weights);
}

int launch_moe_combine(const float* y, const float* w, int n_tok, int n_used, int n, float* out, cudaStream_t s) {
  B2_CHECK_ARG(y && w && out && n_tok > 0 && n_used >= 1 && n > 0, "moe_combine arguments");
  return launch_pdl(moe_combine_kernel, dim3((n + 255) / 256, n_tok), dim3(256), 0, s, y, w, n_used, n, out);
}

}  // namespace b2
