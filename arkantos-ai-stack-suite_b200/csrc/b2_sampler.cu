// On-device sampler chain.  Milda builds its chain in rebuild_sampler
// (Milda/src/engine.cpp:1321-1384) from llama.cpp's samplers and draws a
// token per step with llama_sampler_sample (:1970), then accepts it again
// (:2029).  llama.cpp is not part of the reference tree; its samplers are
// restated from their published source (the version Milda builds against is
// not pinned):
//   penalties(last_n, repeat, freq, present): for every token in the window
//     of the last_n accepted tokens, logit·repeat if logit <= 0 else
//     logit/repeat, then logit − (count·freq + (count > 0)·present);
//   greedy: the first largest logit;
//   top_k(k): the k largest logits, sorted in descending order;
//   top_p(p, 1): softmax over the candidates (max, e = expf(l − max) summed
//     in order, p = e/sum), keep the shortest prefix whose running sum of p
//     reaches p;
//   min_p(p, 1): keep the prefix with logit >= logit_0 + logf(p);
//   temp(t): logit/t;
//   dist(seed): softmax again, then std::discrete_distribution over the p in
//     candidate order driven by a std::mt19937 seeded with `seed`, as the
//     GNU C++ library computes it: the p summed in double, divided by the
//     sum, running sums in double with the last set to 1, and the first
//     running sum not below u = (r1 + r2·2^32)/2^64 (generate_canonical of
//     two 32-bit outputs); one candidate: index 0.
// Equal logits sort by lower token id (llama.cpp's sort leaves their order
// open).  expf is the host C library's (b2_expf_ref); logf(min_p) is taken
// on the host.
//
// Two kernels per sampling step:
//   * sample_slices_kernel: CTA (slice, row) copies its slice of up to
//     kSampSlice logits into shared memory, applies the penalties of the
//     window tokens that fall into it, sorts (logit, id) keys with a bitonic
//     network and writes its best min(k, slice) keys;
//   * sample_chain_kernel: one CTA per row merges the slices' sorted keys
//     into the top k (one warp), runs the rest of the chain on one warp
//     (elementwise steps on the lanes, every sum in order on lane 0; k <= 256
//     values), accepts the token and feeds the next step.
#include <float.h>

#include "b2_common.cuh"
#include "b2_sampler.hpp"

namespace b2 {
namespace {

// (logit, id) as one 64-bit key whose unsigned order is: larger logit first,
// then lower id.
__device__ __forceinline__ unsigned long long make_key(float x, int id) {
  uint32_t u = __float_as_uint(x);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)id);
}
__device__ __forceinline__ float key_logit(unsigned long long k) {
  uint32_t u = (uint32_t)(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}
__device__ __forceinline__ int key_id(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

// Descending bitonic sort of n (a power of two) keys in shared memory.
__device__ void bitonic_desc(unsigned long long* a, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = a[i], y = a[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
}

__device__ __forceinline__ int k_eff(const SamplerDev& p) { return p.temp <= 0.0f ? 1 : p.top_k; }

// Logit of vocabulary entry v of row b in the argmax's gather layout.
__device__ __forceinline__ const float* logit_ptr(const float* logits, int n_tok, int v_local, int b, int v) {
  const int r = v / v_local;
  return logits + ((int64_t)r * n_tok + b) * v_local + (v - r * v_local);
}

__global__ void __launch_bounds__(256) sample_slices_kernel(const float* __restrict__ logits, int n_tok, int row0,
                                                            int n_vocab, int v_local, SamplerDev* const* sps,
                                                            unsigned long long* __restrict__ keys) {
  __shared__ unsigned long long sk[kSampSlice];
  __shared__ float sl[kSampSlice];
  pdl_wait();
  const int pi = blockIdx.x, np = gridDim.x, i = blockIdx.y, b = row0 + i;
  const SamplerDev* sp = sps[i];
  const int per = (n_vocab + np - 1) / np;
  const int va = pi * per, len = max(0, min(n_vocab, va + per) - va);
  for (int t = threadIdx.x; t < len; t += blockDim.x) sl[t] = __ldcg(logit_ptr(logits, n_tok, v_local, b, va + t));
  __syncthreads();
  // penalties of the window tokens in this slice, once per distinct token
  const int rl = sp->ring_len, last_n = sp->last_n;
  const bool pen = last_n != 0 && !(sp->rep == 1.0f && sp->freq == 0.0f && sp->pres == 0.0f);
  if (pen) {
    for (int e = threadIdx.x; e < rl; e += blockDim.x) {
      const int tok = sp->ring[(sp->ring_head + e) % last_n];
      if (tok < va || tok >= va + len) continue;
      bool first = true;
      int count = 0;
      for (int f = 0; f < rl; ++f) {
        const int o = sp->ring[(sp->ring_head + f) % last_n];
        if (o == tok) {
          if (f < e) first = false;
          ++count;
        }
      }
      if (!first) continue;
      float x = sl[tok - va];
      x = x <= 0.0f ? __fmul_rn(x, sp->rep) : __fdiv_rn(x, sp->rep);
      x = __fsub_rn(x, __fadd_rn(__fmul_rn((float)count, sp->freq), __fmul_rn(count > 0 ? 1.0f : 0.0f, sp->pres)));
      sl[tok - va] = x;
    }
  }
  __syncthreads();
  const int kk = k_eff(*sp);
  unsigned long long* dst = keys + ((int64_t)i * kSampParts + pi) * kSampTopKMax;
  if (kk == 1) {
    // greedy: the slice's largest key (a maximum: any order)
    unsigned long long best = 0ull;
    for (int t = threadIdx.x; t < len; t += blockDim.x) {
      const unsigned long long k = make_key(sl[t], va + t);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = sk[w] > best ? sk[w] : best;
      dst[0] = best;
    }
    pdl_launch_dependents();
    return;
  }
  int n2 = 1;
  while (n2 < len) n2 <<= 1;
  for (int t = threadIdx.x; t < n2; t += blockDim.x) sk[t] = t < len ? make_key(sl[t], va + t) : 0ull;
  __syncthreads();
  bitonic_desc(sk, n2);
  for (int t = threadIdx.x; t < kk; t += blockDim.x) dst[t] = t < len ? sk[t] : 0ull;
  pdl_launch_dependents();
}

// ---- mt19937 (Matsumoto & Nishimura 1998, the C++ standard's std::mt19937) ----
__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9D2C5680u;
  y ^= (y << 15) & 0xEFC60000u;
  y ^= y >> 18;
  return y;
}
// The generator's twist (all 624 words renewed in index order), by the whole
// CTA on a shared-memory copy: word k reads words k, k+1 and k+397 (mod 624)
// as they are when its turn comes, so the index ranges [0,227), [227,454),
// [454,623) and {623} each read only words their own range has not written,
// and run as four parallel rounds.
__device__ void mt_twist_cta(uint32_t* mt) {
  const int bounds[5] = {0, 227, 454, 623, 624};
  for (int ph = 0; ph < 4; ++ph) {
    const int k = bounds[ph] + threadIdx.x;
    uint32_t v = 0;
    const bool mine = k < bounds[ph + 1];
    if (mine) {
      const uint32_t y = (mt[k] & 0x80000000u) | (mt[(k + 1) % kMtN] & 0x7FFFFFFFu);
      v = mt[(k + 397) % kMtN] ^ (y >> 1) ^ ((y & 1u) ? 0x9908B0DFu : 0u);
    }
    __syncthreads();
    if (mine) mt[k] = v;
    __syncthreads();
  }
}

__device__ void ring_push(SamplerDev* s, int32_t tok) {
  const int n = s->last_n;
  if (n <= 0) return;
  if (s->ring_len < n) {
    s->ring[(s->ring_head + s->ring_len) % n] = tok;
    ++s->ring_len;
  } else {
    s->ring[s->ring_head] = tok;
    s->ring_head = (s->ring_head + 1) % n;
  }
}

// softmax_impl over l[0..n) (sorted, largest first) by one warp: p =
// expf(l − l_0) on the lanes, their sum in order on lane 0, then each p
// divided by the sum on the lanes.
__device__ void softmax_sorted_warp(const float* l, float* p, int n, const unsigned long long* tab, int lane) {
  const float mx = l[0];
  for (int i = lane; i < n; i += 32) p[i] = b2_expf_ref(__fsub_rn(l[i], mx), tab);
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0)
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, p[i]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int i = lane; i < n; i += 32) p[i] = __fdiv_rn(p[i], sum);
  __syncwarp();
}

__global__ void __launch_bounds__(256) sample_chain_kernel(int n_tok, int row0, int n_vocab, int np,
                                                           SamplerDev* const* sps,
                                                           const unsigned long long* __restrict__ keys,
                                                           int32_t* __restrict__ ids, GreedyFeed feed) {
  extern __shared__ unsigned long long mk[];   // [np][kk]: each slice's best keys, largest first
  __shared__ float cl[kSampTopKMax], cp[kSampTopKMax];
  __shared__ int ci[kSampTopKMax];
  __shared__ unsigned long long tab[32];
  __shared__ double cum[kSampTopKMax];
  pdl_wait();
  const int i = blockIdx.x, b = row0 + i;
  SamplerDev* sp = sps[i];
  exp_table_to_smem(tab, threadIdx.x, blockDim.x);
  const int kk = k_eff(*sp);
  const int per = (n_vocab + np - 1) / np;
  for (int t = threadIdx.x; t < np * kk; t += blockDim.x) {
    const int part = t / kk, j = t - part * kk;
    const int len = max(0, min(n_vocab, part * per + per) - part * per);
    mk[t] = j < len ? __ldcg(keys + ((int64_t)i * kSampParts + part) * kSampTopKMax + j) : 0ull;
  }
  __syncthreads();
  // The K largest keys by merging the slices' sorted lists: warp 0's lane l
  // watches the heads of slices l and l + 32; each round the largest head
  // (keys are distinct: they carry the token id) is taken and its list
  // advances.  The same K keys, in the same order, as sorting them all.
  const int K = min(kk, n_vocab);
  if ((threadIdx.x >> 5) == 0) {
    const int lane = threadIdx.x & 31, pa = lane, pb = lane + 32;
    int ha = 0, hb = 0;
    for (int j = 0; j < K; ++j) {
      const unsigned long long a = (pa < np && ha < kk) ? mk[pa * kk + ha] : 0ull;
      const unsigned long long c = (pb < np && hb < kk) ? mk[pb * kk + hb] : 0ull;
      unsigned long long best = a > c ? a : c;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (best != 0ull) {
        if (best == a) ++ha;
        else if (best == c) ++hb;
      }
      if (lane == 0) {
        cl[j] = key_logit(best);
        ci[j] = key_id(best);
      }
    }
  }
  __syncthreads();
  // warp 0 runs the chain up to the draw (its elementwise expf, divisions
  // and comparisons over the candidates spread on the lanes, every sum on
  // lane 0 in candidate order); the CTA then takes the two generator words
  // the draw needs (twisting the state when it runs out)
  __shared__ int s_size;
  __shared__ uint32_t s_r[2];
  __shared__ uint32_t smt[kMtN];
  if ((threadIdx.x >> 5) == 0) {
    const int lane = threadIdx.x & 31;
    int size = 0;
    if (sp->temp > 0.0f) {
      size = K;
      if (sp->top_p > 0.0f && sp->top_p < 1.0f) {
        softmax_sorted_warp(cl, cp, size, tab, lane);
        // the shortest prefix whose running sum reaches top_p (lane 0)
        int last = size;
        if (lane == 0) {
          float run = 0.0f;
          for (int t = 0; t < size; ++t) {
            run = __fadd_rn(run, cp[t]);
            if (run >= sp->top_p && t + 1 >= 1) {
              last = t + 1;
              break;
            }
          }
        }
        size = __shfl_sync(0xffffffffu, last, 0);
      }
      if (sp->min_p > 0.0f) {
        // the first candidate below the largest + logf(min_p) (candidates
        // sorted: a ballot per group of 32)
        const float min_logit = __fadd_rn(cl[0], sp->logf_min_p);
        int cut = size;
        for (int t0 = 1; t0 < size; t0 += 32) {
          const int t = t0 + lane;
          const unsigned below = __ballot_sync(0xffffffffu, t < size && cl[t] < min_logit);
          if (below) {
            cut = t0 + __ffs(below) - 1;
            break;
          }
        }
        size = cut;
      }
      for (int t = lane; t < size; t += 32) cl[t] = __fdiv_rn(cl[t], sp->temp);
      __syncwarp();
      softmax_sorted_warp(cl, cp, size, tab, lane);
    }
    if (lane == 0) s_size = size;
  }
  __syncthreads();
  if (s_size >= 2) {
    const int mti = sp->mti;
    if (mti >= kMtN - 1) {
      for (int t = threadIdx.x; t < kMtN; t += blockDim.x) smt[t] = sp->mt[t];
      __syncthreads();
      if (threadIdx.x == 0 && mti == kMtN - 1) s_r[0] = mt_temper(smt[kMtN - 1]);
      mt_twist_cta(smt);
      for (int t = threadIdx.x; t < kMtN; t += blockDim.x) sp->mt[t] = smt[t];
      if (threadIdx.x == 0) {
        if (mti == kMtN - 1) {
          s_r[1] = mt_temper(smt[0]);
          sp->mti = 1;
        } else {
          s_r[0] = mt_temper(smt[0]);
          s_r[1] = mt_temper(smt[1]);
          sp->mti = 2;
        }
      }
    } else if (threadIdx.x == 0) {
      s_r[0] = mt_temper(sp->mt[mti]);
      s_r[1] = mt_temper(sp->mt[mti + 1]);
      sp->mti = mti + 2;
    }
    __syncthreads();
  }
  if ((threadIdx.x >> 5) != 0) return;
  const int lane = threadIdx.x & 31;
  const int size = s_size;
  int pick = 0;
  if (size >= 2) {
    // the GNU C++ library's discrete_distribution: the weights summed in
    // double (lane 0, in order), each divided by the sum (lanes), running
    // sums with the last set to 1 (lane 0), the first not below u
    __shared__ double s_sum;
    if (lane == 0) {
      double sum = 0.0;
      for (int t = 0; t < size; ++t) sum = __dadd_rn(sum, (double)cp[t]);
      s_sum = sum;
    }
    __syncwarp();
    const double sum = s_sum;
    for (int t = lane; t < size; t += 32) cum[t] = __ddiv_rn((double)cp[t], sum);
    __syncwarp();
    if (lane == 0) {
      double run = 0.0;
      for (int t = 0; t < size; ++t) {
        run = __dadd_rn(run, cum[t]);
        cum[t] = run;
      }
      cum[size - 1] = 1.0;
      double u =
          __ddiv_rn(__dadd_rn((double)s_r[0], __dmul_rn((double)s_r[1], 4294967296.0)), 18446744073709551616.0);
      if (u >= 1.0) u = 1.0 - 1.1102230246251565e-16;   // nextafter(1, 0)
      // the first running sum not below u among the first size-1
      int lo = 0, hi = size - 1;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cum[mid] < u) lo = mid + 1;
        else hi = mid;
      }
      pick = lo;
    }
  }
  if (lane != 0) return;
  const int32_t tok = ci[pick];
  ring_push(sp, tok);   // llama_sampler_sample accepts the token it returns
  ids[b] = tok;
  if (feed.tok) {
    feed.tok[b] = tok;
    feed.pos[b] += 1;
    const int t = feed.count[b];
    if (t < feed.cap) feed.out[(int64_t)t * n_tok + b] = tok;
    feed.count[b] = t + 1;
  }
}

__global__ void sampler_accept_kernel(SamplerDev* sp, int32_t token) { ring_push(sp, token); }

}  // namespace

void sampler_init_state(SamplerDev* h) {
  h->ring_len = 0;
  h->ring_head = 0;
  h->mt[0] = h->seed;
  for (int k = 1; k < kMtN; ++k) h->mt[k] = 1812433253u * (h->mt[k - 1] ^ (h->mt[k - 1] >> 30)) + (uint32_t)k;
  h->mti = kMtN;
}

int launch_sample(const float* logits, int n_tok, int row0, int n, int n_vocab, int v_local, SamplerDev* const* sps,
                  int32_t* ids, const GreedyFeed& feed, unsigned long long* keys, cudaStream_t s) {
  B2_CHECK_ARG(n >= 1 && n <= 8 && row0 >= 0 && row0 + n <= n_tok && n_vocab > 0, "sample: rows");
  if (n_vocab > kSampParts * kSampSlice) {
    set_error("sampler: vocabularies of up to %d entries are sampled on the device (%d given)",
              kSampParts * kSampSlice, n_vocab);
    return B2_ERR_UNSUPPORTED;
  }
  const int np = std::max(1, std::min(kSampParts, (n_vocab + kSampSlice - 1) / kSampSlice));
  int rc = launch_pdl(sample_slices_kernel, dim3(np, n), dim3(256), 0, s, logits, n_tok, row0, n_vocab, v_local, sps,
                      keys);
  if (rc) return rc;
  const size_t smem = (size_t)np * kSampTopKMax * 8;
  static bool attr_set = false;   // per process: the attribute is per function, not per device
  if (!attr_set) {
    B2_CUDA_TRY(cudaFuncSetAttribute(sample_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)((size_t)kSampParts * kSampTopKMax * 8)));
    attr_set = true;
  }
  return launch_pdl(sample_chain_kernel, dim3(n), dim3(256), smem, s, n_tok, row0, n_vocab, np, sps,
                    (const unsigned long long*)keys, ids, feed);
}

int launch_sampler_accept(SamplerDev* sp, int32_t token, cudaStream_t s) {
  sampler_accept_kernel<<<1, 1, 0, s>>>(sp, token);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

}  // namespace b2
