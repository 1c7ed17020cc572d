// Decode attention over the fp16 KV cache in the reference's order
// (Singularity/src/core/cortex_a5_engine.cpp:1205-1254, with the softmax of
// ref_softmax_f32, Singularity/tests/test_and_bench_a5.cpp:260-278): for
// query head h of token b at position p (kv head h / G),
//   s_t = (Σ_i q_i·k_ti, dims in order) · (1/sqrt(hd))      t = 0..p
//   m = max_t s_t;  e_t = expf(s_t − m);  l = Σ_t e_t (positions in order)
//   p_t = e_t · (1/l);  out_i = Σ_t p_t·v_ti (positions in order)
// every multiply and add a separately rounded fp32 operation, expf the host
// library's (b2_expf_ref), so every output is bit-identical to the
// reference's CPU result.  The sums are sequential chains; the work is laid
// out so that as many chains as possible run side by side.
//
// Two kernels:
//   * attn_scores_kernel: one CTA per (128-position chunk, kv head, query).
//     The chunk's K rows arrive by 1-D bulk copies (one per row, into rows
//     padded by 16 bytes so the per-thread row reads do not collide on
//     banks) while q goes to shared memory;
//     thread t scores position t against the G query heads of the group
//     (G chains over the dims, two heads per packed f32x2 multiply and add)
//     and writes s_t to the score buffer.  The last CTA of each (query, kv
//     head) to finish then runs the softmax of those G heads over all
//     positions: the maximum, e_t (three warps compute a chunk of e while
//     lanes 0..G-1 of warp 0 add the previous chunk into the sums, double
//     buffered), 1/l, and p_t written back over the scores.
//   * attn_pv_kernel: one CTA per (slice of 64/G dims, kv head, query).  A
//     loader warp stages p_t (as pairs) and the V slice (converted to fp32)
//     for chunks of up to 128 positions into three buffers; the chain warp's lane
//     (head, dim pair) runs out += p_t·v_t over the positions in order with
//     packed f32x2 multiplies and adds.  Launched with programmatic dependent
//     launch, it prefetches its V rows into L2 while the scores finish.
// Queries whose sequence id or position is outside the cache attend to
// nothing and get zero outputs.  Every wait is bounded.
#include <float.h>

#include "b2_common.cuh"
#include "b2_layers.hpp"

namespace b2 {
namespace {

constexpr int kScoreP = 128;     // positions per scores CTA (one per thread)
constexpr int kSoftCh = 512;     // positions per softmax chunk

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// acc + a·b on two lanes, the product and the sum each rounded (as a
// separate fp32 multiply then add): p = fma(a, b, −0) is a·b rounded once
// (sign of zero kept), then fma(p, 1, acc) is acc + p rounded once.  A
// packed multiply followed by a packed add can be merged by the code
// generator into one fused rounding; two fmas cannot.  `k` holds (1, 1) and
// (−0, −0) from kernel arguments, so no constant folding turns the fmas back
// into a mergeable multiply and add.
struct Ones {
  uint64_t one, neg_zero;
};
__device__ __forceinline__ uint64_t mul_add2(uint64_t acc, uint64_t a, uint64_t b, const Ones& k) {
  uint64_t p, r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(a), "l"(b), "l"(k.neg_zero));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(p), "l"(k.one), "l"(acc));
  return r;
}

__device__ __forceinline__ int query_positions(const int32_t* pos, const int32_t* seq, int b, int n_seq, int cap,
                                               int* s_out) {
  const int s = seq[b], p = pos[b];
  *s_out = s;
  return (s >= 0 && s < n_seq && p >= 0 && p < cap) ? p + 1 : 0;
}

// Named barriers of the softmax's double buffer: full[buf] = 1 + buf,
// empty[buf] = 3 + buf, each over the CTA's 128 threads.
__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <int HD, int G>
__global__ void __launch_bounds__(kScoreP) attn_scores_kernel(const float* __restrict__ q, int n_head, int n_kv,
                                                              const int32_t* __restrict__ pos,
                                                              const int32_t* __restrict__ seq,
                                                              const uint16_t* __restrict__ kc,
                                                              const KvSeqState* __restrict__ st, int n_seq, int cap,
                                                              float scale, float* __restrict__ sbuf,
                                                              unsigned int* __restrict__ count, int* status,
                                                              float one, float neg_zero) {
  constexpr int P = kScoreP;
  constexpr int NP = (G + 1) / 2;                     // head pairs (the last one half used when G is odd)
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  constexpr int KS = HD * 2 + 16;                     // K row stride in bytes (bank skew)
  uint8_t* ks = smem + 128;                                      // [P] rows of KS bytes
  uint64_t* qs = reinterpret_cast<uint64_t*>(ks + P * KS);       // [HD][NP]: (q_2j[i], q_2j+1[i])
  float* ebuf = reinterpret_cast<float*>(qs + HD * NP);          // softmax: [2][G][kSoftCh]
  __shared__ float mh[4][G];
  __shared__ float inv_l[G];
  __shared__ unsigned int last_cta;
  pdl_wait();
  pdl_launch_dependents();
  const int chunk = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  int s;
  const int n_pos = query_positions(pos, seq, b, n_seq, cap, &s);
  const int n_ch = (n_pos + P - 1) / P;
  if (chunk >= n_ch) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = chunk * P, n = min(P, n_pos - t0);
  const int hq0 = kh * G;
  float* srow = sbuf + ((int64_t)b * n_head + hq0) * cap;   // head g's scores at srow + g * cap
  const KvSeqState sst = st ? st[s] : KvSeqState{0, 0};
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], (uint32_t)(n * HD * 2));
    // one bulk copy per position, into rows of KS bytes
    const int64_t base = ((int64_t)s * n_kv + kh) * cap;
    for (int p = t0; p < t0 + n; ++p)
      bulk_g2s(ks + (p - t0) * KS, kc + (base + kv_slot(sst, p, cap)) * HD, (uint32_t)(HD * 2), &bar[0]);
  }
  // q of the G heads, as head pairs, while the copies fly
  {
    const float* qg = q + ((int64_t)b * n_head + hq0) * HD;
    for (int i = tid; i < HD * NP; i += P) {
      const int d = i / NP, j = i - d * NP;
      const float lo = qg[(2 * j) * HD + d];
      const float hi = (2 * j + 1 < G) ? qg[(2 * j + 1) * HD + d] : 0.0f;
      qs[i] = pack2(lo, hi);
    }
  }
  __syncthreads();
  bool ok = mbar_wait_bounded(&bar[0], 0, status, 5);
  if (ok && tid < n) {
    // the row of position t0 + tid (the KS stride puts the 8 rows of a
    // quarter warp on different banks), then the chains in dim order
    constexpr int NPc = HD / 8;
    const Ones k2{pack2(one, one), pack2(neg_zero, neg_zero)};
    const uint8_t* rp = ks + tid * KS;
    uint64_t acc[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) acc[j] = 0ull;   // (+0, +0)
#pragma unroll
    for (int c = 0; c < NPc; ++c) {
      const uint4 rc = *reinterpret_cast<const uint4*>(rp + 16 * c);
      const uint32_t w4[4] = {rc.x, rc.y, rc.z, rc.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float kv = h2f((uint16_t)((w4[e >> 1] >> (16 * (e & 1))) & 0xFFFFu));
        const uint64_t kk = pack2(kv, kv);
        const int d = 8 * c + e;
#pragma unroll
        for (int j = 0; j < NP; ++j) acc[j] = mul_add2(acc[j], qs[d * NP + j], kk, k2);
      }
    }
    const int t = t0 + tid;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      float lo, hi;
      unpack2(acc[j], lo, hi);
      srow[(int64_t)(2 * j) * cap + t] = __fmul_rn(lo, scale);
      if (2 * j + 1 < G) srow[(int64_t)(2 * j + 1) * cap + t] = __fmul_rn(hi, scale);
    }
  }
  // The last CTA of this (query, kv head) runs the softmax over all positions.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(&count[b * n_kv + kh], 1u);
    last_cta = prev == (unsigned int)(n_ch - 1);
    if (last_cta) count[b * n_kv + kh] = 0u;   // ready for the next launch
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  // m: any order (a maximum)
  {
    float m[G];
#pragma unroll
    for (int g = 0; g < G; ++g) m[g] = -FLT_MAX;
    for (int t = tid; t < n_pos; t += P) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float v = __ldcg(srow + (int64_t)g * cap + t);
        if (v > m[g]) m[g] = v;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], o));
      if (lane == 0) mh[warp][g] = m[g];
    }
  }
  __syncthreads();
  if (tid < G) mh[0][tid] = fmaxf(fmaxf(mh[0][tid], mh[1][tid]), fmaxf(mh[2][tid], mh[3][tid]));
  __syncthreads();
  const float* mg = mh[0];
  // e_t by warps 1..3 into the double buffer (and over the scores); the sums
  // by lanes 0..G-1 of warp 0, positions in order.
  const int n_sc = (n_pos + kSoftCh - 1) / kSoftCh;
  if (warp == 0) {
    float l = 0.0f;
    for (int c = 0; c < n_sc; ++c) {
      const int buf = c & 1, len = min(kSoftCh, n_pos - c * kSoftCh);
      bar_sync(1 + buf, P);   // full
      if (lane < G) {
        const float* e = ebuf + (buf * G + lane) * kSoftCh;
        int i = 0;
        for (; i + 4 <= len; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(e + i);
          l = __fadd_rn(l, v.x);
          l = __fadd_rn(l, v.y);
          l = __fadd_rn(l, v.z);
          l = __fadd_rn(l, v.w);
        }
        for (; i < len; ++i) l = __fadd_rn(l, e[i]);
      }
      __syncwarp();
      bar_arrive(3 + buf, P);   // empty
    }
    if (lane < G) inv_l[lane] = __fdiv_rn(1.0f, l);
  } else {
    const int ptid = tid - 32;   // 96 producer threads
    for (int c = 0; c < n_sc; ++c) {
      const int buf = c & 1, base = c * kSoftCh, len = min(kSoftCh, n_pos - base);
      if (c >= 2) bar_sync(3 + buf, P);   // the chain has read this buffer
      for (int i = ptid; i < G * kSoftCh; i += P - 32) {
        const int g = i / kSoftCh, j = i - g * kSoftCh;
        if (j < len) {
          float* sp = srow + (int64_t)g * cap + base + j;
          const float e = b2_expf_ref(__fsub_rn(__ldcg(sp), mg[g]));
          ebuf[(buf * G + g) * kSoftCh + j] = e;
          *sp = e;
        }
      }
      bar_arrive(1 + buf, P);   // full
    }
    // pair the chain's releases of the last two chunks
    for (int c = max(0, n_sc - 2); c < n_sc; ++c) bar_sync(3 + (c & 1), P);
  }
  __syncthreads();
  // p_t = e_t · (1/l) over the scores
  for (int i = tid; i < G * n_pos; i += P) {
    const int g = i / n_pos, t = i - g * n_pos;
    float* sp = srow + (int64_t)g * cap + t;
    *sp = __fmul_rn(__ldcg(sp), inv_l[g]);
  }
}

// out[b][h][d] for the dims [slice*DS, slice*DS+DS) of the G heads of one kv head.
template <int HD, int G>
__global__ void __launch_bounds__(64) attn_pv_kernel(const int32_t* __restrict__ pos, const int32_t* __restrict__ seq,
                                                     const uint16_t* __restrict__ vc,
                                                     const KvSeqState* __restrict__ st, int n_seq, int n_head,
                                                     int n_kv, int cap, const float* __restrict__ pbuf,
                                                     float* __restrict__ out, float one, float neg_zero) {
  constexpr int DS = 64 / G;            // dims of the slice: G heads x DS/2 pairs = 32 chain lanes
  constexpr int CH = (2048 / DS) < 128 ? (2048 / DS) : 128;   // positions per chunk
  constexpr int NBUF = 3;               // chunks in flight (barrier ids 1..3 full, 4..6 empty)
  constexpr int PST = CH + 4;           // pairs per head row (bank skew)
  constexpr int PIECES = DS / 8;        // 16-byte pieces of fp16 per position
  static_assert(HD % DS == 0 && DS % 8 == 0, "slice");
  __shared__ __align__(16) uint64_t pp[NBUF][G][PST];   // (p_t, p_t)
  __shared__ __align__(16) float vv[NBUF][CH][DS];       // V slice, fp32
  const int slice = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s_q = seq[b], p_q = pos[b];
  const int n_pos = (s_q >= 0 && s_q < n_seq && p_q >= 0 && p_q < cap) ? p_q + 1 : 0;
  const KvSeqState sst = (n_pos && st) ? st[s_q] : KvSeqState{0, 0};
  const int64_t vbase = n_pos ? ((int64_t)s_q * n_kv + kh) * cap : 0;
  const int d0 = slice * DS;
  // V does not depend on the scores: bring this slice's rows towards L2 now.
  if (warp == 1) {
    for (int t = lane; t < n_pos; t += 32) {
      const uint16_t* src = vc + (vbase + kv_slot(sst, t, cap)) * HD + d0;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(src));
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  const float* prow = pbuf + ((int64_t)b * n_head + kh * G) * cap;
  const int n_c = (n_pos + CH - 1) / CH;
  if (warp == 1) {
    // loader: chunk c into buffer c % NBUF once the chain has released it
    for (int c = 0; c < n_c; ++c) {
      const int buf = c % NBUF, base = c * CH, len = min(CH, n_pos - base);
      if (c >= NBUF) bar_sync(4 + buf, 64);
#pragma unroll 4
      for (int i = lane; i < len * PIECES; i += 32) {
        const int t = i / PIECES, pc = i - t * PIECES;
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(vc + (vbase + kv_slot(sst, base + t, cap)) * HD + d0 +
                                                              8 * pc));
        const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
        float* dst = &vv[buf][t][8 * pc];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dst[2 * e] = h2f((uint16_t)(w4[e] & 0xFFFFu));
          dst[2 * e + 1] = h2f((uint16_t)(w4[e] >> 16));
        }
      }
#pragma unroll 4
      for (int i = lane; i < G * len; i += 32) {
        const int g = i / len, t = i - g * len;
        const float pv = __ldcg(prow + (int64_t)g * cap + base + t);
        pp[buf][g][t] = pack2(pv, pv);
      }
      bar_arrive(1 + buf, 64);
    }
    // complete the chain's releases of the last NBUF chunks
    for (int c = max(0, n_c - NBUF); c < n_c; ++c) bar_sync(4 + c % NBUF, 64);
    return;
  }
  // chain warp: lane = (head g, dim pair j)
  const int g = lane / (DS / 2), j = lane - g * (DS / 2);
  const Ones k2{pack2(one, one), pack2(neg_zero, neg_zero)};
  uint64_t acc = 0ull;
  for (int c = 0; c < n_c; ++c) {
    const int buf = c % NBUF, len = min(CH, n_pos - c * CH);
    bar_sync(1 + buf, 64);
    const uint64_t* pr = &pp[buf][g][0];
    int t = 0;
    for (; t + 2 <= len; t += 2) {
      const ulonglong2 p2 = *reinterpret_cast<const ulonglong2*>(pr + t);
      const uint64_t v0 = *reinterpret_cast<const uint64_t*>(&vv[buf][t][2 * j]);
      const uint64_t v1 = *reinterpret_cast<const uint64_t*>(&vv[buf][t + 1][2 * j]);
      acc = mul_add2(acc, p2.x, v0, k2);
      acc = mul_add2(acc, p2.y, v1, k2);
    }
    if (t < len) acc = mul_add2(acc, pr[t], *reinterpret_cast<const uint64_t*>(&vv[buf][t][2 * j]), k2);
    __syncwarp();
    bar_arrive(4 + buf, 64);
  }
  float o0, o1;
  unpack2(acc, o0, o1);
  float* op = out + ((int64_t)b * n_head + kh * G + g) * HD + d0 + 2 * j;
  op[0] = o0;
  op[1] = o1;
}

template <int HD, int G>
int launch_hd_g(const float* q, int n_tok, int n_head, int n_kv, const int32_t* pos, const int32_t* seq,
                const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int n_seq, int cap, float* scores,
                unsigned int* count, float* out, cudaStream_t s, int* status) {
  constexpr int NP = (G + 1) / 2;
  const size_t sm = 128 + (size_t)kScoreP * (HD * 2 + 16) + (size_t)HD * NP * 8 + (size_t)2 * G * kSoftCh * 4;
  B2_CUDA_TRY(cudaFuncSetAttribute(attn_scores_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  const float scale = 1.0f / sqrtf((float)HD);
  int rc = launch_pdl(attn_scores_kernel<HD, G>, dim3((cap + kScoreP - 1) / kScoreP, n_kv, n_tok), dim3(kScoreP), sm,
                      s, q, n_head, n_kv, pos, seq, kc, st, n_seq, cap, scale, scores, count, status, 1.0f, -0.0f);
  if (rc) return rc;
  return launch_pdl(attn_pv_kernel<HD, G>, dim3(HD / (64 / G), n_kv, n_tok), dim3(64), 0, s, pos, seq, vc, st, n_seq,
                    n_head, n_kv, cap, (const float*)scores, out, 1.0f, -0.0f);
}

}  // namespace

size_t attn_scratch_floats(int n_tok, int n_head, int cap) { return (size_t)n_tok * n_head * cap; }

int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int n_seq, int cap, float* scores,
                     unsigned int* count, float* out, cudaStream_t s, int* status) {
  B2_CHECK_ARG(n_kv > 0 && n_head % n_kv == 0 && scores && count && out && cap > 0, "attention arguments");
  const int G = n_head / n_kv;
#define B2_ATTN_CASE(HDV, GV) \
  if (hd == HDV && G == GV)   \
    return launch_hd_g<HDV, GV>(q, n_tok, n_head, n_kv, pos, seq, kc, vc, st, n_seq, cap, scores, count, out, s, status);
  B2_ATTN_CASE(128, 1)
  B2_ATTN_CASE(128, 2)
  B2_ATTN_CASE(128, 4)
  B2_ATTN_CASE(128, 8)
  B2_ATTN_CASE(64, 1)
  B2_ATTN_CASE(64, 2)
  B2_ATTN_CASE(64, 4)
  B2_ATTN_CASE(64, 8)
#undef B2_ATTN_CASE
  set_error("attention: unsupported head_dim %d / group %d", hd, G);
  return B2_ERR_UNSUPPORTED;
}

}  // namespace b2
