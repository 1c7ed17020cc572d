// Decode attention over the fp16 KV cache in the reference's order
// (Singularity/src/core/cortex_a5_engine.cpp:1205-1254, with the softmax of
// ref_softmax_f32, Singularity/tests/test_and_bench_a5.cpp:260-278): for
// query head h of token b at position p (kv head h / G),
//   s_t = (Σ_i q_i·k_ti, dims in order) · (1/sqrt(hd))      t = 0..p
//   m = max_t s_t;  e_t = expf(s_t − m);  l = Σ_t e_t (positions in order)
//   p_t = e_t · (1/l);  out_i = Σ_t p_t·v_ti (positions in order)
// every multiply and add a separately rounded fp32 operation, expf the host
// library's (b2_expf_ref), so every output is bit-identical to the
// reference's CPU result.  The sums over positions are sequential chains:
// the work is laid out so that as many chains as possible run side by side,
// every chain reads shared memory that was filled ahead of it, and nothing
// but the chains themselves is serial.
//
// Scratch per (query, kv head) group, in floats: the scores S [G][capS]
// (capS = cap rounded up to 4), the exponentials E [capS][GP] (GP = max(G,
// 4): one 16-byte-aligned row per position), and the chunk maxima M [G][nchS]
// (nchS = the number of 128-position chunks rounded up to 4).
//
// Three kernels:
//   * attn_scores_kernel: one CTA per (128-position chunk, kv head, query).
//     The chunk's K rows arrive by 1-D bulk copies (one per run of
//     consecutive cache slots: the pinned prefix, the ring's tail, its head)
//     while q goes to shared memory; thread t scores position t against the
//     G query heads (two heads per packed f32x2 operation) and writes s_t;
//     the CTA writes the chunk's maximum per head.
//   * attn_exp_kernel: one CTA per (chunk, kv head, query): m from the chunk
//     maxima (a maximum: any order), then e_t = expf(s_t − m) for every
//     position of the chunk and head into E.
//   * attn_pv_kernel: one CTA per (slice of 64/G dims, kv head, query).
//     First lanes 0..G-1 add e_t in position order (windows of E arrive by
//     bulk copies, in parts the chain starts on as each lands) and take
//     1/l.  Then a loader warp brings each chunk of up to 128 positions in
//     with one 2-D tensor copy of the V slice and one bulk copy of the E
//     rows, turns V into fp32 pairs and forms p_t = e_t·(1/l); the chain
//     warp's lane (head, dim pair) runs out += p_t·v_t over the positions in
//     order as two scalar chains (one per dim).
// Q8_0 caches (llama.cpp's cache type that Milda asks for by default,
// Milda/src/engine.cpp:74-87, 1195-1196): rows of hd int8 codes then the
// hd/32 fp16 block scales (kv_row_bytes).  With a Q8_0 K the CTA quantizes
// its G query heads to Q8_0 (ref_quantize_row_q8_0) and thread t scores its
// position with the reference's Q8_0·Q8_0 block dot (dp4a block sums, then
// sumf += (d_k·d_q)·sumi in block order) times 1/sqrt(hd).  With a Q8_0 V
// the loader brings the slice's codes and the rows' scale words with two
// 2-D tensor copies and converts code·scale (exact in fp32) into the same
// fp32 pairs the chain reads.
// Queries whose sequence id or position is outside the cache attend to
// nothing and get zero outputs.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>

#include "b2_common.cuh"
#include "b2_layers.hpp"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kScoreP = 128;          // positions per scores / exp CTA (one per thread)
constexpr int kPvCh = 128;            // positions per P.V chunk
constexpr int kPvStagesMax = 8;            // P.V stages per CTA: as many as the CTAs per SM leave room for
constexpr int kSumParts = 4;          // bulk copies (and mbarriers) per window of the sum

__host__ __device__ constexpr int gp_of(int g) { return g < 4 ? 4 : g; }
__host__ __device__ inline int cap_s(int cap) { return (cap + 3) & ~3; }
__host__ __device__ inline int nch_s(int cap) { return ((cap + kScoreP - 1) / kScoreP + 3) & ~3; }
// floats of one (query, kv head) group: S [G][capS], E [capS][GP], M [G][nchS]
__host__ __device__ inline int64_t group_floats(int g, int cap) {
  return (int64_t)cap_s(cap) * (g + gp_of(g)) + (int64_t)g * nch_s(cap);
}
__host__ __device__ inline int64_t e_offset(int g, int cap) { return (int64_t)g * cap_s(cap); }
__host__ __device__ inline int64_t m_offset(int g, int cap) { return (int64_t)cap_s(cap) * (g + gp_of(g)); }

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

// A run of logical positions starting at p that sit in consecutive cache
// slots: within the pinned prefix, or within the ring up to its end.
struct SlotRun {
  int p, len;
  int64_t slot;
};
__device__ __forceinline__ SlotRun slot_run(const KvSeqState& st, int p, int end, int cap, int max_len) {
  SlotRun r;
  r.p = p;
  r.slot = kv_slot(st, p, cap);
  int len = min(max_len, end - p);
  if (p < st.n_keep) len = min(len, st.n_keep - p);
  else len = (int)min((int64_t)len, (int64_t)cap - r.slot);
  r.len = len;
  return r;
}

// Shared memory of a scores CTA: barrier, the chunk's K rows, then q (fp16
// K: head pairs [HD][NP] of 8 bytes; Q8_0 K: the G heads' Q8_0 codes [G][HD]
// and scales [G][HD/32] as fp32).
// K rows in shared memory: Q8_0 and Q4_0 rows as cached (hd + 16 and hd/2
// + 16 bytes); fp16 rows padded by 16 bytes, so the rows that the 8 threads
// of a 16-byte load phase read start on different banks.
template <int HD, int KT>
__host__ __device__ constexpr int scores_row_stride() {
  return KT != B2_F16 ? (int)kv_row_bytes(KT, HD) : (int)kv_row_bytes(KT, HD) + 16;
}
template <int HD, int G, int KT>
__host__ __device__ constexpr size_t scores_smem_bytes() {
  return 128 + (size_t)kScoreP * scores_row_stride<HD, KT>() +
         (KT != B2_F16 ? (size_t)G * HD + (size_t)G * (HD / 32) * 4 : (size_t)HD * ((G + 1) / 2) * 8);
}

// Unsigned 4 bytes · signed 4 bytes (the Q4_0 codes against Q8_0 codes).
__device__ __forceinline__ int dp4a_u8s8(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int HD, int G, int KT>
__global__ void __launch_bounds__(kScoreP) attn_scores_kernel(const float* __restrict__ q, int n_head, int n_kv,
                                                              const int32_t* __restrict__ pos,
                                                              const int32_t* __restrict__ seq,
                                                              const uint8_t* __restrict__ kc,
                                                              const KvSeqState* __restrict__ st, int n_seq, int cap,
                                                              float scale, float* __restrict__ sbuf, int* status,
                                                              float one, float neg_zero) {
  constexpr int P = kScoreP;
  constexpr int NP = (G + 1) / 2;              // head pairs (the last one half used when G is odd)
  constexpr int RB = (int)kv_row_bytes(KT, HD);
  constexpr int RS = scores_row_stride<HD, KT>();
  constexpr int KB = P * RS;                   // K rows of the chunk
  constexpr int NB = HD / 32;                  // Q8_0 blocks per row
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint8_t* ks = smem + 128;                                      // [P][RS]
  uint64_t* qs = reinterpret_cast<uint64_t*>(smem + 128 + KB);   // fp16 K: [HD][NP]: (q_2j[i], q_2j+1[i])
  int8_t* qq = reinterpret_cast<int8_t*>(smem + 128 + KB);       // Q8_0 K: codes [G][HD]
  float* qd = reinterpret_cast<float*>(smem + 128 + KB + G * HD);   // Q8_0 K: scales [G][NB]
  __shared__ float mh[P / 32][G];
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
  const int capS = cap_s(cap);
  float* grp = sbuf + ((int64_t)b * n_kv + kh) * group_floats(G, cap);
  float* srow = grp;                           // head g's scores at srow + g * capS
  float* mrow = grp + m_offset(G, cap);        // head g's chunk maxima at mrow + g * nchS
  const KvSeqState sst = st ? st[s] : KvSeqState{0, 0};
  if constexpr (KT != B2_Q8_0) {
    // fp16 rows: one bulk copy per row into its padded slot (the lanes'
    // copies overlap)
    if (tid == 0) {
      mbar_init(&bar[0], 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(&bar[0], (uint32_t)(n * RB));
    }
    __syncthreads();
    if (tid < n) {
      const int64_t slot = kv_slot(sst, t0 + tid, cap);
      bulk_g2s(ks + tid * RS, kc + (((int64_t)s * n_kv + kh) * cap + slot) * RB, (uint32_t)RB, &bar[0]);
    }
  } else if (warp == 0) {
    // one lane per run of consecutive slots (at most three): a bulk copy
    // costs its issuing thread a few hundred cycles, copies from different
    // lanes overlap
    if (lane == 0) {
      mbar_init(&bar[0], 1);
      fence_mbar_init();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(&bar[0], (uint32_t)(n * RB));
    const int64_t base = ((int64_t)s * n_kv + kh) * cap;
    int p = t0;
    for (int r_i = 0; p < t0 + n; ++r_i) {
      const SlotRun r = slot_run(sst, p, t0 + n, cap, P);
      if (lane == r_i) bulk_g2s(ks + (p - t0) * RB, kc + (base + r.slot) * RB, (uint32_t)(r.len * RB), &bar[0]);
      p += r.len;
    }
  }
  // q of the G heads while the copies fly: head pairs for fp16 K; for Q8_0
  // and Q4_0 K each head quantized to Q8_0 (one warp per 32-value block),
  // the dot type that pairs with both
  const float* qg = q + ((int64_t)b * n_head + hq0) * HD;
  if constexpr (KT != B2_F16) {
    for (int blk = warp; blk < G * NB; blk += P / 32) {
      uint16_t d16;
      const int8_t c = quant_q8_0_lane(qg[blk * 32 + lane], &d16);
      qq[blk * 32 + lane] = c;
      if (lane == 0) qd[blk] = h2f(d16);
    }
  } else {
    for (int i = tid; i < HD * NP; i += P) {
      const int d = i / NP, j = i - d * NP;
      const float lo = qg[(2 * j) * HD + d];
      const float hi = (2 * j + 1 < G) ? qg[(2 * j + 1) * HD + d] : 0.0f;
      qs[i] = pack2(lo, hi);
    }
  }
  __syncthreads();
  const bool ok = mbar_wait_bounded(&bar[0], 0, status, 5);
  float sc[2 * NP];
#pragma unroll
  for (int j = 0; j < 2 * NP; ++j) sc[j] = -FLT_MAX;
  if constexpr (KT == B2_Q8_0) {
    if (ok && tid < n) {
      // the Q8_0·Q8_0 block dot of ref_vec_dot_q8_0_q8_0
      // (Singularity/tests/test_and_bench_a5.cpp:205-221): exact block sums,
      // then sumf += (d_k·d_q)·sumi over the blocks in order
      const uint8_t* rp = ks + tid * RB;
      float sumf[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sumf[g] = 0.0f;
#pragma unroll
      for (int bi = 0; bi < NB; ++bi) {
        const uint4 k0 = *reinterpret_cast<const uint4*>(rp + bi * 32);
        const uint4 k1 = *reinterpret_cast<const uint4*>(rp + bi * 32 + 16);
        const float dk = h2f(*reinterpret_cast<const uint16_t*>(rp + HD + 2 * bi));
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const uint4 q0 = *reinterpret_cast<const uint4*>(qq + g * HD + bi * 32);
          const uint4 q1 = *reinterpret_cast<const uint4*>(qq + g * HD + bi * 32 + 16);
          int si = __dp4a((int)k0.x, (int)q0.x, 0);
          si = __dp4a((int)k0.y, (int)q0.y, si);
          si = __dp4a((int)k0.z, (int)q0.z, si);
          si = __dp4a((int)k0.w, (int)q0.w, si);
          si = __dp4a((int)k1.x, (int)q1.x, si);
          si = __dp4a((int)k1.y, (int)q1.y, si);
          si = __dp4a((int)k1.z, (int)q1.z, si);
          si = __dp4a((int)k1.w, (int)q1.w, si);
          sumf[g] = __fadd_rn(sumf[g], __fmul_rn(__fmul_rn(dk, qd[g * NB + bi]), (float)si));
        }
      }
      const int t = t0 + tid;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sc[g] = __fmul_rn(sumf[g], scale);
        srow[(int64_t)g * capS + t] = sc[g];
      }
    }
  } else if constexpr (KT == B2_Q4_0) {
    if (ok && tid < n) {
      // the Q4_0·Q8_0 block dot of ref_vec_dot_q4_0_q8_0
      // (Singularity/tests/test_and_bench_a5.cpp:184-203): sumi =
      // Σ (lo_j − 8)·q_j + (hi_j − 8)·q_{j+16} (exact), then sumf +=
      // (d_k·d_q)·sumi over the blocks in order
      const uint8_t* rp = ks + tid * RS;
      float sumf[G];
#pragma unroll
      for (int g = 0; g < G; ++g) sumf[g] = 0.0f;
#pragma unroll
      for (int bi = 0; bi < NB; ++bi) {
        const uint4 kw = *reinterpret_cast<const uint4*>(rp + bi * 16);
        const uint32_t lo[4] = {kw.x & 0x0F0F0F0Fu, kw.y & 0x0F0F0F0Fu, kw.z & 0x0F0F0F0Fu, kw.w & 0x0F0F0F0Fu};
        const uint32_t hi[4] = {(kw.x >> 4) & 0x0F0F0F0Fu, (kw.y >> 4) & 0x0F0F0F0Fu, (kw.z >> 4) & 0x0F0F0F0Fu,
                                (kw.w >> 4) & 0x0F0F0F0Fu};
        const float dk = h2f(*reinterpret_cast<const uint16_t*>(rp + HD / 2 + 2 * bi));
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const uint4 q0 = *reinterpret_cast<const uint4*>(qq + g * HD + bi * 32);
          const uint4 q1 = *reinterpret_cast<const uint4*>(qq + g * HD + bi * 32 + 16);
          const uint32_t qa[4] = {q0.x, q0.y, q0.z, q0.w}, qb[4] = {q1.x, q1.y, q1.z, q1.w};
          int si = 0, sq = 0;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            si = dp4a_u8s8(lo[w], qa[w], si);
            si = dp4a_u8s8(hi[w], qb[w], si);
            sq = __dp4a(0x01010101, (int)qa[w], sq);
            sq = __dp4a(0x01010101, (int)qb[w], sq);
          }
          sumf[g] = __fadd_rn(sumf[g], __fmul_rn(__fmul_rn(dk, qd[g * NB + bi]), (float)(si - 8 * sq)));
        }
      }
      const int t = t0 + tid;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sc[g] = __fmul_rn(sumf[g], scale);
        srow[(int64_t)g * capS + t] = sc[g];
      }
    }
  } else if (ok && tid < n) {
    // the row of position t0 + tid, then the chains in dim order
    constexpr int NPc = HD / 8;
    const Ones k2{pack2(one, one), pack2(neg_zero, neg_zero)};
    const uint8_t* rp = ks + tid * RS;
    uint64_t acc[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) acc[j] = 0ull;   // (+0, +0)
    // 16 dims per trip (the body stays small enough for the instruction
    // cache); a half2 of K turns into two floats at once, and one 16-byte
    // read brings two head pairs of q
#pragma unroll 2
    for (int c = 0; c < NPc; ++c) {
      const uint4 rc = *reinterpret_cast<const uint4*>(rp + 16 * c);
      const uint32_t w4[4] = {rc.x, rc.y, rc.z, rc.w};
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&w4[e2]));
        const float kv2[2] = {kf.x, kf.y};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int d = 8 * c + 2 * e2 + h;
          const uint64_t kk = pack2(kv2[h], kv2[h]);
          uint64_t qv[NP];
          if constexpr (NP == 1) {
            qv[0] = qs[d];
          } else {
#pragma unroll
            for (int i = 0; i < NP; i += 2) {
              const uint4 v = *reinterpret_cast<const uint4*>(qs + d * NP + i);
              qv[i] = ((uint64_t)v.y << 32) | v.x;
              qv[i + 1] = ((uint64_t)v.w << 32) | v.z;
            }
          }
#pragma unroll
          for (int j = 0; j < NP; ++j) acc[j] = mul_add2(acc[j], qv[j], kk, k2);
        }
      }
    }
    const int t = t0 + tid;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      float lo, hi;
      unpack2(acc[j], lo, hi);
      sc[2 * j] = __fmul_rn(lo, scale);
      sc[2 * j + 1] = __fmul_rn(hi, scale);
      srow[(int64_t)(2 * j) * capS + t] = sc[2 * j];
      if (2 * j + 1 < G) srow[(int64_t)(2 * j + 1) * capS + t] = sc[2 * j + 1];
    }
  }
  // the chunk's maximum per head (a maximum: any order)
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float v = sc[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) mh[warp][g] = v;
  }
  __syncthreads();
  if (tid < G) {
    float v = mh[0][tid];
#pragma unroll
    for (int w = 1; w < P / 32; ++w) v = fmaxf(v, mh[w][tid]);
    mrow[(int64_t)tid * nch_s(cap) + chunk] = v;
  }
}

// e_t = expf(s_t − m) for the chunk's positions, m the maximum over all the
// chunk maxima of the head.
template <int G>
__global__ void __launch_bounds__(kScoreP) attn_exp_kernel(const int32_t* __restrict__ pos,
                                                           const int32_t* __restrict__ seq, int n_seq, int n_kv,
                                                           int cap, float* __restrict__ sbuf) {
  constexpr int P = kScoreP, GP = gp_of(G);
  __shared__ unsigned long long tab[32];
  __shared__ float mh[P / 32][G];
  pdl_wait();
  pdl_launch_dependents();
  const int chunk = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  int s;
  const int n_pos = query_positions(pos, seq, b, n_seq, cap, &s);
  const int n_ch = (n_pos + P - 1) / P;
  if (chunk >= n_ch) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  exp_table_to_smem(tab, tid, P);
  float* grp = sbuf + ((int64_t)b * n_kv + kh) * group_floats(G, cap);
  const float* srow = grp;
  float* erow = grp + e_offset(G, cap);
  const float* mrow = grp + m_offset(G, cap);
  const int capS = cap_s(cap), nchS = nch_s(cap);
  float mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float v = -FLT_MAX;
    for (int c = tid; c < n_ch; c += P) v = fmaxf(v, mrow[g * nchS + c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) mh[warp][g] = v;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float v = mh[0][g];
#pragma unroll
    for (int w = 1; w < P / 32; ++w) v = fmaxf(v, mh[w][g]);
    mg[g] = v;
  }
  const int t = chunk * P + tid;
  if (t < n_pos) {
    float e[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) e[g] = g < G ? b2_expf_ref(__fsub_rn(srow[(int64_t)g * capS + t], mg[g]), tab) : 0.0f;
    float4* dst = reinterpret_cast<float4*>(erow + (int64_t)t * GP);
#pragma unroll
    for (int v = 0; v < GP / 4; ++v) dst[v] = make_float4(e[4 * v], e[4 * v + 1], e[4 * v + 2], e[4 * v + 3]);
  }
}

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Rows of the converted stage hold kPvChP = kPvCh + 2 pairs: 16 bytes of
// padding per row put the rows that the chain lanes read side by side on
// different banks.
constexpr int kPvChP = kPvCh + 2;
// Bytes of a Q8_0 V slice's codes per row: the slice's ds bytes, at least
// 16 (a tensor copy's smallest inner box), starting at the slice's first dim
// rounded down to 16.
__host__ __device__ constexpr int pv_code_bytes(int ds) { return ds < 16 ? 16 : ds; }
// Q4_0: the slice's blocks' 16-byte nibble runs (one for slices of up to 32
// dims), from its first block.
__host__ __device__ constexpr int pv_code_bytes_q4(int ds) { return ds <= 32 ? 16 : ds / 2; }
template <int VT>
__host__ __device__ constexpr int pv_codes(int ds) {
  return VT == B2_Q4_0 ? pv_code_bytes_q4(ds) : pv_code_bytes(ds);
}
// Raw V rows of a stage: fp16 [CH][ds]; Q8_0 codes [CH][pv_code_bytes] then
// the rows' scale words [CH][8] (16 bytes: the hd/32 scales and padding).
template <int VT>
__host__ __device__ constexpr size_t pv_rawv_bytes(int ds) {
  return VT != B2_F16 ? (size_t)kPvCh * (pv_codes<VT>(ds) + 16) : (size_t)kPvCh * ds * 2;
}
template <int G, int VT>
__host__ __device__ constexpr size_t pv_stage_bytes(int ds) {
  // raw V | raw E [CH][GP] | V pairs [ds/2][CHP] | p [G][2·CHP] floats,
  // rounded up to 128 bytes (the tensor copy's destination alignment)
  return (pv_rawv_bytes<VT>(ds) + (size_t)kPvCh * gp_of(G) * 4 + (size_t)(ds / 2) * kPvChP * 8 +
          (size_t)G * kPvChP * 8 + 127) / 128 * 128;
}

// l = Σ_t e_t in position order for lane g < G, over rows e[t * GP + g] of
// shared memory.  Two buffers of 16 values take turns: the next 16 are read
// while the current 16 are added (a warp issues in order: each read sits
// between two adds, in the latency of the chain), and no register copies
// sit between the adds.
template <int GP>
__device__ __forceinline__ float sum_run(const float* e, int a, int b, float l) {
  const int n32 = a + ((b - a) & ~31);
  float A[16], B[16];
  if (n32 > a) {
#pragma unroll
    for (int k = 0; k < 16; ++k) A[k] = e[(a + k) * GP];
  }
  for (int i = a; i < n32; i += 32) {
    // each add followed by the read of the value 16 ahead, so the reads
    // issue in the adds' latency
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      B[k] = e[(i + 16 + k) * GP];
      l = __fadd_rn(l, A[k]);
    }
    const int in = i + 32 < n32 ? i + 32 : i;   // the last trip re-reads in range
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      A[k] = e[(in + k) * GP];
      l = __fadd_rn(l, B[k]);
    }
  }
  // the last (fewer than 32) values: all reads first, then the adds
  const int rem = b - n32;
  float T[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) T[k] = k < rem ? e[(n32 + k) * GP] : 0.0f;
#pragma unroll
  for (int k = 0; k < 32; ++k)
    if (k < rem) l = __fadd_rn(l, T[k]);
  return l;
}

// out[b][h][d] for the dims [slice*DS, slice*DS+DS) of the G heads of one kv
// head.  Sum phase: warp 1's lane 0 copies windows of E into the stage
// memory, in kSumParts parts on their own mbarriers, and warp 0's lanes
// 0..G-1 add them in position order.  P.V phase: warp 1 issues each chunk's
// V rows (one 2-D tensor copy of kPvCh rows x DS dims from the first slot of
// a run) and E rows (one bulk copy) into a raw stage, converts V to fp32
// pairs and forms p = e·(1/l); warp 0's lane (head g, dim pair j) runs out
// += p_t·v_t over the positions in order, one scalar chain per dim.
template <int HD, int G, int VT>
__global__ void __launch_bounds__(64) attn_pv_kernel(const int32_t* __restrict__ pos, const int32_t* __restrict__ seq,
                                                     const __grid_constant__ CUtensorMap vmap,
                                                     const __grid_constant__ CUtensorMap smap,
                                                     const KvSeqState* __restrict__ st, int n_seq, int n_head,
                                                     int n_kv, int cap, const float* __restrict__ sbuf,
                                                     float* __restrict__ out, int* status, int n_stages, int wa,
                                                     float one,
                                                     float neg_zero) {
  constexpr int DS = 64 / G;            // dims of the slice: G heads x DS/2 pairs = 32 chain lanes
  constexpr int CH = kPvCh;
  const int NS = n_stages;
  constexpr int GP = gp_of(G);
  static_assert(HD % DS == 0 && DS % 8 == 0, "slice");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);   // [NS] raw stage landed
  uint64_t* conv = full + kPvStagesMax;                 // [NS] converted
  uint64_t* empty = conv + kPvStagesMax;                // [NS] chain done with the stage
  uint64_t* part = empty + kPvStagesMax;                // [kSumParts] window parts of the sum
  float* inv_l = reinterpret_cast<float*>(part + kSumParts);   // [G]
  constexpr size_t SB = pv_stage_bytes<G, VT>(DS);
  constexpr int RAWV = (int)pv_rawv_bytes<VT>(DS);
  constexpr int DSL = pv_codes<VT>(DS);
  const int WA = wa;                                    // positions per window of the sum (a multiple of 4)
  uint8_t* stages = smem + 256;
  const int slice = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&conv[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kSumParts; ++i) mbar_init(&part[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int s_q = seq[b], p_q = pos[b];
  const int n_pos = (s_q >= 0 && s_q < n_seq && p_q >= 0 && p_q < cap) ? p_q + 1 : 0;
  const KvSeqState sst = (n_pos && st) ? st[s_q] : KvSeqState{0, 0};
  const int row0 = n_pos ? (s_q * n_kv + kh) * cap : 0;   // tensor-map row of slot 0
  const int d0 = slice * DS;
  pdl_wait();
  pdl_launch_dependents();
  const float* erow = sbuf + ((int64_t)b * n_kv + kh) * group_floats(G, cap) + e_offset(G, cap);
  bool ok = true;

  // ---- sum phase ----
  float l = 0.0f;
  for (int w0 = 0, wi = 0; w0 < n_pos; w0 += WA, ++wi) {
    const int len = min(WA, n_pos - w0), len4 = (len + 3) & ~3;
    const int plen = ((len + kSumParts - 1) / kSumParts + 3) & ~3;
    __syncthreads();   // the previous window is consumed
    if (warp == 1 && lane < kSumParts && lane * plen < len && ok) {   // lane i copies part i
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const int a = lane * plen, n4 = min(plen, len4 - a);
      mbar_arrive_expect_tx(&part[lane], (uint32_t)(n4 * GP * 4));
      bulk_g2s(stages + (size_t)a * GP * 4, erow + (int64_t)(w0 + a) * GP, (uint32_t)(n4 * GP * 4), &part[lane]);
    }
    if (warp == 0 && lane < G) {
      const float* e = reinterpret_cast<const float*>(stages) + lane;
      for (int i = 0; i < kSumParts && i * plen < len; ++i) {
        if (ok) ok = mbar_wait_bounded(&part[i], (uint32_t)(wi & 1), status, 10);
        if (ok) l = sum_run<GP>(e, i * plen, min(i * plen + plen, len), l);
      }
    }
    ok = __syncthreads_and(ok);
    if (!ok) {
      // copies of this window still in flight: wait for them (bounded)
      if (warp == 1 && lane == 0)
        for (int i = 0; i < kSumParts && i * plen < len; ++i) mbar_wait_bounded(&part[i], (uint32_t)(wi & 1), nullptr, 0);
      break;
    }
  }
  if (warp == 0 && lane < G) inv_l[lane] = __fdiv_rn(1.0f, l);
  __syncthreads();
  if (!ok) return;

  // ---- P.V phase ----
  if (warp == 1) {
    // Every lane keeps the issue position; lane 0 copies a chunk's V rows,
    // lane 1 its E rows (a bulk copy costs its issuing thread a few hundred
    // cycles, copies from different lanes overlap).
    int p_iss = 0, c_iss = 0;
    auto issue = [&](int si) {
      const SlotRun r = slot_run(sst, p_iss, n_pos, cap, CH);
      uint8_t* sp = stages + si * SB;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[si], (uint32_t)(RAWV + r.len * GP * 4));
        tma_load_2d(sp, &vmap, VT == B2_Q8_0 ? (d0 & ~15) : VT == B2_Q4_0 ? (d0 >> 5) * 16 : d0, row0 + (int)r.slot,
                    &full[si]);
      } else if (lane == 1) {
        bulk_g2s(sp + RAWV, erow + (int64_t)r.p * GP, (uint32_t)(r.len * GP * 4), &full[si]);
      } else if (VT != B2_F16 && lane == 2) {
        // the rows' scale words: 8 fp16 from the end of the codes
        tma_load_2d(sp + CH * DSL, &smap, (int)kv_code_bytes(VT, HD) / 2, row0 + (int)r.slot, &full[si]);
      }
      p_iss += r.len;
      ++c_iss;
    };
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    while (p_iss < n_pos && c_iss < NS) issue(c_iss % NS);
    __syncwarp();
    float inv[G];
#pragma unroll
    for (int g = 0; g < G; ++g) inv[g] = inv_l[g];
    int p = 0;
    for (int c = 0; p < n_pos; ++c) {
      const int si = c % NS;
      const int len = slot_run(sst, p, n_pos, cap, CH).len;
      if (ok) ok = mbar_wait_bounded(&full[si], (uint32_t)((c / NS) & 1), status, 6);
      if (ok && c >= NS) ok = mbar_wait_bounded(&empty[si], (uint32_t)(((c / NS) - 1) & 1), status, 7);
      if (ok) {
        uint8_t* sp = stages + si * SB;
        const float4* re = reinterpret_cast<const float4*>(sp + RAWV);  // [CH][GP/4] raw E
        uint64_t* vp = reinterpret_cast<uint64_t*>(sp + RAWV + CH * GP * 4);   // [DS/2][CHP]
        uint64_t* pp = vp + (DS / 2) * kPvChP;                                // p: [G][2·CHP] floats
        // lane t owns positions t, t + 32, ...: its V row becomes DS/2 pairs
        // and its E row G values p = e·(1/l)
        for (int t = lane; t < len; t += 32) {
          if constexpr (VT == B2_Q8_0) {
            // code · block scale, exact in fp32 (ggml's dequantize_row_q8_0)
            const uint8_t* rc = sp + t * DSL + (d0 & 15);
            const uint16_t* rs = reinterpret_cast<const uint16_t*>(sp + CH * DSL) + t * 8;
#pragma unroll
            for (int c = 0; c < DS / 8; ++c) {
              const uint2 w = *reinterpret_cast<const uint2*>(rc + 8 * c);
              const float d = h2f(rs[(d0 + 8 * c) >> 5]);
              const uint32_t ww[2] = {w.x, w.y};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t h = ww[k >> 1] >> (16 * (k & 1));
                vp[(4 * c + k) * kPvChP + t] =
                    pack2(__fmul_rn((float)(int8_t)(h & 0xFFu), d), __fmul_rn((float)(int8_t)(h >> 8), d));
              }
            }
          } else if constexpr (VT == B2_Q4_0) {
            // (code − 8) · block scale, exact in fp32 (ggml's
            // dequantize_row_q4_0): dim e of a block is byte e % 16's low
            // nibble for e < 16, its high one above
            const uint8_t* rc = sp + t * DSL;
            const uint16_t* rs = reinterpret_cast<const uint16_t*>(sp + CH * DSL) + t * 8;
#pragma unroll
            for (int c = 0; c < DS / 8; ++c) {   // 8 dims: 8 bytes, one half of a block
              const int dd = d0 + 8 * c, e = dd & 31;
              const int bo = ((dd >> 5) - (d0 >> 5)) * 16 + (e & 15);
              const int sh = (e & 16) ? 4 : 0;
              const float d = h2f(rs[dd >> 5]);
              const uint2 w = *reinterpret_cast<const uint2*>(rc + bo);
              const uint32_t ww[2] = {(w.x >> sh) & 0x0F0F0F0Fu, (w.y >> sh) & 0x0F0F0F0Fu};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t h = ww[k >> 1] >> (16 * (k & 1));
                vp[(4 * c + k) * kPvChP + t] = pack2(__fmul_rn((float)((int)(h & 0xFFu) - 8), d),
                                                     __fmul_rn((float)((int)((h >> 8) & 0xFFu) - 8), d));
              }
            }
          } else {
            const uint4* rv = reinterpret_cast<const uint4*>(sp);   // [CH][DS/8] raw V
#pragma unroll
            for (int c = 0; c < DS / 8; ++c) {
              const uint4 w = rv[t * (DS / 8) + c];
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int k = 0; k < 4; ++k)
                vp[(4 * c + k) * kPvChP + t] = pack2(h2f((uint16_t)(ww[k] & 0xFFFFu)), h2f((uint16_t)(ww[k] >> 16)));
            }
          }
#pragma unroll
          for (int c = 0; c < GP / 4; ++c) {
            const float4 e = re[t * (GP / 4) + c];
            const float ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (4 * c + k < G) {
                reinterpret_cast<float*>(pp)[(4 * c + k) * 2 * kPvChP + t] = __fmul_rn(ev[k], inv[4 * c + k]);
              }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[si]);
      if (ok && p_iss < n_pos) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(si);
      }
      __syncwarp();
      p += len;
    }
    // copies still in flight after a failed wait: wait for them (bounded)
    if (!ok && lane == 0) {
      int pp = 0;
      for (int c = 0; pp < p_iss; ++c) {
        const int si = c % NS;
        pp += slot_run(sst, pp, n_pos, cap, CH).len;
        mbar_wait_bounded(&full[si], (uint32_t)((c / NS) & 1), nullptr, 0);
      }
    }
    return;
  }
  // chain warp: lane = (head g, dim pair j), two scalar chains (dims 2j and
  // 2j + 1): each product and each add one rounded fp32 operation
  const int g = lane / (DS / 2), j = lane - g * (DS / 2);
  float acc0 = 0.0f, acc1 = 0.0f;
  int p = 0;
  for (int c = 0; p < n_pos; ++c) {
    const int si = c % NS;
    const int len = slot_run(sst, p, n_pos, cap, CH).len;
    if (ok) ok = mbar_wait_bounded(&conv[si], (uint32_t)((c / NS) & 1), status, 8);
    if (ok) {
      const uint8_t* sp = stages + si * SB;
      const uint64_t* vr = reinterpret_cast<const uint64_t*>(sp + RAWV + CH * GP * 4) + j * kPvChP;
      const float* pf = reinterpret_cast<const float*>(reinterpret_cast<const uint64_t*>(sp + RAWV + CH * GP * 4) +
                                                       (DS / 2) * kPvChP) +
                        g * 2 * kPvChP;
      // positions in groups of 8 (p four per 16-byte load, v pairs two), in
      // two buffers that take turns: the next group is read while the
      // current group's adds run
      const int len16 = len & ~15;
      float4 ap[2], bp[2];
      uint4 av[4], bv[4];
      if (len16 > 0) {
        ap[0] = *reinterpret_cast<const float4*>(pf);
        ap[1] = *reinterpret_cast<const float4*>(pf + 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) av[k] = *reinterpret_cast<const uint4*>(vr + 2 * k);
      }
      for (int t = 0; t < len16; t += 16) {
        // the group's 16 products first, then its adds in position order
        // with the next group's reads between them
        float m0[8], m1[8];
        {
          const float pa[8] = {ap[0].x, ap[0].y, ap[0].z, ap[0].w, ap[1].x, ap[1].y, ap[1].z, ap[1].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            m0[2 * k] = __fmul_rn(pa[2 * k], __uint_as_float(av[k].x));
            m1[2 * k] = __fmul_rn(pa[2 * k], __uint_as_float(av[k].y));
            m0[2 * k + 1] = __fmul_rn(pa[2 * k + 1], __uint_as_float(av[k].z));
            m1[2 * k + 1] = __fmul_rn(pa[2 * k + 1], __uint_as_float(av[k].w));
          }
        }
        bp[0] = *reinterpret_cast<const float4*>(pf + t + 8);
        bp[1] = *reinterpret_cast<const float4*>(pf + t + 12);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          bv[k] = *reinterpret_cast<const uint4*>(vr + t + 8 + 2 * k);
          acc0 = __fadd_rn(acc0, m0[2 * k]);
          acc1 = __fadd_rn(acc1, m1[2 * k]);
          acc0 = __fadd_rn(acc0, m0[2 * k + 1]);
          acc1 = __fadd_rn(acc1, m1[2 * k + 1]);
        }
        {
          const float pb[8] = {bp[0].x, bp[0].y, bp[0].z, bp[0].w, bp[1].x, bp[1].y, bp[1].z, bp[1].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            m0[2 * k] = __fmul_rn(pb[2 * k], __uint_as_float(bv[k].x));
            m1[2 * k] = __fmul_rn(pb[2 * k], __uint_as_float(bv[k].y));
            m0[2 * k + 1] = __fmul_rn(pb[2 * k + 1], __uint_as_float(bv[k].z));
            m1[2 * k + 1] = __fmul_rn(pb[2 * k + 1], __uint_as_float(bv[k].w));
          }
        }
        const int tn = t + 16 < len16 ? t + 16 : t;   // the last trip re-reads in range
        ap[0] = *reinterpret_cast<const float4*>(pf + tn);
        ap[1] = *reinterpret_cast<const float4*>(pf + tn + 4);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          av[k] = *reinterpret_cast<const uint4*>(vr + tn + 2 * k);
          acc0 = __fadd_rn(acc0, m0[2 * k]);
          acc1 = __fadd_rn(acc1, m1[2 * k]);
          acc0 = __fadd_rn(acc0, m0[2 * k + 1]);
          acc1 = __fadd_rn(acc1, m1[2 * k + 1]);
        }
      }
      // the last (fewer than 16) positions: all reads first, then the steps
      const int rem = len - len16;
      float tp[16];
      uint64_t tv[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        tp[k] = k < rem ? pf[len16 + k] : 0.0f;
        tv[k] = k < rem ? vr[len16 + k] : 0ull;
      }
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (k < rem) {
          acc0 = __fadd_rn(acc0, __fmul_rn(tp[k], __uint_as_float((uint32_t)tv[k])));
          acc1 = __fadd_rn(acc1, __fmul_rn(tp[k], __uint_as_float((uint32_t)(tv[k] >> 32))));
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[si]);
    p += len;
  }
  float* op = out + ((int64_t)b * n_head + kh * G + g) * HD + d0 + 2 * j;
  op[0] = acc0;
  op[1] = acc1;
}

// The V cache as 2-D tensors over its rows ([n_seq*n_kv*cap rows]), boxes of
// kPvCh rows: fp16 rows of hd values, ds-dim boxes; Q8_0 rows as bytes
// (boxes of pv_code_bytes(ds) codes) and as 16-bit words (boxes of the 8
// scale words from byte hd).  For fp16 `smap` is a copy of `vmap`.
int make_v_maps(const void* vc, int vt, int64_t n_rows, int hd, int ds, CUtensorMap* vmap, CUtensorMap* smap) {
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess || !fn) {
      set_error("attention: cuTensorMapEncodeTiled unavailable");
      return B2_ERR_CUDA;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  const cuuint64_t rb = (cuuint64_t)kv_row_bytes(vt, hd);
  const cuuint32_t estr[2] = {1, 1};
  auto enc = [&](CUtensorMap* map, CUtensorMapDataType dt, cuuint64_t inner, cuuint32_t box_inner) -> int {
    const cuuint64_t dims[2] = {inner, (cuuint64_t)n_rows};
    const cuuint64_t strides[1] = {rb};
    const cuuint32_t box[2] = {box_inner, (cuuint32_t)kPvCh};
    const CUresult r = encode(map, dt, 2, const_cast<void*>(vc), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("attention: V tensor map rejected (CUresult %d)", (int)r);
      return B2_ERR_CUDA;
    }
    return B2_OK;
  };
  int rc;
  if (vt == B2_Q8_0 || vt == B2_Q4_0) {
    const cuuint32_t cb = (cuuint32_t)(vt == B2_Q8_0 ? pv_code_bytes(ds) : pv_code_bytes_q4(ds));
    if ((rc = enc(vmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, rb, cb))) return rc;
    return enc(smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, rb / 2, 8);
  }
  if ((rc = enc(vmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, (cuuint64_t)hd, (cuuint32_t)ds))) return rc;
  *smap = *vmap;
  return B2_OK;
}

template <int HD, int G, int KT, int VT>
int launch_hd_g(const float* q, int n_tok, int n_head, int n_kv, const int32_t* pos, const int32_t* seq,
                const void* kc, const void* vc, const KvSeqState* st, int n_seq, int cap, float* scratch, float* out,
                cudaStream_t s, int* status) {
  constexpr int DS = 64 / G;
  const size_t sm = scores_smem_bytes<HD, G, KT>();
  B2_CUDA_TRY(
      cudaFuncSetAttribute(attn_scores_kernel<HD, G, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  const float scale = 1.0f / sqrtf((float)HD);
  const dim3 chunks((cap + kScoreP - 1) / kScoreP, n_kv, n_tok);
  int rc = launch_pdl(attn_scores_kernel<HD, G, KT>, chunks, dim3(kScoreP), sm, s, q, n_head, n_kv, pos, seq,
                      static_cast<const uint8_t*>(kc), st, n_seq, cap, scale, scratch, status, 1.0f, -0.0f);
  if (rc) return rc;
  rc = launch_pdl(attn_exp_kernel<G>, chunks, dim3(kScoreP), 0, s, pos, seq, n_seq, n_kv, cap, scratch);
  if (rc) return rc;
  CUtensorMap vmap, smap;
  if ((rc = make_v_maps(vc, VT, (int64_t)n_seq * n_kv * cap, HD, DS, &vmap, &smap))) return rc;
  // Shared memory per CTA: what the grid leaves when its CTAs are spread
  // evenly over the SMs.  It holds up to kPvStagesMax stages of the P.V
  // phase, and in the sum phase a window of E rows: the whole context where
  // it fits (one copy round instead of several).
  const int64_t ctas = (int64_t)(HD / DS) * n_kv * n_tok;
  const int per_sm = (int)std::min<int64_t>(4, std::max<int64_t>(1, (ctas + sm_count() - 1) / sm_count()));
  const size_t budget = (size_t)227 * 1024 / per_sm - 1024 - 256;
  const size_t sb = pv_stage_bytes<G, VT>(DS);
  const int ns = (int)std::max<size_t>(2, std::min<size_t>(kPvStagesMax, budget / sb));
  const size_t e_all = (size_t)cap_s(cap) * gp_of(G) * 4;
  const size_t area = std::max((size_t)ns * sb, std::min(budget, e_all) / 128 * 128);
  const int wa = (int)(area / (gp_of(G) * 4)) & ~3;
  const size_t smv = 256 + area;
  B2_CUDA_TRY(cudaFuncSetAttribute(attn_pv_kernel<HD, G, VT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smv));
  return launch_pdl(attn_pv_kernel<HD, G, VT>, dim3(HD / DS, n_kv, n_tok), dim3(64), smv, s, pos, seq, vmap, smap, st,
                    n_seq, n_head, n_kv, cap, (const float*)scratch, out, status, ns, wa, 1.0f, -0.0f);
}

template <int HD, int G>
int launch_types(const float* q, int n_tok, int n_head, int n_kv, const int32_t* pos, const int32_t* seq,
                 const void* kc, int kt, const void* vc, int vt, const KvSeqState* st, int n_seq, int cap,
                 float* scratch, float* out, cudaStream_t s, int* status) {
#define B2_ATTN_TYPES(KT, VT)                                                                                    \
  if (kt == KT && vt == VT)                                                                                      \
    return launch_hd_g<HD, G, KT, VT>(q, n_tok, n_head, n_kv, pos, seq, kc, vc, st, n_seq, cap, scratch, out, s, \
                                      status);
  B2_ATTN_TYPES(B2_F16, B2_F16)
  B2_ATTN_TYPES(B2_F16, B2_Q8_0)
  B2_ATTN_TYPES(B2_F16, B2_Q4_0)
  B2_ATTN_TYPES(B2_Q8_0, B2_F16)
  B2_ATTN_TYPES(B2_Q8_0, B2_Q8_0)
  B2_ATTN_TYPES(B2_Q8_0, B2_Q4_0)
  B2_ATTN_TYPES(B2_Q4_0, B2_F16)
  B2_ATTN_TYPES(B2_Q4_0, B2_Q8_0)
  B2_ATTN_TYPES(B2_Q4_0, B2_Q4_0)
#undef B2_ATTN_TYPES
  set_error("attention: KV cache types %d / %d (F16, Q8_0 or Q4_0)", kt, vt);
  return B2_ERR_INVALID;
}

}  // namespace

size_t attn_scratch_floats(int n_tok, int n_head, int n_kv, int cap) {
  const int G = n_kv > 0 ? n_head / n_kv : 1;
  return (size_t)n_tok * n_kv * (size_t)group_floats(G, cap);
}

int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const void* kc, int kt, const void* vc, int vt, const KvSeqState* st, int n_seq, int cap,
                     float* scratch, float* out, cudaStream_t s, int* status) {
  B2_CHECK_ARG(n_kv > 0 && n_head % n_kv == 0 && scratch && out && cap > 0, "attention arguments");
  B2_CHECK_ARG((reinterpret_cast<uintptr_t>(scratch) & 15) == 0, "attention scratch must be 16-byte aligned");
  const int G = n_head / n_kv;
#define B2_ATTN_CASE(HDV, GV) \
  if (hd == HDV && G == GV)   \
    return launch_types<HDV, GV>(q, n_tok, n_head, n_kv, pos, seq, kc, kt, vc, vt, st, n_seq, cap, scratch, out, s, \
                                 status);
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
