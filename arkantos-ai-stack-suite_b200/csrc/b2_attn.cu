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
// out so that as many chains as possible run side by side and no chain
// waits on global-memory latency.
//
// Scratch per (query, kv head) group: the scores S [G][capS] (capS = cap
// rounded up to 4) and the probabilities P [capS][GP] (GP = max(G, 4)).
//
// Two kernels:
//   * attn_scores_kernel: one CTA per (128-position chunk, kv head, query).
//     The chunk's K rows arrive by 1-D bulk copies (one per run of
//     consecutive cache slots: the pinned prefix, the ring's tail, its head)
//     while q goes to shared memory; thread t scores position t against the
//     G query heads of the group (G chains over the dims, two heads per
//     packed f32x2 operation) and writes s_t.  The last CTA of each (query,
//     kv head) to finish runs the softmax of those G heads: windows of the
//     score rows come into shared memory by bulk copies, the maximum and
//     e_t are computed there by all threads, lanes 0..G-1 add e_t in
//     position order, and p_t = e_t·(1/l) goes to P.
//   * attn_pv_kernel: one CTA per (slice of 64/G dims, kv head, query).  A
//     loader warp brings each chunk of up to 128 positions in with one 2-D
//     tensor copy of the V slice and one bulk copy of the P rows, then turns
//     V into fp32 and p_t into (p_t, p_t) pairs; the chain warp's lane
//     (head, dim pair) runs out += p_t·v_t over the positions in order with
//     packed f32x2 operations.
// Queries whose sequence id or position is outside the cache attend to
// nothing and get zero outputs.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>

#include "b2_common.cuh"
#include "b2_layers.hpp"

namespace b2 {
namespace {

constexpr int kScoreP = 128;          // positions per scores CTA (one per thread)
constexpr int kWinFloats = 8192;      // softmax window: G x W floats in shared memory
constexpr int kPvCh = 128;            // positions per P.V chunk
constexpr int kPvStages = 4;

__host__ __device__ constexpr int gp_of(int g) { return g < 4 ? 4 : g; }
__host__ __device__ inline int cap_s(int cap) { return (cap + 3) & ~3; }
// floats of one (query, kv head) group: S [G][capS] then P [capS][GP]
__host__ __device__ inline int64_t group_floats(int g, int cap) { return (int64_t)cap_s(cap) * (g + gp_of(g)); }

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
  constexpr int NP = (G + 1) / 2;              // head pairs (the last one half used when G is odd)
  constexpr int GP = gp_of(G);
  constexpr int W = (kWinFloats / G) & ~3;     // softmax window positions
  constexpr int KB = P * HD * 2;               // K rows of the chunk
  constexpr int RB = KB > kWinFloats * 4 ? KB : kWinFloats * 4;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);    // [0] K rows, [1] softmax windows
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem + 128);   // [P][HD] (scores phase)
  float* ws = reinterpret_cast<float*>(smem + 128);         // [G][W] (softmax phase, same bytes)
  uint64_t* qs = reinterpret_cast<uint64_t*>(smem + 128 + RB);   // [HD][NP]: (q_2j[i], q_2j+1[i])
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
  const int capS = cap_s(cap);
  float* grp = sbuf + ((int64_t)b * n_kv + kh) * group_floats(G, cap);
  float* srow = grp;                           // head g's scores at srow + g * capS
  float* prow = grp + (int64_t)G * capS;       // position t's probabilities at prow + t * GP
  const KvSeqState sst = st ? st[s] : KvSeqState{0, 0};
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], (uint32_t)(n * HD * 2));
    const int64_t base = ((int64_t)s * n_kv + kh) * cap;
    for (int p = t0; p < t0 + n;) {
      const SlotRun r = slot_run(sst, p, t0 + n, cap, P);
      bulk_g2s(ks + (p - t0) * HD, kc + (base + r.slot) * HD, (uint32_t)(r.len * HD * 2), &bar[0]);
      p += r.len;
    }
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
    // the row of position t0 + tid, then the chains in dim order
    constexpr int NPc = HD / 8;
    const Ones k2{pack2(one, one), pack2(neg_zero, neg_zero)};
    const uint8_t* rp = reinterpret_cast<const uint8_t*>(ks + tid * HD);
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
      srow[(int64_t)(2 * j) * capS + t] = __fmul_rn(lo, scale);
      if (2 * j + 1 < G) srow[(int64_t)(2 * j + 1) * capS + t] = __fmul_rn(hi, scale);
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
  const int n_win = (n_pos + W - 1) / W;
  uint32_t round = 0;
  // Brings window w of the G score rows into ws [G][W] (a bulk copy per row;
  // rows start on 16 bytes and the length rounds up to 4 floats inside capS).
  auto load_window = [&](int w) -> bool {
    const int p0 = w * W, len = min(W, n_pos - p0), len4 = (len + 3) & ~3;
    __syncthreads();   // every thread is done with the previous window
    if (tid == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&bar[1], (uint32_t)(G * len4 * 4));
      for (int g = 0; g < G; ++g) bulk_g2s(ws + g * W, srow + (int64_t)g * capS + p0, (uint32_t)(len4 * 4), &bar[1]);
    }
    const bool r = mbar_wait_bounded(&bar[1], round & 1, status, 9);
    ++round;
    return r;
  };
  // m: any order (a maximum)
  float mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) mg[g] = -FLT_MAX;
  for (int w = 0; w < n_win && ok; ++w) {
    ok = load_window(w);
    const int len = min(W, n_pos - w * W);
#pragma unroll
    for (int g = 0; g < G; ++g)
      for (int t = tid; t < len; t += P) {
        const float v = ws[g * W + t];
        if (v > mg[g]) mg[g] = v;
      }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mg[g] = fmaxf(mg[g], __shfl_xor_sync(0xffffffffu, mg[g], o));
    if (lane == 0) mh[warp][g] = mg[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) mg[g] = fmaxf(fmaxf(mh[0][g], mh[1][g]), fmaxf(mh[2][g], mh[3][g]));
  // e_t in the window (all threads), then the sums in position order (lanes 0..G-1)
  float l = 0.0f;
  for (int w = 0; w < n_win && ok; ++w) {
    if (n_win > 1) ok = load_window(w);
    const int len = min(W, n_pos - w * W);
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g)
      for (int t = tid; t < len; t += P) ws[g * W + t] = b2_expf_ref(__fsub_rn(ws[g * W + t], mg[g]));
    __syncthreads();
    if (tid < G) {
      const float* e = ws + tid * W;
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
  }
  if (tid < G) inv_l[tid] = __fdiv_rn(1.0f, l);
  __syncthreads();
  // p_t = e_t · (1/l) into P [t][GP]
  for (int w = 0; w < n_win && ok; ++w) {
    const int p0 = w * W, len = min(W, n_pos - p0);
    if (n_win > 1) {
      ok = load_window(w);
      __syncthreads();
#pragma unroll
      for (int g = 0; g < G; ++g)
        for (int t = tid; t < len; t += P) ws[g * W + t] = b2_expf_ref(__fsub_rn(ws[g * W + t], mg[g]));
      __syncthreads();
    }
    for (int i = tid; i < len * G; i += P) {
      const int t = i / G, g = i - t * G;
      prow[(int64_t)(p0 + t) * GP + g] = __fmul_rn(ws[g * W + t], inv_l[g]);
    }
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

template <int G>
__host__ __device__ constexpr size_t pv_stage_bytes(int ds) {
  // raw V (fp16) | raw P [CH][GP] | V fp32 | P pairs [CH][G]
  return (size_t)kPvCh * ds * 2 + (size_t)kPvCh * gp_of(G) * 4 + (size_t)kPvCh * ds * 4 + (size_t)kPvCh * G * 8;
}

// out[b][h][d] for the dims [slice*DS, slice*DS+DS) of the G heads of one kv
// head.  Warp 1: lane 0 issues each chunk's V rows (one 2-D tensor copy of
// kPvCh rows x DS dims from the first slot of a run) and P rows (one bulk
// copy) into a raw stage; the warp converts V to fp32 and P to (p, p)
// pairs.  Warp 0: lane (head g, dim pair j) runs out += p_t·v_t over the
// positions in order.
template <int HD, int G>
__global__ void __launch_bounds__(64) attn_pv_kernel(const int32_t* __restrict__ pos, const int32_t* __restrict__ seq,
                                                     const __grid_constant__ CUtensorMap vmap,
                                                     const KvSeqState* __restrict__ st, int n_seq, int n_head,
                                                     int n_kv, int cap, const float* __restrict__ sbuf,
                                                     float* __restrict__ out, int* status, float one, float neg_zero) {
  constexpr int DS = 64 / G;            // dims of the slice: G heads x DS/2 pairs = 32 chain lanes
  constexpr int CH = kPvCh, NS = kPvStages;
  constexpr int GP = gp_of(G);
  static_assert(HD % DS == 0 && DS % 8 == 0, "slice");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);   // [NS] raw stage landed
  uint64_t* conv = full + NS;                           // [NS] converted
  uint64_t* empty = conv + NS;                          // [NS] chain done with the stage
  constexpr size_t SB = pv_stage_bytes<G>(DS);
  uint8_t* stages = smem + 128;
  const int slice = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&conv[i], 1);
      mbar_init(&empty[i], 1);
    }
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
  const float* prow = sbuf + ((int64_t)b * n_kv + kh) * group_floats(G, cap) + (int64_t)G * cap_s(cap);
  bool ok = true;
  if (warp == 1) {
    int p_iss = 0, c_iss = 0;
    auto issue = [&](int si) {
      const SlotRun r = slot_run(sst, p_iss, n_pos, cap, CH);
      uint8_t* sp = stages + si * SB;
      mbar_arrive_expect_tx(&full[si], (uint32_t)(CH * DS * 2 + r.len * GP * 4));
      tma_load_2d(sp, &vmap, d0, row0 + (int)r.slot, &full[si]);
      bulk_g2s(sp + CH * DS * 2, prow + (int64_t)r.p * GP, (uint32_t)(r.len * GP * 4), &full[si]);
      p_iss += r.len;
      ++c_iss;
    };
    if (lane == 0)
      while (p_iss < n_pos && c_iss < NS) issue(c_iss % NS);
    __syncwarp();
    int p = 0;
    for (int c = 0; p < n_pos; ++c) {
      const int si = c % NS;
      const int len = slot_run(sst, p, n_pos, cap, CH).len;
      if (ok) ok = mbar_wait_bounded(&full[si], (uint32_t)((c / NS) & 1), status, 6);
      if (ok && c >= NS) ok = mbar_wait_bounded(&empty[si], (uint32_t)(((c / NS) - 1) & 1), status, 7);
      if (ok) {
        uint8_t* sp = stages + si * SB;
        const uint32_t* rv = reinterpret_cast<const uint32_t*>(sp);
        const float* rp = reinterpret_cast<const float*>(sp + CH * DS * 2);
        float* fv = reinterpret_cast<float*>(sp + CH * DS * 2 + CH * GP * 4);
        uint64_t* fp = reinterpret_cast<uint64_t*>(sp + CH * DS * 2 + CH * GP * 4 + CH * DS * 4);
        for (int i = lane; i < len * DS / 2; i += 32) {
          const uint32_t w2 = rv[i];
          fv[2 * i] = h2f((uint16_t)(w2 & 0xFFFFu));
          fv[2 * i + 1] = h2f((uint16_t)(w2 >> 16));
        }
        for (int i = lane; i < len * G; i += 32) {
          const int t = i / G, g = i - t * G;
          const float pv = rp[t * GP + g];
          fp[i] = pack2(pv, pv);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&conv[si]);
        if (ok && p_iss < n_pos) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(si);
        }
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
  // chain warp: lane = (head g, dim pair j)
  const int g = lane / (DS / 2), j = lane - g * (DS / 2);
  const Ones k2{pack2(one, one), pack2(neg_zero, neg_zero)};
  uint64_t acc = 0ull;
  int p = 0;
  for (int c = 0; p < n_pos; ++c) {
    const int si = c % NS;
    const int len = slot_run(sst, p, n_pos, cap, CH).len;
    if (ok) ok = mbar_wait_bounded(&conv[si], (uint32_t)((c / NS) & 1), status, 8);
    if (ok) {
      const uint8_t* sp = stages + si * SB;
      const float* vr = reinterpret_cast<const float*>(sp + CH * DS * 2 + CH * GP * 4) + 2 * j;
      const uint64_t* pr = reinterpret_cast<const uint64_t*>(sp + CH * DS * 2 + CH * GP * 4 + CH * DS * 4) + g;
      int t = 0;
      for (; t + 2 <= len; t += 2) {
        const uint64_t p0 = pr[t * G], p1 = pr[(t + 1) * G];
        const uint64_t v0 = *reinterpret_cast<const uint64_t*>(vr + t * DS);
        const uint64_t v1 = *reinterpret_cast<const uint64_t*>(vr + (t + 1) * DS);
        acc = mul_add2(acc, p0, v0, k2);
        acc = mul_add2(acc, p1, v1, k2);
      }
      if (t < len) acc = mul_add2(acc, pr[t * G], *reinterpret_cast<const uint64_t*>(vr + t * DS), k2);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[si]);
    p += len;
  }
  float o0, o1;
  unpack2(acc, o0, o1);
  float* op = out + ((int64_t)b * n_head + kh * G + g) * HD + d0 + 2 * j;
  op[0] = o0;
  op[1] = o1;
}

// The V cache as a 2-D tensor [n_seq*n_kv*cap rows][hd] of fp16, boxes of
// kPvCh rows x ds dims.
int make_v_map(const uint16_t* vc, int64_t n_rows, int hd, int ds, CUtensorMap* map) {
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
  const cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)n_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  const cuuint32_t box[2] = {(cuuint32_t)ds, (cuuint32_t)kPvCh};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(vc), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("attention: V tensor map rejected (CUresult %d)", (int)r);
    return B2_ERR_CUDA;
  }
  return B2_OK;
}

template <int HD, int G>
int launch_hd_g(const float* q, int n_tok, int n_head, int n_kv, const int32_t* pos, const int32_t* seq,
                const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int n_seq, int cap, float* scores,
                unsigned int* count, float* out, cudaStream_t s, int* status) {
  constexpr int NP = (G + 1) / 2;
  constexpr int DS = 64 / G;
  constexpr size_t KB = (size_t)kScoreP * HD * 2, RB = KB > kWinFloats * 4 ? KB : (size_t)kWinFloats * 4;
  const size_t sm = 128 + RB + (size_t)HD * NP * 8;
  B2_CUDA_TRY(cudaFuncSetAttribute(attn_scores_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  const float scale = 1.0f / sqrtf((float)HD);
  int rc = launch_pdl(attn_scores_kernel<HD, G>, dim3((cap + kScoreP - 1) / kScoreP, n_kv, n_tok), dim3(kScoreP), sm,
                      s, q, n_head, n_kv, pos, seq, kc, st, n_seq, cap, scale, scores, count, status, 1.0f, -0.0f);
  if (rc) return rc;
  CUtensorMap vmap;
  if ((rc = make_v_map(vc, (int64_t)n_seq * n_kv * cap, HD, DS, &vmap))) return rc;
  const size_t smv = 128 + (size_t)kPvStages * pv_stage_bytes<G>(DS);
  B2_CUDA_TRY(cudaFuncSetAttribute(attn_pv_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smv));
  return launch_pdl(attn_pv_kernel<HD, G>, dim3(HD / DS, n_kv, n_tok), dim3(64), smv, s, pos, seq, vmap, st, n_seq,
                    n_head, n_kv, cap, (const float*)scores, out, status, 1.0f, -0.0f);
}

}  // namespace

size_t attn_scratch_floats(int n_tok, int n_head, int n_kv, int cap) {
  const int G = n_kv > 0 ? n_head / n_kv : 1;
  return (size_t)n_tok * n_kv * (size_t)group_floats(G, cap);
}

int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int n_seq, int cap, float* scores,
                     unsigned int* count, float* out, cudaStream_t s, int* status) {
  B2_CHECK_ARG(n_kv > 0 && n_head % n_kv == 0 && scores && count && out && cap > 0, "attention arguments");
  B2_CHECK_ARG((reinterpret_cast<uintptr_t>(scores) & 15) == 0, "attention scratch must be 16-byte aligned");
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
