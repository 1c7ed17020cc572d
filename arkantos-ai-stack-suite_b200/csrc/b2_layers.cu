// Decoder-layer kernels around the GEMVs, in the order of the reference's
// forward_token (Singularity/src/core/cortex_a5_engine.cpp:1029-1293):
//   embed         token row dequantization (:1066-1105)
//   add_rmsnorm   residual add fused with RMSNorm (:1121, :1259-1266, :1284-1287)
//   rope_kv       RoPE on q/k (adjacent pairs, :1187-1192) + fp16 K/V store (:1195-1203)
//   attn_split / attn_combine
//                 split-K GQA decode attention over the fp16 cache (:1205-1254)
//   kv_shift      in-place K re-rotation for Milda's KV shift (Milda/src/engine.cpp:1642-1675)
//   argmax        greedy pick with top-2 margin (Milda/src/engine.cpp:1970 samples on host)
// Every kernel takes its per-step values (token ids, positions, sequence ids)
// from device buffers so a captured CUDA graph replays unchanged.
#include <float.h>

#include "b2_common.cuh"
#include "b2_layers.hpp"

namespace b2 {
namespace {

// ---- GGUF row dequantization (one element) -------------------------------------------------
// Same operation order as the oracle's dequantizer (pinned to gguf-py).
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* row, int64_t e) {
  switch (type) {
    case B2_F32: return reinterpret_cast<const float*>(row)[e];
    case B2_F16: return h2f(reinterpret_cast<const uint16_t*>(row)[e]);
    case B2_Q4_0: {
      const uint8_t* blk = row + (e / 32) * 18;
      const int j = (int)(e % 32);
      const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
      const uint8_t byte = blk[2 + (j & 15)];
      const int q = (j < 16 ? (byte & 15) : (byte >> 4)) - 8;
      return __fmul_rn((float)q, d);
    }
    case B2_Q8_0: {
      const uint8_t* blk = row + (e / 32) * 34;
      const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
      return __fmul_rn((float)(int8_t)blk[2 + e % 32], d);
    }
    case B2_Q4_K: {
      const uint8_t* bp = row + (e / 256) * 144;
      const int ee = (int)(e % 256), j = ee >> 5;
      const float d = h2f((uint16_t)(bp[0] | (bp[1] << 8)));
      const float dmin = h2f((uint16_t)(bp[2] | (bp[3] << 8)));
      const uint8_t* sc = bp + 4;
      int s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      const uint8_t byte = bp[16 + (ee >> 6) * 32 + (ee & 31)];
      const int q = (j & 1) ? (byte >> 4) : (byte & 15);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
    }
    case B2_Q6_K: {
      const uint8_t* bp = row + (e / 256) * 210;
      const int ee = (int)(e % 256);
      const int h = ee >> 7, g = (ee >> 5) & 3, l = ee & 31;
      const int lo = (bp[h * 64 + (g & 1) * 32 + l] >> (4 * (g >> 1))) & 15;
      const int hi = (bp[128 + h * 32 + l] >> (2 * g)) & 3;
      const float d = h2f((uint16_t)(bp[208] | (bp[209] << 8)));
      const float sc = (float)(int8_t)bp[192 + (ee >> 4)];
      return __fmul_rn(__fmul_rn(d, sc), (float)((lo | (hi << 4)) - 32));
    }
  }
  return 0.0f;
}

__global__ void embed_kernel(const int32_t* __restrict__ tokens, int n_vocab, int type, const uint8_t* __restrict__ table,
                             int64_t row_bytes, int n_embd, float* __restrict__ x) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  int t = tokens[b];
  if (t < 0 || t >= n_vocab) t = 0;   // out-of-range ids read row 0 (cortex_a5_engine.cpp:1037-1039)
  const uint8_t* row = table + (int64_t)t * row_bytes;
  for (int i = threadIdx.x; i < n_embd; i += blockDim.x) x[(int64_t)b * n_embd + i] = dequant_elem(type, row, i);
}

// ---- residual add + RMSNorm ----------------------------------------------------------------
// x += delta (when delta != nullptr); out = (x·scale)·w with the squares
// rounded to fp32 and summed in double, mean = (float)(sum/n),
// scale = 1/sqrtf(mean + eps) — ggml's rms_norm (llama.cpp CPU backend).
// A double sum of 2^12..2^15 fp32 squares is exact to far below fp32
// resolution, so the tree order here rounds to the same mean as the
// sequential CPU sum (bit-identical outputs, which keeps the following Q8
// activation codes identical even on exact rounding ties).
// With a tensor-parallel exchange (in.n > 0) the residual delta is the sum of
// the ranks' partial outputs in rank order, ((p0 + p1) + p2) + ..., read from
// the local gather buffer once every rank's flag shows this phase's epoch.
__global__ void add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w,
                                   float* __restrict__ out, int n, float eps, PeerIn in, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  float* xr = x + (int64_t)b * n;
  const float* dr = delta ? delta + (int64_t)b * n : nullptr;
  if (in.n) {
    if (threadIdx.x == 0) {
      wait_peer_flags(in.flags, in.n, *in.epoch, status, 3);
      __threadfence();
    }
    __syncthreads();
  }
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = xr[i];
    if (in.n) {
      const float* pp = in.parts + (int64_t)b * n + i;
      float sum = __ldcg(pp);
      for (int j = 1; j < in.n; ++j) sum = __fadd_rn(sum, __ldcg(pp + j * in.slot));
      v = __fadd_rn(v, sum);
      xr[i] = v;
    } else if (dr) {
      v = __fadd_rn(v, dr[i]);
      xr[i] = v;
    }
    ss += (double)__fmul_rn(v, v);
  }
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = __double2float_rn(__ddiv_rn(red[0], (double)n));
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  float* orow = out + (int64_t)b * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

// ---- RoPE + KV store -------------------------------------------------------------------------
__device__ __forceinline__ int64_t kv_slot(const KvSeqState& st, int p, int cap) {
  const int ring = cap - st.n_keep;
  if (p < st.n_keep || ring <= 0) return p;
  int r = (st.ring_head + (p - st.n_keep)) % ring;
  return st.n_keep + r;
}

__global__ void rope_kv_kernel(const float* __restrict__ qkv, int n_head, int n_kv, int hd, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ seq, const float* __restrict__ rope, float* __restrict__ q_out,
                               uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, const KvSeqState* __restrict__ st,
                               int cap) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int p = pos[b], s = seq[b];
  const int row_len = (n_head + 2 * n_kv) * hd;
  const float* src = qkv + (int64_t)b * row_len;
  const float* cs = rope + (int64_t)p * hd;
  const int64_t slot = kv_slot(st[s], p, cap);
  const int half = hd / 2;
  for (int i = threadIdx.x; i < (n_head + n_kv) * half; i += blockDim.x) {
    const int h = i / half, pr = i - h * half;
    const float x0 = src[h * hd + 2 * pr], x1 = src[h * hd + 2 * pr + 1];
    const float c = cs[2 * pr], sn = cs[2 * pr + 1];
    const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    if (h < n_head) {
      q_out[(int64_t)b * n_head * hd + h * hd + 2 * pr] = y0;
      q_out[(int64_t)b * n_head * hd + h * hd + 2 * pr + 1] = y1;
    } else {
      const int kh = h - n_head;
      uint16_t* dst = kc + (((int64_t)s * n_kv + kh) * cap + slot) * hd + 2 * pr;
      dst[0] = f2h_rn(y0);
      dst[1] = f2h_rn(y1);
    }
  }
  for (int i = threadIdx.x; i < n_kv * hd; i += blockDim.x) {
    const int kh = i / hd, d = i - kh * hd;
    vc[(((int64_t)s * n_kv + kh) * cap + slot) * hd + d] = f2h_rn(src[(n_head + n_kv) * hd + i]);
  }
}

// ---- split-K decode attention ----------------------------------------------------------------
// CTA (split, kv head, query): positions [split*P, split*P+P) ∩ [0, pos+1) of
// the query's sequence, for the G query heads sharing the kv head.  Writes
// unnormalised partial outputs with their running max and sum.
template <int HD, int G>
__global__ void __launch_bounds__(128) attn_split_kernel(const float* __restrict__ q, int n_head, int n_kv,
                                                         const int32_t* __restrict__ pos, const int32_t* __restrict__ seq,
                                                         const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
                                                         const KvSeqState* __restrict__ st, int cap, int P, float scale,
                                                         float* __restrict__ part_o, float* __restrict__ part_ml,
                                                         int n_split) {
  pdl_wait();
  pdl_launch_dependents();
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int n_pos = pos[b] + 1, s = seq[b];
  const int t0 = split * P, t1 = min(t0 + P, n_pos);
  const int hq0 = kh * G;
  float* po = part_o + (((int64_t)b * n_head + hq0) * n_split + split) * HD;
  float* pml = part_ml + (((int64_t)b * n_head + hq0) * n_split + split) * 2;
  if (t0 >= t1) {
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
      const int g = i / HD, d = i - g * HD;
      po[(int64_t)g * n_split * HD + d] = 0.0f;
    }
    if (threadIdx.x < G) {
      pml[(int64_t)threadIdx.x * n_split * 2 + 0] = -FLT_MAX;
      pml[(int64_t)threadIdx.x * n_split * 2 + 1] = 0.0f;
    }
    return;
  }
  extern __shared__ float sm[];
  float* qs = sm;               // [G][HD]
  float* sc = qs + G * HD;      // [G][P]
  __shared__ float red[G][4];
  const KvSeqState sst = st[s];
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x)
    qs[i] = q[((int64_t)b * n_head + hq0) * HD + i];
  __syncthreads();
  const uint16_t* kbase = kc + ((int64_t)s * n_kv + kh) * cap * HD;
  const uint16_t* vbase = vc + ((int64_t)s * n_kv + kh) * cap * HD;
  const int n = t1 - t0;
  // scores: one thread per position
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t slot = kv_slot(sst, t0 + i, cap);
    const uint4* kr = reinterpret_cast<const uint4*>(kbase + slot * HD);
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll 4
    for (int c = 0; c < HD / 8; ++c) {
      const uint4 u = __ldg(kr + c);
      const __half2* h2 = reinterpret_cast<const __half2*>(&u);
      float kf[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        kf[2 * j] = f.x;
        kf[2 * j + 1] = f.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g] = fmaf(qs[g * HD + c * 8 + j], kf[j], acc[g]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g * P + i] = __fmul_rn(acc[g], scale);
  }
  __syncthreads();
  // per-head max and exp-sum over this split
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = -FLT_MAX;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, sc[g * P + i]);
    m = warp_max(m);
    if (lane == 0) red[g][warp] = m;
  }
  __syncthreads();
  float mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) mg[g] = fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]));
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float e = b2_expf(__fsub_rn(sc[g * P + i], mg[g]));
      sc[g * P + i] = e;
      l = __fadd_rn(l, e);
    }
    l = warp_sum(l);
    if (lane == 0) red[g][warp] = l;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    pml[(int64_t)g * n_split * 2 + 0] = mg[g];
    pml[(int64_t)g * n_split * 2 + 1] = __fadd_rn(__fadd_rn(__fadd_rn(red[g][0], red[g][1]), red[g][2]), red[g][3]);
  }
  // P·V: threads over head dims (HD/2 __half2 pairs per thread group)
  constexpr int PAIRS = HD / 2;                     // 64 for HD=128, 32 for HD=64
  constexpr int TSPLIT = 128 / PAIRS;               // position interleave: 2 or 4
  const int pr = threadIdx.x % PAIRS, ts = threadIdx.x / PAIRS;
  float o0[G], o1[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o0[g] = o1[g] = 0.0f;
  for (int i = ts; i < n; i += TSPLIT) {
    const int64_t slot = kv_slot(sst, t0 + i, cap);
    const float2 v = __half22float2(__ldg(reinterpret_cast<const __half2*>(vbase + slot * HD) + pr));
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pgi = sc[g * P + i];
      o0[g] = fmaf(pgi, v.x, o0[g]);
      o1[g] = fmaf(pgi, v.y, o1[g]);
    }
  }
  __syncthreads();
  // reduce the TSPLIT position interleaves through shared memory (reuse qs)
  float* acc = qs;   // [TSPLIT][G][HD]
  if (TSPLIT * G * HD > G * HD + G * P) return;  // not reached for the instantiated shapes
#pragma unroll
  for (int g = 0; g < G; ++g) {
    acc[(ts * G + g) * HD + 2 * pr] = o0[g];
    acc[(ts * G + g) * HD + 2 * pr + 1] = o1[g];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i - g * HD;
    float v = 0.0f;
#pragma unroll
    for (int t = 0; t < TSPLIT; ++t) v = __fadd_rn(v, acc[(t * G + g) * HD + d]);
    po[(int64_t)g * n_split * HD + d] = v;
  }
}

// Combines the chunks of one query head: M = max m_s, L = Σ_s e^(m_s−M)·l_s,
// out = (Σ_s e^(m_s−M)·O_s) · (1/L), chunks in order, each step one rounded
// operation.
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int n_head,
                                    int hd, int n_split, float* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y;
  const float* ml = part_ml + ((int64_t)b * n_head + h) * n_split * 2;
  const float* po = part_o + ((int64_t)b * n_head + h) * n_split * hd;
  float M = -FLT_MAX;
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.0f;
  for (int s = 0; s < n_split; ++s)
    if (ml[2 * s + 1] > 0.0f) L = __fadd_rn(L, __fmul_rn(b2_expf(__fsub_rn(ml[2 * s], M)), ml[2 * s + 1]));
  const float invL = __fdiv_rn(1.0f, L);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float v = 0.0f;
    for (int s = 0; s < n_split; ++s)
      if (ml[2 * s + 1] > 0.0f)
        v = __fadd_rn(v, __fmul_rn(b2_expf(__fsub_rn(ml[2 * s], M)), po[(int64_t)s * hd + d]));
    out[((int64_t)b * n_head + h) * hd + d] = __fmul_rn(v, invL);
  }
}

// ---- KV shift ----------------------------------------------------------------------------
// Rotates K rows of logical positions [p_begin, p_end) of sequence s (slots
// computed with the state before the shift) by the angle table cs[hd] of the
// position delta, in place: fp16 -> fp32 -> rotate -> fp16 (RNE).
__global__ void kv_shift_kernel(uint16_t* __restrict__ kc, int n_kv, int hd, int s, KvSeqState stt, int cap, int p_begin,
                                int p_end, const float* __restrict__ cs) {
  const int half = hd / 2;
  const int64_t total = (int64_t)(p_end - p_begin) * n_kv * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int pr = (int)(i % half);
    const int kh = (int)((i / half) % n_kv);
    const int p = p_begin + (int)(i / ((int64_t)half * n_kv));
    const int64_t slot = kv_slot(stt, p, cap);
    uint16_t* row = kc + (((int64_t)s * n_kv + kh) * cap + slot) * hd;
    const float x0 = h2f(row[2 * pr]), x1 = h2f(row[2 * pr + 1]);
    const float c = cs[2 * pr], sn = cs[2 * pr + 1];
    row[2 * pr] = f2h_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    row[2 * pr + 1] = f2h_rn(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
  }
}

// Moves K/V rows of logical [src0, src0+n) to logical [dst0, dst0+n) of one
// sequence (dst0 < src0, processed in ascending order by a single CTA per
// head so overlapping ranges move safely), rotating K by cs (delta table).
__global__ void kv_compact_kernel(uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int n_kv, int hd, int s,
                                  KvSeqState stt, int cap, int dst0, int src0, int n, const float* __restrict__ cs) {
  const int kh = blockIdx.x;
  const int half = hd / 2;
  for (int t = 0; t < n; ++t) {
    const int64_t ss = kv_slot(stt, src0 + t, cap), ds = kv_slot(stt, dst0 + t, cap);
    uint16_t* ksrc = kc + (((int64_t)s * n_kv + kh) * cap + ss) * hd;
    uint16_t* kdst = kc + (((int64_t)s * n_kv + kh) * cap + ds) * hd;
    uint16_t* vsrc = vc + (((int64_t)s * n_kv + kh) * cap + ss) * hd;
    uint16_t* vdst = vc + (((int64_t)s * n_kv + kh) * cap + ds) * hd;
    float y0 = 0.f, y1 = 0.f;
    uint16_t vv0 = 0, vv1 = 0;
    if (threadIdx.x < half) {
      const int pr = threadIdx.x;
      const float x0 = h2f(ksrc[2 * pr]), x1 = h2f(ksrc[2 * pr + 1]);
      const float c = cs[2 * pr], sn = cs[2 * pr + 1];
      y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
      vv0 = vsrc[2 * pr];
      vv1 = vsrc[2 * pr + 1];
    }
    __syncthreads();
    if (threadIdx.x < half) {
      const int pr = threadIdx.x;
      kdst[2 * pr] = f2h_rn(y0);
      kdst[2 * pr + 1] = f2h_rn(y1);
      vdst[2 * pr] = vv0;
      vdst[2 * pr + 1] = vv1;
    }
    __syncthreads();
  }
}

// ---- greedy argmax -----------------------------------------------------------------------
// Logits of token b, vocabulary entry v, live at
//   logits[(v / v_local) * n_tok * v_local + b * v_local + v % v_local]
// (tensor-parallel gather layout; v_local = n_vocab without TP).  Ties pick
// the lowest id.  Writes id, top-1 value and top-1 − top-2 margin.  With a
// feed (device-side greedy loop) it also makes the id the next step's token of
// row b, advances the row's position and appends the id to the row's output
// list; the step's other kernels have finished reading tok/pos by then.
__global__ void argmax_kernel(const float* __restrict__ logits, int n_tok, int n_vocab, int v_local,
                              int32_t* __restrict__ ids, float* __restrict__ top, GreedyFeed feed, PeerIn in,
                              int* status) {
  pdl_wait();
  if (!feed.tok) pdl_launch_dependents();
  if (in.n) {   // the ranks' head shards arrive in the gather layout
    if (threadIdx.x == 0) {
      wait_peer_flags(in.flags, in.n, *in.epoch, status, 4);
      __threadfence();
    }
    __syncthreads();
  }
  const int b = blockIdx.x;
  float v1 = -FLT_MAX, v2 = -FLT_MAX;
  int i1 = 0x7fffffff;
  for (int v = threadIdx.x; v < n_vocab; v += blockDim.x) {
    const float x = __ldcg(logits + (int64_t)(v / v_local) * n_tok * v_local + (int64_t)b * v_local + v % v_local);
    if (x > v1 || (x == v1 && v < i1)) {
      v2 = v1;
      v1 = x;
      i1 = v;
    } else if (x > v2) {
      v2 = x;
    }
  }
  __shared__ float s1[32], s2[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a1 = __shfl_xor_sync(0xffffffffu, v1, o);
    const float a2 = __shfl_xor_sync(0xffffffffu, v2, o);
    const int ai = __shfl_xor_sync(0xffffffffu, i1, o);
    if (a1 > v1 || (a1 == v1 && ai < i1)) {
      v2 = fmaxf(v1, a2);
      v1 = a1;
      i1 = ai;
    } else {
      v2 = fmaxf(v2, a1);
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s1[w] = v1;
    s2[w] = v2;
    si[w] = i1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b1 = s1[0], b2 = s2[0];
    int bi = si[0];
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
      if (s1[k] > b1 || (s1[k] == b1 && si[k] < bi)) {
        b2 = fmaxf(b1, s2[k]);
        b1 = s1[k];
        bi = si[k];
      } else {
        b2 = fmaxf(b2, s1[k]);
      }
    }
    ids[b] = bi;
    top[2 * b] = b1;
    top[2 * b + 1] = b1 - b2;
    if (feed.tok) {
      feed.tok[b] = bi;
      feed.pos[b] += 1;
      const int t = feed.count[b];
      if (t < feed.cap) feed.out[(int64_t)t * n_tok + b] = bi;
      feed.count[b] = t + 1;
    }
  }
}

template <typename K, typename... Args>
int launch_pdl(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...));
  return B2_OK;
}

}  // namespace

int launch_embed(const int32_t* tokens, int n_tok, int n_vocab, int type, const uint8_t* table, int64_t row_bytes,
                 int n_embd, float* x, cudaStream_t s) {
  return launch_pdl(embed_kernel, dim3(n_tok), dim3(256), 0, s, tokens, n_vocab, type, table, row_bytes, n_embd, x);
}

int launch_add_rmsnorm(float* x, const float* delta, const float* w, float* out, int n_tok, int n, float eps,
                       cudaStream_t s, const PeerIn* in, int* status) {
  return launch_pdl(add_rmsnorm_kernel, dim3(n_tok), dim3(512), 0, s, x, delta, w, out, n, eps, in ? *in : PeerIn{},
                    status);
}

int launch_rope_kv(const float* qkv, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                   const float* rope, float* q_out, uint16_t* kc, uint16_t* vc, const KvSeqState* st, int cap,
                   cudaStream_t s) {
  return launch_pdl(rope_kv_kernel, dim3(n_tok), dim3(256), 0, s, qkv, n_head, n_kv, hd, pos, seq, rope, q_out, kc, vc,
                    st, cap);
}

int attn_splits(int cap, int P) { return (cap + P - 1) / P; }

int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int cap, int P, float* part_o,
                     float* part_ml, float* out, cudaStream_t s) {
  const int G = n_head / n_kv;
  const int n_split = attn_splits(cap, P);
  const float scale = 1.0f / sqrtf((float)hd);
  const dim3 grid(n_split, n_kv, n_tok);
  int rc = B2_ERR_UNSUPPORTED;
  auto smem_for = [&](int g) {
    const size_t a = (size_t)(g * hd + g * P) * 4;
    const size_t b = (size_t)(128 / (hd / 2)) * g * hd * 4;
    return std::max(a, b);
  };
#define B2_ATTN_CASE(HDV, GV)                                                                                       \
  if (hd == HDV && G == GV) {                                                                                       \
    const size_t sm = smem_for(GV);                                                                                 \
    if (sm > 48 * 1024)                                                                                             \
      B2_CUDA_TRY(cudaFuncSetAttribute(attn_split_kernel<HDV, GV>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                       (int)sm));                                                                   \
    rc = launch_pdl(attn_split_kernel<HDV, GV>, grid, dim3(128), sm, s, q, n_head, n_kv, pos, seq, kc, vc, st, cap, \
                    P, scale, part_o, part_ml, n_split);                                                            \
  }
  B2_ATTN_CASE(128, 1)
  B2_ATTN_CASE(128, 2)
  B2_ATTN_CASE(128, 4)
  B2_ATTN_CASE(128, 8)
  B2_ATTN_CASE(64, 1)
  B2_ATTN_CASE(64, 2)
  B2_ATTN_CASE(64, 4)
  B2_ATTN_CASE(64, 8)
#undef B2_ATTN_CASE
  if (rc == B2_ERR_UNSUPPORTED) {
    set_error("attention: unsupported head_dim %d / group %d", hd, G);
    return rc;
  }
  if (rc != B2_OK) return rc;
  return launch_pdl(attn_combine_kernel, dim3(n_head, n_tok), dim3(hd), 0, s, (const float*)part_o,
                    (const float*)part_ml, n_head, hd, n_split, out);
}

int launch_kv_shift(uint16_t* kc, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int p_begin, int p_end,
                    const float* cs, cudaStream_t s) {
  if (p_end <= p_begin) return B2_OK;
  const int64_t total = (int64_t)(p_end - p_begin) * n_kv * (hd / 2);
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 4 * kSMs);
  kv_shift_kernel<<<grid, 256, 0, s>>>(kc, n_kv, hd, seq, st, cap, p_begin, p_end, cs);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_kv_compact(uint16_t* kc, uint16_t* vc, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int dst0,
                      int src0, int n, const float* cs, cudaStream_t s) {
  if (n <= 0) return B2_OK;
  kv_compact_kernel<<<n_kv, std::max(32, hd / 2), 0, s>>>(kc, vc, n_kv, hd, seq, st, cap, dst0, src0, n, cs);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_argmax(const float* logits, int n_tok, int n_vocab, int v_local, int32_t* ids, float* top, cudaStream_t s,
                  const GreedyFeed& feed, const PeerIn* in, int* status) {
  return launch_pdl(argmax_kernel, dim3(n_tok), dim3(1024), 0, s, logits, n_tok, n_vocab, v_local, ids, top, feed,
                    in ? *in : PeerIn{}, status);
}

}  // namespace b2
