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
#include "b2_quant.cuh"

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

// Residual add + RMSNorm fused with the next GEMV's activation quantization:
// one CTA per token, thread i owning values [8i, 8i+8) (n = 8·blockDim), so
// warp w holds Q8_K super-block w and four consecutive lanes one Q8_0 block.
// The residual sum, the double sum of squares and the scaling are the same
// operations as add_rmsnorm_kernel; the quantizers are the reference's
// (b2_quant.cuh) and write the image the GEMV copies.
__global__ void add_rmsnorm_q_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                     const float* __restrict__ w, float* __restrict__ out, int n, float eps, PeerIn in,
                                     int* status, ActImage img) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, i0 = 8 * tid;
  float* xr = x + (int64_t)b * n + i0;
  if (in.n) {
    if (tid == 0) {
      wait_peer_flags(in.flags, in.n, *in.epoch, status, 3);
      __threadfence();
    }
    __syncthreads();
  }
  float v[8];
  {
    const float4 a0 = *reinterpret_cast<const float4*>(xr), a1 = *reinterpret_cast<const float4*>(xr + 4);
    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
    v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
  }
  if (in.n || delta) {
    float dsum[8];
    if (in.n) {
      for (int r = 0; r < in.n; ++r) {
        const float* pp = in.parts + r * in.slot + (int64_t)b * n + i0;
        const float4 p0 = __ldcg(reinterpret_cast<const float4*>(pp)), p1 = __ldcg(reinterpret_cast<const float4*>(pp + 4));
        const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) dsum[j] = r ? __fadd_rn(dsum[j], pv[j]) : pv[j];
      }
    } else {
      const float* dr = delta + (int64_t)b * n + i0;
      const float4 d0 = *reinterpret_cast<const float4*>(dr), d1 = *reinterpret_cast<const float4*>(dr + 4);
      dsum[0] = d0.x; dsum[1] = d0.y; dsum[2] = d0.z; dsum[3] = d0.w;
      dsum[4] = d1.x; dsum[5] = d1.y; dsum[6] = d1.z; dsum[7] = d1.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], dsum[j]);
    *reinterpret_cast<float4*>(xr) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(xr + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += (double)__fmul_rn(v[j], v[j]);
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    double t = tid < (blockDim.x >> 5) ? red[tid] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (tid == 0) red[0] = t;
  }
  __syncthreads();
  const float mean = __double2float_rn(__ddiv_rn(red[0], (double)n));
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  float y[8];
  {
    const float4 w0 = *reinterpret_cast<const float4*>(w + i0), w1 = *reinterpret_cast<const float4*>(w + i0 + 4);
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__fmul_rn(v[j], scale), wv[j]);
  }
  if (out) {
    float* orow = out + (int64_t)b * n + i0;
    *reinterpret_cast<float4*>(orow) = make_float4(y[0], y[1], y[2], y[3]);
    *reinterpret_cast<float4*>(orow + 4) = make_float4(y[4], y[5], y[6], y[7]);
  }
  if (img.type == B2_Q4_K || img.type == B2_Q6_K) {
    int8_t q[8];
    int bs = 0;
    const float d = quant_q8_k_lane(y, q, &bs);
    store_q8k_unit(img, b, tid >> 5, q, d, bs);
  } else {
    // Q8_0 block tid/4 over lanes 4k..4k+3 (ref_quantize_row_q8_0)
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fmul_rn(amax, 1.0f / 127.0f);
    const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
    uint32_t wd[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sc = __fmul_rn(y[j], id);
      const float tt = sc >= 0.0f ? __fadd_rn(sc, 0.5f) : __fsub_rn(sc, 0.5f);
      int q = __float2int_rz(tt);
      q = q < -127 ? -127 : (q > 127 ? 127 : q);
      sum += q;
      wd[j >> 2] |= ((uint32_t)(uint8_t)q) << (8 * (j & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    uint32_t wb[8];
    const int g0 = lane & ~3;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      wb[2 * m] = __shfl_sync(0xffffffffu, wd[0], g0 + m);
      wb[2 * m + 1] = __shfl_sync(0xffffffffu, wd[1], g0 + m);
    }
    if ((lane & 3) == 0) store_q8_0_block(img, b, tid >> 2, wb, h2f(f2h_rn(d)), sum);
  }
}

// ---- RoPE + KV store -------------------------------------------------------------------------

__global__ void rope_kv_kernel(const float* __restrict__ qkv, int n_head, int n_kv, int hd, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ seq, const float* __restrict__ rope, float* __restrict__ q_out,
                               uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, const KvSeqState* __restrict__ st,
                               int n_seq, int cap) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int p = pos[b], s = seq[b];
  if (s < 0 || s >= n_seq || p < 0 || p >= cap) {   // outside the cache: zero q, store nothing
    for (int i = threadIdx.x; i < n_head * hd; i += blockDim.x) q_out[(int64_t)b * n_head * hd + i] = 0.0f;
    return;
  }
  const int row_len = (n_head + 2 * n_kv) * hd;
  const float* src = qkv + (int64_t)b * row_len;
  const float* cs = rope + (int64_t)p * hd;
  const int64_t slot = kv_slot(st ? st[s] : KvSeqState{0, 0}, p, cap);
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
// CTA (chunk, kv head, query): positions [chunk*128, chunk*128+128) ∩ [0, pos+1)
// of the query's sequence, for the G query heads sharing the kv head.  The
// chunk's K and V rows are brought into shared memory by cp.async.bulk (1-D
// TMA; a chunk crossing the ring's seam or the pinned prefix is up to three
// copies) while q goes to shared memory; then, per head:
//   scores: lane i of an 8-lane group holds dims [B*i, B*i+B) and
//     [HD/2 + B*i, HD/2 + B*i + B) (B = HD/16) of q and k (16-byte rows of a
//     position per group, so the K reads are bank-conflict free); an fmaf
//     chain over its dims in that order, a butterfly over the 8 lanes (xor 4,
//     2, 1), times 1/sqrt(HD).  Each lane group scores 4 positions against
//     all G heads at once (q from shared memory, packed f32x2 FMAs);
//   m = the chunk's max; e = exp(s − m); the chunk sum l = ((W0 + W1) + W2) + W3
//     with W_w the 32-lane butterfly (xor 16..1) of e over positions 32w..32w+31;
//   P·V: output dim d keeps four sums a_r of e·v over the positions i with
//     i mod 4 == r (fmaf chains in position order; warp r of a dim half takes
//     them, one position for all heads at a time), then (a0 + a1) + (a2 + a3).
// Writes the unnormalised partial output with its max and sum.  With
// fz.count, the last CTA of each (query, kv head) to finish also combines the
// chunks (attn_combine's arithmetic) into fz.out and, with fz.img, quantizes
// those G·HD outputs into the O projection's activation image.  Every wait is
// bounded; a query outside the cache attends to nothing.
constexpr int kAttnP = 128;
struct AttnFuse {
  unsigned int* count = nullptr;   // [n_tok][n_kv] arrivals, zero between launches (null: separate combine)
  float* out = nullptr;            // [n_tok][n_head][hd]
  ActImage img;                    // O projection image (img.img null: none)
};

// Two fp32 FMAs in one instruction (fma.rn.f32x2): each lane is rounded like fmaf.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// B fp16 values at p (16-byte aligned for B = 8, 8-byte for B = 4) -> fp32.
template <int B>
__device__ __forceinline__ void ld_half_row(const uint16_t* p, float (&f)[B]) {
  if constexpr (B == 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[2 * e] = h2f((uint16_t)(ww[e] & 0xFFFFu));
      f[2 * e + 1] = h2f((uint16_t)(ww[e] >> 16));
    }
  } else {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    f[0] = h2f((uint16_t)(w.x & 0xFFFFu));
    f[1] = h2f((uint16_t)(w.x >> 16));
    f[2] = h2f((uint16_t)(w.y & 0xFFFFu));
    f[3] = h2f((uint16_t)(w.y >> 16));
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(256, 3) attn_chunk_kernel(const float* __restrict__ q, int n_head, int n_kv,
                                                            const int32_t* __restrict__ pos,
                                                            const int32_t* __restrict__ seq,
                                                            const uint16_t* __restrict__ kc,
                                                            const uint16_t* __restrict__ vc,
                                                            const KvSeqState* __restrict__ st, int n_seq, int cap,
                                                            float scale, float* __restrict__ part_o,
                                                            float* __restrict__ part_ml, int n_split, int* status,
                                                            AttnFuse fz) {
  constexpr int P = kAttnP, B = HD / 16;
  constexpr int PAIRS = HD / 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);        // [0]: K rows, [1]: V rows
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem + 128);   // [P][HD]
  uint16_t* vs = ks + P * HD;                                 // [P][HD]
  float* qs = reinterpret_cast<float*>(vs + P * HD);          // [G][HD]
  float* sc = qs + G * HD;                                    // [P][G]: scores, then e
  __shared__ float mh[G], lh[G], wred[G][4];
  __shared__ unsigned int last_cta;
  pdl_wait();
  pdl_launch_dependents();
  const int chunk = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int s = seq[b], pb = pos[b];
  const int n_pos = (s >= 0 && s < n_seq && pb >= 0 && pb < cap) ? pb + 1 : 0;
  const int t0 = chunk * P, n = min(P, n_pos - t0);
  const int hq0 = kh * G;
  float* po = part_o + (((int64_t)b * n_head + hq0) * n_split + chunk) * HD;
  float* pml = part_ml + (((int64_t)b * n_head + hq0) * n_split + chunk) * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (n <= 0) {
    for (int i = tid; i < G * HD; i += blockDim.x) po[(int64_t)(i / HD) * n_split * HD + i % HD] = 0.0f;
    if (tid < G) {
      pml[(int64_t)tid * n_split * 2 + 0] = -FLT_MAX;
      pml[(int64_t)tid * n_split * 2 + 1] = 0.0f;
    }
  } else {
    const KvSeqState sst = st ? st[s] : KvSeqState{0, 0};
    const int64_t base = ((int64_t)s * n_kv + kh) * cap;   // row of slot 0
    if (tid == 0) {
      mbar_init(&bar[0], 1);
      mbar_init(&bar[1], 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(&bar[0], (uint32_t)(n * HD * 2));
      mbar_arrive_expect_tx(&bar[1], (uint32_t)(n * HD * 2));
      // logical positions [t0, t0+n) as runs of consecutive slots; all K
      // runs first, so the scores can start while V is still arriving
      for (int kv = 0; kv < 2; ++kv) {
        int p = t0;
        while (p < t0 + n) {
          const int64_t slot = kv_slot(sst, p, cap);
          int len = t0 + n - p;
          if (p < sst.n_keep) len = min(len, sst.n_keep - p);
          else len = (int)min((int64_t)len, (int64_t)cap - slot);   // up to the end of the ring
          bulk_g2s((kv ? vs : ks) + (p - t0) * HD, (kv ? vc : kc) + (base + slot) * HD, (uint32_t)(len * HD * 2),
                   &bar[kv]);
          p += len;
        }
      }
    }
    // q of the G heads into shared memory while the copies fly
    {
      const float4* qg = reinterpret_cast<const float4*>(q + ((int64_t)b * n_head + hq0) * HD);
      for (int i = tid; i < G * HD / 4; i += blockDim.x) reinterpret_cast<float4*>(qs)[i] = qg[i];
    }
    __syncthreads();
    mbar_wait_bounded(&bar[0], 0, status, 5);

    // ---- scores: lane group grp of warp w takes positions w*16 + it*4 + grp, HG heads per pass ----
    {
      constexpr int HG = G < 4 ? G : 4;
      const int li = lane & 7, grp = lane >> 3;
#pragma unroll 1
      for (int hb = 0; hb < G; hb += HG) {
        float acc[4][HG];
#pragma unroll
        for (int it = 0; it < 4; ++it)
#pragma unroll
          for (int h = 0; h < HG; ++h) acc[it][h] = 0.0f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int d0 = j * (HD / 2) + B * li;
          float qv[HG][B];
#pragma unroll
          for (int h = 0; h < HG; ++h)
#pragma unroll
            for (int d = 0; d < B; d += 4) {
              const float4 v = *reinterpret_cast<const float4*>(qs + (hb + h) * HD + d0 + d);
              qv[h][d] = v.x;
              qv[h][d + 1] = v.y;
              qv[h][d + 2] = v.z;
              qv[h][d + 3] = v.w;
            }
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int i = warp * 16 + it * 4 + grp;
            float kf[B];
            if (i < n) {
              ld_half_row<B>(ks + i * HD + d0, kf);
            } else {
#pragma unroll
              for (int d = 0; d < B; ++d) kf[d] = 0.0f;
            }
#pragma unroll
            for (int d = 0; d < B; ++d) {
              if constexpr (HG == 1) {
                acc[it][0] = fmaf(qv[0][d], kf[d], acc[it][0]);
              } else {
#pragma unroll
                for (int h = 0; h < HG; h += 2)
                  ffma2(acc[it][h], acc[it][h + 1], qv[h][d], qv[h + 1][d], kf[d], kf[d]);
              }
            }
          }
        }
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int i = warp * 16 + it * 4 + grp;
#pragma unroll
          for (int h = 0; h < HG; ++h) {
            float a = acc[it][h];
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
            a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
            if (li == h && i < n) sc[i * G + hb + h] = __fmul_rn(a, scale);
          }
        }
      }
    }
    __syncthreads();
    // ---- max, exp and the chunk sum: 128 threads per head, 2 heads per round ----
#pragma unroll 1
    for (int h0 = 0; h0 < G; h0 += 2) {
      const int h = h0 + (tid >> 7), w = (tid >> 5) & 3, i = tid & 127;
      const bool act = h < G;
      float v = (act && i < n) ? sc[i * G + h] : -FLT_MAX;
      v = warp_max(v);
      if (act && lane == 0) wred[h][w] = v;
      __syncthreads();
      const float m = act ? fmaxf(fmaxf(wred[h][0], wred[h][1]), fmaxf(wred[h][2], wred[h][3])) : 0.0f;
      float e = 0.0f;
      if (act && i < n) {
        e = b2_expf(__fsub_rn(sc[i * G + h], m));
        sc[i * G + h] = e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, o));
      __syncthreads();   // every wred max read before the sums reuse it
      if (act && lane == 0) wred[h][w] = e;
      __syncthreads();
      if (act && i == 0) {
        mh[h] = m;
        lh[h] = __fadd_rn(__fadd_rn(__fadd_rn(wred[h][0], wred[h][1]), wred[h][2]), wred[h][3]);
      }
    }
    __syncthreads();
    mbar_wait_bounded(&bar[1], 0, status, 5);   // V, which landed while the scores ran
    // ---- P·V: warp (residue r, dim half), lane = dim pair; all heads per position ----
    float* pv = reinterpret_cast<float*>(ks);   // [4 residues][G][HD] partials, K is no longer needed
    {
      const int r = warp & 3, pr = (warp >> 2) * 32 + lane;
      if (pr < PAIRS) {
        float acc[G][2];
#pragma unroll
        for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = 0.0f;
        for (int i = r; i < n; i += 4) {
          const uint32_t vv = *reinterpret_cast<const uint32_t*>(vs + i * HD + 2 * pr);
          const float v0 = h2f((uint16_t)(vv & 0xFFFFu)), v1 = h2f((uint16_t)(vv >> 16));
          float e[G];
#pragma unroll
          for (int h = 0; h < G; h += (G >= 4 ? 4 : 1)) {
            if constexpr (G >= 4) {
              const float4 e4 = *reinterpret_cast<const float4*>(sc + i * G + h);
              e[h] = e4.x;
              e[h + 1] = e4.y;
              e[h + 2] = e4.z;
              e[h + 3] = e4.w;
            } else {
              e[h] = sc[i * G + h];
            }
          }
#pragma unroll
          for (int h = 0; h < G; ++h) ffma2(acc[h][0], acc[h][1], e[h], e[h], v0, v1);
        }
        __syncwarp();
#pragma unroll
        for (int h = 0; h < G; ++h)
          *reinterpret_cast<float2*>(pv + (r * G + h) * HD + 2 * pr) = make_float2(acc[h][0], acc[h][1]);
      }
    }
    __syncthreads();
    for (int hd2 = tid; hd2 < G * HD; hd2 += blockDim.x) {
      const int h = hd2 / HD, d = hd2 - h * HD;
      const float a0 = pv[(0 * G + h) * HD + d], a1 = pv[(1 * G + h) * HD + d];
      const float a2 = pv[(2 * G + h) * HD + d], a3 = pv[(3 * G + h) * HD + d];
      po[(int64_t)h * n_split * HD + d] = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    }
    if (tid < G) {
      pml[(int64_t)tid * n_split * 2 + 0] = mh[tid];
      pml[(int64_t)tid * n_split * 2 + 1] = lh[tid];
    }
  }
  if (fz.count == nullptr) return;
  // ---- the last CTA of this (query, kv head) combines the chunks ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned int* cnt = fz.count + (int64_t)b * n_kv + kh;
    last_cta = atomicAdd(cnt, 1u) == (unsigned int)(n_split - 1);
    if (last_cta) *cnt = 0u;   // ready for the next launch
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  // Chunk weights e_c = exp(m_c − M) per head (staged once), L = Σ_c e_c·l_c
  // in chunk order, then out[d] = (Σ_c e_c·O_c[d]) · (1/L) — attn_combine's
  // arithmetic, with the partials read from L2 eight chunks at a time.
  float* ec = reinterpret_cast<float*>(smem + 128);   // [G][n_split] (0: chunk attended to nothing)
  float* ob = ec + G * n_split;                        // [G][HD] outputs of this kv head
  __shared__ float inv_l[G];
  if (warp < G) {
    const float* ml = part_ml + ((int64_t)b * n_head + hq0 + warp) * n_split * 2;
    float M = -FLT_MAX;
    for (int c = lane; c < n_split; c += 32) M = fmaxf(M, __ldcg(ml + 2 * c));
    M = warp_max(M);
    for (int c = lane; c < n_split; c += 32) {
      const float lc = __ldcg(ml + 2 * c + 1);
      ec[warp * n_split + c] = lc > 0.0f ? b2_expf(__fsub_rn(__ldcg(ml + 2 * c), M)) : 0.0f;
    }
    __syncwarp();
    if (lane == 0) {
      float L = 0.0f;
      for (int c = 0; c < n_split; ++c) {
        const float lc = __ldcg(ml + 2 * c + 1);
        if (lc > 0.0f) L = __fadd_rn(L, __fmul_rn(ec[warp * n_split + c], lc));
      }
      inv_l[warp] = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;   // L == 0: a query that attended to nothing
    }
  }
  __syncthreads();
  for (int hd2 = tid; hd2 < G * HD; hd2 += blockDim.x) {
    const int h = hd2 / HD, d = hd2 - h * HD;
    const float* pq = part_o + ((int64_t)b * n_head + hq0 + h) * n_split * HD + d;
    const float* eh = ec + h * n_split;
    float v = 0.0f;
    for (int c0 = 0; c0 < n_split; c0 += 8) {
      float pv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pv[j] = c0 + j < n_split ? __ldcg(pq + (int64_t)(c0 + j) * HD) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < n_split && eh[c0 + j] != 0.0f) v = __fadd_rn(v, __fmul_rn(eh[c0 + j], pv[j]));
    }
    const float o = __fmul_rn(v, inv_l[h]);
    fz.out[((int64_t)b * n_head + hq0 + h) * HD + d] = o;
    ob[hd2] = o;
  }
  if (fz.img.img == nullptr) return;
  __syncthreads();
  // quantize the G*HD outputs (columns [hq0*HD, (hq0+G)*HD) of the O input row)
  const int col0 = hq0 * HD;
  if (fz.img.type == B2_Q4_K || fz.img.type == B2_Q6_K) {
    // one 256-value unit per warp, 8 values per lane
    for (int u = warp; u < G * HD / 256; u += blockDim.x / 32) {
      float v8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v8[j] = ob[u * 256 + lane * 8 + j];
      int8_t q8[8];
      int bs = 0;
      const float d = quant_q8_k_lane(v8, q8, &bs);
      store_q8k_unit(fz.img, b, col0 / 256 + u, q8, d, bs);
    }
  } else {
    // one 32-value block per thread (ref_quantize_row_q8_0)
    for (int u = tid; u < G * HD / 32; u += blockDim.x) {
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(ob[u * 32 + j]));
      const float d = __fmul_rn(amax, 1.0f / 127.0f);
      const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
      uint32_t w8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int sum = 0;
      for (int j = 0; j < 32; ++j) {
        const float scv = __fmul_rn(ob[u * 32 + j], id);
        const float tt = scv >= 0.0f ? __fadd_rn(scv, 0.5f) : __fsub_rn(scv, 0.5f);
        int qv = __float2int_rz(tt);
        qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
        sum += qv;
        w8[j >> 2] |= ((uint32_t)(uint8_t)qv) << (8 * (j & 3));
      }
      store_q8_0_block(fz.img, b, col0 / 32 + u, w8, h2f(f2h_rn(d)), sum);
    }
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
  const float invL = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;   // L == 0: a query that attended to nothing
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
// computed with the state before the shift) by the angle table of the
// position delta, in place: fp16 -> fp32 -> rotate -> fp16 (RNE).  The table
// comes by value (no upload, so the call is stream-ordered and capturable).
__global__ void kv_shift_kernel(uint16_t* __restrict__ kc, int n_kv, int hd, int s, KvSeqState stt, int cap, int p_begin,
                                int p_end, RotTable rt) {
  __shared__ float cs[2 * kRotPairs];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) cs[i] = rt.cs[i];
  __syncthreads();
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
                                  KvSeqState stt, int cap, int dst0, int src0, int n, RotTable rt) {
  __shared__ float cs[2 * kRotPairs];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) cs[i] = rt.cs[i];
  __syncthreads();
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
// Each token's vocabulary is scanned by np CTAs (contiguous slices); the last
// of them to finish (arrival counter) merges the slices' (top-1, top-2, id)
// and writes the result.  The merge is order-independent: the top-1 is the
// largest value with the lowest id, the top-2 the largest of the rest.
// Top-1 / top-2 merge with the reference's tie rule (the lower index wins).
__device__ __forceinline__ void top2_merge(float& v1, float& v2, int& i1, float a1, float a2, int ai) {
  if (a1 > v1 || (a1 == v1 && ai < i1)) {
    v2 = fmaxf(v1, a2);
    v1 = a1;
    i1 = ai;
  } else {
    v2 = fmaxf(v2, a1);
  }
}

__global__ void argmax_kernel(const float* __restrict__ logits, int n_tok, int n_vocab, int v_local,
                              int32_t* __restrict__ ids, float* __restrict__ top, GreedyFeed feed, PeerIn in,
                              int* status, uint32_t* __restrict__ part, unsigned int* __restrict__ count) {
  pdl_wait();
  if (!feed.tok) pdl_launch_dependents();
  if (in.n) {   // the ranks' head shards arrive in the gather layout
    if (threadIdx.x == 0) {
      wait_peer_flags(in.flags, in.n, *in.epoch, status, 4);
      __threadfence();
    }
    __syncthreads();
  }
  // CTA (pi, b) scans vocabulary slice pi of token b: contiguous runs of the
  // [shard][n_tok][v_local] gather layout, one run per shard it crosses.
  const int b = blockIdx.y, np = gridDim.x, pi = blockIdx.x;
  const int per = (n_vocab + np - 1) / np;
  const int va = pi * per, vb = min(n_vocab, va + per);
  float v1 = -FLT_MAX, v2 = -FLT_MAX;
  int i1 = 0x7fffffff;
  for (int r = va / v_local; r * v_local < vb; ++r) {
    const int a = max(va, r * v_local), e = min(vb, (r + 1) * v_local);
    const float* row = logits + ((int64_t)r * n_tok + b) * v_local - (int64_t)r * v_local;   // indexed by v
    for (int v = a + (int)threadIdx.x; v < e; v += blockDim.x) {
      const float x = __ldcg(row + v);
      if (x > v1 || (x == v1 && v < i1)) {
        v2 = v1;
        v1 = x;
        i1 = v;
      } else if (x > v2) {
        v2 = x;
      }
    }
  }
  __shared__ float s1[32], s2[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a1 = __shfl_xor_sync(0xffffffffu, v1, o);
    const float a2 = __shfl_xor_sync(0xffffffffu, v2, o);
    const int ai = __shfl_xor_sync(0xffffffffu, i1, o);
    top2_merge(v1, v2, i1, a1, a2, ai);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s1[w] = v1;
    s2[w] = v2;
    si[w] = i1;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float b1 = s1[0], b2 = s2[0];
  int bi = si[0];
  for (int k = 1; k < (int)(blockDim.x >> 5); ++k) top2_merge(b1, b2, bi, s1[k], s2[k], si[k]);
  if (np > 1) {
    // the last CTA of token b to finish merges the slices
    uint32_t* pp = part + ((int64_t)b * np + pi) * 3;
    pp[0] = __float_as_uint(b1);
    pp[1] = __float_as_uint(b2);
    pp[2] = (uint32_t)bi;
    __threadfence();
    if (atomicAdd(&count[b], 1u) != (unsigned int)(np - 1)) return;
    __threadfence();
    const uint32_t* p0 = part + (int64_t)b * np * 3;
    b1 = __uint_as_float(__ldcg(p0));
    b2 = __uint_as_float(__ldcg(p0 + 1));
    bi = (int)__ldcg(p0 + 2);
    for (int k = 1; k < np; ++k)
      top2_merge(b1, b2, bi, __uint_as_float(__ldcg(p0 + 3 * k)), __uint_as_float(__ldcg(p0 + 3 * k + 1)),
                 (int)__ldcg(p0 + 3 * k + 2));
    count[b] = 0;   // ready for the next launch
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

bool add_rmsnorm_q_supported(int n, int act_type) {
  (void)act_type;
  return n % 256 == 0 && n / 8 <= 1024;
}

int launch_add_rmsnorm_q(float* x, const float* delta, const float* w, float* out, int n_tok, int n, float eps,
                         const ActImage& img, cudaStream_t s, const PeerIn* in, int* status) {
  if (!add_rmsnorm_q_supported(n, img.type) || img.kq < n || img.img == nullptr) return B2_ERR_UNSUPPORTED;
  return launch_pdl(add_rmsnorm_q_kernel, dim3(n_tok), dim3(n / 8), 0, s, x, delta, w, out, n, eps,
                    in ? *in : PeerIn{}, status, img);
}

int launch_rope_kv(const float* qkv, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                   const float* rope, float* q_out, uint16_t* kc, uint16_t* vc, const KvSeqState* st, int n_seq, int cap,
                   cudaStream_t s) {
  return launch_pdl(rope_kv_kernel, dim3(n_tok), dim3(256), 0, s, qkv, n_head, n_kv, hd, pos, seq, rope, q_out, kc, vc,
                    st, n_seq, cap);
}

int attn_splits(int cap) { return (cap + kAttnP - 1) / kAttnP; }

// The fused combine stages G*n_split chunk weights and G*hd outputs in the
// K buffer of the last CTA.
bool attn_combine_fusable(int n_head, int n_kv, int hd, int cap) {
  const int G = n_head / n_kv;
  return (size_t)G * (attn_splits(cap) + hd) * 4 <= (size_t)kAttnP * hd * 2;
}

bool attn_fusable(int n_head, int n_kv, int hd, int act_type) {
  const int G = n_head / n_kv;
  return (act_type == B2_Q4_K || act_type == B2_Q6_K) ? (G * hd) % 256 == 0 : (G * hd) % 32 == 0;
}

int launch_attention(const float* q, int n_tok, int n_head, int n_kv, int hd, const int32_t* pos, const int32_t* seq,
                     const uint16_t* kc, const uint16_t* vc, const KvSeqState* st, int n_seq, int cap, float* part_o,
                     float* part_ml, float* out, cudaStream_t s, int* status, unsigned int* count,
                     const ActImage* img) {
  const int G = n_head / n_kv;
  const int n_split = attn_splits(cap);
  const float scale = 1.0f / sqrtf((float)hd);
  const dim3 grid(n_split, n_kv, n_tok);
  AttnFuse fz;
  B2_CHECK_ARG(!count || attn_combine_fusable(n_head, n_kv, hd, cap), "attention: combine not fusable");
  if (count) {
    fz.count = count;
    fz.out = out;
    if (img) {
      B2_CHECK_ARG(attn_fusable(n_head, n_kv, hd, img->type) && img->img, "attention: image not fusable");
      fz.img = *img;
    }
  }
  int rc = B2_ERR_UNSUPPORTED;
#define B2_ATTN_CASE(HDV, GV)                                                                                       \
  if (hd == HDV && G == GV) {                                                                                       \
    const size_t sm = 128 + (size_t)2 * kAttnP * HDV * 2 + (size_t)GV * HDV * 4 + (size_t)GV * kAttnP * 4;          \
    B2_CUDA_TRY(cudaFuncSetAttribute(attn_chunk_kernel<HDV, GV>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                     (int)sm));                                                                     \
    rc = launch_pdl(attn_chunk_kernel<HDV, GV>, grid, dim3(256), sm, s, q, n_head, n_kv, pos, seq, kc, vc, st,      \
                    n_seq, cap, scale, part_o, part_ml, n_split, status, fz);                                       \
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
  if (rc != B2_OK || count) return rc;
  return launch_pdl(attn_combine_kernel, dim3(n_head, n_tok), dim3(hd), 0, s, (const float*)part_o,
                    (const float*)part_ml, n_head, hd, n_split, out);
}

int launch_kv_shift(uint16_t* kc, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int p_begin, int p_end,
                    const RotTable& cs, cudaStream_t s) {
  B2_CHECK_ARG(hd <= 2 * kRotPairs, "head_dim too large for the rotation table");
  if (p_end <= p_begin) return B2_OK;
  const int64_t total = (int64_t)(p_end - p_begin) * n_kv * (hd / 2);
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 4 * kSMs);
  kv_shift_kernel<<<grid, 256, 0, s>>>(kc, n_kv, hd, seq, st, cap, p_begin, p_end, cs);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_kv_compact(uint16_t* kc, uint16_t* vc, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int dst0,
                      int src0, int n, const RotTable& cs, cudaStream_t s) {
  B2_CHECK_ARG(hd <= 2 * kRotPairs, "head_dim too large for the rotation table");
  if (n <= 0) return B2_OK;
  kv_compact_kernel<<<n_kv, std::max(32, hd / 2), 0, s>>>(kc, vc, n_kv, hd, seq, st, cap, dst0, src0, n, cs);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

// SwiGLU over (gate, up) row pairs, as the GEMV's SwiGLU epilogue computes
// it: h[t][f] = silu(gu[t][2f]) * gu[t][2f+1], the same rounded operations.
__global__ void swiglu_pairs_kernel(const float* __restrict__ gu, int64_t n_tok, int ff, float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = n_tok * ff;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / ff, f = i - t * ff;
    const float2 v = *reinterpret_cast<const float2*>(gu + t * 2 * ff + 2 * f);
    h[i] = __fmul_rn(__fdiv_rn(v.x, __fadd_rn(1.0f, b2_expf(-v.x))), v.y);
  }
}

int launch_swiglu_pairs(const float* gu, int n_tok, int ff, float* h, cudaStream_t s) {
  const int64_t total = (int64_t)n_tok * ff;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 8 * kSMs));
  return launch_pdl(swiglu_pairs_kernel, dim3(grid), dim3(256), 0, s, gu, (int64_t)n_tok, ff, h);
}

int launch_argmax(const float* logits, int n_tok, int n_vocab, int v_local, int32_t* ids, float* top, cudaStream_t s,
                  const GreedyFeed& feed, const PeerIn* in, int* status, uint32_t* scratch) {
  // With scratch, each token's vocabulary is split over up to kArgmaxParts
  // CTAs (the last one merges); without, one CTA per token.
  const int np = scratch ? std::max(1, std::min(kArgmaxParts, n_vocab / 2048)) : 1;
  B2_CHECK_ARG(n_tok >= 1 && n_tok <= kArgmaxTok, "argmax: too many tokens");
  uint32_t* part = scratch;
  unsigned int* count = scratch ? reinterpret_cast<unsigned int*>(scratch + (size_t)kArgmaxTok * kArgmaxParts * 3)
                                : nullptr;
  return launch_pdl(argmax_kernel, dim3(np, n_tok), dim3(np > 1 ? 256 : 1024), 0, s, logits, n_tok, n_vocab, v_local,
                    ids, top, feed, in ? *in : PeerIn{}, status, part, count);
}

}  // namespace b2
