// Decoder-layer kernels around the GEMVs, in the order of the reference's
// forward_token (Singularity/src/core/cortex_a5_engine.cpp:1029-1293):
//   embed         token row dequantization (:1066-1105)
//   add_rmsnorm   residual add fused with RMSNorm (:1121, :1259-1266, :1284-1287)
//   rope_kv       RoPE on q/k (adjacent pairs, :1187-1192) + K/V store (:1195-1203) into an
//                 fp16, Q8_0 or Q4_0 cache (llama.cpp cache types, Milda/src/engine.cpp:74-87)
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
      peer_wait(in, status, 3);
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
      peer_wait(in, status, 3);
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
// Cache rows (one kv head at one slot) in the cache type's storage
// (kv_row_bytes): fp16 values, or Q8_0 as hd int8 codes then the hd/32 fp16
// block scales (quantized as ref_quantize_row_q8_0,
// Singularity/tests/test_and_bench_a5.cpp:223-245).
__device__ __forceinline__ uint8_t* kv_row(uint8_t* c, int type, int hd, int s, int n_kv, int kh, int cap,
                                           int64_t slot) {
  return c + (((int64_t)s * n_kv + kh) * cap + slot) * kv_row_bytes(type, hd);
}
// Byte of a Q4_0 row holding value i (its low nibble for i % 32 < 16).
__device__ __forceinline__ int q4_byte(int i) { return (i >> 5) * 16 + (i & 15); }
// Value i of a row (fp16, or code · block scale: exact in fp32; Q4_0 codes
// are offset by 8).
template <int T>
__device__ __forceinline__ float kv_load(const uint8_t* row, int hd, int i) {
  if constexpr (T == B2_Q8_0) {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(row + hd + 2 * (i >> 5)));
    return __fmul_rn((float)(int8_t)row[i], d);
  } else if constexpr (T == B2_Q4_0) {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(row + hd / 2 + 2 * (i >> 5)));
    const int nib = (row[q4_byte(i)] >> ((i & 16) ? 4 : 0)) & 15;
    return __fmul_rn((float)(nib - 8), d);
  } else {
    return h2f(reinterpret_cast<const uint16_t*>(row)[i]);
  }
}
// Q4_0 block scale of ggml's quantize_row_q4_0_ref from the value of largest
// magnitude (the first such; +0 when all are zero): d = max/−8, id = 1/d.
__device__ __forceinline__ void q4_0_scale(float mx, float* d, float* id) {
  *d = __fdiv_rn(mx, -8.0f);
  *id = *d != 0.0f ? __fdiv_rn(1.0f, *d) : 0.0f;
}
// Code of x: min(15, trunc(x·id + 8.5)).
__device__ __forceinline__ uint32_t q4_0_code(float x, float id) {
  const int c = __float2int_rz(__fadd_rn(__fmul_rn(x, id), 8.5f));
  return (uint32_t)(c < 15 ? c : 15);
}
// Stores value i of a row; for Q8_0 and Q4_0 the whole warp stores one
// 32-value block (lane = value i % 32), the block's scale from lane 0.
template <int T>
__device__ __forceinline__ void kv_store(uint8_t* row, int hd, int i, float y) {
  if constexpr (T == B2_Q8_0) {
    uint16_t d16;
    const int8_t q = quant_q8_0_lane(y, &d16);
    row[i] = (uint8_t)q;
    if ((threadIdx.x & 31) == 0) *reinterpret_cast<uint16_t*>(row + hd + 2 * (i >> 5)) = d16;
  } else if constexpr (T == B2_Q4_0) {
    const int lane = threadIdx.x & 31;
    float av = fabsf(y), v = y;
    int idx = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float a2 = __shfl_xor_sync(0xffffffffu, av, o), v2 = __shfl_xor_sync(0xffffffffu, v, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (a2 > av || (a2 == av && i2 < idx)) {
        av = a2;
        v = v2;
        idx = i2;
      }
    }
    float d, id;
    q4_0_scale(av > 0.0f ? v : 0.0f, &d, &id);
    const uint32_t c = q4_0_code(y, id);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, c, 16);   // value i + 16's code
    if (lane < 16) row[q4_byte(i)] = (uint8_t)(c | (hi << 4));
    if (lane == 0) *reinterpret_cast<uint16_t*>(row + hd / 2 + 2 * (i >> 5)) = f2h_rn(d);
  } else {
    reinterpret_cast<uint16_t*>(row)[i] = f2h_rn(y);
  }
}
// Adjacent-pair rotation of value i, from its own value x and its pair
// partner's (lane i ^ 1): x0·c − x1·s for even i, x0·s + x1·c for odd i.
__device__ __forceinline__ float rotate_lane(float x, int i, const float* cs) {
  const float other = __shfl_xor_sync(0xffffffffu, x, 1);
  const int pr = i & ~1;
  const float c = cs[pr], sn = cs[pr + 1];
  const float x0 = (i & 1) ? other : x, x1 = (i & 1) ? x : other;
  return (i & 1) ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)) : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
}

// One CTA per token: q heads rotated into q_out; K heads rotated and V heads
// stored into the caches, one warp per 32-value block (hd % 32 == 0).
template <int KT, int VT>
__global__ void rope_kv_kernel(const float* __restrict__ qkv, int n_head, int n_kv, int hd, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ seq, const float* __restrict__ rope, float* __restrict__ q_out,
                               uint8_t* __restrict__ kc, uint8_t* __restrict__ vc, const KvSeqState* __restrict__ st,
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
  for (int i = threadIdx.x; i < n_head * half; i += blockDim.x) {
    const int h = i / half, pr = i - h * half;
    const float x0 = src[h * hd + 2 * pr], x1 = src[h * hd + 2 * pr + 1];
    const float c = cs[2 * pr], sn = cs[2 * pr + 1];
    q_out[(int64_t)b * n_head * hd + h * hd + 2 * pr] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    q_out[(int64_t)b * n_head * hd + h * hd + 2 * pr + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n_warps = blockDim.x >> 5;
  const int nb = hd / 32;
  for (int blk = warp; blk < 2 * n_kv * nb; blk += n_warps) {
    const bool is_v = blk >= n_kv * nb;
    const int kh = (blk - (is_v ? n_kv * nb : 0)) / nb;
    const int i = (blk % nb) * 32 + lane;
    if (!is_v) {
      const float y = rotate_lane(src[(n_head + kh) * hd + i], i, cs);
      kv_store<KT>(kv_row(kc, KT, hd, s, n_kv, kh, cap, slot), hd, i, y);
    } else {
      kv_store<VT>(kv_row(vc, VT, hd, s, n_kv, kh, cap, slot), hd, i, src[(n_head + n_kv + kh) * hd + i]);
    }
  }
}

// ---- KV shift ----------------------------------------------------------------------------
// Rotates K rows of logical positions [p_begin, p_end) of sequence s (slots
// computed with the state before the shift) by the angle table of the
// position delta, in place: value -> fp32 -> rotate -> the cache type's
// storage (fp16 RNE, or Q8_0 requantized per block as
// ref_quantize_row_q8_0).  Each thread takes 4 consecutive values (two
// rotation pairs): one 8-byte fp16 load and store, or one 4-byte code word,
// with the 8 threads of a 32-value block sharing its maximum by shuffles.
// The table comes by value (no upload, so the call is stream-ordered and
// capturable).
template <int KT>
__global__ void kv_shift_kernel(uint8_t* __restrict__ kc, int n_kv, int hd, int s, KvSeqState stt, int cap, int p_begin,
                                int p_end, RotTable rt) {
  __shared__ float cs[2 * kRotPairs];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) cs[i] = rt.cs[i];
  __syncthreads();
  const int qpr = hd / 4;                               // threads per row (16 or 32: whole 8-lane groups)
  const int total = (p_end - p_begin) * n_kv * qpr;     // multiple of 16
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * blockDim.x;
  // warp-uniform trip count: every lane of a warp runs every trip (shuffles)
  for (int base = (blockIdx.x * blockDim.x + threadIdx.x) & ~31; base < total; base += stride) {
    const int q = base + lane;
    const bool on = q < total;
    const int row = on ? q / qpr : 0, i = (q - row * qpr) * 4;
    const int kh = row % n_kv, p = p_begin + row / n_kv;
    uint8_t* rp = kv_row(kc, KT, hd, s, n_kv, kh, cap, on ? kv_slot(stt, p, cap) : 0);
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (KT == B2_Q8_0) {
      if (on) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(rp + i);
        const float d = h2f(*reinterpret_cast<const uint16_t*>(rp + hd + 2 * (i >> 5)));
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = __fmul_rn((float)(int8_t)(w >> (8 * k)), d);
      }
    } else if constexpr (KT == B2_Q4_0) {
      if (on) {
        // values i..i+3 share one word of nibbles (low for i % 32 < 16)
        const uint32_t w = *reinterpret_cast<const uint32_t*>(rp + q4_byte(i)) >> ((i & 16) ? 4 : 0);
        const float d = h2f(*reinterpret_cast<const uint16_t*>(rp + hd / 2 + 2 * (i >> 5)));
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = __fmul_rn((float)((int)((w >> (8 * k)) & 15u) - 8), d);
      }
    } else if (on) {
      const uint2 w = *reinterpret_cast<const uint2*>(rp + 2 * i);
      x[0] = h2f((uint16_t)(w.x & 0xFFFFu));
      x[1] = h2f((uint16_t)(w.x >> 16));
      x[2] = h2f((uint16_t)(w.y & 0xFFFFu));
      x[3] = h2f((uint16_t)(w.y >> 16));
    }
    float y[4];
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      const float c = cs[(i + k) & (2 * kRotPairs - 1)], sn = cs[(i + k + 1) & (2 * kRotPairs - 1)];
      y[k] = __fsub_rn(__fmul_rn(x[k], c), __fmul_rn(x[k + 1], sn));
      y[k + 1] = __fadd_rn(__fmul_rn(x[k], sn), __fmul_rn(x[k + 1], c));
    }
    if constexpr (KT == B2_Q4_0) {
      // the block's 32 values sit on 8 consecutive lanes: the value of
      // largest magnitude (the first such), then codes; the lanes of values
      // 16..31 hand their codes to the lanes of values 0..15 (lane ^ 4), whose
      // bytes take them as high nibbles
      float av = fabsf(y[0]), v = y[0];
      int idx = i;
#pragma unroll
      for (int k = 1; k < 4; ++k)
        if (fabsf(y[k]) > av) {
          av = fabsf(y[k]);
          v = y[k];
          idx = i + k;
        }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        const float a2 = __shfl_xor_sync(0xffffffffu, av, o), v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (a2 > av || (a2 == av && i2 < idx)) {
          av = a2;
          v = v2;
          idx = i2;
        }
      }
      float d, id;
      q4_0_scale(av > 0.0f ? v : 0.0f, &d, &id);
      uint32_t w = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) w |= q4_0_code(y[k], id) << (8 * k);
      const uint32_t hi = __shfl_xor_sync(0xffffffffu, w, 4);
      if (on && (i & 16) == 0) {
        *reinterpret_cast<uint32_t*>(rp + q4_byte(i)) = w | (hi << 4);
        if ((i & 31) == 0) *reinterpret_cast<uint16_t*>(rp + hd / 2 + 2 * (i >> 5)) = f2h_rn(d);
      }
    } else if constexpr (KT == B2_Q8_0) {
      // the block's 32 values sit on 8 consecutive lanes
      float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float d = __fmul_rn(amax, 1.0f / 127.0f);
      const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
      uint32_t w = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float sc = __fmul_rn(y[k], id);
        const float t = sc >= 0.0f ? __fadd_rn(sc, 0.5f) : __fsub_rn(sc, 0.5f);
        int c = __float2int_rz(t);
        c = c < -127 ? -127 : (c > 127 ? 127 : c);
        w |= (uint32_t)(uint8_t)(int8_t)c << (8 * k);
      }
      if (on) {
        *reinterpret_cast<uint32_t*>(rp + i) = w;
        if ((i & 31) == 0) *reinterpret_cast<uint16_t*>(rp + hd + 2 * (i >> 5)) = f2h_rn(d);
      }
    } else if (on) {
      uint2 w;
      w.x = (uint32_t)f2h_rn(y[0]) | ((uint32_t)f2h_rn(y[1]) << 16);
      w.y = (uint32_t)f2h_rn(y[2]) | ((uint32_t)f2h_rn(y[3]) << 16);
      *reinterpret_cast<uint2*>(rp + 2 * i) = w;
    }
  }
}

// Moves K/V rows of logical [src0, src0+n) to logical [dst0, dst0+n) of one
// sequence (dst0 < src0, processed in ascending order by a single CTA per
// head so overlapping ranges move safely), rotating K by cs (delta table)
// and storing it back in the cache type's storage.  hd threads, one value
// each.
template <int KT, int VT>
__global__ void kv_compact_kernel(uint8_t* __restrict__ kc, uint8_t* __restrict__ vc, int n_kv, int hd, int s,
                                  KvSeqState stt, int cap, int dst0, int src0, int n, RotTable rt) {
  __shared__ float cs[2 * kRotPairs];
  for (int i = threadIdx.x; i < hd; i += blockDim.x) cs[i] = rt.cs[i];
  __syncthreads();
  const int kh = blockIdx.x, i = threadIdx.x;
  const int vb = (int)kv_row_bytes(VT, hd);
  for (int t = 0; t < n; ++t) {
    const int64_t ss = kv_slot(stt, src0 + t, cap), ds = kv_slot(stt, dst0 + t, cap);
    const uint8_t* ksrc = kv_row(kc, KT, hd, s, n_kv, kh, cap, ss);
    uint8_t* kdst = kv_row(kc, KT, hd, s, n_kv, kh, cap, ds);
    const uint8_t* vsrc = kv_row(vc, VT, hd, s, n_kv, kh, cap, ss);
    uint8_t* vdst = kv_row(vc, VT, hd, s, n_kv, kh, cap, ds);
    const float y = rotate_lane(kv_load<KT>(ksrc, hd, i), i, cs);
    // the V row moves as bytes: 2 per value for fp16, codes then scales for
    // Q8_0 and Q4_0
    constexpr int vq = VT != B2_F16;
    const int cb = (int)kv_code_bytes(VT, hd);
    uint16_t v0 = 0;
    uint8_t v1 = 0;
    if constexpr (vq) {
      if (i < cb) v1 = vsrc[i];
      if (i < (vb - cb) / 2) v0 = reinterpret_cast<const uint16_t*>(vsrc + cb)[i];
    } else {
      v0 = reinterpret_cast<const uint16_t*>(vsrc)[i];
    }
    __syncthreads();
    kv_store<KT>(kdst, hd, i, y);
    if constexpr (vq) {
      if (i < cb) vdst[i] = v1;
      if (i < (vb - cb) / 2) reinterpret_cast<uint16_t*>(vdst + cb)[i] = v0;
    } else {
      reinterpret_cast<uint16_t*>(vdst)[i] = v0;
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
      peer_wait(in, status, 4);
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
                   const float* rope, float* q_out, void* kc, int kt, void* vc, int vt, const KvSeqState* st, int n_seq,
                   int cap, cudaStream_t s) {
  B2_CHECK_ARG(kv_type_ok(kt) && kv_type_ok(vt), "KV cache types must be F16, Q8_0 or Q4_0");
  B2_CHECK_ARG(hd % 32 == 0, "head_dim must be a multiple of 32");
  uint8_t* k8 = static_cast<uint8_t*>(kc);
  uint8_t* v8 = static_cast<uint8_t*>(vc);
#define B2_ROPE_KV(KT, VT)                                                                                           \
  if (kt == KT && vt == VT)                                                                                          \
    return launch_pdl(rope_kv_kernel<KT, VT>, dim3(n_tok), dim3(256), 0, s, qkv, n_head, n_kv, hd, pos, seq, rope, \
                      q_out, k8, v8, st, n_seq, cap);
  B2_ROPE_KV(B2_F16, B2_F16)
  B2_ROPE_KV(B2_F16, B2_Q8_0)
  B2_ROPE_KV(B2_F16, B2_Q4_0)
  B2_ROPE_KV(B2_Q8_0, B2_F16)
  B2_ROPE_KV(B2_Q8_0, B2_Q8_0)
  B2_ROPE_KV(B2_Q8_0, B2_Q4_0)
  B2_ROPE_KV(B2_Q4_0, B2_F16)
  B2_ROPE_KV(B2_Q4_0, B2_Q8_0)
  B2_ROPE_KV(B2_Q4_0, B2_Q4_0)
#undef B2_ROPE_KV
  return B2_ERR_INVALID;
}

int launch_kv_shift(void* kc, int kt, int n_kv, int hd, int seq, const KvSeqState& st, int cap, int p_begin, int p_end,
                    const RotTable& cs, cudaStream_t s) {
  B2_CHECK_ARG(hd <= 2 * kRotPairs, "head_dim too large for the rotation table");
  B2_CHECK_ARG(hd % 32 == 0 && kv_type_ok(kt), "KV shift: head_dim % 32 and an F16, Q8_0 or Q4_0 cache");
  if (p_end <= p_begin) return B2_OK;
  const int64_t quads = (int64_t)(p_end - p_begin) * n_kv * (hd / 4);
  B2_CHECK_ARG(quads < (int64_t)1 << 30, "KV shift range too large");
  const int grid = (int)std::min<int64_t>((quads + 255) / 256, 4 * kSMs);
  uint8_t* k8 = static_cast<uint8_t*>(kc);
  if (kt == B2_Q8_0) kv_shift_kernel<B2_Q8_0><<<grid, 256, 0, s>>>(k8, n_kv, hd, seq, st, cap, p_begin, p_end, cs);
  else if (kt == B2_Q4_0) kv_shift_kernel<B2_Q4_0><<<grid, 256, 0, s>>>(k8, n_kv, hd, seq, st, cap, p_begin, p_end, cs);
  else kv_shift_kernel<B2_F16><<<grid, 256, 0, s>>>(k8, n_kv, hd, seq, st, cap, p_begin, p_end, cs);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_kv_compact(void* kc, int kt, void* vc, int vt, int n_kv, int hd, int seq, const KvSeqState& st, int cap,
                      int dst0, int src0, int n, const RotTable& cs, cudaStream_t s) {
  B2_CHECK_ARG(hd <= 2 * kRotPairs, "head_dim too large for the rotation table");
  B2_CHECK_ARG(hd % 32 == 0 && kv_type_ok(kt) && kv_type_ok(vt),
               "KV compact: head_dim % 32, F16, Q8_0 or Q4_0 caches");
  if (n <= 0) return B2_OK;
  uint8_t* k8 = static_cast<uint8_t*>(kc);
  uint8_t* v8 = static_cast<uint8_t*>(vc);
#define B2_COMPACT(KT, VT)                                                                                       \
  if (kt == KT && vt == VT)                                                                                      \
    kv_compact_kernel<KT, VT><<<n_kv, hd, 0, s>>>(k8, v8, n_kv, hd, seq, st, cap, dst0, src0, n, cs);
  B2_COMPACT(B2_F16, B2_F16)
  B2_COMPACT(B2_F16, B2_Q8_0)
  B2_COMPACT(B2_F16, B2_Q4_0)
  B2_COMPACT(B2_Q8_0, B2_F16)
  B2_COMPACT(B2_Q8_0, B2_Q8_0)
  B2_COMPACT(B2_Q8_0, B2_Q4_0)
  B2_COMPACT(B2_Q4_0, B2_F16)
  B2_COMPACT(B2_Q4_0, B2_Q8_0)
  B2_COMPACT(B2_Q4_0, B2_Q4_0)
#undef B2_COMPACT
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

// out[i] = ((p_0[i] + p_1[i]) + p_2[i]) + ... over n_parts partials laid out
// [n_parts][n]: the ranks' partial projections summed in rank order.
__global__ void rank_sum_kernel(const float* __restrict__ parts, int n_parts, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = parts[i];
    for (int r = 1; r < n_parts; ++r) acc = __fadd_rn(acc, parts[(int64_t)r * n + i]);
    out[i] = acc;
  }
}

int launch_rank_sum(const float* parts, int n_parts, int64_t n, float* out, cudaStream_t s) {
  B2_CHECK_ARG(parts && out && n_parts >= 1 && n > 0, "rank_sum arguments");
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 8 * kSMs);
  rank_sum_kernel<<<grid, 256, 0, s>>>(parts, n_parts, n, out);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

// SwiGLU over (gate, up) row pairs, as the GEMV's SwiGLU epilogue computes
// it: h[t][f] = silu(gu[t][2f]) * gu[t][2f+1] in the reference's order
// (silu_mul_ref).
__global__ void swiglu_pairs_kernel(const float* __restrict__ gu, int64_t n_tok, int ff, float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = n_tok * ff;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / ff, f = i - t * ff;
    const float2 v = *reinterpret_cast<const float2*>(gu + t * 2 * ff + 2 * f);
    h[i] = silu_mul_ref(v.x, v.y);
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
