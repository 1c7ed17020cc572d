// Warp-level activation quantizers, bit-exact with the reference CPU path.
//
// Q8_0 follows ref_quantize_row_q8_0 (Singularity/tests/test_and_bench_a5.cpp:223-245):
//   d = amax*(1/127) -> fp16 (RNE), id = 127/amax, q = trunc(x*id ± 0.5), |q| <= 127.
// Q8_K follows ggml's quantize_row_q8_K: max = value of largest magnitude
//   (first such index), iscale = -127/max, q = rint(iscale*x) capped at 127,
//   d = 1/iscale, bsums over 16-value groups.
// Every fp operation is an explicitly rounded intrinsic, so no contraction
// or fast-math rewrite can change a code.
#pragma once

#include "b2_common.cuh"

namespace b2 {

// One 32-value block per warp, one value per lane.  Returns the lane's code;
// *d16 receives the fp16 scale bits (same on all lanes).
__device__ __forceinline__ int8_t quant_q8_0_lane(float x, uint16_t* d16) {
  const float ax = fabsf(x);
  const float amax = warp_max(ax);
  const float d = __fmul_rn(amax, 1.0f / 127.0f);
  const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
  *d16 = f2h_rn(d);
  const float scaled = __fmul_rn(x, id);
  const float t = scaled >= 0.0f ? __fadd_rn(scaled, 0.5f) : __fsub_rn(scaled, 0.5f);
  int q = __float2int_rz(t);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

// One 256-value super-block per warp, 8 consecutive values per lane
// (v[0..7] = x[8*lane .. 8*lane+7]).  Writes the lane's 8 codes to q[],
// returns d; *bsum receives the 16-group sum for group lane/2 (valid on even
// lanes).
__device__ __forceinline__ float quant_q8_k_lane(const float v[8], int8_t q[8], int* bsum) {
  const int lane = threadIdx.x & 31;
  float amax = 0.0f, vmax = 0.0f;
  int idx = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float ax = fabsf(v[i]);
    if (ax > amax) {
      amax = ax;
      vmax = v[i];
      idx = lane * 8 + i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float a2 = __shfl_xor_sync(0xffffffffu, amax, o);
    const float v2 = __shfl_xor_sync(0xffffffffu, vmax, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (a2 > amax || (a2 == amax && i2 < idx)) {
      amax = a2;
      vmax = v2;
      idx = i2;
    }
  }
  if (amax == 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
    *bsum = 0;
    return 0.0f;
  }
  const float iscale = __fdiv_rn(-127.0f, vmax);
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int c = __float2int_rn(__fmul_rn(iscale, v[i]));
    c = c > 127 ? 127 : c;
    q[i] = static_cast<int8_t>(c);
    s += c;
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  *bsum = s;
  return __fdiv_rn(1.0f, iscale);
}

// ---- stores into a GEMV activation image (ActImage carve-up) -------------------------------
// Codes of token t start at t*kq, in natural order (unit u of Q8_K at
// u*256, block b of Q8_0 at b*32).

// One Q8_K unit b of token t, called by a whole warp (lane = 8-value group):
// codes q[8] of the lane, scale d, and the lane's 16-group sum bs (valid on
// even lanes, as quant_q8_k_lane returns it).
__device__ __forceinline__ void store_q8k_unit(const ActImage& a, int t, int b, const int8_t (&q)[8], float d,
                                               int bs) {
  const int lane = threadIdx.x & 31;
  const uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) | ((uint32_t)(uint8_t)q[2] << 16) |
                      ((uint32_t)(uint8_t)q[3] << 24);
  const uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) | ((uint32_t)(uint8_t)q[6] << 16) |
                      ((uint32_t)(uint8_t)q[7] << 24);
  uint8_t* unit = a.img + (int64_t)t * a.kq + (int64_t)b * 256;
  *reinterpret_cast<uint2*>(unit + lane * 8) = make_uint2(w0, w1);
  float* dxs = reinterpret_cast<float*>(a.img + a.off_dx);
  int16_t* bss = reinterpret_cast<int16_t*>(a.img + a.off_bs);
  if (lane == 0) dxs[t * a.nu + b] = d;
  if (a.type == B2_Q6_K) {
    if ((lane & 1) == 0) bss[(t * a.nu + b) * 16 + lane / 2] = (int16_t)bs;
  } else {
    const int b32 = bs + __shfl_xor_sync(0xffffffffu, bs, 2);
    if ((lane & 3) == 0) bss[(t * a.nu + b) * 8 + lane / 4] = (int16_t)b32;
  }
}

// One Q8_0 block b of token t from one thread: its 8 code words, the fp16
// scale as fp32 and the code sum (kept for Q4_0's offset term).
__device__ __forceinline__ void store_q8_0_block(const ActImage& a, int t, int b, const uint32_t (&w)[8], float dq,
                                                 int sum) {
  uint8_t* trow = a.img + (int64_t)t * a.kq;
  *reinterpret_cast<uint4*>(trow + b * 32) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(trow + b * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
  reinterpret_cast<float*>(a.img + a.off_dx)[t * a.nu + b] = dq;
  if (a.type == B2_Q4_0) reinterpret_cast<int16_t*>(a.img + a.off_bs)[t * a.nu + b] = (int16_t)sum;
}

}  // namespace b2
