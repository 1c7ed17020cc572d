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

}  // namespace b2
