// Activation quantization to planar Q8 buffers, conversion back to GGUF
// blocks, exact integer block dots, and on-device dequantization of a
// repacked matrix (parity paths).
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

// One warp per 32-block (Q8_0) or 256-block (Q8_K) of one token row.
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, int64_t k,
                                     int64_t kp, int8_t* __restrict__ qs, float* __restrict__ d) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t nbk = kp / 32;
  const int64_t total = (int64_t)n_tok * nbk;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = wid; i < total; i += nw) {
    const int t = (int)(i / nbk);
    const int64_t kb = i - (int64_t)t * nbk;
    const int64_t e = kb * 32 + lane;
    const float xv = e < k ? x[t * x_stride + e] : 0.0f;
    uint16_t d16;
    const int8_t q = quant_q8_0_lane(xv, &d16);
    qs[t * kp + e] = q;
    if (lane == 0) d[t * nbk + kb] = h2f(d16);
  }
}

__global__ void quantize_q8_k_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, int64_t k,
                                     int64_t kp, int8_t* __restrict__ qs, float* __restrict__ d,
                                     int16_t* __restrict__ bsum) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t nbk = kp / 256;
  const int64_t total = (int64_t)n_tok * nbk;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = wid; i < total; i += nw) {
    const int t = (int)(i / nbk);
    const int64_t kb = i - (int64_t)t * nbk;
    const int64_t e0 = kb * 256 + lane * 8;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (e0 + j) < k ? x[t * x_stride + e0 + j] : 0.0f;
    int8_t q[8];
    int bs;
    const float dd = quant_q8_k_lane(v, q, &bs);
#pragma unroll
    for (int j = 0; j < 8; ++j) qs[t * kp + e0 + j] = q[j];
    if ((lane & 1) == 0) bsum[t * (kp / 16) + kb * 16 + lane / 2] = (int16_t)bs;
    if (lane == 0) d[t * nbk + kb] = dd;
  }
}

// Planar activations -> GGUF blocks (Q8_0: fp16 d + 32 int8; Q8_K: fp32 d,
// 256 int8, 16 int16 sums).  One thread per output byte.
__global__ void act_to_blocks_kernel(int type, const int8_t* qs, const float* d, const int16_t* bsum, int n_tok,
                                     int64_t k, int64_t kp, uint8_t* out) {
  const int64_t bs = type == B2_Q8_0 ? 32 : 256;
  const int64_t bb = type == B2_Q8_0 ? 34 : 292;
  const int64_t nb = k / bs;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_tok * nb * bb) return;
  const int64_t blk = i / bb;
  const int j = (int)(i - blk * bb);
  const int t = (int)(blk / nb);
  const int64_t b = blk - (int64_t)t * nb;
  uint32_t v;
  if (type == B2_Q8_0) {
    if (j < 2) {
      const uint32_t h = f2h_rn(d[t * (kp / 32) + b]);
      v = (h >> (8 * j)) & 0xFFu;
    } else {
      v = (uint8_t)qs[t * kp + b * 32 + (j - 2)];
    }
  } else {
    if (j < 4) {
      v = (__float_as_uint(d[t * (kp / 256) + b]) >> (8 * j)) & 0xFFu;
    } else if (j < 260) {
      v = (uint8_t)qs[t * kp + b * 256 + (j - 4)];
    } else {
      const int g = (j - 260) >> 1;
      const uint32_t s = (uint16_t)bsum[t * (kp / 16) + b * 16 + g];
      v = (s >> (8 * ((j - 260) & 1))) & 0xFFu;
    }
  }
  out[i] = (uint8_t)v;
}

// Exact integer block dots of one row of a tiled matrix against token 0 of
// `a`: one thread per unit, which rebuilds the unit's GGUF bytes from its slot.
__global__ void block_dots_kernel(QMatrix m, int64_t row, const int8_t* qs, const int16_t* bsum, int32_t* out_i,
                                  int32_t* out_m) {
  const int b = (int)((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (b >= m.nu) return;
  uint8_t bp[210];
  slot_to_unit(m.type, m.data + slot_offset(m, row / 8, b), (int)(row % 8), bp);
  const int64_t col = (int64_t)b * unit_elems(m.type);
  if (m.type == B2_Q4_0) {
    const uint8_t* q = bp + 2;
    int s = 0;
    for (int j = 0; j < 16; ++j) s += ((int)(q[j] & 15) - 8) * qs[col + j] + ((int)(q[j] >> 4) - 8) * qs[col + j + 16];
    out_i[b] = s;
  } else if (m.type == B2_Q8_0) {
    const int8_t* q = reinterpret_cast<const int8_t*>(bp + 2);
    int s = 0;
    for (int j = 0; j < 32; ++j) s += (int)q[j] * qs[col + j];
    out_i[b] = s;
  } else if (m.type == B2_Q4_K) {
    const uint8_t* sc = bp + 4;
    int is = 0, ms = 0;
    for (int j = 0; j < 8; ++j) {
      int s, mm;
      if (j < 4) {
        s = sc[j] & 63;
        mm = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
        mm = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      int dot = 0;
      for (int l = 0; l < 32; ++l) {
        const int e = j * 32 + l;
        const uint8_t byte = bp[16 + (e >> 6) * 32 + (e & 31)];
        const int qv = ((e >> 5) & 1) ? (byte >> 4) : (byte & 15);
        dot += qv * qs[col + e];
      }
      is += s * dot;
      ms += mm * ((int)bsum[col / 16 + 2 * j] + (int)bsum[col / 16 + 2 * j + 1]);
    }
    out_i[b] = is;
    if (out_m) out_m[b] = ms;
  } else {
    const int8_t* sc = reinterpret_cast<const int8_t*>(bp + 192);
    int is = 0;
    for (int g = 0; g < 16; ++g) {
      int dot = 0;
      for (int l = 0; l < 16; ++l) {
        const int e = g * 16 + l;
        const int h = e >> 7, gg = (e >> 5) & 3, ll = e & 31;
        const int lo = (bp[h * 64 + (gg & 1) * 32 + ll] >> (4 * (gg >> 1))) & 15;
        const int hi = (bp[128 + h * 32 + ll] >> (2 * gg)) & 3;
        dot += ((lo | (hi << 4)) - 32) * qs[col + e];
      }
      is += (int)sc[g] * dot;
    }
    out_i[b] = is;
  }
}

// fp32 dequantization of a tiled matrix: one thread per (row, unit), the same
// operation order as the GGUF layouts define (Q4_0: (q-8)·d; Q8_0: q·d;
// Q4_K: (d·sc)·q − dmin·m; Q6_K: (d·sc)·q).
__global__ void dequantize_kernel(QMatrix m, float* dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m.n_rows * m.nu) return;
  const int64_t r = i / m.nu;
  const int u = (int)(i - r * m.nu);
  uint8_t bp[210];
  slot_to_unit(m.type, m.data + slot_offset(m, r / 8, u), (int)(r % 8), bp);
  const int ue = unit_elems(m.type);
  float* out = dst + r * m.k + (int64_t)u * ue;
  if (m.type == B2_Q4_0) {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(bp));
    for (int j = 0; j < 32; ++j) {
      const uint8_t byte = bp[2 + (j & 15)];
      out[j] = __fmul_rn((float)((j < 16 ? (byte & 15) : (byte >> 4)) - 8), d);
    }
  } else if (m.type == B2_Q8_0) {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(bp));
    for (int j = 0; j < 32; ++j) out[j] = __fmul_rn((float)reinterpret_cast<const int8_t*>(bp + 2)[j], d);
  } else if (m.type == B2_Q4_K) {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(bp));
    const float dmin = h2f(*reinterpret_cast<const uint16_t*>(bp + 2));
    const uint8_t* sc = bp + 4;
    for (int e = 0; e < 256; ++e) {
      const int j = e >> 5;
      int s, mm;
      if (j < 4) {
        s = sc[j] & 63;
        mm = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
        mm = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      const uint8_t byte = bp[16 + (e >> 6) * 32 + (e & 31)];
      const int q = (j & 1) ? (byte >> 4) : (byte & 15);
      out[e] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)mm));
    }
  } else {
    const float d = h2f(*reinterpret_cast<const uint16_t*>(bp + 208));
    for (int e = 0; e < 256; ++e) {
      const int h = e >> 7, g = (e >> 5) & 3, l = e & 31;
      const int lo = (bp[h * 64 + (g & 1) * 32 + l] >> (4 * (g >> 1))) & 15;
      const int hi = (bp[128 + h * 32 + l] >> (2 * g)) & 3;
      const int q = (lo | (hi << 4)) - 32;
      const float sc = (float)reinterpret_cast<const int8_t*>(bp + 192)[e >> 4];
      out[e] = __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
  }
}

int grid_for(int64_t n, int block) { return (int)std::min<int64_t>((n + block - 1) / block, 1 << 30); }

// One thread runs the tensor-parallel exchange's bounded flag wait.
__global__ void flag_wait_kernel(const unsigned long long* flags, int n, unsigned long long target, int* status) {
  wait_peer_flags(flags, n, target, status, kPeerWaitStatus);
}

}  // namespace

int launch_flag_wait(const unsigned long long* flags, int n, unsigned long long target, int* status,
                     cudaStream_t s) {
  flag_wait_kernel<<<1, 1, 0, s>>>(flags, n, target, status);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_quantize_act(int act_type, const float* x, int64_t x_stride, int n_tok, int64_t k, ActQ& out,
                        cudaStream_t s) {
  B2_CHECK_ARG(out.kp >= k && out.n_tok >= n_tok, "activation buffer too small");
  const int block = 256;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(block);
  cfg.stream = s;
  if (act_type == B2_Q8_0) {
    const int64_t warps = (int64_t)n_tok * (out.kp / 32);
    cfg.gridDim = dim3(std::max(1, std::min(grid_for(warps * 32, block), 4 * kSMs)));
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_q8_0_kernel, x, x_stride, n_tok, k, out.kp, out.qs, out.d));
  } else if (act_type == B2_Q8_K) {
    const int64_t warps = (int64_t)n_tok * (out.kp / 256);
    cfg.gridDim = dim3(std::max(1, std::min(grid_for(warps * 32, block), 4 * kSMs)));
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_q8_k_kernel, x, x_stride, n_tok, k, out.kp, out.qs, out.d,
                                   out.bsum));
  } else {
    set_error("quantize_act: unsupported activation type %d", act_type);
    return B2_ERR_UNSUPPORTED;
  }
  out.type = act_type;
  return B2_OK;
}

int launch_act_to_blocks(const ActQ& a, int64_t k, void* blocks, cudaStream_t s) {
  const int64_t nbytes = (int64_t)a.n_tok * (int64_t)row_bytes(a.type, k);
  if (nbytes == 0) return B2_OK;
  act_to_blocks_kernel<<<grid_for(nbytes, 256), 256, 0, s>>>(a.type, a.qs, a.d, a.bsum, a.n_tok, k, a.kp,
                                                         static_cast<uint8_t*>(blocks));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_block_dots(const QMatrix& w, const ActQ& a, int64_t row, int32_t* out_i, int32_t* out_m, cudaStream_t s) {
  B2_CHECK_ARG(row >= 0 && row < w.n_rows, "block_dots row");
  block_dots_kernel<<<grid_for(w.nu, 128), 128, 0, s>>>(w, row, a.qs, a.bsum, out_i, out_m);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_dequantize(const QMatrix& w, float* dst, cudaStream_t s) {
  const int64_t n = w.n_rows * w.nu;
  if (n == 0) return B2_OK;
  dequantize_kernel<<<grid_for(n, 128), 128, 0, s>>>(w, dst);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

}  // namespace b2
