// Host-side code: error text, GGUF block bookkeeping, the upload repack,
// GGUF weight quantizers, the seeded synthetic-weight generator and the RoPE
// table.  No device code.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "b2_internal.hpp"

namespace b2 {

namespace {
thread_local char g_err[1024] = "";
thread_local bool g_pdl = true;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}
const char* last_error() { return g_err; }
bool pdl_enabled() { return g_pdl; }

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}
void set_pdl(bool on) { g_pdl = on; }

int block_elems(int type) {
  switch (type) {
    case B2_Q4_0: case B2_Q8_0: return 32;
    case B2_Q4_K: case B2_Q6_K: case B2_Q8_K: return 256;
    default: return 1;
  }
}

size_t row_bytes(int type, int64_t k) {
  switch (type) {
    case B2_F32: return (size_t)k * 4;
    case B2_F16: return (size_t)k * 2;
    case B2_Q4_0: return (size_t)(k / 32) * 18;
    case B2_Q8_0: return (size_t)(k / 32) * 34;
    case B2_Q4_K: return (size_t)(k / 256) * 144;
    case B2_Q6_K: return (size_t)(k / 256) * 210;
    case B2_Q8_K: return (size_t)(k / 256) * 292;
    default: return 0;
  }
}

bool is_weight_type(int type) {
  return type == B2_Q4_0 || type == B2_Q8_0 || type == B2_Q4_K || type == B2_Q6_K;
}

// ---- tile layout ----------------------------------------------------------------------
void plan_qmatrix(QMatrix& m) {
  m.nu = (int)(m.k / unit_elems(m.type));
  m.splits = tile_splits(m.type, m.k);
  m.ulen = (m.nu + m.splits - 1) / m.splits;
  m.slot_bytes = tile_slot_bytes(m.type);
  m.n_tiles = (m.n_rows + 7) / 8;
  m.tile_bytes = (int64_t)m.splits * m.ulen * m.slot_bytes;
}

UploadStager::~UploadStager() {
  if (stream) cudaStreamSynchronize(stream);
  for (int b = 0; b < 2; ++b) {
    if (h[b]) cudaFreeHost(h[b]);
    if (ev[b]) cudaEventDestroy(ev[b]);
  }
  if (stream) cudaStreamDestroy(stream);
}

int UploadStager::init(size_t per_buffer) {
  if (!stream) {
    B2_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    for (int b = 0; b < 2; ++b) B2_CUDA_TRY(cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming));
  }
  if (per_buffer <= bytes) return B2_OK;
  B2_CUDA_TRY(cudaStreamSynchronize(stream));
  for (int b = 0; b < 2; ++b) {
    if (h[b]) cudaFreeHost(h[b]);
    h[b] = nullptr;
  }
  bytes = 0;
  for (int b = 0; b < 2; ++b) {
    const cudaError_t e = cudaMallocHost(&h[b], per_buffer);
    if (e != cudaSuccess) {
      set_error("upload staging: pinned allocation of %zu bytes: %s", per_buffer, cudaGetErrorString(e));
      return B2_ERR_OOM;
    }
  }
  bytes = per_buffer;
  return B2_OK;
}

int UploadStager::finish() {
  if (stream) B2_CUDA_TRY(cudaStreamSynchronize(stream));
  return B2_OK;
}

int upload_tiles(QMatrix& m, const uint8_t* const* rows, UploadStager* st) {
  plan_qmatrix(m);
  cudaGetDevice(&m.device);
  m.data = nullptr;
  UploadStager local;
  if (!st) st = &local;
  int rc = st->init(std::max<size_t>((size_t)64 << 20, (size_t)m.tile_bytes));
  if (rc) return rc;
  const int64_t bytes = m.bytes();
  cudaError_t e = cudaMalloc(&m.data, (size_t)std::max<int64_t>(bytes, 16));
  if (e != cudaSuccess) {
    m.data = nullptr;
    set_error("matrix upload: device allocation of %lld bytes: %s", (long long)bytes, cudaGetErrorString(e));
    return B2_ERR_OOM;
  }
  // Slabs of whole tiles, alternating between the two pinned buffers: a
  // buffer is refilled once its previous copy has completed; the tiles of a
  // slab are split over host threads.
  const int64_t slab = std::max<int64_t>(1, (int64_t)st->bytes / std::max<int64_t>(1, m.tile_bytes));
  const int nt = (int)std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  for (int64_t t0 = 0; t0 < m.n_tiles && rc == B2_OK; t0 += slab) {
    const int64_t t1 = std::min(m.n_tiles, t0 + slab), n = t1 - t0;
    const int b = st->next;
    st->next ^= 1;
    e = cudaEventSynchronize(st->ev[b]);
    if (e != cudaSuccess) {
      set_error("matrix upload: staging wait: %s", cudaGetErrorString(e));
      rc = B2_ERR_CUDA;
      break;
    }
    uint8_t* h = st->h[b];
    auto work = [&](int64_t a, int64_t c) {
      if (c > a) repack_tiles_host(m, rows, a, c, h + (a - t0) * m.tile_bytes);
    };
    std::vector<std::thread> th;
    for (int t = 1; t < nt; ++t) th.emplace_back(work, t0 + n * t / nt, t0 + n * (t + 1) / nt);
    work(t0, t0 + n / nt);
    for (auto& x : th) x.join();
    e = cudaMemcpyAsync(m.data + t0 * m.tile_bytes, h, (size_t)(n * m.tile_bytes), cudaMemcpyHostToDevice,
                        st->stream);
    if (e == cudaSuccess) e = cudaEventRecord(st->ev[b], st->stream);
    if (e != cudaSuccess) {
      set_error("matrix upload: copy: %s", cudaGetErrorString(e));
      rc = B2_ERR_CUDA;
    }
  }
  if (rc == B2_OK && st == &local) rc = st->finish();
  if (rc != B2_OK) {
    st->finish();
    cudaFree(m.data);
    m.data = nullptr;
  }
  return rc;
}

void repack_tiles_host(const QMatrix& m, const uint8_t* const* rows, int64_t t0, int64_t t1, uint8_t* out) {
  const int ub = gguf_unit_bytes(m.type);
  memset(out, 0, (size_t)((t1 - t0) * m.tile_bytes));
  for (int64_t t = t0; t < t1; ++t) {
    uint8_t* tile = out + (t - t0) * m.tile_bytes;
    for (int g = 0; g < 8; ++g) {
      const int64_t r = t * 8 + g;
      if (r >= m.n_rows) break;
      for (int u = 0; u < m.nu; ++u)
        unit_to_slot(m.type, rows[r] + (size_t)u * ub, g, tile + slot_offset(m, 0, u));
    }
  }
}

// ---- fp16 (host) ---------------------------------------------------------------------
uint16_t host_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
  if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
  const int e = (int)(ax >> 23) - 127;
  if (e >= -14) {
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    const uint32_t mant = ax & 0x7FFFFFu;
    uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
  }
  const int shift = -1 - e;
  if (shift > 25) return sign;
  const uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
  uint32_t h = mant >> shift;
  const uint32_t rem = mant & ((1u << shift) - 1u);
  const uint32_t half = 1u << (shift - 1);
  if (rem > half || (rem == half && (h & 1u))) h += 1u;
  return (uint16_t)(sign | h);
}

float host_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
  uint32_t bits;
  if (e == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      uint32_t mm = mant, ee = 113;
      while (!(mm & 0x400u)) {
        mm <<= 1;
        --ee;
      }
      bits = sign | (ee << 23) | ((mm & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// ---- GGUF weight quantizers --------------------------------------------------------
namespace {
inline int nearest(float v) { return (int)lrintf(v); }

// ggml quantize_row_q4_0_ref.
void quant_row_q4_0(const float* x, uint8_t* out, int64_t k) {
  for (int64_t b = 0; b < k / 32; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < 32; ++j) {
      const float v = xb[j];
      if (amax < fabsf(v)) {
        amax = fabsf(v);
        max = v;
      }
    }
    const float d = max / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    BlockQ4_0* y = reinterpret_cast<BlockQ4_0*>(out) + b;
    y->d = host_f32_to_f16(d);
    for (int j = 0; j < 16; ++j) {
      const float x0 = xb[j] * id, x1 = xb[16 + j] * id;
      const int q0 = std::min(15, (int)(int8_t)(x0 + 8.5f));
      const int q1 = std::min(15, (int)(int8_t)(x1 + 8.5f));
      y->qs[j] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

// ggml quantize_row_q8_0_ref.
void quant_row_q8_0(const float* x, uint8_t* out, int64_t k) {
  for (int64_t b = 0; b < k / 32; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = std::max(amax, fabsf(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    BlockQ8_0* y = reinterpret_cast<BlockQ8_0*>(out) + b;
    y->d = host_f32_to_f16(d);
    for (int j = 0; j < 32; ++j) y->qs[j] = (int8_t)roundf(xb[j] * id);
  }
}

// Q4_K: per 32-value sub-block an affine [min, max] map onto 0..15, scales
// and mins quantized to 6 bits against the super-block d / dmin.
void quant_row_q4_k(const float* x, uint8_t* out, int64_t k) {
  for (int64_t b = 0; b < k / 256; ++b) {
    const float* xb = x + b * 256;
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
      float lo = 0.0f, hi = -INFINITY;
      for (int l = 0; l < 32; ++l) {
        lo = std::min(lo, xb[j * 32 + l]);
        hi = std::max(hi, xb[j * 32 + l]);
      }
      hi = std::max(hi, lo);
      scale[j] = (hi - lo) / 15.0f;
      minv[j] = -lo;
      max_scale = std::max(max_scale, scale[j]);
      max_min = std::max(max_min, minv[j]);
    }
    BlockQ4_K* y = reinterpret_cast<BlockQ4_K*>(out) + b;
    y->d = host_f32_to_f16(max_scale / 63.0f);
    y->dmin = host_f32_to_f16(max_min / 63.0f);
    const float d = host_f16_to_f32(y->d), dmin = host_f16_to_f32(y->dmin);
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
      ls[j] = (uint8_t)(d > 0.0f ? std::clamp(nearest(scale[j] / d), 0, 63) : 0);
      lm[j] = (uint8_t)(dmin > 0.0f ? std::clamp(nearest(minv[j] / dmin), 0, 63) : 0);
    }
    for (int j = 0; j < 4; ++j) {
      y->scales[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
      y->scales[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
      y->scales[j + 8] = (uint8_t)((ls[j + 4] & 0x0F) | ((lm[j + 4] & 0x0F) << 4));
    }
    memset(y->qs, 0, sizeof y->qs);
    for (int e = 0; e < 256; ++e) {
      const int j = e >> 5;
      const float es = d * (float)ls[j], em = dmin * (float)lm[j];
      const int q = es > 0.0f ? std::clamp(nearest((xb[e] + em) / es), 0, 15) : 0;
      y->qs[(e >> 6) * 32 + (e & 31)] |= (uint8_t)(q << (4 * ((e >> 5) & 1)));
    }
  }
}

// Q6_K: per 16-value group a signed scale (the largest-magnitude value maps
// to −32), group scales quantized to int8 against the super-block d.
void quant_row_q6_k(const float* x, uint8_t* out, int64_t k) {
  for (int64_t b = 0; b < k / 256; ++b) {
    const float* xb = x + b * 256;
    float sg[16];
    float max_abs_scale = 0.0f;
    for (int g = 0; g < 16; ++g) {
      float amax = 0.0f, vmax = 0.0f;
      for (int l = 0; l < 16; ++l) {
        const float v = xb[g * 16 + l];
        if (fabsf(v) > amax) {
          amax = fabsf(v);
          vmax = v;
        }
      }
      sg[g] = vmax / -32.0f;
      max_abs_scale = std::max(max_abs_scale, fabsf(sg[g]));
    }
    BlockQ6_K* y = reinterpret_cast<BlockQ6_K*>(out) + b;
    y->d = host_f32_to_f16(max_abs_scale / 127.0f);
    const float d = host_f16_to_f32(y->d);
    int ls[16];
    for (int g = 0; g < 16; ++g) {
      ls[g] = d > 0.0f ? std::clamp(nearest(sg[g] / d), -128, 127) : 0;
      y->scales[g] = (int8_t)ls[g];
    }
    memset(y->ql, 0, sizeof y->ql);
    memset(y->qh, 0, sizeof y->qh);
    for (int e = 0; e < 256; ++e) {
      const float es = d * (float)ls[e >> 4];
      const int q = es != 0.0f ? std::clamp(nearest(xb[e] / es), -32, 31) : 0;
      const int q6 = q + 32;
      const int h = e >> 7, g = (e >> 5) & 3, l = e & 31;
      y->ql[h * 64 + (g & 1) * 32 + l] |= (uint8_t)((q6 & 0x0F) << (4 * (g >> 1)));
      y->qh[h * 32 + l] |= (uint8_t)((q6 >> 4) << (2 * g));
    }
  }
}
}  // namespace

int quantize_weights(int type, const float* src, int64_t n_rows, int64_t k, void* dst, int n_threads) {
  if (!is_weight_type(type)) {
    set_error("quantize_weights: unsupported type %d", type);
    return B2_ERR_UNSUPPORTED;
  }
  if (k % block_elems(type) != 0) {
    set_error("quantize_weights: k=%lld not a multiple of the block size", (long long)k);
    return B2_ERR_INVALID;
  }
  const size_t rb = row_bytes(type, k);
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const float* x = src + r * k;
      uint8_t* o = static_cast<uint8_t*>(dst) + r * rb;
      switch (type) {
        case B2_Q4_0: quant_row_q4_0(x, o, k); break;
        case B2_Q8_0: quant_row_q8_0(x, o, k); break;
        case B2_Q4_K: quant_row_q4_k(x, o, k); break;
        case B2_Q6_K: quant_row_q6_k(x, o, k); break;
      }
    }
  };
  const int nt = (int)std::max<int64_t>(1, std::min<int64_t>(n_threads < 1 ? 1 : n_threads, n_rows));
  std::vector<std::thread> th;
  for (int t = 1; t < nt; ++t) th.emplace_back(work, n_rows * t / nt, n_rows * (t + 1) / nt);
  work(0, n_rows / nt);
  for (auto& x : th) x.join();
  return B2_OK;
}

// ---- synthetic weights ---------------------------------------------------------------
namespace {
inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
}  // namespace

// Approximately normal values from a counter-based hash: value i of stream
// `seed` is the centred sum of the four 16-bit fields of mix64(seed, i), an
// Irwin-Hall(4) variate scaled to unit variance (support +-3.46 sigma, excess
// kurtosis -0.3).  It needs no transcendental function, so the loop
// vectorizes and the multi-GB synthetic checkpoints fill at memory speed;
// any slice [offset, offset + n) equals the same slice of a longer call.
int synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float std_dev, float* out, int n_threads) {
  const uint64_t base = seed * 0xD1B54A32D192ED03ull;
  // var(sum of 4 U(0,65536)) = 4 * 65536^2 / 12
  const float scale = std_dev * (float)(1.7320508075688772 / 65536.0);
  auto work = [&](int64_t i0, int64_t i1) {
    for (int64_t i = i0; i < i1; ++i) {
      const uint64_t h = mix64(base + offset + (uint64_t)i);
      const int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
                        (int32_t)(h >> 48) - 131070;
      out[i] = mean + scale * (float)s;
    }
  };
  const int nt = (int)std::max<int64_t>(1, std::min<int64_t>(n_threads < 1 ? 1 : n_threads, n / 4096 + 1));
  std::vector<std::thread> th;
  for (int t = 1; t < nt; ++t) th.emplace_back(work, n * t / nt, n * (t + 1) / nt);
  work(0, n / nt);
  for (auto& x : th) x.join();
  return B2_OK;
}

void rope_table(float theta, int head_dim, int p0, int n_pos, float* out) {
  for (int p = 0; p < n_pos; ++p) {
    for (int i = 0; i < head_dim / 2; ++i) {
      const double freq = pow((double)theta, -2.0 * (double)i / (double)head_dim);
      const double ang = (double)(p0 + p) * freq;
      out[(size_t)p * head_dim + 2 * i] = (float)cos(ang);
      out[(size_t)p * head_dim + 2 * i + 1] = (float)sin(ang);
    }
  }
}

}  // namespace b2
