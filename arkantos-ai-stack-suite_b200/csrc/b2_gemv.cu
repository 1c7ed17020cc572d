// Decode GEMV / skinny GEMM over repacked GGUF weights (Q4_0, Q8_0, Q4_K, Q6_K)
// for 1..8 token rows — the B200 version of the reference's matmul_quantized
// (Singularity/src/core/cortex_a5_engine.cpp:997-1027), whose per-row dot is
// ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 (Singularity/tests/test_and_bench_a5.cpp:184-221)
// and, for K-quants, ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K.
//
// Structure (one persistent CTA per SM, rows split evenly between CTAs):
//   * warp 8 is a producer: its lanes issue one cp.async.bulk (1-D TMA) per
//     (row, plane) of a 16-row x kc-column stage into a ring of smem stages,
//     completing on a full[] mbarrier.  It starts before the grid dependency
//     resolves, so weights stream while the previous kernel drains.
//   * warps 0..7 wait on the grid dependency (PDL), bring the activations
//     into smem (quantizing fp32 in place, bit-exact with the reference's
//     quantizer, or copying pre-quantized planes), then consume stages: each
//     warp owns two rows of a stage, lanes stride over blocks, integer dots
//     with dp4a, per-block fp32 scale products, warp-shuffle reduction.
//   * epilogue: store, residual add, or SwiGLU over interleaved gate/up rows.
// Every mbarrier wait is bounded; on expiry the kernel writes a status code
// and returns.
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kNCW = 8;                  // consumer warps
constexpr int kRW = 2;                   // rows per consumer warp per stage
constexpr int kRG = kNCW * kRW;          // rows per stage
constexpr int kThreads = (kNCW + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 2 * kMaxStages * 8;

struct GemvP {
  const uint8_t* p0;
  const uint8_t* p1;
  int64_t p0_row, p0_chunk, p1_row, p1_chunk;
  int kc, n_chunks;
  int64_t kp, k;
  int64_t row_begin, row_end;
  const float* x;
  int64_t x_stride;
  const int8_t* aq;
  const float* ad;
  const int16_t* absum;
  float* y;
  int64_t y_stride;
  int epilogue;
  int n_stages;
  uint32_t stage_bytes;
  int* status;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kNCW * 32) : "memory"); }

// ---- activation prologue ---------------------------------------------------------
template <int WT, int B>
__device__ void load_act(const GemvP& p, int8_t* aq, float* ad, int16_t* ab, int warp, int lane) {
  const int64_t kp = p.kp;
  if (p.x != nullptr) {
    // Issue every load of a batch of blocks before quantizing any of them, so
    // a warp waits for one memory round trip per batch, not one per block.
    if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
      constexpr int U = 16;
      const int64_t nbk = kp / 32;
      const int64_t total = (int64_t)B * nbk;
      for (int64_t i0 = warp; i0 < total; i0 += (int64_t)kNCW * U) {
        float xv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + (int64_t)u * kNCW;
          float v = 0.0f;
          if (i < total) {
            const int t = (int)(i / nbk);
            const int64_t e = (i - (int64_t)t * nbk) * 32 + lane;
            if (e < p.k) v = __ldg(p.x + t * p.x_stride + e);
          }
          xv[u] = v;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + (int64_t)u * kNCW;
          if (i < total) {
            const int t = (int)(i / nbk);
            const int64_t kb = i - (int64_t)t * nbk;
            uint16_t d16;
            const int8_t q = quant_q8_0_lane(xv[u], &d16);
            aq[t * kp + kb * 32 + lane] = q;
            if (lane == 0) ad[t * nbk + kb] = h2f(d16);
          }
        }
      }
    } else {
      constexpr int U = 4;
      const int64_t nbk = kp / 256;
      const int64_t total = (int64_t)B * nbk;
      for (int64_t i0 = warp; i0 < total; i0 += (int64_t)kNCW * U) {
        float v[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + (int64_t)u * kNCW;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
          if (i < total) {
            const int t = (int)(i / nbk);
            const int64_t e0 = (i - (int64_t)t * nbk) * 256 + lane * 8;
            if (e0 < p.k) {   // k is a multiple of 256: all 8 values are in range
              const float4* src = reinterpret_cast<const float4*>(p.x + t * p.x_stride + e0);
              a = __ldg(src);
              c = __ldg(src + 1);
            }
          }
          v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
          v[u][4] = c.x; v[u][5] = c.y; v[u][6] = c.z; v[u][7] = c.w;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t i = i0 + (int64_t)u * kNCW;
          if (i < total) {
            const int t = (int)(i / nbk);
            const int64_t kb = i - (int64_t)t * nbk;
            const int64_t e0 = kb * 256 + lane * 8;
            int8_t q[8];
            int bs;
            const float d = quant_q8_k_lane(v[u], q, &bs);
            uint2 packed;
            packed.x = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) | ((uint32_t)(uint8_t)q[2] << 16) |
                       ((uint32_t)(uint8_t)q[3] << 24);
            packed.y = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) | ((uint32_t)(uint8_t)q[6] << 16) |
                       ((uint32_t)(uint8_t)q[7] << 24);
            *reinterpret_cast<uint2*>(aq + t * kp + e0) = packed;
            if ((lane & 1) == 0) ab[t * (kp / 16) + kb * 16 + lane / 2] = (int16_t)bs;
            if (lane == 0) ad[t * nbk + kb] = d;
          }
        }
      }
    }
  } else {
    const int tid = warp * 32 + lane;
    const int64_t nq = (int64_t)B * kp / 16;
    for (int64_t i = tid; i < nq; i += kNCW * 32)
      reinterpret_cast<uint4*>(aq)[i] = reinterpret_cast<const uint4*>(p.aq)[i];
    const int64_t nd = (WT == B2_Q4_0 || WT == B2_Q8_0) ? (int64_t)B * kp / 32 : (int64_t)B * kp / 256;
    for (int64_t i = tid; i < nd; i += kNCW * 32) ad[i] = p.ad[i];
    if constexpr (WT == B2_Q4_K || WT == B2_Q6_K) {
      const int64_t nb = (int64_t)B * kp / 16;
      for (int64_t i = tid; i < nb; i += kNCW * 32) ab[i] = p.absum[i];
    }
  }
}

// ---- per-stage compute -------------------------------------------------------------
template <int WT, int B>
__device__ __forceinline__ void compute_stage(const GemvP& p, const uint8_t* sp0, const uint8_t* sp1, int c,
                                              const int8_t* aq, const float* ad, const int16_t* ab, int warp,
                                              int lane, float (&acc)[kRW][B]) {
  const int64_t kp = p.kp;
  const int kc = p.kc;
  if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
    const int nb = kc / 32;
    const int64_t nbk = kp / 32;
    for (int blk = lane; blk < nb; blk += 32) {
      constexpr int W32 = (WT == B2_Q4_0) ? 4 : 8;   // 32-bit words of weight data per block
      uint32_t wv[kRW][W32];
      float dw[kRW];
#pragma unroll
      for (int j = 0; j < kRW; ++j) {
        const int lr = warp * kRW + j;
        const uint4* wp = reinterpret_cast<const uint4*>(sp0 + lr * p.p0_chunk + blk * (W32 * 4));
#pragma unroll
        for (int v = 0; v < W32 / 4; ++v) {
          const uint4 u = wp[v];
          wv[j][4 * v + 0] = u.x;
          wv[j][4 * v + 1] = u.y;
          wv[j][4 * v + 2] = u.z;
          wv[j][4 * v + 3] = u.w;
        }
        dw[j] = h2f(*reinterpret_cast<const uint16_t*>(sp1 + lr * p.p1_chunk + blk * 2));
      }
      const int64_t kb = (int64_t)c * nb + blk;
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(aq + t * kp + kb * 32);
        const uint4 xa = xp[0], xb = xp[1];
        const float dx = ad[t * nbk + kb];
#pragma unroll
        for (int j = 0; j < kRW; ++j) {
          int s;
          if constexpr (WT == B2_Q4_0) {
            s = __dp4a(nib_lo_s8(wv[j][0]), (int)xa.x, 0);
            s = __dp4a(nib_lo_s8(wv[j][1]), (int)xa.y, s);
            s = __dp4a(nib_lo_s8(wv[j][2]), (int)xa.z, s);
            s = __dp4a(nib_lo_s8(wv[j][3]), (int)xa.w, s);
            s = __dp4a(nib_hi_s8(wv[j][0]), (int)xb.x, s);
            s = __dp4a(nib_hi_s8(wv[j][1]), (int)xb.y, s);
            s = __dp4a(nib_hi_s8(wv[j][2]), (int)xb.z, s);
            s = __dp4a(nib_hi_s8(wv[j][3]), (int)xb.w, s);
          } else {
            s = __dp4a((int)wv[j][0], (int)xa.x, 0);
            s = __dp4a((int)wv[j][1], (int)xa.y, s);
            s = __dp4a((int)wv[j][2], (int)xa.z, s);
            s = __dp4a((int)wv[j][3], (int)xa.w, s);
            s = __dp4a((int)wv[j][4], (int)xb.x, s);
            s = __dp4a((int)wv[j][5], (int)xb.y, s);
            s = __dp4a((int)wv[j][6], (int)xb.z, s);
            s = __dp4a((int)wv[j][7], (int)xb.w, s);
          }
          acc[j][t] = __fadd_rn(acc[j][t], __fmul_rn(__fmul_rn(dw[j], dx), (float)s));
        }
      }
    }
  } else if constexpr (WT == B2_Q4_K) {
    const int nsb = kc / 256;
    const int ntask = nsb * 4;
    const int64_t nsbk = kp / 256;
    for (int task = lane; task < ntask; task += 32) {
      const int sb = task >> 2, c4 = task & 3;
      const int64_t col0 = (int64_t)c * kc + sb * 256;   // first column of the super-block
      uint4 q0[kRW], q1[kRW];
      float dd[kRW], dm[kRW];
      int sc0[kRW], sc1[kRW], m0[kRW], m1[kRW];
#pragma unroll
      for (int j = 0; j < kRW; ++j) {
        const uint8_t* bp = sp0 + (warp * kRW + j) * p.p0_chunk + sb * 144;
        const uint32_t dpair = *reinterpret_cast<const uint32_t*>(bp);
        dd[j] = h2f((uint16_t)(dpair & 0xFFFFu));
        dm[j] = h2f((uint16_t)(dpair >> 16));
        const uint8_t* s = bp + 4;
        const int ja = 2 * c4, jb = 2 * c4 + 1;
        if (ja < 4) {
          sc0[j] = s[ja] & 63;
          m0[j] = s[ja + 4] & 63;
          sc1[j] = s[jb] & 63;
          m1[j] = s[jb + 4] & 63;
        } else {
          sc0[j] = (s[ja + 4] & 0x0F) | ((s[ja - 4] >> 6) << 4);
          m0[j] = (s[ja + 4] >> 4) | ((s[ja] >> 6) << 4);
          sc1[j] = (s[jb + 4] & 0x0F) | ((s[jb - 4] >> 6) << 4);
          m1[j] = (s[jb + 4] >> 4) | ((s[jb] >> 6) << 4);
        }
        q0[j] = *reinterpret_cast<const uint4*>(bp + 16 + c4 * 32);
        q1[j] = *reinterpret_cast<const uint4*>(bp + 32 + c4 * 32);
      }
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(aq + t * kp + col0 + c4 * 64);
        const uint4 xa0 = xp[0], xa1 = xp[1], xb0 = xp[2], xb1 = xp[3];
        const uint2 bs = *reinterpret_cast<const uint2*>(ab + t * (kp / 16) + col0 / 16 + c4 * 4);
        const int b01 = (int)(int16_t)(bs.x & 0xFFFFu) + (int)(int16_t)(bs.x >> 16);
        const int b23 = (int)(int16_t)(bs.y & 0xFFFFu) + (int)(int16_t)(bs.y >> 16);
        const float dy = ad[t * nsbk + col0 / 256];
#pragma unroll
        for (int j = 0; j < kRW; ++j) {
          const uint32_t m4 = 0x0F0F0F0Fu;
          int lo = __dp4a((int)(q0[j].x & m4), (int)xa0.x, 0);
          lo = __dp4a((int)(q0[j].y & m4), (int)xa0.y, lo);
          lo = __dp4a((int)(q0[j].z & m4), (int)xa0.z, lo);
          lo = __dp4a((int)(q0[j].w & m4), (int)xa0.w, lo);
          lo = __dp4a((int)(q1[j].x & m4), (int)xa1.x, lo);
          lo = __dp4a((int)(q1[j].y & m4), (int)xa1.y, lo);
          lo = __dp4a((int)(q1[j].z & m4), (int)xa1.z, lo);
          lo = __dp4a((int)(q1[j].w & m4), (int)xa1.w, lo);
          int hi = __dp4a((int)((q0[j].x >> 4) & m4), (int)xb0.x, 0);
          hi = __dp4a((int)((q0[j].y >> 4) & m4), (int)xb0.y, hi);
          hi = __dp4a((int)((q0[j].z >> 4) & m4), (int)xb0.z, hi);
          hi = __dp4a((int)((q0[j].w >> 4) & m4), (int)xb0.w, hi);
          hi = __dp4a((int)((q1[j].x >> 4) & m4), (int)xb1.x, hi);
          hi = __dp4a((int)((q1[j].y >> 4) & m4), (int)xb1.y, hi);
          hi = __dp4a((int)((q1[j].z >> 4) & m4), (int)xb1.z, hi);
          hi = __dp4a((int)((q1[j].w >> 4) & m4), (int)xb1.w, hi);
          const int isum = sc0[j] * lo + sc1[j] * hi;
          const int msum = m0[j] * b01 + m1[j] * b23;
          acc[j][t] = __fadd_rn(acc[j][t], __fmul_rn(__fmul_rn(dd[j], dy), (float)isum));
          acc[j][t] = __fsub_rn(acc[j][t], __fmul_rn(__fmul_rn(dm[j], dy), (float)msum));
        }
      }
    }
  } else {  // Q6_K
    const int nsb = kc / 256;
    const int ntask = nsb * 4;
    const int64_t nsbk = kp / 256;
    for (int task = lane; task < ntask; task += 32) {
      const int sb = task >> 2, h = (task >> 1) & 1, gp = task & 1;
      const int64_t col0 = (int64_t)c * kc + sb * 256;
      uint32_t la[kRW][8], lb[kRW][8];
      int sca0[kRW], sca1[kRW], scb0[kRW], scb1[kRW];
      float d6[kRW];
#pragma unroll
      for (int j = 0; j < kRW; ++j) {
        const int lr = warp * kRW + j;
        const uint8_t* bp = sp0 + lr * p.p0_chunk + sb * 208;
        const uint4 l0 = *reinterpret_cast<const uint4*>(bp + h * 64 + gp * 32);
        const uint4 l1 = *reinterpret_cast<const uint4*>(bp + h * 64 + gp * 32 + 16);
        const uint4 h0 = *reinterpret_cast<const uint4*>(bp + 128 + h * 32);
        const uint4 h1 = *reinterpret_cast<const uint4*>(bp + 128 + h * 32 + 16);
        const uint32_t qlw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t qhw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t a = (qlw[i] & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * gp)) & 0x03030303u) << 4);
          const uint32_t b = ((qlw[i] >> 4) & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * gp + 4)) & 0x03030303u) << 4);
          la[j][i] = (a + 0x60606060u) ^ 0x80808080u;
          lb[j][i] = (b + 0x60606060u) ^ 0x80808080u;
        }
        const int8_t* sc = reinterpret_cast<const int8_t*>(bp + 192);
        sca0[j] = sc[h * 8 + 2 * gp];
        sca1[j] = sc[h * 8 + 2 * gp + 1];
        scb0[j] = sc[h * 8 + 2 * (gp + 2)];
        scb1[j] = sc[h * 8 + 2 * (gp + 2) + 1];
        d6[j] = h2f(*reinterpret_cast<const uint16_t*>(sp1 + lr * p.p1_chunk + sb * 2));
      }
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const int8_t* xb = aq + t * kp + col0 + h * 128;
        const uint4 xa0 = *reinterpret_cast<const uint4*>(xb + gp * 32);
        const uint4 xa1 = *reinterpret_cast<const uint4*>(xb + gp * 32 + 16);
        const uint4 xb0 = *reinterpret_cast<const uint4*>(xb + (gp + 2) * 32);
        const uint4 xb1 = *reinterpret_cast<const uint4*>(xb + (gp + 2) * 32 + 16);
        const float dy = ad[t * nsbk + col0 / 256];
#pragma unroll
        for (int j = 0; j < kRW; ++j) {
          int a0 = __dp4a((int)la[j][0], (int)xa0.x, 0);
          a0 = __dp4a((int)la[j][1], (int)xa0.y, a0);
          a0 = __dp4a((int)la[j][2], (int)xa0.z, a0);
          a0 = __dp4a((int)la[j][3], (int)xa0.w, a0);
          int a1 = __dp4a((int)la[j][4], (int)xa1.x, 0);
          a1 = __dp4a((int)la[j][5], (int)xa1.y, a1);
          a1 = __dp4a((int)la[j][6], (int)xa1.z, a1);
          a1 = __dp4a((int)la[j][7], (int)xa1.w, a1);
          int b0 = __dp4a((int)lb[j][0], (int)xb0.x, 0);
          b0 = __dp4a((int)lb[j][1], (int)xb0.y, b0);
          b0 = __dp4a((int)lb[j][2], (int)xb0.z, b0);
          b0 = __dp4a((int)lb[j][3], (int)xb0.w, b0);
          int b1 = __dp4a((int)lb[j][4], (int)xb1.x, 0);
          b1 = __dp4a((int)lb[j][5], (int)xb1.y, b1);
          b1 = __dp4a((int)lb[j][6], (int)xb1.z, b1);
          b1 = __dp4a((int)lb[j][7], (int)xb1.w, b1);
          const int isum = sca0[j] * a0 + sca1[j] * a1 + scb0[j] * b0 + scb1[j] * b1;
          acc[j][t] = __fadd_rn(acc[j][t], __fmul_rn(__fmul_rn(d6[j], dy), (float)isum));
        }
      }
    }
  }
}

template <int WT, int B>
__global__ void __launch_bounds__(kThreads, (B <= 4) ? 2 : 1) gemv_kernel(const GemvP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint8_t* ring = smem + kBarBytes;
  int8_t* aq = reinterpret_cast<int8_t*>(ring + (size_t)p.n_stages * p.stage_bytes);
  const int64_t kp = p.kp;
  float* ad = reinterpret_cast<float*>(aq + (size_t)B * kp);
  const int64_t nd = (WT == B2_Q4_0 || WT == B2_Q8_0) ? kp / 32 : kp / 256;
  // bsum rows are read 8 bytes at a time: keep the array 16-byte aligned.
  int16_t* ab = reinterpret_cast<int16_t*>(reinterpret_cast<uint8_t*>(ad) + (((size_t)B * nd * 4 + 15) / 16 * 16));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = p.n_stages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // Balanced contiguous row range of this CTA, in whole row pairs.
  const int64_t n = p.row_end - p.row_begin;
  const int64_t n_pairs = (n + 1) / 2;
  const int64_t pr0 = n_pairs * blockIdx.x / gridDim.x;
  const int64_t pr1 = n_pairs * (blockIdx.x + 1) / gridDim.x;
  const int64_t r0 = p.row_begin + 2 * pr0;
  const int64_t r1 = min(p.row_begin + 2 * pr1, p.row_end);
  const int n_groups = r1 > r0 ? (int)((r1 - r0 + kRG - 1) / kRG) : 0;
  const int total = n_groups * p.n_chunks;

  if (warp == kNCW) {
    // ---------------- producer ----------------
    for (int st = 0; st < total; ++st) {
      const int s = st % ns;
      const uint32_t ph = (uint32_t)(st / ns) & 1u;
      if (st >= ns && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.status, 2)) return;
      const int g = st / p.n_chunks, c = st - g * p.n_chunks;
      const int64_t rb = r0 + (int64_t)g * kRG;
      const int rows = (int)min((int64_t)kRG, r1 - rb);
      uint8_t* sp0 = ring + (size_t)s * p.stage_bytes;
      uint8_t* sp1 = sp0 + kRG * p.p0_chunk;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * (p.p0_chunk + p.p1_chunk)));
      __syncwarp();
      if (lane < rows) {
        bulk_g2s(sp0 + lane * p.p0_chunk, p.p0 + (rb + lane) * p.p0_row + (int64_t)c * p.p0_chunk,
                 (uint32_t)p.p0_chunk, &full[s]);
        if (p.p1_chunk)
          bulk_g2s(sp1 + lane * p.p1_chunk, p.p1 + (rb + lane) * p.p1_row + (int64_t)c * p.p1_chunk,
                   (uint32_t)p.p1_chunk, &full[s]);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  load_act<WT, B>(p, aq, ad, ab, warp, lane);
  consumer_sync();

  int st = 0;
  for (int g = 0; g < n_groups; ++g) {
    float acc[kRW][B];
#pragma unroll
    for (int j = 0; j < kRW; ++j)
#pragma unroll
      for (int t = 0; t < B; ++t) acc[j][t] = 0.0f;
    for (int c = 0; c < p.n_chunks; ++c, ++st) {
      const int s = st % ns;
      const uint32_t ph = (uint32_t)(st / ns) & 1u;
      if (!mbar_wait_bounded(&full[s], ph, p.status, 1)) return;
      const uint8_t* sp0 = ring + (size_t)s * p.stage_bytes;
      const uint8_t* sp1 = sp0 + kRG * p.p0_chunk;
      compute_stage<WT, B>(p, sp0, sp1, c, aq, ad, ab, warp, lane, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    const int64_t rb = r0 + (int64_t)g * kRG + warp * kRW;
    float v[kRW][B];
#pragma unroll
    for (int j = 0; j < kRW; ++j)
#pragma unroll
      for (int t = 0; t < B; ++t) v[j][t] = warp_sum(acc[j][t]);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < B; ++t) {
        float* yt = p.y + t * p.y_stride;
        if (p.epilogue == EPI_SWIGLU) {
          if (rb + 1 < r1) {
            const float gt = v[0][t], up = v[1][t];
            yt[rb / 2] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
          }
        } else {
#pragma unroll
          for (int j = 0; j < kRW; ++j) {
            if (rb + j < r1) {
              if (p.epilogue == EPI_ACCUM) yt[rb + j] = __fadd_rn(yt[rb + j], v[j][t]);
              else yt[rb + j] = v[j][t];
            }
          }
        }
      }
    }
  }
}

template <int WT, int B>
int launch_t(const GemvP& p, int grid, size_t smem, cudaStream_t s) {
  auto kern = gemv_kernel<WT, B>;
  static size_t configured = 0;
  if (smem > configured) {
    B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
  return B2_OK;
}

template <int WT>
int launch_w(const GemvP& p, int B, int grid, size_t smem, cudaStream_t s) {
  switch (B) {
    case 1: return launch_t<WT, 1>(p, grid, smem, s);
    case 2: return launch_t<WT, 2>(p, grid, smem, s);
    case 3: return launch_t<WT, 3>(p, grid, smem, s);
    case 4: return launch_t<WT, 4>(p, grid, smem, s);
    case 5: return launch_t<WT, 5>(p, grid, smem, s);
    case 6: return launch_t<WT, 6>(p, grid, smem, s);
    case 7: return launch_t<WT, 7>(p, grid, smem, s);
    case 8: return launch_t<WT, 8>(p, grid, smem, s);
  }
  set_error("gemv: n_tok %d outside [1, 8]", B);
  return B2_ERR_INVALID;
}

}  // namespace

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  const QMatrix& w = *a.w;
  B2_CHECK_ARG(a.n_tok >= 1 && a.n_tok <= 8, "n_tok must be in [1, 8]");
  B2_CHECK_ARG(a.row_begin >= 0 && a.row_end <= w.n_rows && a.row_begin <= a.row_end, "row range");
  B2_CHECK_ARG(a.y != nullptr, "y");
  B2_CHECK_ARG(a.x != nullptr || a.act != nullptr, "x or act");
  if (a.row_end == a.row_begin) return B2_OK;
  GemvP p = {};
  p.p0 = w.plane0;
  p.p1 = w.plane1;
  p.p0_row = w.p0_row;
  p.p0_chunk = w.p0_chunk;
  p.p1_row = w.p1_row;
  p.p1_chunk = w.p1_chunk;
  p.kc = w.kc;
  p.n_chunks = w.n_chunks;
  p.kp = w.kp;
  p.k = w.k;
  p.row_begin = a.row_begin;
  p.row_end = a.row_end;
  p.x = a.act ? nullptr : a.x;
  p.x_stride = a.x_stride;
  if (a.act) {
    B2_CHECK_ARG(a.act->kp == w.kp && a.act->type == act_type_for(w.type) && a.act->n_tok >= a.n_tok,
                 "activation planes do not match the matrix");
    p.aq = a.act->qs;
    p.ad = a.act->d;
    p.absum = a.act->bsum;
  }
  p.y = a.y;
  p.y_stride = a.y_stride;
  p.epilogue = a.epilogue;
  p.status = a.status;
  const bool k_quant = (w.type == B2_Q4_K || w.type == B2_Q6_K);
  // Same carve-up as the kernel: qs [B][kp] | d [B][nd] fp32 (16 B aligned end) | bsum [B][kp/16].
  const size_t nd = (size_t)(k_quant ? w.kp / 256 : w.kp / 32);
  const size_t act_bytes = (size_t)a.n_tok * w.kp + ((size_t)a.n_tok * nd * 4 + 15) / 16 * 16 +
                           (k_quant ? (size_t)a.n_tok * (w.kp / 16) * 2 : 0);
  const size_t stage = ((size_t)kRG * (w.p0_chunk + w.p1_chunk) + 127) / 128 * 128;
  const size_t smem_cap = 227 * 1024;
  size_t avail = smem_cap - kBarBytes - ((act_bytes + 127) / 128 * 128);
  int ns = (int)std::min<size_t>(kMaxStages, avail / stage);
  if (ns > 4) ns = 4;
  if (ns < 2) {
    set_error("gemv: shared memory too small for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  p.n_stages = ns;
  p.stage_bytes = (uint32_t)stage;
  const size_t smem = kBarBytes + (size_t)ns * stage + ((act_bytes + 127) / 128 * 128);
  int dev = 0, n_sm = kSMs;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t rows = a.row_end - a.row_begin;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(n_sm, (rows + kRG - 1) / kRG));
  switch (w.type) {
    case B2_Q4_0: return launch_w<B2_Q4_0>(p, a.n_tok, grid, smem, s);
    case B2_Q8_0: return launch_w<B2_Q8_0>(p, a.n_tok, grid, smem, s);
    case B2_Q4_K: return launch_w<B2_Q4_K>(p, a.n_tok, grid, smem, s);
    case B2_Q6_K: return launch_w<B2_Q6_K>(p, a.n_tok, grid, smem, s);
  }
  set_error("gemv: unsupported weight type %d", w.type);
  return B2_ERR_UNSUPPORTED;
}

}  // namespace b2
