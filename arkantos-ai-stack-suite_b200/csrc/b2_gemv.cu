// Decode GEMV / skinny GEMM over repacked GGUF weights (Q4_0, Q8_0, Q4_K, Q6_K)
// for 1..8 token rows — the B200 version of the reference's matmul_quantized
// (Singularity/src/core/cortex_a5_engine.cpp:997-1027), whose per-row dot is
// ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 (Singularity/tests/test_and_bench_a5.cpp:184-221)
// and, for K-quants, ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K.
//
// Structure (one persistent CTA per SM, rows split evenly between CTAs):
//   * warp 8 is the producer: for each stage of RG consecutive whole rows its
//     lane 0 issues one cp.async.bulk (1-D TMA) per plane — the rows of a
//     repacked plane are contiguous — into a ring of smem stages, completing
//     on a full[] mbarrier.  It runs ahead of the grid dependency, so weights
//     stream while the previous kernel drains (PDL).
//   * warps 0..7 wait on the grid dependency, bring the activations into smem
//     (quantizing fp32 in the CTA, bit-exact with the reference's quantizer,
//     or copying pre-quantized planes), then consume stages: 8/RG warps share
//     a row, lanes stride over its blocks, integer dots with dp4a, per-block
//     fp32 scale products, warp-shuffle reduction, then the warps of a row
//     combine through shared memory.
//   * epilogue: store, residual add, or SwiGLU over interleaved gate/up rows.
// Every mbarrier wait is bounded; on expiry the kernel writes a status code
// and returns.
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kNCW = 8;                  // consumer warps
constexpr int kThreads = (kNCW + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 2 * kMaxStages * 8;
constexpr int kMaxTok = 8;

struct GemvP {
  const uint8_t* p0;
  const uint8_t* p1;
  int64_t p0_row, p1_row;
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
  int rg;                 // rows per stage (1, 2, 4 or 8)
  uint32_t stage_bytes;
  int* status;
  PeerOut peer;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kNCW * 32) : "memory"); }

// Output (token t, row) of the store / residual-add epilogues; with a
// tensor-parallel exchange the value goes to this rank's slot of every rank.
__device__ __forceinline__ void store_y(const GemvP& p, int t, int64_t row, float v) {
  const int64_t off = t * p.y_stride + row;
  if (p.peer.n) {
    for (int j = 0; j < p.peer.n; ++j) p.peer.dst[j][off] = v;
    return;
  }
  float* yp = p.y + off;
  *yp = p.epilogue == EPI_ACCUM ? __fadd_rn(*yp, v) : v;
}

// After every consumer thread of the CTA has stored: count the CTA; the last
// CTA of the grid publishes the next epoch to every rank's flag.  Stores reach
// peers before the count (fence.sys by the counting thread after the CTA
// barrier), and the count before the flags (fence.sys in the last CTA).
__device__ __forceinline__ void signal_peers(const GemvP& p) {
  __threadfence_system();
  const unsigned int prev = atomicAdd(p.peer.done, 1u);
  if (prev == gridDim.x - 1) {
    __threadfence_system();
    const unsigned long long e = *p.peer.epoch + 1ull;
    *p.peer.epoch = e;
    *p.peer.done = 0u;
    for (int j = 0; j < p.peer.n; ++j) st_release_sys_u64(p.peer.flag[j], e);
  }
}

// ---- activation prologue ---------------------------------------------------------
template <int WT, int B>
__device__ void load_act(const GemvP& p, int8_t* aq, float* ad, int16_t* ab, int warp, int lane) {
  const int64_t kp = p.kp;
  const int tid = warp * 32 + lane;
  if (p.x != nullptr) {
    if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
      // One 32-value block per thread: eight float4 loads in flight, then the
      // reference quantizer on registers (no shuffles).
      const int64_t nbk = kp / 32;
      for (int64_t i = tid; i < (int64_t)B * nbk; i += kNCW * 32) {
        const int t = (int)(i / nbk);
        const int64_t kb = i - (int64_t)t * nbk;
        float v[32];
        if (kb * 32 < p.k) {   // k is a multiple of 32: the block is entirely in range
          const float4* src = reinterpret_cast<const float4*>(p.x + t * p.x_stride + kb * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 f = __ldg(src + j);
            v[4 * j] = f.x;
            v[4 * j + 1] = f.y;
            v[4 * j + 2] = f.z;
            v[4 * j + 3] = f.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.0f;
        }
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fmul_rn(amax, 1.0f / 127.0f);
        const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sc = __fmul_rn(v[j], id);
          const float tt = sc >= 0.0f ? __fadd_rn(sc, 0.5f) : __fsub_rn(sc, 0.5f);
          int q = __float2int_rz(tt);
          q = q < -127 ? -127 : (q > 127 ? 127 : q);
          w[j >> 2] |= ((uint32_t)(uint8_t)q) << (8 * (j & 3));
        }
        uint4* dst = reinterpret_cast<uint4*>(aq + t * kp + kb * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        ad[t * nbk + kb] = h2f(f2h_rn(d));
      }
    } else {
      // One 256-value super-block per warp, batches of U in flight.
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

// ---- one row of a stage ---------------------------------------------------------------
// Lanes of the warps sharing the row stride over its blocks starting at
// `first` with step `step`; partial sums accumulate into acc[B].
template <int WT, int B>
__device__ __forceinline__ void compute_row(const uint8_t* rp0, const uint8_t* rp1, int64_t kp, const int8_t* aq,
                                            const float* ad, const int16_t* ab, int first, int step, float (&acc)[B]) {
  if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
    const int nb = (int)(kp / 32);
    constexpr int W32 = (WT == B2_Q4_0) ? 4 : 8;
#pragma unroll 2
    for (int blk = first; blk < nb; blk += step) {
      uint32_t wv[W32];
      const uint4* wp = reinterpret_cast<const uint4*>(rp0 + blk * (W32 * 4));
#pragma unroll
      for (int v = 0; v < W32 / 4; ++v) {
        const uint4 u = wp[v];
        wv[4 * v + 0] = u.x;
        wv[4 * v + 1] = u.y;
        wv[4 * v + 2] = u.z;
        wv[4 * v + 3] = u.w;
      }
      const float dw = h2f(reinterpret_cast<const uint16_t*>(rp1)[blk]);
      int lo[4], hi[4];
      if constexpr (WT == B2_Q4_0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = nib_lo_s8(wv[j]);
          hi[j] = nib_hi_s8(wv[j]);
        }
      }
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(aq + t * kp + blk * 32);
        const uint4 xa = xp[0], xb = xp[1];
        int s;
        if constexpr (WT == B2_Q4_0) {
          s = __dp4a(lo[0], (int)xa.x, 0);
          s = __dp4a(lo[1], (int)xa.y, s);
          s = __dp4a(lo[2], (int)xa.z, s);
          s = __dp4a(lo[3], (int)xa.w, s);
          s = __dp4a(hi[0], (int)xb.x, s);
          s = __dp4a(hi[1], (int)xb.y, s);
          s = __dp4a(hi[2], (int)xb.z, s);
          s = __dp4a(hi[3], (int)xb.w, s);
        } else {
          s = __dp4a((int)wv[0], (int)xa.x, 0);
          s = __dp4a((int)wv[1], (int)xa.y, s);
          s = __dp4a((int)wv[2], (int)xa.z, s);
          s = __dp4a((int)wv[3], (int)xa.w, s);
          s = __dp4a((int)wv[4], (int)xb.x, s);
          s = __dp4a((int)wv[5], (int)xb.y, s);
          s = __dp4a((int)wv[6], (int)xb.z, s);
          s = __dp4a((int)wv[7], (int)xb.w, s);
        }
        acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dw, ad[t * (kp / 32) + blk]), (float)s));
      }
    }
  } else if constexpr (WT == B2_Q4_K) {
    const int ntask = (int)(kp / 256) * 4;
    for (int task = first; task < ntask; task += step) {
      const int sb = task >> 2, c4 = task & 3;
      const uint8_t* bp = rp0 + sb * 144;
      const uint32_t dpair = *reinterpret_cast<const uint32_t*>(bp);
      const float dd = h2f((uint16_t)(dpair & 0xFFFFu));
      const float dm = h2f((uint16_t)(dpair >> 16));
      const uint8_t* s = bp + 4;
      const int ja = 2 * c4, jb = 2 * c4 + 1;
      int sc0, sc1, m0, m1;
      if (ja < 4) {
        sc0 = s[ja] & 63;
        m0 = s[ja + 4] & 63;
        sc1 = s[jb] & 63;
        m1 = s[jb + 4] & 63;
      } else {
        sc0 = (s[ja + 4] & 0x0F) | ((s[ja - 4] >> 6) << 4);
        m0 = (s[ja + 4] >> 4) | ((s[ja] >> 6) << 4);
        sc1 = (s[jb + 4] & 0x0F) | ((s[jb - 4] >> 6) << 4);
        m1 = (s[jb + 4] >> 4) | ((s[jb] >> 6) << 4);
      }
      const uint4 q0 = *reinterpret_cast<const uint4*>(bp + 16 + c4 * 32);
      const uint4 q1 = *reinterpret_cast<const uint4*>(bp + 32 + c4 * 32);
      const uint32_t m4 = 0x0F0F0F0Fu;
      const int l[8] = {(int)(q0.x & m4), (int)(q0.y & m4), (int)(q0.z & m4), (int)(q0.w & m4),
                        (int)(q1.x & m4), (int)(q1.y & m4), (int)(q1.z & m4), (int)(q1.w & m4)};
      const int h[8] = {(int)((q0.x >> 4) & m4), (int)((q0.y >> 4) & m4), (int)((q0.z >> 4) & m4),
                        (int)((q0.w >> 4) & m4), (int)((q1.x >> 4) & m4), (int)((q1.y >> 4) & m4),
                        (int)((q1.z >> 4) & m4), (int)((q1.w >> 4) & m4)};
      const int64_t col0 = (int64_t)sb * 256;
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(aq + t * kp + col0 + c4 * 64);
        const uint4 xa0 = xp[0], xa1 = xp[1], xb0 = xp[2], xb1 = xp[3];
        const uint2 bs = *reinterpret_cast<const uint2*>(ab + t * (kp / 16) + col0 / 16 + c4 * 4);
        const int b01 = (int)(int16_t)(bs.x & 0xFFFFu) + (int)(int16_t)(bs.x >> 16);
        const int b23 = (int)(int16_t)(bs.y & 0xFFFFu) + (int)(int16_t)(bs.y >> 16);
        const float dy = ad[t * (kp / 256) + sb];
        int lo = __dp4a(l[0], (int)xa0.x, 0);
        lo = __dp4a(l[1], (int)xa0.y, lo);
        lo = __dp4a(l[2], (int)xa0.z, lo);
        lo = __dp4a(l[3], (int)xa0.w, lo);
        lo = __dp4a(l[4], (int)xa1.x, lo);
        lo = __dp4a(l[5], (int)xa1.y, lo);
        lo = __dp4a(l[6], (int)xa1.z, lo);
        lo = __dp4a(l[7], (int)xa1.w, lo);
        int hi = __dp4a(h[0], (int)xb0.x, 0);
        hi = __dp4a(h[1], (int)xb0.y, hi);
        hi = __dp4a(h[2], (int)xb0.z, hi);
        hi = __dp4a(h[3], (int)xb0.w, hi);
        hi = __dp4a(h[4], (int)xb1.x, hi);
        hi = __dp4a(h[5], (int)xb1.y, hi);
        hi = __dp4a(h[6], (int)xb1.z, hi);
        hi = __dp4a(h[7], (int)xb1.w, hi);
        const int isum = sc0 * lo + sc1 * hi;
        const int msum = m0 * b01 + m1 * b23;
        acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dd, dy), (float)isum));
        acc[t] = __fsub_rn(acc[t], __fmul_rn(__fmul_rn(dm, dy), (float)msum));
      }
    }
  } else {  // Q6_K
    const int ntask = (int)(kp / 256) * 4;
    for (int task = first; task < ntask; task += step) {
      const int sb = task >> 2, hh = (task >> 1) & 1, gp = task & 1;
      const uint8_t* bp = rp0 + sb * 208;
      const uint4 l0 = *reinterpret_cast<const uint4*>(bp + hh * 64 + gp * 32);
      const uint4 l1 = *reinterpret_cast<const uint4*>(bp + hh * 64 + gp * 32 + 16);
      const uint4 h0 = *reinterpret_cast<const uint4*>(bp + 128 + hh * 32);
      const uint4 h1 = *reinterpret_cast<const uint4*>(bp + 128 + hh * 32 + 16);
      const uint32_t qlw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
      const uint32_t qhw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      int la[8], lb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t a = (qlw[i] & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * gp)) & 0x03030303u) << 4);
        const uint32_t b = ((qlw[i] >> 4) & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * gp + 4)) & 0x03030303u) << 4);
        la[i] = (int)((a + 0x60606060u) ^ 0x80808080u);
        lb[i] = (int)((b + 0x60606060u) ^ 0x80808080u);
      }
      const int8_t* sc = reinterpret_cast<const int8_t*>(bp + 192);
      const int sca0 = sc[hh * 8 + 2 * gp], sca1 = sc[hh * 8 + 2 * gp + 1];
      const int scb0 = sc[hh * 8 + 2 * (gp + 2)], scb1 = sc[hh * 8 + 2 * (gp + 2) + 1];
      const float d6 = h2f(reinterpret_cast<const uint16_t*>(rp1)[sb]);
      const int64_t col0 = (int64_t)sb * 256 + hh * 128;
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const int8_t* xb = aq + t * kp + col0;
        const uint4 xa0 = *reinterpret_cast<const uint4*>(xb + gp * 32);
        const uint4 xa1 = *reinterpret_cast<const uint4*>(xb + gp * 32 + 16);
        const uint4 xb0 = *reinterpret_cast<const uint4*>(xb + (gp + 2) * 32);
        const uint4 xb1 = *reinterpret_cast<const uint4*>(xb + (gp + 2) * 32 + 16);
        const float dy = ad[t * (kp / 256) + sb];
        int a0 = __dp4a(la[0], (int)xa0.x, 0);
        a0 = __dp4a(la[1], (int)xa0.y, a0);
        a0 = __dp4a(la[2], (int)xa0.z, a0);
        a0 = __dp4a(la[3], (int)xa0.w, a0);
        int a1 = __dp4a(la[4], (int)xa1.x, 0);
        a1 = __dp4a(la[5], (int)xa1.y, a1);
        a1 = __dp4a(la[6], (int)xa1.z, a1);
        a1 = __dp4a(la[7], (int)xa1.w, a1);
        int b0 = __dp4a(lb[0], (int)xb0.x, 0);
        b0 = __dp4a(lb[1], (int)xb0.y, b0);
        b0 = __dp4a(lb[2], (int)xb0.z, b0);
        b0 = __dp4a(lb[3], (int)xb0.w, b0);
        int b1 = __dp4a(lb[4], (int)xb1.x, 0);
        b1 = __dp4a(lb[5], (int)xb1.y, b1);
        b1 = __dp4a(lb[6], (int)xb1.z, b1);
        b1 = __dp4a(lb[7], (int)xb1.w, b1);
        const int isum = sca0 * a0 + sca1 * a1 + scb0 * b0 + scb1 * b1;
        acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(d6, dy), (float)isum));
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
  __shared__ float red[2][kNCW][kMaxTok];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = p.n_stages;
  const int rg = p.rg;
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
  const int total = r1 > r0 ? (int)((r1 - r0 + rg - 1) / rg) : 0;
  const uint32_t p1_off = (uint32_t)(rg * p.p0_row);

  if (warp == kNCW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int st = 0; st < total; ++st) {
        const int s = st % ns;
        const uint32_t ph = (uint32_t)(st / ns) & 1u;
        if (st >= ns && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.status, 2)) return;
        const int64_t rb = r0 + (int64_t)st * rg;
        const int rows = (int)min((int64_t)rg, r1 - rb);
        uint8_t* sp = ring + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * (p.p0_row + p.p1_row)));
        bulk_g2s(sp, p.p0 + rb * p.p0_row, (uint32_t)(rows * p.p0_row), &full[s]);
        if (p.p1_row) bulk_g2s(sp + p1_off, p.p1 + rb * p.p1_row, (uint32_t)(rows * p.p1_row), &full[s]);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  // A timed-out wait does not leave the loop early: the warp keeps taking the
  // same named barriers as the others (skipping its waits and math), so the
  // CTA always reaches its end and, with an exchange, still signals peers.
  pdl_wait();
  load_act<WT, B>(p, aq, ad, ab, warp, lane);
  consumer_sync();
  bool ok = true;

  const int wpr = kNCW / rg;               // warps per row
  const int my_row = warp / wpr;           // row of the stage this warp works on
  const int sub = warp - my_row * wpr;
  const int first = sub * 32 + lane, step = wpr * 32;
  const int tid = warp * 32 + lane;
  for (int st = 0; st < total; ++st) {
    const int s = st % ns;
    const uint32_t ph = (uint32_t)(st / ns) & 1u;
    if (ok) ok = mbar_wait_bounded(&full[s], ph, p.status, 1);
    const uint8_t* sp = ring + (size_t)s * p.stage_bytes;
    const int64_t rb = r0 + (int64_t)st * rg;
    const int rows = (int)min((int64_t)rg, r1 - rb);
    float acc[B];
#pragma unroll
    for (int t = 0; t < B; ++t) acc[t] = 0.0f;
    if (ok && my_row < rows)
      compute_row<WT, B>(sp + my_row * p.p0_row, sp + p1_off + my_row * p.p1_row, kp, aq, ad, ab, first, step, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (wpr == 1 && p.epilogue != EPI_SWIGLU) {
      // Each warp owns a whole row: reduce and write, no cross-warp step.
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && my_row < rows) store_y(p, t, rb + my_row, v);
      }
      continue;
    }
#pragma unroll
    for (int t = 0; t < B; ++t) {
      const float v = warp_sum(acc[t]);
      if (lane == 0) red[st & 1][warp][t] = v;
    }
    consumer_sync();
    // Combine the warps of each row; one thread per (row, token) writes.
    if (p.epilogue == EPI_SWIGLU) {
      if (tid < (rows / 2) * B) {
        const int pr = tid / B, t = tid - pr * B;
        float g = 0.0f, u = 0.0f;
        for (int w = 0; w < wpr; ++w) {
          g = __fadd_rn(g, red[st & 1][(2 * pr) * wpr + w][t]);
          u = __fadd_rn(u, red[st & 1][(2 * pr + 1) * wpr + w][t]);
        }
        const int64_t row = rb + 2 * pr;
        p.y[t * p.y_stride + row / 2] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, b2_expf(-g))), u);
      }
    } else if (tid < rows * B) {
      const int r = tid / B, t = tid - r * B;
      float v = 0.0f;
      for (int w = 0; w < wpr; ++w) v = __fadd_rn(v, red[st & 1][r * wpr + w][t]);
      store_y(p, t, rb + r, v);
    }
  }
  if (p.peer.n) {
    __threadfence_system();   // this thread's peer stores, before the CTA is counted
    consumer_sync();
    if (warp == 0 && lane == 0) signal_peers(p);
  }
}

// 227 KB opt-in per block, less 1 KB for the kernel's static shared memory.
constexpr int kSmemCap = 227 * 1024 - 1024;

template <int WT, int B>
int set_smem_attr() {
  B2_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<WT, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap));
  return B2_OK;
}

template <int WT>
int set_smem_attr_all() {
  int rc = set_smem_attr<WT, 1>();
  if (!rc) rc = set_smem_attr<WT, 2>();
  if (!rc) rc = set_smem_attr<WT, 3>();
  if (!rc) rc = set_smem_attr<WT, 4>();
  if (!rc) rc = set_smem_attr<WT, 5>();
  if (!rc) rc = set_smem_attr<WT, 6>();
  if (!rc) rc = set_smem_attr<WT, 7>();
  if (!rc) rc = set_smem_attr<WT, 8>();
  return rc;
}

template <int WT, int B>
int launch_t(const GemvP& p, int grid, size_t smem, cudaStream_t s) {
  auto kern = gemv_kernel<WT, B>;
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

int prepare_gemv_kernels() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return B2_OK;
  int rc = set_smem_attr_all<B2_Q4_0>();
  if (!rc) rc = set_smem_attr_all<B2_Q8_0>();
  if (!rc) rc = set_smem_attr_all<B2_Q4_K>();
  if (!rc) rc = set_smem_attr_all<B2_Q6_K>();
  if (!rc && dev >= 0 && dev < 64) done[dev] = true;
  return rc;
}

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  int prc = prepare_gemv_kernels();
  if (prc) return prc;
  const QMatrix& w = *a.w;
  B2_CHECK_ARG(a.n_tok >= 1 && a.n_tok <= kMaxTok, "n_tok must be in [1, 8]");
  B2_CHECK_ARG(a.row_begin >= 0 && a.row_end <= w.n_rows && a.row_begin <= a.row_end, "row range");
  B2_CHECK_ARG(a.y != nullptr, "y");
  B2_CHECK_ARG(a.x != nullptr || a.act != nullptr, "x or act");
  B2_CHECK_ARG(w.n_chunks == 1, "matrix layout");
  B2_CHECK_ARG(a.epilogue != EPI_SWIGLU || (a.row_begin % 2) == 0, "SwiGLU rows must start on a pair");
  if (a.row_end == a.row_begin) return B2_OK;
  GemvP p = {};
  p.p0 = w.plane0;
  p.p1 = w.plane1;
  p.p0_row = w.p0_row;
  p.p1_row = w.p1_row;
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
  if (a.peer && a.peer->n > 0) {
    B2_CHECK_ARG(a.epilogue == EPI_STORE && a.peer->n <= kMaxTp && a.peer->done && a.peer->epoch,
                 "peer exchange needs the store epilogue and its counters");
    p.peer = *a.peer;
  } else {
    p.peer = PeerOut{};
  }
  const bool k_quant = (w.type == B2_Q4_K || w.type == B2_Q6_K);
  // Same carve-up as the kernel: qs [B][kp] | d [B][nd] fp32 (16 B aligned end) | bsum [B][kp/16].
  const size_t nd = (size_t)(k_quant ? w.kp / 256 : w.kp / 32);
  const size_t act_bytes = (size_t)a.n_tok * w.kp + ((size_t)a.n_tok * nd * 4 + 15) / 16 * 16 +
                           (k_quant ? (size_t)a.n_tok * (w.kp / 16) * 2 : 0);
  const size_t row_b = (size_t)(w.p0_row + w.p1_row);
  // Rows per stage: up to 8 whole rows within ~24 KB (at least 2 for SwiGLU pairs).
  int rg = 8;
  while (rg > 1 && (size_t)rg * row_b > 24 * 1024) rg /= 2;
  if (a.epilogue == EPI_SWIGLU && rg < 2) rg = 2;
  const size_t stage = ((size_t)rg * row_b + 127) / 128 * 128;
  const size_t smem_cap = kSmemCap;
  const size_t fixed = kBarBytes + ((act_bytes + 127) / 128 * 128);
  if (fixed + 2 * stage > smem_cap) {
    set_error("gemv: shared memory too small for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  int ns = (int)std::min<size_t>(6, (smem_cap - fixed) / stage);
  // Keep two CTAs per SM possible when the activations are small.
  while (ns > 3 && fixed + (size_t)ns * stage > 112 * 1024) --ns;
  p.n_stages = ns;
  p.rg = rg;
  p.stage_bytes = (uint32_t)stage;
  const size_t smem = fixed + (size_t)ns * stage;
  const int n_sm = sm_count();
  const int64_t rows = a.row_end - a.row_begin;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(n_sm, (rows + rg - 1) / rg));
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
