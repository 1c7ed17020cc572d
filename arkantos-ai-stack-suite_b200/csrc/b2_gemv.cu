// Decode GEMV / skinny GEMM over tiled GGUF weights (Q4_0, Q8_0, Q4_K, Q6_K)
// for 1..8 token rows — the B200 version of the reference's matmul_quantized
// (Singularity/src/core/cortex_a5_engine.cpp:997-1027), whose per-row dot is
// ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 (Singularity/tests/test_and_bench_a5.cpp:184-221)
// and, for K-quants, ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K.
//
// Weights are in the tile layout (8-row tiles, S unit ranges per row, see
// QMatrix).  One CTA per SM takes a contiguous run of tile groups; a group is
// P = 8/S tiles whose S ranges are worked by the 8 consumer warps (warp w:
// tile w/S, range w%S).
//   * warp 8 is the producer: lane 0 streams each stage — for every tile of
//     the group the next U unit slots of all its ranges, one contiguous
//     cp.async.bulk (1-D TMA) per tile — into a ring of shared-memory stages
//     completing on full[] mbarriers.  It starts before the grid dependency
//     resolves, so weights stream while the previous kernel drains (PDL).
//   * the activations are quantized once per launch by a small kernel
//     (bit-exact with the reference's quantizers) into an image of the
//     shared-memory layout; the producer copies that image into every CTA
//     once the grid dependency resolves, and warps 0..7 then take the
//     stages.  Integer dots are exact: for 1-2 tokens with dp4a (lane =
//     tile row x unit residue mod 4), for 3-8 tokens with int8 mma.sync
//     (m16n8k32; m16n8k16 for Q6_K's 16-weight groups; tokens are the M
//     rows, the tile's 8 rows the N columns).  Each unit's integer sums are
//     scaled in fp32 as the reference does, into four partial sums by unit
//     residue mod 4; a range's sum is (a0 + a1) + (a2 + a3) and the S ranges
//     of a row are added in order through shared memory — one order for
//     every batch size (restated by the oracle's orc_tile_row_dot).
//   * epilogue: store, residual add, SwiGLU over interleaved gate/up rows,
//     or the tensor-parallel exchange into every rank's gather buffer.
// Every mbarrier wait is bounded; a warp whose wait expires records a status
// code and runs to the end without waiting or computing, so the named
// barriers stay matched and the CTA always exits.
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

// Consumer warps: 16 for the mma kernels (the two warps of a range split its
// four unit residues into pairs), 8 for the dp4a kernels; plus one producer.
constexpr int kMaxNCW = 16;
constexpr int ncw_for(int mode) { return mode == 0 ? 16 : 8; }
constexpr int kMaxStages = 6;
constexpr int kBarBytes = 128;           // full[kMaxStages], empty[kMaxStages], act, padded
constexpr int kMaxTok = 8;
constexpr int kDp4aMaxTok = 2;           // dp4a up to this many tokens, mma.sync above
constexpr uint32_t kM4 = 0x0F0F0F0Fu;

struct GemvP {
  const uint8_t* w;
  int type, nu, S, L, slot_bytes;
  int64_t tile_bytes, n_rows, n_tiles, k;
  int n_tok, n_act_tok;   // tokens computed; token rows quantized into shared memory (8 for mma)
  const float* x;
  int64_t x_stride;
  float* y;
  int64_t y_stride;
  int epilogue;
  int U, n_stages;
  uint32_t stage_bytes;   // P tiles x U x S slots
  int kq;                 // activation row bytes (k rounded up to 128)
  uint32_t off_dx, off_bs, act_bytes;   // activation carve-up (bytes from the activation base)
  const uint8_t* act_img; // the quantized activations in that carve-up (global), or null:
                          // the consumers quantize x into shared memory themselves
  int* status;
  PeerOut peer;
};

__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}
// The S warps of tile slot p (barrier ids 2..9).
__device__ __forceinline__ void tile_sync(int p, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + p), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Activation image (global and in shared memory): codes [n_act_tok][kq] |
// fp32 scale per (token, unit) | int16 block sums per (token, unit).  The
// codes of token t start at t*kq.  For the dp4a kernels they are in natural
// order; for the mma kernels each token's codes are stored in fragment order:
//   Q8_K (256-value units, 64 words w): the 16 words thread q of a warp
//     needs, idx = 2j + h <-> word 8j + 4h + q, sit in 16-byte chunks i = idx/4
//     at physical chunk ((4i + q) + 4*(t & 1)) & 15 of the unit's 256 bytes;
//   Q8_0 (32-value blocks): words q and q+4 of block u are one 8-byte slot,
//     slot ((u & 3)*4 + q + 4*(t & 3)) & 15 of the 128 bytes of blocks u & ~3.
// The rotations by token spread the 8 tokens of a fragment load over all
// banks.
__device__ __forceinline__ void act_frag16(const uint8_t* trow, int u, int g, int q, uint32_t (&a)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 v = lds128(trow + u * 256 + (((4 * i + q) + 4 * (g & 1)) & 15) * 16);
    a[4 * i] = v.x;
    a[4 * i + 1] = v.y;
    a[4 * i + 2] = v.z;
    a[4 * i + 3] = v.w;
  }
}
__device__ __forceinline__ uint2 act_frag2(const uint8_t* trow, int u, int g, int q) {
  return *reinterpret_cast<const uint2*>(trow + (u >> 2) * 128 + ((((u & 3) * 4 + q) + 4 * (g & 3)) & 15) * 8);
}
__device__ __forceinline__ uint4 act_chunk16(const uint8_t* trow, int c) { return lds128(trow + c * 16); }

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// D[16x8] = A[16xK] (tokens x k, int8; rows 8..15 zero) * B[Kx8] (k x weight rows).
__device__ __forceinline__ void mma_k32_s8u8(int& c0, int& c1, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  int4 d;   // d.z, d.w: rows 8..15 of D, the zero token rows
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d.x), "=r"(d.y), "=r"(d.z), "=r"(d.w)
      : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0), "r"(b1), "r"(0));
  c0 = d.x;
  c1 = d.y;
}
__device__ __forceinline__ void mma_k32_s8s8(int& c0, int& c1, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  int4 d;   // d.z, d.w: rows 8..15 of D, the zero token rows
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d.x), "=r"(d.y), "=r"(d.z), "=r"(d.w)
      : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0), "r"(b1), "r"(0));
  c0 = d.x;
  c1 = d.y;
}
__device__ __forceinline__ void mma_k16_s8u8(int& c0, int& c1, uint32_t a0, uint32_t b0) {
  int4 d;   // d.z, d.w: rows 8..15 of D, the zero token rows
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(d.x), "=r"(d.y), "=r"(d.z), "=r"(d.w)
               : "r"(a0), "r"(0), "r"(b0), "r"(0));
  c0 = d.x;
  c1 = d.y;
}

__device__ __forceinline__ int ubyte(uint32_t w, int b) { return (int)((w >> (8 * b)) & 0xFFu); }
__device__ __forceinline__ int sbyte(uint32_t w, int b) { return (int)(int8_t)((w >> (8 * b)) & 0xFFu); }

// Q4_K 6-bit scales and mins of one row's 12 packed bytes (words s0, s1, s2):
// sc[0..3], m[0..3], sc[4..7], m[4..7] as the bytes of four words.
__device__ __forceinline__ void q4k_scales(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t& sl, uint32_t& ml,
                                           uint32_t& sh, uint32_t& mh) {
  sl = s0 & 0x3F3F3F3Fu;
  ml = s1 & 0x3F3F3F3Fu;
  sh = (s2 & kM4) | ((s0 >> 2) & 0x30303030u);
  mh = ((s2 >> 4) & kM4) | ((s1 >> 2) & 0x30303030u);
}

// ---- activation image ------------------------------------------------------------------
// fp32 x [n_tok][k] -> the image: codes, the fp32 scale of every unit, and the
// block sums the unit terms need (Q4_0: per 32; Q4_K: per 32 as pairs of
// Q8_K sums; Q6_K: Q8_K's per 16).  Token rows n_tok..n_act_tok-1 are zero.
// Threads tid of nthreads (a multiple of 32) share the work; img is global
// memory (the quantize kernel) or the GEMV's shared memory.
template <bool MMA>
__device__ void quantize_image(const float* __restrict__ x, int64_t x_stride, int n_tok, int n_act_tok, int type,
                               int nu, int kq, uint32_t off_dx, uint32_t off_bs, uint8_t* img, int64_t tid,
                               int64_t nthreads) {
  float* dxs = reinterpret_cast<float*>(img + off_dx);
  int16_t* bss = reinterpret_cast<int16_t*>(img + off_bs);
  if (type == B2_Q4_0 || type == B2_Q8_0) {
    // One 32-value block per thread: eight float4 loads in flight, then the
    // reference quantizer on registers.
    for (int64_t i = tid; i < (int64_t)n_act_tok * nu; i += nthreads) {
      const int t = (int)(i / nu), b = (int)(i - (int64_t)t * nu);
      uint32_t w[8];
      int sum = 0;
      float dq = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 0;
      if (t < n_tok) {
        const float4* src = reinterpret_cast<const float4*>(x + t * x_stride + (int64_t)b * 32);
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = __ldg(src + j);
          v[4 * j] = f.x;
          v[4 * j + 1] = f.y;
          v[4 * j + 2] = f.z;
          v[4 * j + 3] = f.w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fmul_rn(amax, 1.0f / 127.0f);
        const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sc = __fmul_rn(v[j], id);
          const float tt = sc >= 0.0f ? __fadd_rn(sc, 0.5f) : __fsub_rn(sc, 0.5f);
          int q = __float2int_rz(tt);
          q = q < -127 ? -127 : (q > 127 ? 127 : q);
          sum += q;
          w[j >> 2] |= ((uint32_t)(uint8_t)q) << (8 * (j & 3));
        }
        dq = h2f(f2h_rn(d));
      }
      uint8_t* trow = img + (int64_t)t * kq;
      if constexpr (MMA) {
        uint8_t* base = trow + (b >> 2) * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint2*>(base + ((((b & 3) * 4 + q) + 4 * (t & 3)) & 15) * 8) = make_uint2(w[q], w[q + 4]);
      } else {
        *reinterpret_cast<uint4*>(trow + b * 32) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(trow + b * 32 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
      }
      dxs[t * nu + b] = dq;
      if (type == B2_Q4_0) bss[t * nu + b] = (int16_t)sum;
    }
  } else {
    // One 256-value super-block per warp, 8 values per lane.
    const int lane = threadIdx.x & 31;
    for (int64_t i = tid >> 5; i < (int64_t)n_act_tok * nu; i += nthreads >> 5) {
      const int t = (int)(i / nu), b = (int)(i - (int64_t)t * nu);
      int8_t q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int bs = 0;
      float d = 0.0f;
      if (t < n_tok) {   // warp-uniform
        const float4* src = reinterpret_cast<const float4*>(x + t * x_stride + (int64_t)b * 256 + lane * 8);
        const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
        const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        d = quant_q8_k_lane(v, q, &bs);
      }
      const uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
                          ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
      const uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
                          ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
      uint8_t* unit = img + (int64_t)t * kq + (int64_t)b * 256;
      if constexpr (MMA) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int wi = 2 * lane + h2;   // word 8j + 4h + q of the unit
          const int j = wi >> 3, h = (wi >> 2) & 1, qq = wi & 3;
          const int idx = 2 * j + h;
          *reinterpret_cast<uint32_t*>(unit + ((((idx >> 2) * 4 + qq) + 4 * (t & 1)) & 15) * 16 + (idx & 3) * 4) =
              h2 ? w1 : w0;
        }
      } else {
        *reinterpret_cast<uint2*>(unit + lane * 8) = make_uint2(w0, w1);
      }
      if (lane == 0) dxs[t * nu + b] = d;
      if (type == B2_Q6_K) {
        if ((lane & 1) == 0) bss[(t * nu + b) * 16 + lane / 2] = (int16_t)bs;
      } else {
        const int b32 = bs + __shfl_xor_sync(0xffffffffu, bs, 2);
        if ((lane & 3) == 0) bss[(t * nu + b) * 8 + lane / 4] = (int16_t)b32;
      }
    }
  }
}

template <bool MMA>
__global__ void quantize_image_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, int n_act_tok,
                                      int type, int nu, int kq, uint32_t off_dx, uint32_t off_bs, uint8_t* img) {
  pdl_wait();
  pdl_launch_dependents();
  quantize_image<MMA>(x, x_stride, n_tok, n_act_tok, type, nu, kq, off_dx, off_bs, img,
                      (int64_t)blockIdx.x * blockDim.x + threadIdx.x, (int64_t)gridDim.x * blockDim.x);
}

// ---- mma path: one unit for token g (= lane/4), tile rows 2q, 2q+1 (q = lane%4) ------------
template <int WT>
__device__ __forceinline__ void mma_unit(const GemvP& p, const uint8_t* sl, const uint8_t* act, int u, int g, int q,
                                         float& acc0, float& acc1) {
  const uint8_t* trow = act + g * p.kq;
  const float* dxs = reinterpret_cast<const float*>(act + p.off_dx);
  const int16_t* bss = reinterpret_cast<const int16_t*>(act + p.off_bs);
  const float dx = dxs[g * p.nu + u];
  if constexpr (WT == B2_Q4_0) {
    const uint32_t w = lds32(sl + 16 * g + 4 * q);
    const uint2 a = act_frag2(trow, u, g, q);
    int c0, c1;
    mma_k32_s8u8(c0, c1, a.x, a.y, w & kM4, (w >> 4) & kM4);
    const int corr = 8 * (int)bss[g * p.nu + u];
    const uint32_t dw = lds32(sl + 128 + 4 * q);
    acc0 = __fadd_rn(acc0, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw & 0xFFFFu)), dx), (float)(c0 - corr)));
    acc1 = __fadd_rn(acc1, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw >> 16)), dx), (float)(c1 - corr)));
  } else if constexpr (WT == B2_Q8_0) {
    const uint2 a = act_frag2(trow, u, g, q);
    int c0, c1;
    mma_k32_s8s8(c0, c1, a.x, a.y, lds32(sl + 16 * g + 4 * q), lds32(sl + 128 + 16 * g + 4 * q));
    const uint32_t dw = lds32(sl + 256 + 4 * q);
    acc0 = __fadd_rn(acc0, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw & 0xFFFFu)), dx), (float)c0));
    acc1 = __fadd_rn(acc1, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw >> 16)), dx), (float)c1));
  } else if constexpr (WT == B2_Q4_K) {
    const uint8_t* m0 = sl + 1024 + 32 * q;   // d|dmin|scales of rows 2q and 2q+1
    uint32_t sl0, ml0, sh0, mh0, sl1, ml1, sh1, mh1;
    q4k_scales(lds32(m0 + 4), lds32(m0 + 8), lds32(m0 + 12), sl0, ml0, sh0, mh0);
    q4k_scales(lds32(m0 + 20), lds32(m0 + 24), lds32(m0 + 28), sl1, ml1, sh1, mh1);
    const uint8_t* qrow = sl + 128 * g;
    uint32_t af[16];
    act_frag16(trow, u, g, q, af);
    int is0 = 0, is1 = 0;
#pragma unroll
    for (int jc = 0; jc < 4; ++jc) {
      const uint32_t w0 = lds32(qrow + 16 * ((2 * jc + g) & 7) + 4 * q);
      const uint32_t w1 = lds32(qrow + 16 * ((2 * jc + 1 + g) & 7) + 4 * q);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * jc + h;
        const uint32_t b0 = h ? (w0 >> 4) & kM4 : w0 & kM4;
        const uint32_t b1 = h ? (w1 >> 4) & kM4 : w1 & kM4;
        int c0, c1;
        mma_k32_s8u8(c0, c1, af[2 * j], af[2 * j + 1], b0, b1);
        const int s0 = j < 4 ? ubyte(sl0, j) : ubyte(sh0, j - 4);
        const int s1 = j < 4 ? ubyte(sl1, j) : ubyte(sh1, j - 4);
        is0 += s0 * c0;
        is1 += s1 * c1;
      }
    }
    const uint4 b32 = lds128(reinterpret_cast<const uint8_t*>(bss + (g * p.nu + u) * 8));
    int ms0 = __dp2a_lo((int)b32.x, (int)ml0, 0);
    ms0 = __dp2a_hi((int)b32.y, (int)ml0, ms0);
    ms0 = __dp2a_lo((int)b32.z, (int)mh0, ms0);
    ms0 = __dp2a_hi((int)b32.w, (int)mh0, ms0);
    int ms1 = __dp2a_lo((int)b32.x, (int)ml1, 0);
    ms1 = __dp2a_hi((int)b32.y, (int)ml1, ms1);
    ms1 = __dp2a_lo((int)b32.z, (int)mh1, ms1);
    ms1 = __dp2a_hi((int)b32.w, (int)mh1, ms1);
    const uint32_t dd0 = lds32(m0), dd1 = lds32(m0 + 16);
    acc0 = __fadd_rn(acc0, __fmul_rn(__fmul_rn(h2f((uint16_t)(dd0 & 0xFFFFu)), dx), (float)is0));
    acc0 = __fsub_rn(acc0, __fmul_rn(__fmul_rn(h2f((uint16_t)(dd0 >> 16)), dx), (float)ms0));
    acc1 = __fadd_rn(acc1, __fmul_rn(__fmul_rn(h2f((uint16_t)(dd1 & 0xFFFFu)), dx), (float)is1));
    acc1 = __fsub_rn(acc1, __fmul_rn(__fmul_rn(h2f((uint16_t)(dd1 >> 16)), dx), (float)ms1));
  } else {  // Q6_K
    const uint8_t* qlr = sl + 128 * g;
    const uint8_t* qhr = sl + 1024 + 64 * g;
    const uint8_t* scp = sl + 1536 + 32 * q;   // scales of rows 2q and 2q+1
    const int16_t* bs = bss + (g * p.nu + u) * 16;
    uint32_t af[16];
    act_frag16(trow, u, g, q, af);
    int is0 = 0, is1 = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint32_t qh0 = lds32(qhr + 16 * ((2 * hh + g) & 3) + 4 * q);
      const uint32_t qh1 = lds32(qhr + 16 * ((2 * hh + 1 + g) & 3) + 4 * q);
      const uint32_t sa0 = lds32(scp + 8 * hh), sb0 = lds32(scp + 8 * hh + 4);
      const uint32_t sa1 = lds32(scp + 16 + 8 * hh), sb1 = lds32(scp + 16 + 8 * hh + 4);
#pragma unroll
      for (int a1 = 0; a1 < 2; ++a1) {
        const uint32_t ql0 = lds32(qlr + 16 * ((4 * hh + 2 * a1 + g) & 7) + 4 * q);
        const uint32_t ql1 = lds32(qlr + 16 * ((4 * hh + 2 * a1 + 1 + g) & 7) + 4 * q);
#pragma unroll
        for (int nh = 0; nh < 2; ++nh) {
          const int a = a1 + 2 * nh;   // quartile of the half
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const uint32_t ql = hf ? ql1 : ql0;
            const uint32_t qh = hf ? qh1 : qh0;
            const uint32_t lo = nh ? (ql >> 4) & kM4 : ql & kM4;
            const uint32_t b0 = lo | (((qh >> (2 * a)) & 0x03030303u) << 4);
            const int i = hh * 8 + a * 2 + hf;   // 16-weight group of the super-block
            int c0, c1;
            mma_k16_s8u8(c0, c1, af[i], b0);
            const int b = 32 * (int)bs[i];
            const int gi = a * 2 + hf;           // group within the half
            const int s0 = gi < 4 ? sbyte(sa0, gi) : sbyte(sb0, gi - 4);
            const int s1 = gi < 4 ? sbyte(sa1, gi) : sbyte(sb1, gi - 4);
            is0 += s0 * (c0 - b);
            is1 += s1 * (c1 - b);
          }
        }
      }
    }
    const uint32_t dw = lds32(sl + 1664 + 4 * q);
    acc0 = __fadd_rn(acc0, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw & 0xFFFFu)), dx), (float)is0));
    acc1 = __fadd_rn(acc1, __fmul_rn(__fmul_rn(h2f((uint16_t)(dw >> 16)), dx), (float)is1));
  }
}

// ---- dp4a path: one unit, tile row g, tokens 0..B-1 -----------------------------------------
template <int WT, int B>
__device__ __forceinline__ void dp4a_unit(const GemvP& p, const uint8_t* sl, const uint8_t* act, int u, int g,
                                          float (&acc)[B]) {
  const float* dxs = reinterpret_cast<const float*>(act + p.off_dx);
  const int16_t* bss = reinterpret_cast<const int16_t*>(act + p.off_bs);
  if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
    uint32_t lo[4], hi[4];
    float dw;
    if constexpr (WT == B2_Q4_0) {
      const uint4 w = lds128(sl + 16 * g);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo[j] = ww[j] & kM4;
        hi[j] = (ww[j] >> 4) & kM4;
      }
      dw = h2f(*reinterpret_cast<const uint16_t*>(sl + 128 + 2 * g));
    } else {
      const uint4 a = lds128(sl + 16 * g), b = lds128(sl + 128 + 16 * g);
      lo[0] = a.x; lo[1] = a.y; lo[2] = a.z; lo[3] = a.w;
      hi[0] = b.x; hi[1] = b.y; hi[2] = b.z; hi[3] = b.w;
      dw = h2f(*reinterpret_cast<const uint16_t*>(sl + 256 + 2 * g));
    }
#pragma unroll
    for (int t = 0; t < B; ++t) {
      const uint8_t* trow = act + t * p.kq;
      const uint4 xa = act_chunk16(trow, 2 * u), xb = act_chunk16(trow, 2 * u + 1);
      int s;
      if constexpr (WT == B2_Q4_0) {
        s = dp4a_us(lo[0], xa.x, 0);
        s = dp4a_us(lo[1], xa.y, s);
        s = dp4a_us(lo[2], xa.z, s);
        s = dp4a_us(lo[3], xa.w, s);
        s = dp4a_us(hi[0], xb.x, s);
        s = dp4a_us(hi[1], xb.y, s);
        s = dp4a_us(hi[2], xb.z, s);
        s = dp4a_us(hi[3], xb.w, s);
        s -= 8 * (int)bss[t * p.nu + u];
      } else {
        s = dp4a_ss(lo[0], xa.x, 0);
        s = dp4a_ss(lo[1], xa.y, s);
        s = dp4a_ss(lo[2], xa.z, s);
        s = dp4a_ss(lo[3], xa.w, s);
        s = dp4a_ss(hi[0], xb.x, s);
        s = dp4a_ss(hi[1], xb.y, s);
        s = dp4a_ss(hi[2], xb.z, s);
        s = dp4a_ss(hi[3], xb.w, s);
      }
      acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dw, dxs[t * p.nu + u]), (float)s));
    }
  } else if constexpr (WT == B2_Q4_K) {
    const uint4 meta = lds128(sl + 1024 + 16 * g);
    uint32_t sl4, ml4, sh4, mh4;
    q4k_scales(meta.y, meta.z, meta.w, sl4, ml4, sh4, mh4);
    const float dd = h2f((uint16_t)(meta.x & 0xFFFFu)), dm = h2f((uint16_t)(meta.x >> 16));
    const uint8_t* qrow = sl + 128 * g;
    int is[B];
#pragma unroll
    for (int t = 0; t < B; ++t) is[t] = 0;
#pragma unroll
    for (int jc = 0; jc < 4; ++jc) {
      const uint4 qa = lds128(qrow + 16 * ((2 * jc + g) & 7));
      const uint4 qb = lds128(qrow + 16 * ((2 * jc + 1 + g) & 7));
      const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const int s_lo = jc < 2 ? ubyte(sl4, 2 * jc) : ubyte(sh4, 2 * jc - 4);
      const int s_hi = jc < 2 ? ubyte(sl4, 2 * jc + 1) : ubyte(sh4, 2 * jc - 3);
#pragma unroll
      for (int t = 0; t < B; ++t) {
        const uint8_t* trow = act + t * p.kq;
        const int c0 = u * 16 + 4 * jc;   // the 64 activation bytes of this 32-byte qs pair
        const uint4 x0 = act_chunk16(trow, c0), x1 = act_chunk16(trow, c0 + 1);
        const uint4 x2 = act_chunk16(trow, c0 + 2), x3 = act_chunk16(trow, c0 + 3);
        const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
        int dl = 0, dh = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dl = dp4a_us(qw[i] & kM4, xl[i], dl);
          dh = dp4a_us((qw[i] >> 4) & kM4, xh[i], dh);
        }
        is[t] += s_lo * dl + s_hi * dh;
      }
    }
#pragma unroll
    for (int t = 0; t < B; ++t) {
      const uint4 b32 = lds128(reinterpret_cast<const uint8_t*>(bss + (t * p.nu + u) * 8));
      int m = __dp2a_lo((int)b32.x, (int)ml4, 0);
      m = __dp2a_hi((int)b32.y, (int)ml4, m);
      m = __dp2a_lo((int)b32.z, (int)mh4, m);
      m = __dp2a_hi((int)b32.w, (int)mh4, m);
      const float dx = dxs[t * p.nu + u];
      acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dd, dx), (float)is[t]));
      acc[t] = __fsub_rn(acc[t], __fmul_rn(__fmul_rn(dm, dx), (float)m));
    }
  } else {  // Q6_K
    const uint8_t* qlr = sl + 128 * g;
    const uint8_t* qhr = sl + 1024 + 64 * g;
    const uint4 sc4 = lds128(sl + 1536 + 16 * g);
    const uint32_t scw[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
    const float d6 = h2f(*reinterpret_cast<const uint16_t*>(sl + 1664 + 2 * g));
    int is[B];
#pragma unroll
    for (int t = 0; t < B; ++t) is[t] = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint4 h0 = lds128(qhr + 16 * ((2 * hh + g) & 3)), h1 = lds128(qhr + 16 * ((2 * hh + 1 + g) & 3));
      const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
      for (int a1 = 0; a1 < 2; ++a1) {
        const uint4 l0 = lds128(qlr + 16 * ((4 * hh + 2 * a1 + g) & 7));
        const uint4 l1 = lds128(qlr + 16 * ((4 * hh + 2 * a1 + 1 + g) & 7));
        const uint32_t ql[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int nh = 0; nh < 2; ++nh) {
          const int a = a1 + 2 * nh;   // quartile of the half
          uint32_t v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            v[i] = (nh ? (ql[i] >> 4) & kM4 : ql[i] & kM4) | (((qh[i] >> (2 * a)) & 0x03030303u) << 4);
          const int g0 = hh * 8 + a * 2;   // groups g0 (l 0..15) and g0+1 (l 16..31)
          const int s0 = sbyte(scw[g0 >> 2], g0 & 3), s1 = sbyte(scw[(g0 + 1) >> 2], (g0 + 1) & 3);
#pragma unroll
          for (int t = 0; t < B; ++t) {
            const uint8_t* trow = act + t * p.kq;
            const uint4 xa = act_chunk16(trow, u * 16 + g0), xb = act_chunk16(trow, u * 16 + g0 + 1);
            int d0 = dp4a_us(v[0], xa.x, 0);
            d0 = dp4a_us(v[1], xa.y, d0);
            d0 = dp4a_us(v[2], xa.z, d0);
            d0 = dp4a_us(v[3], xa.w, d0);
            int d1 = dp4a_us(v[4], xb.x, 0);
            d1 = dp4a_us(v[5], xb.y, d1);
            d1 = dp4a_us(v[6], xb.z, d1);
            d1 = dp4a_us(v[7], xb.w, d1);
            const int16_t* bs = bss + (t * p.nu + u) * 16;
            is[t] += s0 * (d0 - 32 * (int)bs[g0]) + s1 * (d1 - 32 * (int)bs[g0 + 1]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < B; ++t)
      acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(d6, dxs[t * p.nu + u]), (float)is[t]));
  }
}

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
// peers before the count (fence.sys by each storing thread, then the CTA
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

// Finishes a tile: red[(r*WR + h)*64 + e] holds the partial of range r (half
// h of its residues when WR = 2) for element e = token*8 + row; one warp adds
// them — range sums (A + B), then the ranges in order — and writes.
template <int WR>
__device__ __forceinline__ float tile_total(const float* red, int S, int e) {
  float v = WR == 2 ? __fadd_rn(red[e], red[64 + e]) : red[e];
  for (int r = 1; r < S; ++r)
    v = __fadd_rn(v, WR == 2 ? __fadd_rn(red[r * 128 + e], red[r * 128 + 64 + e]) : red[r * 64 + e]);
  return v;
}

template <int WR>
__device__ __forceinline__ void finish_tile(const GemvP& p, const float* red, int64_t tile, int lane) {
  if (p.epilogue == EPI_SWIGLU) {
    // lane = token*4 + pair; tile rows (2*pair, 2*pair+1) are (gate, up) of one feature
    const int t = lane >> 2, pr = lane & 3;
    const int64_t row = tile * 8 + 2 * pr;
    if (t < p.n_tok && row < p.n_rows) {
      const float gs = tile_total<WR>(red, p.S, t * 8 + 2 * pr);
      const float us = tile_total<WR>(red, p.S, t * 8 + 2 * pr + 1);
      p.y[t * p.y_stride + row / 2] = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, b2_expf(-gs))), us);
    }
    return;
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int e = lane + 32 * hh;
    const int t = e >> 3, rr = e & 7;
    const int64_t row = tile * 8 + rr;
    if (t < p.n_tok && row < p.n_rows) store_y(p, t, row, tile_total<WR>(red, p.S, e));
  }
}

template <int WT, int MODE>   // MODE 0: mma.sync; 1, 2: dp4a over that many tokens
__global__ void __launch_bounds__((ncw_for(MODE) + 1) * 32, 1) gemv_kernel(const GemvP p) {
  constexpr int NW = ncw_for(MODE);        // consumer warps
  constexpr int WR = MODE == 0 ? 2 : 1;    // warps per range
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* act_bar = empty + kMaxStages;
  uint8_t* ring = smem + kBarBytes;
  uint8_t* act = ring + (size_t)p.n_stages * p.stage_bytes;
  __shared__ float red[2][NW][64];   // [group parity][warp = (slot*S + range)*WR + half][token*8 + row]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = p.n_stages;
  const int S = p.S, P = 8 / S;      // tile slots: P tiles of S ranges of WR warps
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    mbar_init(act_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // Tile groups of this CTA (contiguous, balanced) and the stage sequence.
  const int64_t n_groups = (p.n_tiles + P - 1) / P;
  const int64_t g0 = n_groups * blockIdx.x / gridDim.x, g1 = n_groups * (blockIdx.x + 1) / gridDim.x;
  const int n_ch = (p.L + p.U - 1) / p.U;   // stages per group
  const int64_t total = (g1 - g0) * n_ch;
  const uint32_t piece = (uint32_t)p.U * S * p.slot_bytes;   // one tile's part of a stage

  if (warp == NW) {
    // ---------------- producer ----------------
    // The first ns stages need no free slot and go out at once; then, once the
    // previous kernel (the activation quantizer) has finished, the image.
    if (lane == 0) {
      auto issue = [&](int64_t st) {
        const int s = (int)(st % ns);
        const int64_t grp = g0 + st / n_ch;
        const int ch = (int)(st % n_ch);
        const int i0 = ch * p.U, ni = min(p.U, p.L - i0);
        const uint32_t bytes = (uint32_t)ni * S * p.slot_bytes;
        uint32_t tx = 0;
        for (int pp = 0; pp < P; ++pp)
          if (grp * P + pp < p.n_tiles) tx += bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        uint8_t* sp = ring + (size_t)s * p.stage_bytes;
        for (int pp = 0; pp < P; ++pp) {
          const int64_t tile = grp * P + pp;
          if (tile < p.n_tiles)
            bulk_g2s(sp + pp * piece, p.w + tile * p.tile_bytes + (int64_t)i0 * S * p.slot_bytes, bytes, &full[s]);
        }
      };
      const int64_t first = total < ns ? total : ns;
      for (int64_t st = 0; st < first; ++st) issue(st);
      if (p.act_img) {
        pdl_wait();
        mbar_arrive_expect_tx(act_bar, p.act_bytes);
        bulk_g2s(act, p.act_img, p.act_bytes, act_bar);
      }
      for (int64_t st = first; st < total; ++st) {
        const uint32_t ph = (uint32_t)(st / ns) & 1u;
        if (!mbar_wait_bounded(&empty[st % ns], ph ^ 1u, p.status, 2)) return;
        issue(st);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  bool ok = true;
  if (p.act_img) {
    ok = mbar_wait_bounded(act_bar, 0, p.status, 3);
  } else {
    quantize_image<MODE == 0>(p.x, p.x_stride, p.n_tok, p.n_act_tok, p.type, p.nu, p.kq, p.off_dx, p.off_bs, act,
                              warp * 32 + lane, NW * 32);
    consumer_sync(NW * 32);
  }

  const int slot_p = warp / (S * WR), r = (warp / WR) % S, half = warp % WR;
  const int g = lane >> 2, q = lane & 3;     // mma: token g, tile rows 2q, 2q+1
  const int dg = lane & 7, dq = lane >> 3;   // dp4a: tile row dg, unit residue dq
  constexpr int NB = MODE == 0 ? 1 : MODE;
  float acc[2][2];   // mma partial sums [residue of the pair][row]
  float dacc[NB];    // dp4a partial sums [token] of residue dq
  int64_t st = 0;
  for (int64_t grp = g0; grp < g1; ++grp) {
    const int64_t tile = grp * P + slot_p;
    const bool live = tile < p.n_tiles;
    acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.0f;
#pragma unroll
    for (int t = 0; t < NB; ++t) dacc[t] = 0.0f;
    for (int ch = 0; ch < n_ch; ++ch, ++st) {
      const int s = (int)(st % ns);
      const uint32_t ph = (uint32_t)(st / ns) & 1u;
      if (ok) ok = mbar_wait_bounded(&full[s], ph, p.status, 1);
      const int i0 = ch * p.U, ni = min(p.U, p.L - i0);
      if (ok && live) {
        const uint8_t* base = ring + (size_t)s * p.stage_bytes + slot_p * piece;
        // this stage holds units [ua, ub) of the warp's range
        const int ua = r * p.L + i0, ub = min(ua + ni, p.nu);
        const size_t us = (size_t)S * p.slot_bytes;   // slot stride between consecutive units
        const uint8_t* rbase = base + (size_t)r * p.slot_bytes;   // unit ua of the range
        if constexpr (MODE == 0) {
          // units of residue 2*half (acc[0]) and 2*half+1 (acc[1]), in increasing order
          int u = ua;
          while (u < ub) {
            const int res = u & 3;
            if ((res >> 1) != half) {
              u += half ? 2 - res : 4 - res;
            } else if ((res & 1) == 0 && u + 1 < ub) {
              mma_unit<WT>(p, rbase + (size_t)(u - ua) * us, act, u, g, q, acc[0][0], acc[0][1]);
              mma_unit<WT>(p, rbase + (size_t)(u + 1 - ua) * us, act, u + 1, g, q, acc[1][0], acc[1][1]);
              u += 4;
            } else if ((res & 1) == 0) {
              mma_unit<WT>(p, rbase + (size_t)(u - ua) * us, act, u, g, q, acc[0][0], acc[0][1]);
              ++u;
            } else {
              mma_unit<WT>(p, rbase + (size_t)(u - ua) * us, act, u, g, q, acc[1][0], acc[1][1]);
              u += 3;
            }
          }
        } else {
          // the four lane groups take four consecutive units (residues 0..3) at once
          for (int u4 = ua & ~3; u4 < ub; u4 += 4) {
            const int u = u4 + dq;
            if (u >= ua && u < ub) dp4a_unit<WT, NB>(p, rbase + (size_t)(u - ua) * us, act, u, dg, dacc);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // The warp's partial into red[parity][warp][token*8 + row]: (a_2h + a_2h+1)
    // for an mma warp, (a0 + a1) + (a2 + a3) for a dp4a warp.
    float* rw = red[grp & 1][warp];
    if constexpr (MODE == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) rw[g * 8 + 2 * q + e] = __fadd_rn(acc[0][e], acc[1][e]);
    } else {
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        // residues dq and dq^1 are 8 lanes apart, dq and dq^2 16 lanes apart
        float v = __fadd_rn(dacc[t], __shfl_xor_sync(0xffffffffu, dacc[t], 8));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 16));
        if (dq == 0) rw[t * 8 + dg] = v;
      }
    }
    if (S * WR > 1) tile_sync(slot_p, S * WR * 32);
    else __syncwarp();
    if (r == 0 && half == 0 && live) finish_tile<WR>(p, red[grp & 1][slot_p * S * WR], tile, lane);
  }
  if (p.peer.n) {
    __threadfence_system();   // this thread's peer stores, before the CTA is counted
    consumer_sync(NW * 32);
    if (warp == 0 && lane == 0) signal_peers(p);
  }
}

// 227 KB opt-in per block, less the kernel's static shared memory.
constexpr int kSmemCap = 227 * 1024 - (int)sizeof(float) * 2 * kMaxNCW * 64 - 1024;

template <int WT, int MODE>
int set_attr() {
  B2_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<WT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap));
  return B2_OK;
}

template <int WT>
int set_attr_all() {
  int rc = set_attr<WT, 0>();
  if (!rc) rc = set_attr<WT, 1>();
  if (!rc) rc = set_attr<WT, 2>();
  return rc;
}

template <int WT, int MODE>
int launch_t(const GemvP& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((ncw_for(MODE) + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<WT, MODE>, p));
  return B2_OK;
}

template <int WT>
int launch_w(const GemvP& p, int grid, size_t smem, cudaStream_t s) {
  if (p.n_tok > kDp4aMaxTok) return launch_t<WT, 0>(p, grid, smem, s);
  if (p.n_tok == 1) return launch_t<WT, 1>(p, grid, smem, s);
  return launch_t<WT, 2>(p, grid, smem, s);
}

// Carve-up of the activation image for w at n_tok tokens.
struct ActGeom {
  int n_act_tok, kq;
  uint32_t off_dx, off_bs, bytes;
};
ActGeom act_geom(const QMatrix& w, int n_tok) {
  ActGeom g;
  g.n_act_tok = n_tok > kDp4aMaxTok ? kMaxTok : n_tok;
  g.kq = (int)((w.k + 127) / 128 * 128);
  const int bs_per_unit = w.type == B2_Q4_0 ? 1 : w.type == B2_Q4_K ? 8 : w.type == B2_Q6_K ? 16 : 0;
  const size_t qs_b = (size_t)g.n_act_tok * g.kq;
  const size_t dx_b = ((size_t)g.n_act_tok * w.nu * 4 + 15) / 16 * 16;
  const size_t bs_b = ((size_t)g.n_act_tok * w.nu * bs_per_unit * 2 + 15) / 16 * 16;
  g.off_dx = (uint32_t)qs_b;
  g.off_bs = (uint32_t)(qs_b + dx_b);
  g.bytes = (uint32_t)(qs_b + dx_b + bs_b);
  return g;
}

int launch_quantize_image(const QMatrix& w, const float* x, int64_t x_stride, int n_tok, const ActGeom& g,
                          uint8_t* img, cudaStream_t s) {
  const bool k_quant = w.type == B2_Q4_K || w.type == B2_Q6_K;
  const int64_t work = (int64_t)g.n_act_tok * w.nu * (k_quant ? 32 : 1);   // threads wanted
  const int block = 256;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((work + block - 1) / block, 4 * sm_count()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (n_tok > kDp4aMaxTok)
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_image_kernel<true>, x, x_stride, n_tok, g.n_act_tok, w.type, w.nu,
                                   g.kq, g.off_dx, g.off_bs, img));
  else
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_image_kernel<false>, x, x_stride, n_tok, g.n_act_tok, w.type,
                                   w.nu, g.kq, g.off_dx, g.off_bs, img));
  return B2_OK;
}

}  // namespace

size_t gemv_act_image_bytes(const QMatrix& w, int n_tok) { return act_geom(w, n_tok).bytes; }

// Small activations (<= 32 KB of fp32) are quantized by every CTA itself;
// larger ones go through the image in global memory.
bool gemv_needs_image(const QMatrix& w, int n_tok) { return (size_t)n_tok * w.k * 4 > 32 * 1024; }

int prepare_gemv_kernels() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return B2_OK;
  int rc = set_attr_all<B2_Q4_0>();
  if (!rc) rc = set_attr_all<B2_Q8_0>();
  if (!rc) rc = set_attr_all<B2_Q4_K>();
  if (!rc) rc = set_attr_all<B2_Q6_K>();
  if (!rc && dev >= 0 && dev < 64) done[dev] = true;
  return rc;
}

int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  int prc = prepare_gemv_kernels();
  if (prc) return prc;
  const QMatrix& w = *a.w;
  B2_CHECK_ARG(a.n_tok >= 1 && a.n_tok <= kMaxTok, "n_tok must be in [1, 8]");
  B2_CHECK_ARG(a.y != nullptr && a.x != nullptr, "x and y");
  B2_CHECK_ARG(w.data != nullptr && w.nu > 0, "matrix");
  B2_CHECK_ARG(a.epilogue != EPI_SWIGLU || (w.n_rows % 2) == 0, "SwiGLU needs (gate, up) row pairs");
  B2_CHECK_ARG((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.x_stride % 4) == 0,
               "x must be 16-byte aligned with a stride of whole float4s");
  B2_CHECK_ARG(!gemv_needs_image(w, a.n_tok) ||
                   (a.act_img != nullptr && (reinterpret_cast<uintptr_t>(a.act_img) & 15) == 0),
               "activation image scratch (16-byte aligned)");
  GemvP p = {};
  p.w = w.data;
  p.type = w.type;
  p.nu = w.nu;
  p.S = w.splits;
  p.L = w.ulen;
  p.slot_bytes = w.slot_bytes;
  p.tile_bytes = w.tile_bytes;
  p.n_rows = w.n_rows;
  p.n_tiles = w.n_tiles;
  p.k = w.k;
  p.n_tok = a.n_tok;
  p.n_act_tok = a.n_tok > kDp4aMaxTok ? kMaxTok : a.n_tok;
  p.x = a.x;
  p.x_stride = a.x_stride;
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
  const ActGeom ag = act_geom(w, a.n_tok);
  p.kq = ag.kq;
  p.off_dx = ag.off_dx;
  p.off_bs = ag.off_bs;
  p.act_bytes = ag.bytes;
  // Small activations are quantized by each CTA itself (no extra kernel and
  // no dependency on a shared image between consecutive launches); large ones
  // once, into the image every CTA copies.
  const bool in_kernel = !gemv_needs_image(w, a.n_tok);
  p.act_img = in_kernel ? nullptr : a.act_img;
  // Stages of P tiles x U unit steps of all S ranges, U as large as fits ~32 KB.
  const int P = 8 / w.splits;
  const size_t step_b = (size_t)P * w.splits * w.slot_bytes;
  int U = (int)std::max<size_t>(1, (32 * 1024) / step_b);
  U = std::min(U, w.ulen);
  const size_t stage = step_b * U;
  const size_t fixed = kBarBytes + p.act_bytes;
  if (fixed + 2 * stage > (size_t)kSmemCap) {
    set_error("gemv: shared memory too small for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  // With small activations stay within ~100 KB, so that two CTAs fit on an SM
  // and the next launch's producer can stream while this one drains.
  const size_t cap = (in_kernel && fixed + 3 * stage <= 100 * 1024) ? 100 * 1024 : (size_t)kSmemCap;
  const int ns = (int)std::min<size_t>(kMaxStages, (cap - fixed) / stage);
  p.U = U;
  p.n_stages = ns;
  p.stage_bytes = (uint32_t)stage;
  const size_t smem = fixed + (size_t)ns * stage;
  const int64_t groups = (w.n_tiles + P - 1) / P;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(), groups));
  if (!in_kernel) {
    const int qrc = launch_quantize_image(w, a.x, a.x_stride, a.n_tok, ag, a.act_img, s);
    if (qrc) return qrc;
  }
  switch (w.type) {
    case B2_Q4_0: return launch_w<B2_Q4_0>(p, grid, smem, s);
    case B2_Q8_0: return launch_w<B2_Q8_0>(p, grid, smem, s);
    case B2_Q4_K: return launch_w<B2_Q4_K>(p, grid, smem, s);
    case B2_Q6_K: return launch_w<B2_Q6_K>(p, grid, smem, s);
  }
  set_error("gemv: unsupported weight type %d", w.type);
  return B2_ERR_UNSUPPORTED;
}

}  // namespace b2
