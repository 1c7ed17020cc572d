// Decode GEMV / skinny GEMM over tiled GGUF weights (Q4_0, Q8_0, Q4_K, Q6_K)
// for 1..8 token rows — the B200 version of the reference's matmul_quantized
// (Singularity/src/core/cortex_a5_engine.cpp:997-1027), whose per-row dot is
// ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 (Singularity/tests/test_and_bench_a5.cpp:184-221)
// and, for K-quants, ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K.
//
// Weights are in the tile layout (8-row tiles, S unit ranges per row, see
// QMatrix).  One CTA per SM takes a contiguous run of items: tile pairs
// (16 rows) for the mma kernels, groups of P = 8/S tiles for dp4a.
//   * the last warp is the producer: lane 0 streams each stage — for every
//     tile of the item the next U unit slots of all its ranges, one
//     contiguous cp.async.bulk (1-D TMA) per tile — into a ring of
//     shared-memory stages completing on full[] mbarriers.  It starts before
//     the grid dependency resolves, so weights stream while the previous
//     kernel drains (PDL).
//   * the activations are quantized (bit-exact with the reference's
//     quantizers) either by every CTA into shared memory (small inputs) or
//     once per launch by a small kernel into an image of the shared-memory
//     layout that the producer copies in after the grid dependency resolves.
//   * integer dots are exact: for 1-2 tokens with dp4a (8 warps; warp = tile
//     of the group x range, lane = tile row x unit residue mod 4); for 3-8
//     tokens with int8 mma.sync m16n8k32 (m16n8k16 for Q6_K's 16-weight
//     groups) with the tile pair's 16 weight rows as M and the tokens as N
//     (16 warps in sets of S; a set works one tile pair, a warp one range of
//     it for all four unit residues).  Each unit's integer sums are scaled in
//     fp32 as the reference does, into four partial sums by unit residue mod
//     4; a range's sum is (a0 + a1) + (a2 + a3) and the S ranges of a row are
//     added in order through shared memory — one order for every batch size
//     (restated by the oracle's orc_tile_row_dot).
//   * epilogue: store, residual add, SwiGLU over interleaved gate/up rows,
//     or the tensor-parallel exchange into every rank's gather buffer.
// Every mbarrier wait is bounded; a warp whose wait expires records a status
// code and runs to the end without waiting or computing, so the named
// barriers stay matched and the CTA always exits.
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

// Consumer warps: 16 for the mma kernels, 8 for the dp4a kernels; plus one
// producer.
constexpr int kMaxNCW = 16;
constexpr int ncw_for(int mode) { return mode == 0 ? 16 : 8; }
constexpr int kMaxStages = 16;
constexpr int kBarBytes = 512;           // full[kMaxStages], empty[kMaxStages], act, padded
constexpr int kMaxTok = 8;
constexpr int kDp4aMaxTok = 2;           // dp4a up to this many tokens, mma.sync above
constexpr uint32_t kM4 = 0x0F0F0F0Fu;

constexpr int kMaxMat = 64;          // matrices of one multi-matrix launch
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
  RopeKvEpi rope;
  // The matrices of the launch (same type and shape, one shared x): items
  // run over matrix 0's, then matrix 1's, ...; wl[0] = w, yl[0] = y for one.
  int n_mat;
  int64_t ipm;            // items per matrix
  const uint8_t* wl[kMaxMat];
  float* yl[kMaxMat];
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

// Activation image (global and in shared memory): the ActImage carve-up,
// stored by store_q8k_unit / store_q8_0_block (b2_quant.cuh).
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

// Rows-as-M forms: D[16x8] = A[16xK] (weight rows of a tile pair) * B[Kx8]
// (k x tokens).  d[0..3] = (row g, token 2q), (row g, 2q+1), (row g+8, 2q),
// (row g+8, 2q+1) for lane = 4g + q.
__device__ __forceinline__ void mma16_k32_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma16_k32_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma16_k16_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(0));
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
__device__ void quantize_image(const float* __restrict__ x, int64_t x_stride, int n_tok, const ActImage& img,
                               int64_t tid, int64_t nthreads) {
  const int nu = img.nu;
  if (img.type == B2_Q4_0 || img.type == B2_Q8_0) {
    // One 32-value block per thread: eight float4 loads in flight, then the
    // reference quantizer on registers.
    for (int64_t i = tid; i < (int64_t)img.n_act_tok * nu; i += nthreads) {
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
      store_q8_0_block(img, t, b, w, dq, sum);
    }
  } else {
    // One 256-value super-block per warp, 8 values per lane.
    const int lane = threadIdx.x & 31;
    for (int64_t i = tid >> 5; i < (int64_t)img.n_act_tok * nu; i += nthreads >> 5) {
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
      store_q8k_unit(img, t, b, q, d, bs);
    }
  }
}

__global__ void quantize_image_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, const ActImage img) {
  pdl_wait();
  pdl_launch_dependents();
  quantize_image(x, x_stride, n_tok, img, (int64_t)blockIdx.x * blockDim.x + threadIdx.x,
                 (int64_t)gridDim.x * blockDim.x);
}

// ---- mma path: one unit of a 16-row tile pair for tokens 0..7 ------------------------------
// sa, sb: the unit's slot in tile a (rows 0..7 -> D rows 0..7) and tile b
// (D rows 8..15).  Lane 4g + q holds outputs i = 2*tb + e: tile row g of
// tile tb (0: a, 1: b) for token 2q + e.  Each output's fp32 update is the
// reference's per-unit sequence.
template <int WT>
__device__ __forceinline__ void mma2_unit(const GemvP& p, const uint8_t* sa, const uint8_t* sb, const uint8_t* act,
                                          int u, int g, int q, float (&acc)[4]) {
  const float* dxs = reinterpret_cast<const float*>(act + p.off_dx);
  const int16_t* bss = reinterpret_cast<const int16_t*>(act + p.off_bs);
  const float dx0 = dxs[(2 * q) * p.nu + u], dx1 = dxs[(2 * q + 1) * p.nu + u];
  const uint8_t* trow = act + g * p.kq;   // B column g = token g
  if constexpr (WT == B2_Q4_0) {
    const uint32_t wa = lds32(sa + 16 * g + 4 * q), wb = lds32(sb + 16 * g + 4 * q);
    const uint2 b = act_frag2(trow, u, g, q);
    int c[4];
    mma16_k32_u8s8(c, wa & kM4, wb & kM4, (wa >> 4) & kM4, (wb >> 4) & kM4, b.x, b.y);
    const int corr0 = 8 * (int)bss[(2 * q) * p.nu + u], corr1 = 8 * (int)bss[(2 * q + 1) * p.nu + u];
    const float da = h2f(*reinterpret_cast<const uint16_t*>(sa + 128 + 2 * g));
    const float db = h2f(*reinterpret_cast<const uint16_t*>(sb + 128 + 2 * g));
    acc[0] = __fadd_rn(acc[0], __fmul_rn(__fmul_rn(da, dx0), (float)(c[0] - corr0)));
    acc[1] = __fadd_rn(acc[1], __fmul_rn(__fmul_rn(da, dx1), (float)(c[1] - corr1)));
    acc[2] = __fadd_rn(acc[2], __fmul_rn(__fmul_rn(db, dx0), (float)(c[2] - corr0)));
    acc[3] = __fadd_rn(acc[3], __fmul_rn(__fmul_rn(db, dx1), (float)(c[3] - corr1)));
  } else if constexpr (WT == B2_Q8_0) {
    const uint2 b = act_frag2(trow, u, g, q);
    int c[4];
    mma16_k32_s8s8(c, lds32(sa + 16 * g + 4 * q), lds32(sb + 16 * g + 4 * q), lds32(sa + 128 + 16 * g + 4 * q),
                   lds32(sb + 128 + 16 * g + 4 * q), b.x, b.y);
    const float da = h2f(*reinterpret_cast<const uint16_t*>(sa + 256 + 2 * g));
    const float db = h2f(*reinterpret_cast<const uint16_t*>(sb + 256 + 2 * g));
    acc[0] = __fadd_rn(acc[0], __fmul_rn(__fmul_rn(da, dx0), (float)c[0]));
    acc[1] = __fadd_rn(acc[1], __fmul_rn(__fmul_rn(da, dx1), (float)c[1]));
    acc[2] = __fadd_rn(acc[2], __fmul_rn(__fmul_rn(db, dx0), (float)c[2]));
    acc[3] = __fadd_rn(acc[3], __fmul_rn(__fmul_rn(db, dx1), (float)c[3]));
  } else if constexpr (WT == B2_Q4_K) {
    const uint4 ma = lds128(sa + 1024 + 16 * g), mb = lds128(sb + 1024 + 16 * g);
    uint32_t sla, mla, sha, mha, slb, mlb, shb, mhb;
    q4k_scales(ma.y, ma.z, ma.w, sla, mla, sha, mha);
    q4k_scales(mb.y, mb.z, mb.w, slb, mlb, shb, mhb);
    const uint8_t* qa = sa + 128 * g;
    const uint8_t* qb = sb + 128 * g;
    uint32_t af[16];
    act_frag16(trow, u, g, q, af);
    int is[4] = {0, 0, 0, 0};
#pragma unroll
    for (int jc = 0; jc < 4; ++jc) {
      const uint32_t wa0 = lds32(qa + 16 * ((2 * jc + g) & 7) + 4 * q);
      const uint32_t wa1 = lds32(qa + 16 * ((2 * jc + 1 + g) & 7) + 4 * q);
      const uint32_t wb0 = lds32(qb + 16 * ((2 * jc + g) & 7) + 4 * q);
      const uint32_t wb1 = lds32(qb + 16 * ((2 * jc + 1 + g) & 7) + 4 * q);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * jc + h;
        int c[4];
        if (h == 0)
          mma16_k32_u8s8(c, wa0 & kM4, wb0 & kM4, wa1 & kM4, wb1 & kM4, af[2 * j], af[2 * j + 1]);
        else
          mma16_k32_u8s8(c, (wa0 >> 4) & kM4, (wb0 >> 4) & kM4, (wa1 >> 4) & kM4, (wb1 >> 4) & kM4, af[2 * j],
                         af[2 * j + 1]);
        const int sa_j = j < 4 ? ubyte(sla, j) : ubyte(sha, j - 4);
        const int sb_j = j < 4 ? ubyte(slb, j) : ubyte(shb, j - 4);
        is[0] += sa_j * c[0];
        is[1] += sa_j * c[1];
        is[2] += sb_j * c[2];
        is[3] += sb_j * c[3];
      }
    }
    const uint4 b0 = lds128(reinterpret_cast<const uint8_t*>(bss + ((2 * q) * p.nu + u) * 8));
    const uint4 b1 = lds128(reinterpret_cast<const uint8_t*>(bss + ((2 * q + 1) * p.nu + u) * 8));
    auto msum = [](const uint4& bq, uint32_t ml, uint32_t mh) {
      int m = __dp2a_lo((int)bq.x, (int)ml, 0);
      m = __dp2a_hi((int)bq.y, (int)ml, m);
      m = __dp2a_lo((int)bq.z, (int)mh, m);
      return __dp2a_hi((int)bq.w, (int)mh, m);
    };
    const int ms[4] = {msum(b0, mla, mha), msum(b1, mla, mha), msum(b0, mlb, mhb), msum(b1, mlb, mhb)};
    const float dd[2] = {h2f((uint16_t)(ma.x & 0xFFFFu)), h2f((uint16_t)(mb.x & 0xFFFFu))};
    const float dm[2] = {h2f((uint16_t)(ma.x >> 16)), h2f((uint16_t)(mb.x >> 16))};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float dx = (i & 1) ? dx1 : dx0;
      acc[i] = __fadd_rn(acc[i], __fmul_rn(__fmul_rn(dd[i >> 1], dx), (float)is[i]));
      acc[i] = __fsub_rn(acc[i], __fmul_rn(__fmul_rn(dm[i >> 1], dx), (float)ms[i]));
    }
  } else {  // Q6_K: 16 groups of 16 weights, m16n8k16
    const uint8_t* qla = sa + 128 * g;
    const uint8_t* qlb = sb + 128 * g;
    const uint8_t* qha = sa + 1024 + 64 * g;
    const uint8_t* qhb = sb + 1024 + 64 * g;
    const uint4 sca = lds128(sa + 1536 + 16 * g), scb = lds128(sb + 1536 + 16 * g);
    const uint32_t swa[4] = {sca.x, sca.y, sca.z, sca.w}, swb[4] = {scb.x, scb.y, scb.z, scb.w};
    const int16_t* bs0 = bss + ((2 * q) * p.nu + u) * 16;
    const int16_t* bs1 = bss + ((2 * q + 1) * p.nu + u) * 16;
    uint32_t af[16];
    act_frag16(trow, u, g, q, af);
    int is[4] = {0, 0, 0, 0};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        // qh word of l = 16*hf + 4q.. of half hh; ql words of quartiles a = 0/2 (lo/hi nibble of
        // chunk 4hh + hf) and a = 1/3 (chunk 4hh + 2 + hf)
        const uint32_t ha = lds32(qha + 16 * ((2 * hh + hf + g) & 3) + 4 * q);
        const uint32_t hb = lds32(qhb + 16 * ((2 * hh + hf + g) & 3) + 4 * q);
#pragma unroll
        for (int a1 = 0; a1 < 2; ++a1) {
          const uint32_t la = lds32(qla + 16 * ((4 * hh + 2 * a1 + hf + g) & 7) + 4 * q);
          const uint32_t lb = lds32(qlb + 16 * ((4 * hh + 2 * a1 + hf + g) & 7) + 4 * q);
#pragma unroll
          for (int nh = 0; nh < 2; ++nh) {
            const int a = a1 + 2 * nh;          // quartile of the half
            const int i = hh * 8 + a * 2 + hf;  // 16-weight group of the super-block
            const uint32_t va = (nh ? (la >> 4) & kM4 : la & kM4) | (((ha >> (2 * a)) & 0x03030303u) << 4);
            const uint32_t vb = (nh ? (lb >> 4) & kM4 : lb & kM4) | (((hb >> (2 * a)) & 0x03030303u) << 4);
            int c[4];
            mma16_k16_u8s8(c, va, vb, af[i]);
            const int o0 = 32 * (int)bs0[i], o1 = 32 * (int)bs1[i];
            const int s_a = sbyte(swa[i >> 2], i & 3), s_b = sbyte(swb[i >> 2], i & 3);
            is[0] += s_a * (c[0] - o0);
            is[1] += s_a * (c[1] - o1);
            is[2] += s_b * (c[2] - o0);
            is[3] += s_b * (c[3] - o1);
          }
        }
      }
    }
    const float da = h2f(*reinterpret_cast<const uint16_t*>(sa + 1664 + 2 * g));
    const float db = h2f(*reinterpret_cast<const uint16_t*>(sb + 1664 + 2 * g));
    acc[0] = __fadd_rn(acc[0], __fmul_rn(__fmul_rn(da, dx0), (float)is[0]));
    acc[1] = __fadd_rn(acc[1], __fmul_rn(__fmul_rn(da, dx1), (float)is[1]));
    acc[2] = __fadd_rn(acc[2], __fmul_rn(__fmul_rn(db, dx0), (float)is[2]));
    acc[3] = __fadd_rn(acc[3], __fmul_rn(__fmul_rn(db, dx1), (float)is[3]));
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
        int s0 = dp4a_us(lo[0], xa.x, 0), s1 = dp4a_us(hi[0], xb.x, 0);
        s0 = dp4a_us(lo[1], xa.y, s0);
        s1 = dp4a_us(hi[1], xb.y, s1);
        s0 = dp4a_us(lo[2], xa.z, s0);
        s1 = dp4a_us(hi[2], xb.z, s1);
        s0 = dp4a_us(lo[3], xa.w, s0);
        s1 = dp4a_us(hi[3], xb.w, s1);
        s = s0 + s1 - 8 * (int)bss[t * p.nu + u];
      } else {
        int s0 = dp4a_ss(lo[0], xa.x, 0), s1 = dp4a_ss(hi[0], xb.x, 0);
        s0 = dp4a_ss(lo[1], xa.y, s0);
        s1 = dp4a_ss(hi[1], xb.y, s1);
        s0 = dp4a_ss(lo[2], xa.z, s0);
        s1 = dp4a_ss(hi[2], xb.z, s1);
        s0 = dp4a_ss(lo[3], xa.w, s0);
        s1 = dp4a_ss(hi[3], xb.w, s1);
        s = s0 + s1;
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
__device__ __forceinline__ void store_y(const GemvP& p, float* y, int t, int64_t row, float v) {
  const int64_t off = t * p.y_stride + row;
  if (p.peer.n) {
    for (int j = 0; j < p.peer.n; ++j) p.peer.dst[j][off] = v;
    return;
  }
  float* yp = y + off;
  *yp = p.epilogue == EPI_ACCUM ? __fadd_rn(*yp, v) : v;
}

// After every consumer thread of the CTA has stored (a CTA barrier): count
// the CTA; the last CTA of the grid publishes the next epoch to every rank's
// flag.  Stores reach peers before the count (the barrier, then this
// thread's fence.sys), and the count before the flags (fence.sys in the last
// CTA).
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

// Sum of the S range partials of output e, ranges added in order.  red
// holds S blocks of `stride` floats (block r: range r).
__device__ __forceinline__ float range_total(const float* red, int S, int stride, int e) {
  float v = red[e];
  for (int r = 1; r < S; ++r) v = __fadd_rn(v, red[r * stride + e]);
  return v;
}

// Writes the outputs of `nt` consecutive 8-row tiles starting at tile t0 from
// red (S blocks of nt*64 floats, element e = token*(8*nt) + tile_row), one
// warp: store / residual add / peer store, or SwiGLU over (gate, up) row
// pairs of a tile.
// The fused QKV epilogue for one (token, row pair): see RopeKvEpi.
__device__ __forceinline__ void rope_kv_store(const RopeKvEpi& e, int t, int64_t row, float x0, float x1) {
  const int s = e.seq[t], ps = e.pos[t];
  const int h = (int)(row / e.hd), pr = (int)(row - (int64_t)h * e.hd) / 2;
  if (s < 0 || s >= e.n_seq || ps < 0 || ps >= e.cap) {   // outside the cache: zero q, store nothing
    if (h < e.n_head) {
      float* qo = e.q_out + (int64_t)t * e.n_head * e.hd + row;
      qo[0] = 0.0f;
      qo[1] = 0.0f;
    }
    return;
  }
  const int64_t slot = kv_slot(e.st ? e.st[s] : KvSeqState{0, 0}, ps, e.cap);
  if (h < e.n_head + e.n_kv) {
    const float c = e.rope[(int64_t)ps * e.hd + 2 * pr], sn = e.rope[(int64_t)ps * e.hd + 2 * pr + 1];
    const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    if (h < e.n_head) {
      float* qo = e.q_out + (int64_t)t * e.n_head * e.hd + row;
      qo[0] = y0;
      qo[1] = y1;
    } else {
      uint16_t* dst = e.kc + (((int64_t)s * e.n_kv + (h - e.n_head)) * e.cap + slot) * e.hd + 2 * pr;
      dst[0] = f2h_rn(y0);
      dst[1] = f2h_rn(y1);
    }
  } else {
    uint16_t* dst = e.vc + (((int64_t)s * e.n_kv + (h - e.n_head - e.n_kv)) * e.cap + slot) * e.hd + 2 * pr;
    dst[0] = f2h_rn(x0);
    dst[1] = f2h_rn(x1);
  }
}

template <int NT>
__device__ __forceinline__ void finish_tiles(const GemvP& p, const float* red, int64_t t0, int lane, float* y) {
  constexpr int R = 8 * NT;   // rows per item
  if (p.epilogue == EPI_ROPE_KV) {
    // R/2 row pairs x 8 tokens
#pragma unroll
    for (int k = 0; k < (R / 2 * 8 + 31) / 32; ++k) {
      const int e = lane + 32 * k;
      if (e >= R / 2 * 8) break;
      const int t = e / (R / 2), f = e % (R / 2);
      const int64_t row = t0 * 8 + 2 * f;
      if (t < p.n_tok && row < p.n_rows)
        rope_kv_store(p.rope, t, row, range_total(red, p.S, R * 8, t * R + 2 * f),
                      range_total(red, p.S, R * 8, t * R + 2 * f + 1));
    }
    return;
  }
  if (p.epilogue == EPI_SWIGLU) {
    // R/2 features x 8 tokens: feature f = rows (2f, 2f+1)
#pragma unroll
    for (int k = 0; k < (R / 2 * 8 + 31) / 32; ++k) {
      const int e = lane + 32 * k;
      if (e >= R / 2 * 8) break;
      const int t = e / (R / 2), f = e % (R / 2);
      const int64_t row = t0 * 8 + 2 * f;
      if (t < p.n_tok && row < p.n_rows) {
        const float gs = range_total(red, p.S, R * 8, t * R + 2 * f);
        const float us = range_total(red, p.S, R * 8, t * R + 2 * f + 1);
        p.y[t * p.y_stride + row / 2] = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, b2_expf(-gs))), us);
      }
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < R * 8 / 32; ++k) {
    const int e = lane + 32 * k;
    const int t = e / R, rr = e % R;
    const int64_t row = t0 * 8 + rr;
    if (t < p.n_tok && row < p.n_rows) store_y(p, y, t, row, range_total(red, p.S, R * 8, e));
  }
}

// MODE 0 (3..8 tokens, int8 mma.sync, weight rows as the M dimension): items
// are tile pairs (16 rows).  The 16 consumer warps form NSET = 16/S sets of S
// warps; set j works items j, j + NSET, ... of the CTA's run, warp r of a set
// one unit range of the pair for all four residues.  A stage holds one item's
// next U units of all ranges, so the sets consume the ring concurrently.
// MODES 1, 2 (dp4a over 1-2 tokens): items are P = 8/S tiles; all 8 consumer
// warps (tile w/S, range w%S) work every stage.
template <int WT, int MODE>
__global__ void __launch_bounds__((ncw_for(MODE) + 1) * 32, 1) gemv_kernel(const GemvP p) {
  constexpr int NW = ncw_for(MODE);        // consumer warps
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* act_bar = empty + kMaxStages;
  uint8_t* ring = smem + kBarBytes;
  uint8_t* act = ring + (size_t)p.n_stages * p.stage_bytes;
  // mma: [iteration parity][set][range][token*16 + pair row]; dp4a: [group parity][tile slot][range][token*8 + row]
  __shared__ float red[2][kMaxNCW * 128];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = p.n_stages;
  const int S = p.S;
  const int P = MODE == 0 ? 2 : 8 / S;   // tiles per item
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MODE == 0 ? S : NW);
    }
    mbar_init(act_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // Items of this CTA (contiguous, balanced) and the stage sequence.  The
  // consumer sets (MODE 0: NSET sets; dp4a: one) each own a ring of nss =
  // ns/NSET consecutive slots and take their stages in order, so a set never
  // waits on a slot whose previous use (by the same set) is still in flight.
  // Set j works items j, j + NSET, ...; its local stage l is chunk l % n_ch of
  // its item l / n_ch and lives in slot j*nss + l % nss.
  const int64_t n_items = p.ipm * p.n_mat;
  const int64_t g0 = n_items * blockIdx.x / gridDim.x, g1 = n_items * (blockIdx.x + 1) / gridDim.x;
  const int n_ch = (p.L + p.U - 1) / p.U;   // stages per item
  const int nset = MODE == 0 ? min(NW / S, 8) : 1;
  const int nss = ns / nset;
  const uint32_t piece = (uint32_t)p.U * S * p.slot_bytes;   // one tile's part of a stage

  if (warp == NW) {
    // ---------------- producer ----------------
    // Stages go out round-robin over the sets by local stage; the first nss
    // of every set need no free slot.  Once those are out and the previous
    // kernel (the activation quantizer) has finished, the image.
    if (lane == 0) {
      const int64_t items_here = g1 - g0;
      const int64_t max_local = ((items_here + nset - 1) / nset) * n_ch;
      bool act_sent = p.act_img == nullptr;
      // l = blk * n_ch + ch = use * nss + ring_pos, kept as counters: one
      // thread issues every stage, so no division (64-bit ones are long
      // software sequences) sits between a freed slot and its refill.
      int64_t blk = 0, use = 0;
      int ch = 0, ring_pos = 0;
      int64_t mi = p.n_mat > 1 ? g0 / p.ipm : 0;   // matrix cursor (several matrices: one set, items ascend)
      for (int64_t l = 0; l < max_local; ++l) {
        if (l == nss && !act_sent) {
          pdl_wait();
          mbar_arrive_expect_tx(act_bar, p.act_bytes);
          bulk_g2s(act, p.act_img, p.act_bytes, act_bar);
          act_sent = true;
        }
        for (int j = 0; j < nset; ++j) {
          const int64_t i = j + (int64_t)nset * blk;   // item index within the CTA's run
          if (i >= items_here) continue;
          const int sl = j * nss + ring_pos;
          if (use > 0 && !mbar_wait_bounded(&empty[sl], (uint32_t)((use - 1) & 1), p.status, 2)) return;
          const int64_t gitem = g0 + i;
          while (p.n_mat > 1 && (mi + 1) * p.ipm <= gitem) ++mi;
          const int64_t item = gitem - mi * p.ipm;   // item within matrix mi
          const uint8_t* wm = p.wl[mi];
          const int i0 = ch * p.U, ni = min(p.U, p.L - i0);
          const uint32_t bytes = (uint32_t)ni * S * p.slot_bytes;
          uint32_t tx = 0;
          for (int pp = 0; pp < P; ++pp)
            if (item * P + pp < p.n_tiles) tx += bytes;
          mbar_arrive_expect_tx(&full[sl], tx);
          uint8_t* sp = ring + (size_t)sl * p.stage_bytes;
          if (ni == p.L && tx == (uint32_t)P * bytes) {
            // whole tiles, all live: the P tiles are adjacent in memory, one copy
            bulk_g2s(sp, wm + item * P * p.tile_bytes, tx, &full[sl]);
            continue;
          }
          for (int pp = 0; pp < P; ++pp) {
            const int64_t tile = item * P + pp;
            if (tile < p.n_tiles)
              bulk_g2s(sp + pp * piece, wm + tile * p.tile_bytes + (int64_t)i0 * S * p.slot_bytes, bytes, &full[sl]);
          }
        }
        if (++ch == n_ch) {
          ch = 0;
          ++blk;
        }
        if (++ring_pos == nss) {
          ring_pos = 0;
          ++use;
        }
      }
      if (!act_sent) {
        pdl_wait();
        mbar_arrive_expect_tx(act_bar, p.act_bytes);
        bulk_g2s(act, p.act_img, p.act_bytes, act_bar);
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
    ActImage ai;
    ai.img = act;
    ai.kq = p.kq;
    ai.nu = p.nu;
    ai.type = p.type;
    ai.n_act_tok = p.n_act_tok;
    ai.mma = MODE == 0;
    ai.off_dx = p.off_dx;
    ai.off_bs = p.off_bs;
    quantize_image(p.x, p.x_stride, p.n_tok, ai, warp * 32 + lane, NW * 32);
    consumer_sync(NW * 32);
  }
  const size_t us = (size_t)S * p.slot_bytes;   // slot stride between consecutive units of a range

  if constexpr (MODE == 0) {
    const int set = warp / S, r = warp % S;
    const int g = lane >> 2, q = lane & 3;      // D rows g, g+8; tokens 2q, 2q+1
    int it = 0;
    int ring_pos = 0;      // this set's local stage modulo nss, and its ring pass parity
    uint32_t ph = 0;
    // (with S = 1 only the first 8 of the 16 warps form sets; the rest idle)
    for (int64_t i = set; set < nset && g0 + i < g1; i += nset, ++it) {
      const int64_t item = g0 + i;
      float acc[4][4];   // [unit residue][output]
#pragma unroll
      for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.0f;
      for (int ch = 0; ch < n_ch; ++ch) {
        const int s = set * nss + ring_pos;   // local stage it*n_ch + ch of this set
        if (ok) ok = mbar_wait_bounded(&full[s], ph, p.status, 1);
        if (++ring_pos == nss) {
          ring_pos = 0;
          ph ^= 1u;
        }
        const int i0 = ch * p.U, ni = min(p.U, p.L - i0);
        const int ua = r * p.L + i0, ub = min(ua + ni, p.nu);   // units of this stage in range r
        if (ok) {
          const uint8_t* sa = ring + (size_t)s * p.stage_bytes + (size_t)r * p.slot_bytes;
          const uint8_t* sb = sa + piece;
          for (int u4 = ua & ~3; u4 < ub; u4 += 4) {
#pragma unroll
            for (int a = 0; a < 4; ++a) {
              const int u = u4 + a;
              if (u >= ua && u < ub) mma2_unit<WT>(p, sa + (u - ua) * us, sb + (u - ua) * us, act, u, g, q, acc[a]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // range partial (a0 + a1) + (a2 + a3) into red[it&1][set][r][token*16 + row]
      float* rw = red[it & 1] + (set * S + r) * 128;
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        const float v = __fadd_rn(__fadd_rn(acc[0][o], acc[1][o]), __fadd_rn(acc[2][o], acc[3][o]));
        rw[(2 * q + (o & 1)) * 16 + g + 8 * (o >> 1)] = v;
      }
      if (S > 1) tile_sync(set, S * 32);
      else __syncwarp();
      if (r == 0 && ok) finish_tiles<2>(p, red[it & 1] + set * S * 128, item * 2, lane, p.y);
    }
  } else {
    const int slot_p = warp / S, r = warp % S;
    const int dg = lane & 7, dq = lane >> 3;    // tile row dg, unit residue dq
    constexpr int NB = MODE;
    float dacc[NB];    // partial sums [token] of residue dq
    int ring_pos = 0;      // stage counter modulo ns, and the ring pass parity
    uint32_t ph = 0;
    int64_t mi = p.n_mat > 1 ? g0 / p.ipm : 0;   // matrix cursor
    for (int64_t grp = g0; grp < g1; ++grp) {
      while (p.n_mat > 1 && (mi + 1) * p.ipm <= grp) ++mi;
      const int64_t tile = (grp - mi * p.ipm) * P + slot_p;
      const bool live = tile < p.n_tiles;
#pragma unroll
      for (int t = 0; t < NB; ++t) dacc[t] = 0.0f;
      for (int ch = 0; ch < n_ch; ++ch) {
        const int s = ring_pos;
        if (ok) ok = mbar_wait_bounded(&full[s], ph, p.status, 1);
        if (++ring_pos == ns) {
          ring_pos = 0;
          ph ^= 1u;
        }
        const int i0 = ch * p.U, ni = min(p.U, p.L - i0);
        if (ok && live) {
          const uint8_t* rbase = ring + (size_t)s * p.stage_bytes + slot_p * piece + (size_t)r * p.slot_bytes;
          // this stage holds units [ua, ub) of the warp's range; the four lane
          // groups take four consecutive units (residues 0..3) at once
          const int ua = r * p.L + i0, ub = min(ua + ni, p.nu);
#pragma unroll 4
          for (int u4 = ua & ~3; u4 < ub; u4 += 4) {
            const int u = u4 + dq;
            if (u >= ua && u < ub) dp4a_unit<WT, NB>(p, rbase + (size_t)(u - ua) * us, act, u, dg, dacc);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // (a0 + a1) + (a2 + a3): residues dq and dq^1 are 8 lanes apart, dq and dq^2 16
      float* rw = red[grp & 1] + (slot_p * S + r) * 64;
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        float v = __fadd_rn(dacc[t], __shfl_xor_sync(0xffffffffu, dacc[t], 8));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 16));
        if (dq == 0) rw[t * 8 + dg] = v;
      }
      if (S > 1) tile_sync(slot_p, S * 32);
      else __syncwarp();
      if (r == 0 && live && ok) finish_tiles<1>(p, red[grp & 1] + slot_p * S * 64, tile, lane, p.yl[mi]);
    }
  }
  if (p.peer.n) {
    // Every consumer thread's peer stores are ordered before the CTA barrier;
    // the signalling thread's system-scope fence after it makes them all
    // visible before the count (the grid-barrier pattern: barrier, then one
    // thread's fence and atomic).
    consumer_sync(NW * 32);
    if (warp == 0 && lane == 0) signal_peers(p);
  }
}

// 227 KB opt-in per block, less the kernel's static shared memory.
constexpr int kSmemCap = 227 * 1024 - (int)sizeof(float) * 2 * kMaxNCW * 128 - 1024;

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

int launch_quantize_image(const float* x, int64_t x_stride, int n_tok, const ActImage& g, cudaStream_t s) {
  const bool k_quant = g.type == B2_Q4_K || g.type == B2_Q6_K;
  const int64_t work = (int64_t)g.n_act_tok * g.nu * (k_quant ? 32 : 1);   // threads wanted
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
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_image_kernel, x, x_stride, n_tok, g));
  return B2_OK;
}

}  // namespace

// Carve-up of the activation image for w at n_tok tokens.
ActImage gemv_act_image(const QMatrix& w, int n_tok, uint8_t* img) {
  ActImage g;
  g.img = img;
  g.type = w.type;
  g.nu = w.nu;
  g.mma = n_tok > kDp4aMaxTok;
  g.n_act_tok = g.mma ? kMaxTok : n_tok;
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

size_t gemv_act_image_bytes(const QMatrix& w, int n_tok) { return gemv_act_image(w, n_tok, nullptr).bytes; }

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
  B2_CHECK_ARG(a.image_ready || a.x != nullptr, "x");
  B2_CHECK_ARG(a.epilogue == EPI_ROPE_KV ? a.rope != nullptr : a.y != nullptr, "outputs");
  B2_CHECK_ARG(w.data != nullptr && w.nu > 0, "matrix");
  B2_CHECK_ARG(a.epilogue != EPI_SWIGLU || (w.n_rows % 2) == 0, "SwiGLU needs (gate, up) row pairs");
  B2_CHECK_ARG(a.image_ready || ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.x_stride % 4) == 0),
               "x must be 16-byte aligned with a stride of whole float4s");
  B2_CHECK_ARG(!(gemv_needs_image(w, a.n_tok) || a.image_ready) ||
                   (a.act_img != nullptr && (reinterpret_cast<uintptr_t>(a.act_img) & 15) == 0),
               "activation image scratch (16-byte aligned)");
  if (a.epilogue == EPI_ROPE_KV) {
    const RopeKvEpi& r = *a.rope;
    B2_CHECK_ARG(r.pos && r.seq && r.rope && r.q_out && r.kc && r.vc && r.hd > 0 && (r.hd % 8) == 0 &&
                     w.n_rows == (int64_t)(r.n_head + 2 * r.n_kv) * r.hd,
                 "RoPE/KV epilogue arguments");
  }
  GemvP p = {};
  p.w = w.data;
  p.n_mat = a.n_mat;
  if (a.n_mat == 1) {
    p.wl[0] = w.data;
    p.yl[0] = a.y;
  } else {
    B2_CHECK_ARG(a.n_mat >= 1 && a.n_mat <= kMaxMat && a.wlist && a.ylist, "multi-matrix GEMV: 1..64 matrices");
    B2_CHECK_ARG(a.n_tok <= kDp4aMaxTok && a.epilogue == EPI_STORE && !(a.peer && a.peer->n > 0) && !a.image_ready,
                 "multi-matrix GEMV: 1-2 tokens, plain store");
    for (int i = 0; i < a.n_mat; ++i) {
      const QMatrix& wi = *a.wlist[i];
      B2_CHECK_ARG(wi.data && wi.type == w.type && wi.n_rows == w.n_rows && wi.k == w.k && a.ylist[i],
                   "multi-matrix GEMV: matrices of one type and shape, an output each");
      p.wl[i] = wi.data;
      p.yl[i] = a.ylist[i];
    }
  }
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
  const ActImage ag = gemv_act_image(w, a.n_tok, a.act_img);
  p.kq = ag.kq;
  p.off_dx = ag.off_dx;
  p.off_bs = ag.off_bs;
  p.act_bytes = ag.bytes;
  // Small activations are quantized by each CTA itself (no extra kernel and
  // no dependency on a shared image between consecutive launches); large ones
  // once, into the image every CTA copies.
  const bool in_kernel = !a.image_ready && !gemv_needs_image(w, a.n_tok);
  p.act_img = in_kernel ? nullptr : a.act_img;
  if (a.epilogue == EPI_ROPE_KV) p.rope = *a.rope;
  // Stages of P tiles x U unit steps of all S ranges.  mma: one tile pair per
  // stage, U as large as fits (up to whole tiles: then the stage is one bulk
  // copy of up to ~128 KB).  An SM's bulk copies are served at a near-fixed
  // rate of copies, not bytes, so few large copies stream fastest: measured
  // on the 8B shapes, whole-tile stages with one slot per consumer set beat
  // ~18 KB stages with two slots per set (gate/up 26.3 -> 23.1 us, head 161
  // -> 133 us).  Where whole tiles do not fit, the largest U that gives every
  // set a slot.  dp4a: P = 8/S tiles, ~32 KB.  With small activations stay
  // within ~100 KB when that still gives the pipeline it needs, so that two
  // CTAs fit on an SM and the next launch's producer can stream while this
  // one drains.
  const bool mma = a.n_tok > kDp4aMaxTok;
  const int P = mma ? 2 : 8 / w.splits;
  const int nset = mma ? std::min(16 / w.splits, 8) : 1;
  const size_t step_b = (size_t)P * w.splits * w.slot_bytes;
  const size_t fixed = kBarBytes + p.act_bytes;
  int U = 0, ns = 0;
  size_t stage = 0;
  auto fit = [&](size_t cap_, int want_per_set) -> bool {
    for (int u = std::min<int>(w.ulen, (int)std::max<size_t>(1, (mma ? 128 * 1024 : 32 * 1024) / step_b)); u >= 1;
         --u) {
      const size_t st = step_b * u;
      if (fixed + st > cap_) continue;
      int n = (int)std::min<size_t>(kMaxStages, (cap_ - fixed) / st);
      n = n / nset * nset;
      if (n >= want_per_set * nset) {
        U = u;
        ns = n;
        stage = st;
        return true;
      }
    }
    return false;
  };
  // (A multi-matrix launch streams long enough that the deepest ring wins.)
  const bool ok_fit = (in_kernel && a.n_mat == 1 && fit(100 * 1024, mma ? 2 : 3)) ||
                      (mma && fit((size_t)kSmemCap, 1)) || fit((size_t)kSmemCap, 2) || fit((size_t)kSmemCap, 1);
  if (!ok_fit) {
    set_error("gemv: shared memory too small for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  p.U = U;
  p.n_stages = ns;
  p.stage_bytes = (uint32_t)stage;
  const size_t smem = fixed + (size_t)ns * stage;
  p.ipm = (w.n_tiles + P - 1) / P;
  const int64_t items = p.ipm * p.n_mat;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(), items));
  if (!in_kernel && !a.image_ready) {
    const int qrc = launch_quantize_image(a.x, a.x_stride, a.n_tok, ag, s);
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
