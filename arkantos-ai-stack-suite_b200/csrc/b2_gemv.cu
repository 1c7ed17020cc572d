// Decode GEMV / skinny GEMM over tiled GGUF weights (Q4_0, Q8_0, Q4_K, Q6_K)
// for 1..8 token rows — the B200 version of the reference's matmul_quantized
// (Singularity/src/core/cortex_a5_engine.cpp:997-1027), whose per-row dot is
// ref_vec_dot_q4_0_q8_0 / _q8_0_q8_0 (Singularity/tests/test_and_bench_a5.cpp:184-221)
// and, for K-quants, ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K.
//
// Summation order: the reference's.  Every output y[t][r] is the left fold
// over the row's units in order, sumf = ((0 + p_0) + p_1) + ... (Q4_K:
// ((sumf + a_u) − b_u) per unit), where each unit's terms are the exact
// integer block sums scaled exactly as the CPU vec_dot scales them.  So every
// output is bit-identical to the reference's per-row result.
//
// Weights are in the tile layout (8-row tiles, units in order, see QMatrix).
// A CTA takes a contiguous run of items (a tile for 1-2 tokens, a pair of
// tiles for 3-8).  With many items per CTA its warps own items round-robin
// and fold each item's rows through all units themselves; with few (at most
// kKsMaxItems) each item gets a group of S warps that split its units in
// chunks: a warp computes its chunk's unit terms, then takes the running sums
// from the warp of the previous chunk (a shared-memory slot and an mbarrier),
// adds its terms in unit order and passes the sums on, so the fold keeps the
// reference's order while up to 16 warps stream and compute.  Every warp
// streams its own chunks: lane 0 issues 1-D bulk copies (cp.async.bulk, no
// multicast) of U consecutive unit slots into the warp's ring of stages,
// each completing on its own mbarrier, and refills a stage as soon as the
// warp has read it.  The first stages are issued before the grid dependency
// resolves, so with programmatic dependent launch a GEMV's weights stream
// while the previous kernel finishes.
//   * activations are quantized bit-exactly with the reference's quantizers,
//     either by the CTA itself into shared memory (small inputs) or once per
//     launch by a producer kernel into an image that one bulk copy brings in;
//   * 1-2 tokens: dp4a, lane = tile row g (lane & 7) x unit residue j
//     (lane >> 3); the four lanes of a row exchange their unit terms by
//     shuffles and all fold them in unit order;
//   * 3-8 tokens: int8 mma.sync (m16n8k32; m16n8k16 for Q6_K's 16-weight
//     groups) with the 16 rows of a tile pair as M (tile A's row g as row g,
//     tile B's as row g + 8) and the tokens as N; lane 4g+q folds rows g of
//     both tiles for tokens 2q and 2q+1;
//   * epilogue: store, residual add, SwiGLU over interleaved gate/up rows,
//     RoPE + fp16 KV store over the fused QKV rows, or the tensor-parallel
//     exchange into every rank's gather buffer.
// Every mbarrier wait is bounded: a warp whose wait expires records a status
// code, stops computing and issuing, waits (bounded) for the copies it still
// has in flight, and the CTA always exits.
#include <stdlib.h>

#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kMaxWarps = 16;
constexpr int kMaxStages = 8;            // ring stages per warp
// Shared memory header: full[kMaxWarps][kMaxStages] mbarriers (per warp, or per
// group with split items), the activation mbarrier, turn[kMaxWarps], the
// split groups' used[kMaxWarps][kMaxStages] counters and issued[kMaxWarps].
constexpr int kUsedOff = (kMaxWarps * kMaxStages + 1 + kMaxWarps) * 8;
constexpr int kIssuedOff = kUsedOff + kMaxWarps * kMaxStages * 4;
constexpr int kHdrBytes = (kIssuedOff + kMaxWarps * 4 + 127) / 128 * 128;
constexpr int kMaxTok = 8;
constexpr int kDp4aMaxTok = 2;           // dp4a up to this many tokens, mma.sync above
constexpr int kKsMaxItems = 8;           // items per CTA up to which the warps of a group split each item
constexpr int kKsPairUnits = 2;          // units per chunk of a split tile pair
// 4-unit groups per chunk of a split dp4a tile (two for Q4_K at 2 tokens,
// whose unit terms take the most registers)
__host__ __device__ constexpr int ks_dp4a_groups(int type, int n_tok) { return type == B2_Q4_K && n_tok == 2 ? 2 : 4; }
constexpr uint32_t kM4 = 0x0F0F0F0Fu;

constexpr int kMaxMat = 64;          // matrices of one multi-matrix launch
struct GemvP {
  int type, nu, slot_bytes;
  int64_t tile_bytes, n_rows, n_tiles, k;
  int n_tok;
  const float* x;
  int64_t x_stride;
  int64_t y_stride;
  int epilogue;
  int U, n_ch, n_stages;   // units per stage, stages per item, ring stages per warp
  int Ug;                  // units per group stage (split items)
  int ipt;                 // tiles per item: 1, or 2 (the rows-as-M pairs of MODE 3)
  int S;                   // warps per item (split items, KS), else 1
  uint32_t tok_bytes;      // the groups' slots for passing sums (KS)
  uint32_t half_bytes;     // one tile's share of a stage: U (Ug with split items) unit slots
  uint32_t stage_bytes;    // ipt * half_bytes
  int kq;                  // activation row stride in bytes
  uint32_t off_dx, off_bs, act_bytes, act_region;   // activation carve-up and its shared-memory size
  const uint8_t* act_img;  // the quantized activations (global), or null: the CTA quantizes x itself
  int* status;
  PeerOut peer;
  RopeKvEpi rope;
  // The matrices of the launch (same type and shape, one shared x): tiles
  // run over matrix 0's, then matrix 1's, ...
  int n_mat;
  int64_t tpm;             // tiles per matrix
  const uint8_t* wl[kMaxMat];
  float* yl[kMaxMat];
  // Grouped experts (mixture of experts): matrix i of the launch is expert
  // mat_ids[i] (device ids, read after the grid dependency) of a stack whose
  // experts lie mat_stride bytes apart from wl[0]; its output is yl[0] +
  // i·y_mat_stride.  Null: the host lists above.
  const int32_t* mat_ids;
  int n_expert;
  int64_t mat_stride, y_mat_stride;
  // Per-matrix inputs (grouped experts): matrix i reads x + i·x_mat_stride;
  // the CTAs split into n_mat equal sets, set i over matrix i's tiles only,
  // so each CTA quantizes the one input its items need.  0: one shared x.
  int64_t x_mat_stride;
  // Row-fold form (gemv_rows_kernel): rows of the terms table per token
  // (8 x the most tiles a CTA takes), floats per table row, and the bytes of
  // the CTA's weights in shared memory.
  int rf_rows, rf_stride;
  uint32_t rf_w_bytes;
};

// Weights and output of matrix mi of the launch.  Expert ids outside
// [0, n_expert) are clamped (the copies stay inside the stack).
__device__ __forceinline__ const uint8_t* mat_weights(const GemvP& p, int64_t mi) {
  if (!p.mat_ids) return p.wl[mi];
  const int e = min(max(__ldg(p.mat_ids + mi), 0), p.n_expert - 1);
  return p.wl[0] + (int64_t)e * p.mat_stride;
}
__device__ __forceinline__ float* mat_out(const GemvP& p, int64_t mi) {
  return p.mat_ids ? p.yl[0] + mi * p.y_mat_stride : p.yl[mi];
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// Rows-as-M forms: D[16x8] = A[16xK] (weight row g of tile A as row g, of
// tile B as row g + 8) * B[Kx8] (k x tokens).  Lane 4g+q gets d[0] = (row
// gA, token 2q), d[1] = (gA, 2q+1), d[2] = (gB, 2q), d[3] = (gB, 2q+1).
__device__ __forceinline__ void mma_k32_u8s8_rows(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_k32_s8s8_rows(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_k16_u8s8_rows(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
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
// Σ_j m_j · bsum_j over the 8 32-groups (bq: 8 int16 group sums of one token).
__device__ __forceinline__ int q4k_msum(const uint4& bq, uint32_t ml, uint32_t mh) {
  int m = __dp2a_lo((int)bq.x, (int)ml, 0);
  m = __dp2a_hi((int)bq.y, (int)ml, m);
  m = __dp2a_lo((int)bq.z, (int)mh, m);
  return __dp2a_hi((int)bq.w, (int)mh, m);
}

// ---- activation image ------------------------------------------------------------------
// fp32 x [n_tok][k] -> the image (ActImage carve-up, codes in natural order):
// codes, the fp32 scale of every unit, and the block sums the unit terms
// need (Q4_0: per 32; Q4_K: per 32 as pairs of Q8_K sums; Q6_K: Q8_K's per
// 16).  Threads tid of nthreads (a multiple of 32) share the work; img is
// global memory (the quantize kernel) or the GEMV's shared memory.
__device__ void quantize_image(const float* __restrict__ x, int64_t x_stride, int n_tok, const ActImage& img,
                               int64_t tid, int64_t nthreads) {
  const int nu = img.nu;
  if (img.type == B2_Q4_0 || img.type == B2_Q8_0) {
    // One 32-value block per 8 lanes, one float4 per lane; the block's amax
    // and code sum by xor shuffles inside the 8 lanes (max and integer sums
    // are exact in any order, and every code is the reference quantizer's
    // own formula).  Each round loads four float4s per lane before any
    // arithmetic.  Rounds are warp-uniform: tid and nthreads are whole warps
    // and the lane count is a multiple of 8, so a group of 8 lanes is wholly
    // inside or outside the range.
    const int total = n_tok * nu * 8;   // lanes; token t's block b is lane group t·nu + b
    const int lane = (int)(tid & 31);
    float* dxs = reinterpret_cast<float*>(img.img + img.off_dx);
    int16_t* bss = reinterpret_cast<int16_t*>(img.img + img.off_bs);
    for (int64_t base = tid - lane; base < total; base += 4 * nthreads) {
      float4 f[4];
      int tk[4], bk[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t i = base + r * nthreads + lane;
        int b = 0, t = 0;
        f[r] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < total) {
          b = (int)(i >> 3);
          while (b >= nu) {   // at most n_tok - 1 steps
            b -= nu;
            ++t;
          }
          f[r] = __ldg(reinterpret_cast<const float4*>(x + t * x_stride + b * 32) + (i & 7));
        }
        tk[r] = t;
        bk[r] = b;
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (base + r * nthreads >= total) break;   // warp-uniform
        const int part = lane & 7, t = tk[r], b = bk[r];
        const float v[4] = {f[r].x, f[r].y, f[r].z, f[r].w};
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        const float d = __fmul_rn(amax, 1.0f / 127.0f);
        const float id = (amax != 0.0f) ? __fdiv_rn(127.0f, amax) : 0.0f;
        uint32_t wd = 0;
        int sum = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float sc = __fmul_rn(v[j], id);
          const float tt = sc >= 0.0f ? __fadd_rn(sc, 0.5f) : __fsub_rn(sc, 0.5f);
          int q = __float2int_rz(tt);
          q = q < -127 ? -127 : (q > 127 ? 127 : q);
          sum += q;
          wd |= ((uint32_t)(uint8_t)q) << (8 * j);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (base + r * nthreads + lane < total) {
          *reinterpret_cast<uint32_t*>(img.img + t * img.kq + b * 32 + part * 4) = wd;
          if (part == 0) {
            dxs[t * nu + b] = h2f(f2h_rn(d));
            if (img.type == B2_Q4_0) bss[t * nu + b] = (int16_t)sum;
          }
        }
      }
    }
  } else {
    // One 256-value super-block per warp, 8 values per lane.
    const int lane = threadIdx.x & 31;
    for (int64_t i = tid >> 5; i < (int64_t)n_tok * nu; i += nthreads >> 5) {
      const int t = (int)(i / nu), b = (int)(i - (int64_t)t * nu);
      int8_t q[8];
      int bs = 0;
      const float4* src = reinterpret_cast<const float4*>(x + t * x_stride + (int64_t)b * 256 + lane * 8);
      const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
      const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
      const float d = quant_q8_k_lane(v, q, &bs);
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

// ---- dp4a path: the terms of one unit u, tile row g, tokens 0..B-1 ---------------------------
// pa[t] is the unit's product (d_w·d_x)·isum; for Q4_K pb[t] is the min term
// (dmin·d_x)·msum, subtracted after pa is added.
template <int WT, int B>
__device__ __forceinline__ void dp4a_terms(const GemvP& p, const uint8_t* sl, const uint8_t* act, int u, int g,
                                           float (&pa)[B], float (&pb)[B]) {
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
      const uint8_t* xr = act + t * p.kq + u * 32;
      const uint4 xa = lds128(xr), xb = lds128(xr + 16);
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
      pa[t] = __fmul_rn(__fmul_rn(dw, dxs[t * p.nu + u]), (float)s);
      pb[t] = 0.0f;
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
        const uint8_t* xr = act + t * p.kq + u * 256 + 64 * jc;   // the 64 codes of this 32-byte qs pair
        const uint4 x0 = lds128(xr), x1 = lds128(xr + 16), x2 = lds128(xr + 32), x3 = lds128(xr + 48);
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
      const int m = q4k_msum(lds128(reinterpret_cast<const uint8_t*>(bss + (t * p.nu + u) * 8)), ml4, mh4);
      const float dx = dxs[t * p.nu + u];
      pa[t] = __fmul_rn(__fmul_rn(dd, dx), (float)is[t]);
      pb[t] = __fmul_rn(__fmul_rn(dm, dx), (float)m);
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
            const uint8_t* xr = act + t * p.kq + u * 256 + 16 * g0;
            const uint4 xa = lds128(xr), xb = lds128(xr + 16);
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
    for (int t = 0; t < B; ++t) {
      pa[t] = __fmul_rn(__fmul_rn(d6, dxs[t * p.nu + u]), (float)is[t]);
      pb[t] = 0.0f;
    }
  }
}

// Q4_0 / Q8_0 terms of unit u for all 8 rows of a tile from one lane (the
// row-fold form): the unit's activation codes, scale and block sum are read
// once, then each row's block sum and its update term exactly as dp4a_terms
// forms them, (d_r·dx_t)·isum, stored at out[t·tok_stride + r·row_stride].
template <int WT, int NB>
__device__ __forceinline__ void unit_terms8(const GemvP& p, const uint8_t* sl, const uint8_t* act, int u, float* out,
                                            int row_stride, int tok_stride) {
  static_assert(WT == B2_Q4_0 || WT == B2_Q8_0, "Q4_0 / Q8_0 slots");
  const float* dxs = reinterpret_cast<const float*>(act + p.off_dx);
  const int16_t* bss = reinterpret_cast<const int16_t*>(act + p.off_bs);
  uint4 xa[NB], xb[NB];
  float dx[NB];
  int off[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) {
    const uint8_t* xr = act + t * p.kq + u * 32;
    xa[t] = lds128(xr);
    xb[t] = lds128(xr + 16);
    dx[t] = dxs[t * p.nu + u];
    off[t] = WT == B2_Q4_0 ? 8 * (int)bss[t * p.nu + u] : 0;
  }
  const uint4 dq = lds128(sl + (WT == B2_Q4_0 ? 128 : 256));   // the 8 rows' fp16 scales
  const uint32_t dqw[4] = {dq.x, dq.y, dq.z, dq.w};
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const float dw = h2f((uint16_t)(dqw[r >> 1] >> (16 * (r & 1))));
    uint32_t lo[4], hi[4];
    if constexpr (WT == B2_Q4_0) {
      const uint4 w = lds128(sl + 16 * r);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        lo[c] = ww[c] & kM4;
        hi[c] = (ww[c] >> 4) & kM4;
      }
    } else {
      const uint4 a = lds128(sl + 16 * r), b = lds128(sl + 128 + 16 * r);
      lo[0] = a.x; lo[1] = a.y; lo[2] = a.z; lo[3] = a.w;
      hi[0] = b.x; hi[1] = b.y; hi[2] = b.z; hi[3] = b.w;
    }
#pragma unroll
    for (int t = 0; t < NB; ++t) {
      int s0, s1;
      if constexpr (WT == B2_Q4_0) {
        s0 = dp4a_us(lo[0], xa[t].x, 0);
        s1 = dp4a_us(hi[0], xb[t].x, 0);
        s0 = dp4a_us(lo[1], xa[t].y, s0);
        s1 = dp4a_us(hi[1], xb[t].y, s1);
        s0 = dp4a_us(lo[2], xa[t].z, s0);
        s1 = dp4a_us(hi[2], xb[t].z, s1);
        s0 = dp4a_us(lo[3], xa[t].w, s0);
        s1 = dp4a_us(hi[3], xb[t].w, s1);
      } else {
        s0 = dp4a_ss(lo[0], xa[t].x, 0);
        s1 = dp4a_ss(hi[0], xb[t].x, 0);
        s0 = dp4a_ss(lo[1], xa[t].y, s0);
        s1 = dp4a_ss(hi[1], xb[t].y, s1);
        s0 = dp4a_ss(lo[2], xa[t].z, s0);
        s1 = dp4a_ss(hi[2], xb[t].z, s1);
        s0 = dp4a_ss(lo[3], xa[t].w, s0);
        s1 = dp4a_ss(hi[3], xb[t].w, s1);
      }
      out[t * tok_stride + r * row_stride] = __fmul_rn(__fmul_rn(dw, dx[t]), (float)(s0 + s1 - off[t]));
    }
  }
}

// ---- rows-as-M path: the terms of one unit u of two tiles for lane 4g+q ---------------------
// i = 2·(tile B) + (token 2q+1): a[i] / b[i] as in dp4a_terms for row g of
// tile A (i = 0, 1) or of tile B (i = 2, 3) and token 2q (i even) or 2q+1.
// The B fragment is token g's codes.  Tokens at or past n_tok read the last
// token's data instead: a column of the mma only feeds the outputs of its own
// token, and those outputs are never stored.  Everything that depends only
// on the lane is worked out once per warp (PairLane), so a unit costs its
// reads, the integer work and the reference's float updates.
struct PairLane {
  const uint8_t* x;      // token g's codes + 4q (the B fragment's column and k offset)
  const float* dx0;      // unit scales of tokens 2q and 2q+1
  const float* dx1;
  const int16_t* bs0;    // block sums of tokens 2q and 2q+1
  const int16_t* bs1;
  int rot[8];            // 16·((c + g) mod 8) + 4q: the lane's word of 16-byte chunk c of row g (Q4_K qs, Q6_K ql)
  int roth[4];           // 16·((c + g) mod 4) + 4q (Q6_K qh)
  int g, q4;             // row g, 4q
};
__device__ __forceinline__ PairLane pair_lane(const GemvP& p, const uint8_t* act, int g, int q) {
  PairLane L;
  const int last = p.n_tok - 1;
  const int tg = min(g, last), t0 = min(2 * q, last), t1 = min(2 * q + 1, last);
  const int nb = p.type == B2_Q4_0 ? 1 : p.type == B2_Q4_K ? 8 : p.type == B2_Q6_K ? 16 : 0;
  L.x = act + tg * p.kq + 4 * q;
  L.dx0 = reinterpret_cast<const float*>(act + p.off_dx) + t0 * p.nu;
  L.dx1 = reinterpret_cast<const float*>(act + p.off_dx) + t1 * p.nu;
  L.bs0 = reinterpret_cast<const int16_t*>(act + p.off_bs) + t0 * p.nu * nb;
  L.bs1 = reinterpret_cast<const int16_t*>(act + p.off_bs) + t1 * p.nu * nb;
#pragma unroll
  for (int c = 0; c < 8; ++c) L.rot[c] = 16 * ((c + g) & 7) + 4 * q;
#pragma unroll
  for (int c = 0; c < 4; ++c) L.roth[c] = 16 * ((c + g) & 3) + 4 * q;
  L.g = g;
  L.q4 = 4 * q;
  return L;
}

template <int WT>
__device__ __forceinline__ void mma_pair_terms(const PairLane& L, const uint8_t* sa, const uint8_t* sb, int u,
                                               float (&a)[4], float (&b)[4]) {
  const int g = L.g;
  const float dx0 = L.dx0[u], dx1 = L.dx1[u];
  if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
    const uint8_t* xb = L.x + u * 32;
    const uint32_t b0 = lds32(xb), b1 = lds32(xb + 16);
    const int q4 = L.q4;
    int c[4];
    float dA, dB;
    if constexpr (WT == B2_Q4_0) {
      const uint32_t wa = lds32(sa + 16 * g + q4), wb = lds32(sb + 16 * g + q4);
      mma_k32_u8s8_rows(c, wa & kM4, wb & kM4, (wa >> 4) & kM4, (wb >> 4) & kM4, b0, b1);
      const int k0 = 8 * (int)L.bs0[u], k1 = 8 * (int)L.bs1[u];
      c[0] -= k0;
      c[1] -= k1;
      c[2] -= k0;
      c[3] -= k1;
      dA = h2f(*reinterpret_cast<const uint16_t*>(sa + 128 + 2 * g));
      dB = h2f(*reinterpret_cast<const uint16_t*>(sb + 128 + 2 * g));
    } else {
      mma_k32_s8s8_rows(c, lds32(sa + 16 * g + q4), lds32(sb + 16 * g + q4), lds32(sa + 128 + 16 * g + q4),
                        lds32(sb + 128 + 16 * g + q4), b0, b1);
      dA = h2f(*reinterpret_cast<const uint16_t*>(sa + 256 + 2 * g));
      dB = h2f(*reinterpret_cast<const uint16_t*>(sb + 256 + 2 * g));
    }
    a[0] = __fmul_rn(__fmul_rn(dA, dx0), (float)c[0]);
    a[1] = __fmul_rn(__fmul_rn(dA, dx1), (float)c[1]);
    a[2] = __fmul_rn(__fmul_rn(dB, dx0), (float)c[2]);
    a[3] = __fmul_rn(__fmul_rn(dB, dx1), (float)c[3]);
    b[0] = b[1] = b[2] = b[3] = 0.0f;
  } else if constexpr (WT == B2_Q4_K) {
    const uint4 ma = lds128(sa + 1024 + 16 * g), mb = lds128(sb + 1024 + 16 * g);
    uint32_t slA, mlA, shA, mhA, slB, mlB, shB, mhB;
    q4k_scales(ma.y, ma.z, ma.w, slA, mlA, shA, mhA);
    q4k_scales(mb.y, mb.z, mb.w, slB, mlB, shB, mhB);
    const uint8_t* qa = sa + 128 * g;
    const uint8_t* qb = sb + 128 * g;
    const uint8_t* xu = L.x + u * 256;
    int is[4] = {0, 0, 0, 0};
#pragma unroll
    for (int jc = 0; jc < 4; ++jc) {
      const int c0 = L.rot[2 * jc], c1 = L.rot[2 * jc + 1];
      const uint32_t w0a = lds32(qa + c0), w1a = lds32(qa + c1), w0b = lds32(qb + c0), w1b = lds32(qb + c1);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * jc + h;   // 32-weight group
        const uint32_t b0 = lds32(xu + 32 * j), b1 = lds32(xu + 32 * j + 16);
        const int sh = 4 * h;
        int c[4];
        mma_k32_u8s8_rows(c, (w0a >> sh) & kM4, (w0b >> sh) & kM4, (w1a >> sh) & kM4, (w1b >> sh) & kM4, b0, b1);
        const int sA = j < 4 ? ubyte(slA, j) : ubyte(shA, j - 4);
        const int sB = j < 4 ? ubyte(slB, j) : ubyte(shB, j - 4);
        is[0] += sA * c[0];
        is[1] += sA * c[1];
        is[2] += sB * c[2];
        is[3] += sB * c[3];
      }
    }
    const uint4 bq0 = lds128(reinterpret_cast<const uint8_t*>(L.bs0 + u * 8));
    const uint4 bq1 = lds128(reinterpret_cast<const uint8_t*>(L.bs1 + u * 8));
    const int ms[4] = {q4k_msum(bq0, mlA, mhA), q4k_msum(bq1, mlA, mhA), q4k_msum(bq0, mlB, mhB),
                       q4k_msum(bq1, mlB, mhB)};
    const float ddA = h2f((uint16_t)(ma.x & 0xFFFFu)), dmA = h2f((uint16_t)(ma.x >> 16));
    const float ddB = h2f((uint16_t)(mb.x & 0xFFFFu)), dmB = h2f((uint16_t)(mb.x >> 16));
    const float dd[4] = {ddA, ddA, ddB, ddB}, dm[4] = {dmA, dmA, dmB, dmB}, dx[4] = {dx0, dx1, dx0, dx1};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = __fmul_rn(__fmul_rn(dd[i], dx[i]), (float)is[i]);
      b[i] = __fmul_rn(__fmul_rn(dm[i], dx[i]), (float)ms[i]);
    }
  } else {  // Q6_K: 16 groups of 16 weights, m16n8k16
    const uint8_t* qla = sa + 128 * g;
    const uint8_t* qlb = sb + 128 * g;
    const uint8_t* qha = sa + 1024 + 64 * g;
    const uint8_t* qhb = sb + 1024 + 64 * g;
    const uint4 sca = lds128(sa + 1536 + 16 * g), scb = lds128(sb + 1536 + 16 * g);
    const uint32_t swa[4] = {sca.x, sca.y, sca.z, sca.w}, swb[4] = {scb.x, scb.y, scb.z, scb.w};
    const int16_t* bs0 = L.bs0 + u * 16;
    const int16_t* bs1 = L.bs1 + u * 16;
    const uint8_t* xu = L.x + u * 256;
    int is[4] = {0, 0, 0, 0};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int ch = L.roth[2 * hh + hf];
        const uint32_t hwa = lds32(qha + ch), hwb = lds32(qhb + ch);
#pragma unroll
        for (int a1 = 0; a1 < 2; ++a1) {
          const int cl = L.rot[4 * hh + 2 * a1 + hf];
          const uint32_t lwa = lds32(qla + cl), lwb = lds32(qlb + cl);
#pragma unroll
          for (int nh = 0; nh < 2; ++nh) {
            const int aq = a1 + 2 * nh;          // quartile of the half
            const int i = hh * 8 + aq * 2 + hf;  // 16-weight group of the super-block
            const uint32_t va = ((lwa >> (4 * nh)) & kM4) | (((hwa >> (2 * aq)) & 0x03030303u) << 4);
            const uint32_t vb = ((lwb >> (4 * nh)) & kM4) | (((hwb >> (2 * aq)) & 0x03030303u) << 4);
            const uint32_t b0 = lds32(xu + 16 * i);
            int c[4];
            mma_k16_u8s8_rows(c, va, vb, b0);
            const int o0 = 32 * (int)bs0[i], o1 = 32 * (int)bs1[i];
            const int sA = sbyte(swa[i >> 2], i & 3), sB = sbyte(swb[i >> 2], i & 3);
            is[0] += sA * (c[0] - o0);
            is[1] += sA * (c[1] - o1);
            is[2] += sB * (c[2] - o0);
            is[3] += sB * (c[3] - o1);
          }
        }
      }
    }
    const float dA = h2f(*reinterpret_cast<const uint16_t*>(sa + 1664 + 2 * g));
    const float dB = h2f(*reinterpret_cast<const uint16_t*>(sb + 1664 + 2 * g));
    a[0] = __fmul_rn(__fmul_rn(dA, dx0), (float)is[0]);
    a[1] = __fmul_rn(__fmul_rn(dA, dx1), (float)is[1]);
    a[2] = __fmul_rn(__fmul_rn(dB, dx0), (float)is[2]);
    a[3] = __fmul_rn(__fmul_rn(dB, dx1), (float)is[3]);
    b[0] = b[1] = b[2] = b[3] = 0.0f;
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

// After every thread of the CTA has stored (a CTA barrier): count the CTA;
// the last CTA of the grid publishes the next epoch to every rank's flag.
// Stores reach peers before the count (the barrier, then this thread's
// fence.sys), and the count before the flags (fence.sys in the last CTA).
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

// Epilogue of one (token, row pair) (rows r0 = 2f and r0 + 1 of the
// output; for SwiGLU the pair is (gate_f, up_f)).
__device__ __forceinline__ void emit_pair(const GemvP& p, float* y, int t, int64_t r0, float v0, float v1) {
  if (p.epilogue == EPI_ROPE_KV) {
    if (r0 < p.n_rows) rope_kv_store(p.rope, t, r0, v0, v1);
  } else if (p.epilogue == EPI_SWIGLU) {
    if (r0 < p.n_rows) y[t * p.y_stride + r0 / 2] = silu_mul_ref(v0, v1);
  } else {
    if (r0 < p.n_rows) store_y(p, y, t, r0, v0);
    if (r0 + 1 < p.n_rows) store_y(p, y, t, r0 + 1, v1);
  }
}

// Whole items (S = 1): warp w takes items t0 + w, t0 + w + nw, ... of the
// CTA's run [t0, t1), chunk ch of n_ch of each (U units per chunk), through
// its own ring of stages, slot l % n_stages.  An item is a tile, or with
// ipt = 2 the tile pair (2·item, 2·item + 1) whose chunk copies land in the
// two halves of a stage (a missing second tile of an odd count is not
// copied; its rows are never stored).

// A bulk copy costs its issuing thread about 300 cycles whatever its size,
// while copies issued by different lanes overlap, so a stage's copies (and
// the stages of a ring fill) go out from different lanes.  Part `part` of a
// stage: part 0 arms the barrier with the whole stage's bytes and copies
// tile A's units [u0, u0 + n) of item `item`; part 1 copies tile B's (pairs;
// not for a missing second tile of an odd count, whose rows are never
// stored).  The barrier's transaction count may run ahead of the arming; the
// phase cannot complete before the arming arrival.
__device__ __forceinline__ void copy_part(const GemvP& p, int64_t item, int u0, int n, uint32_t half, uint8_t* dst,
                                          uint64_t* bar, int part) {
  const uint32_t bytes = (uint32_t)n * (uint32_t)p.slot_bytes;
  if (p.ipt == 2) {
    const int64_t ta = 2 * item;
    const bool two = ta + 1 < p.tpm;
    const uint8_t* src = p.wl[0] + ta * p.tile_bytes + (int64_t)u0 * p.slot_bytes;
    if (part == 0) {
      mbar_arrive_expect_tx(bar, two ? 2 * bytes : bytes);
      bulk_g2s(dst, src, bytes, bar);
    } else if (two) {
      bulk_g2s(dst + half, src + p.tile_bytes, bytes, bar);
    }
  } else if (part == 0) {
    const int64_t mi = p.n_mat > 1 ? item / p.tpm : 0;
    const int64_t tl = item - mi * p.tpm;
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(dst, mat_weights(p, mi) + tl * p.tile_bytes + (int64_t)u0 * p.slot_bytes, bytes, bar);
  }
}

// Stage l of a whole-items warp: item item0 + (l / n_ch)·nw, chunk l % n_ch,
// slot l % n_stages; lanes [l·ipt, l·ipt + ipt) of `lane0` onwards issue it.
__device__ __forceinline__ void issue_stage(const GemvP& p, int64_t item0, int64_t l, int nw, uint8_t* ring,
                                            uint64_t* full, int part) {
  const int s = (int)(l % p.n_stages);
  const int64_t it = l / p.n_ch;
  const int u0 = (int)(l - it * p.n_ch) * p.U;
  copy_part(p, item0 + it * nw, u0, min(p.U, p.nu - u0), p.half_bytes, ring + (size_t)s * p.stage_bytes, &full[s],
            part);
}

// Split items (KS): the S warps of a group share one item and one ring of
// stages of Ug units (both tiles of a pair: one bulk copy per tile and
// stage, so that few, large copies carry the weights).  Warp s of the group
// takes chunks s, s + S, ... of U units; chunk c lies in stage c / (Ug / U).
// The last warp to finish with a stage refills it (an acq_rel counter per
// stage slot), so no warp waits for another to release a stage.
__device__ __forceinline__ void issue_gstage(const GemvP& p, int64_t item, int k, uint8_t* ring, uint64_t* full,
                                             int* issued, int part) {
  const int slot = k % p.n_stages, u0 = k * p.Ug;
  copy_part(p, item, u0, min(p.Ug, p.nu - u0), p.half_bytes, ring + (size_t)slot * p.stage_bytes, &full[slot], part);
  if (part == 0) atomicAdd(issued, 1);
}
__device__ __forceinline__ unsigned int atom_add_acq_rel(unsigned int* a, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(a)), "r"(v) : "memory");
  return old;
}
// After the warp has read chunk c (stage k): count it, and if it was the
// stage's last chunk, refill the slot with stage k + n_stages (lanes 0 and 1
// for the two tiles of a pair).
__device__ __forceinline__ void release_chunk(const GemvP& p, int64_t item, int k, int cps, int n_gst,
                                              unsigned int* used, uint8_t* ring, uint64_t* full, int* issued,
                                              bool ok, int lane) {
  __syncwarp();
  int refill = 0;
  if (lane == 0) {
    const int slot = k % p.n_stages;
    const unsigned int prev = atom_add_acq_rel(&used[slot], 1u);
    refill = prev == (unsigned int)((k / p.n_stages + 1) * cps - 1) && ok && k + p.n_stages < n_gst;
    if (refill) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  refill = __shfl_sync(0xffffffffu, refill, 0);
  if (refill && lane < p.ipt) issue_gstage(p, item, k + p.n_stages, ring, full, issued, lane);
}

// The running sums of a split item pass from the warp of chunk c to the warp
// of chunk c + 1 through the group's slot of shared memory, so every output
// is still the left fold over its units in order.  A warp computes its
// chunk's unit terms into registers and releases the stage before it waits
// for the incoming sums; then it adds its terms in unit order and passes the
// sums on (or, for the last chunk, runs the epilogue).  A warp whose wait
// expired still passes the sums on, so the rest of the ring ends without
// waiting out its own limits.
__device__ __forceinline__ bool receive_sums(uint64_t* turn, uint32_t& n_rx, const float* slot, int lane, int n,
                                             float* acc, bool ok, int* status) {
  if (ok) ok = mbar_wait_bounded(turn, n_rx & 1, status, 2);
  ok = __all_sync(0xffffffffu, ok);
  ++n_rx;
  if (ok)
    for (int i = 0; i < n; ++i) acc[i] = slot[lane * 4 + i];
  return ok;
}
__device__ __forceinline__ void pass_sums(uint64_t* next_turn, float* slot, int lane, int n, const float* acc) {
  for (int i = 0; i < n; ++i) slot[lane * 4 + i] = acc[i];
  __syncwarp();   // every lane's sums before the arrive (release) of lane 0
  if (lane == 0) mbar_arrive(next_turn);
}

// Epilogue of tile pair `item` for lane 4g+q (MODE 3): rows g of both tiles,
// tokens 2q and 2q+1.
__device__ __forceinline__ void pair_epilogue(const GemvP& p, float* y, int64_t item, int g, int q, const float (&acc)[4],
                                              bool ok) {
  float other[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) other[i] = __shfl_xor_sync(0xffffffffu, acc[i], 4);   // row g ^ 1
  if (!ok) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = 2 * q + (i & 1);
    const int64_t row = (2 * item + (i >> 1)) * 8 + g;
    if (t >= p.n_tok) continue;
    if (p.epilogue == EPI_ROPE_KV || p.epilogue == EPI_SWIGLU) {
      if ((g & 1) == 0) emit_pair(p, y, t, row, acc[i], other[i]);
    } else if (row < p.n_rows) {
      store_y(p, y, t, row, acc[i]);
    }
  }
}

// Epilogue of tile tl for lane (g, j) (dp4a modes): lanes j < NB store token j
// of row g (the token selected without indexing the register arrays).
template <int NB>
__device__ __forceinline__ void tile_epilogue(const GemvP& p, float* y, int64_t tl, int g, int j, const float (&acc)[NB],
                                              bool ok) {
  float other[NB];
#pragma unroll
  for (int t = 0; t < NB; ++t) other[t] = __shfl_xor_sync(0xffffffffu, acc[t], 1);   // row g ^ 1
  float mine = acc[0], theirs = other[0];
#pragma unroll
  for (int t = 1; t < NB; ++t)
    if (j == t) {
      mine = acc[t];
      theirs = other[t];
    }
  if (ok && j < NB) {
    const int64_t row = tl * 8 + g;
    if (p.epilogue == EPI_ROPE_KV || p.epilogue == EPI_SWIGLU) {
      if ((g & 1) == 0) emit_pair(p, y, j, row, mine, theirs);
    } else if (row < p.n_rows) {
      store_y(p, y, j, row, mine);
    }
  }
}

// The row's units u4, u4+1, ... (fewer than 4 at the end) in order, from
// lanes g, g+8, ... (dp4a modes).
template <int WT, int NB>
__device__ __forceinline__ void fold4(float (&acc)[NB], const float (&pa)[NB], const float (&pb)[NB], int n_in, int g) {
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    if (jj < n_in) {
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        acc[t] = __fadd_rn(acc[t], __shfl_sync(0xffffffffu, pa[t], g + 8 * jj));
        if constexpr (WT == B2_Q4_K) acc[t] = __fsub_rn(acc[t], __shfl_sync(0xffffffffu, pb[t], g + 8 * jj));
      }
    }
  }
}

// MODES 1, 2: dp4a over 1 or 2 tokens; MODE 3: 3..8 tokens on int8
// mma.sync with the 16 rows of a tile pair as M.  KS: the S warps of a group
// split one item; otherwise every warp folds whole items.
template <int WT, int MODE, bool KS>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) gemv_kernel(const GemvP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nw = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = KS ? p.S : 1;
  const int R = nw / S, grp = warp / S, split = warp - grp * S;
  const int ring_id = KS ? grp : warp;   // the group's ring (KS) or the warp's own
  uint64_t* full = reinterpret_cast<uint64_t*>(smem) + ring_id * kMaxStages;
  uint64_t* act_bar = reinterpret_cast<uint64_t*>(smem) + kMaxWarps * kMaxStages;
  uint64_t* turn = act_bar + 1;   // [kMaxWarps]: the sums arrived for this warp (KS)
  unsigned int* used = reinterpret_cast<unsigned int*>(smem + kUsedOff) + grp * kMaxStages;   // KS
  int* issued_g = reinterpret_cast<int*>(smem + kIssuedOff) + grp;                            // KS
  float* sums = reinterpret_cast<float*>(smem + kHdrBytes);   // [R][32 lanes][4] (KS)
  uint8_t* act = smem + kHdrBytes + p.tok_bytes;
  uint8_t* ring = act + p.act_region + (size_t)ring_id * p.n_stages * p.stage_bytes;
  float* slot = sums + grp * 128;

  if (lane == 0) {
    if (!KS || split == 0) {
      for (int s = 0; s < p.n_stages; ++s) mbar_init(&full[s], 1);
      if (KS) {
        for (int s = 0; s < p.n_stages; ++s) used[s] = 0u;
        *issued_g = 0;
      }
    }
    if (KS) mbar_init(&turn[warp], 1);
    if (warp == 0) mbar_init(act_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // This CTA's items (contiguous, balanced; with per-matrix inputs, within
  // its matrix).
  const int64_t n_items = MODE == 3 ? (p.tpm + 1) / 2 : p.tpm * p.n_mat;
  int64_t t0 = n_items * blockIdx.x / gridDim.x, t1 = n_items * (blockIdx.x + 1) / gridDim.x;
  const float* xin = p.x;
  if (p.x_mat_stride) {
    const int cpm = gridDim.x / p.n_mat, mi = blockIdx.x / cpm, lc = blockIdx.x - mi * cpm;
    t0 = mi * p.tpm + p.tpm * lc / cpm;
    t1 = mi * p.tpm + p.tpm * (lc + 1) / cpm;
    xin = p.x + mi * p.x_mat_stride;
  }
  // KS: the group's one item; otherwise the warp's items, every nw-th.
  const int64_t item0 = t0 + (KS ? grp : warp);
  const int64_t my_items = KS ? (grp < R && item0 < t1 ? 1 : 0) : (item0 < t1 ? (t1 - item0 + nw - 1) / nw : 0);
  const int my_chunks = KS ? (split < p.n_ch ? (p.n_ch - split + S - 1) / S : 0) : p.n_ch;
  const int cps = KS ? p.Ug / p.U : 1;               // chunks per group stage
  const int n_gst = KS ? (p.nu + p.Ug - 1) / p.Ug : 0;
  const int64_t n_stages_total = KS ? 0 : my_items * p.n_ch;
  // Weights do not depend on the previous kernel (except which experts a
  // grouped launch reads): fill the ring now, one stage per lane (two lanes
  // per stage for pairs).
  if (p.mat_ids) pdl_wait();
  int64_t issued = 0;   // whole items: stages issued so far (every lane keeps the count)
  {
    const int st_lane = lane / p.ipt, part = lane - st_lane * p.ipt;
    if constexpr (KS) {
      if (my_items && split == 0 && st_lane < n_gst && st_lane < p.n_stages)
        issue_gstage(p, item0, st_lane, ring, full, issued_g, part);
    } else {
      issued = min(n_stages_total, (int64_t)p.n_stages);
      if (st_lane < issued) issue_stage(p, item0, st_lane, nw, ring, full, part);
    }
  }
  __syncwarp();

  // Activations: after the grid dependency resolves.
  pdl_wait();
  bool ok = true;
  if (p.act_img) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(act_bar, p.act_bytes);
      bulk_g2s(act, p.act_img, p.act_bytes, act_bar);
    }
    ok = mbar_wait_bounded(act_bar, 0, p.status, 3);
  } else {
    ActImage ai;
    ai.img = act;
    ai.kq = p.kq;
    ai.nu = p.nu;
    ai.type = p.type;
    ai.n_act_tok = p.n_tok;
    ai.off_dx = p.off_dx;
    ai.off_bs = p.off_bs;
    quantize_image(xin, p.x_stride, p.n_tok, ai, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  ok = __all_sync(0xffffffffu, ok);

  int64_t consumed = 0;   // stages consumed (whole items)
  uint32_t n_rx = 0;      // sums received (KS)
  const bool last_split = !KS || ((p.n_ch - 1) % S == split);   // this warp ends the item
  for (int64_t it = 0; it < my_items; ++it) {
    const int64_t item = item0 + it * nw;   // KS: one item
    const int64_t mi = p.n_mat > 1 ? item / p.tpm : 0;
    const int64_t tl = item - mi * p.tpm;
    float* y = mat_out(p, mi);
    if constexpr (MODE == 3) {
      const int g = lane >> 2, q = lane & 3;   // rows g of tiles 2·item and 2·item+1, tokens 2q and 2q+1
      const PairLane PL = pair_lane(p, act, g, q);
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int kc = 0; kc < my_chunks; ++kc) {
        if constexpr (!KS) {
          const int s = (int)(consumed % p.n_stages);
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (uint32_t)((consumed / p.n_stages) & 1), p.status, 1));
          const uint8_t* st = ring + (size_t)s * p.stage_bytes;
          const int u0 = kc * p.U, u1 = min(u0 + p.U, p.nu);
          if (ok) {
            // two units at a time: both units' terms, then the adds in order
            for (int ub = u0; ub < u1; ub += 2) {
              float a[2][4], b[2][4];
#pragma unroll
              for (int k = 0; k < 2; ++k)
                if (ub + k < u1) {
                  const uint8_t* sa = st + (size_t)(ub + k - u0) * p.slot_bytes;
                  mma_pair_terms<WT>(PL, sa, sa + p.half_bytes, ub + k, a[k], b[k]);
                }
#pragma unroll
              for (int k = 0; k < 2; ++k)
                if (ub + k < u1) {
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    acc[i] = __fadd_rn(acc[i], a[k][i]);
                    if constexpr (WT == B2_Q4_K) acc[i] = __fsub_rn(acc[i], b[k][i]);
                  }
                }
            }
          }
          __syncwarp();
          if (ok && issued < n_stages_total) {
            if (lane < p.ipt) {
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              issue_stage(p, item0, issued, nw, ring, full, lane);
            }
            ++issued;
          }
          ++consumed;
        } else {
          constexpr int UM = kKsPairUnits;
          const int ch = split + kc * S, k = ch / cps, sl = k % p.n_stages;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[sl], (uint32_t)((k / p.n_stages) & 1), p.status, 1));
          const uint8_t* st = ring + (size_t)sl * p.stage_bytes + (size_t)(ch - k * cps) * p.U * p.slot_bytes;
          const int u0 = ch * p.U, u1 = min(u0 + p.U, p.nu);
          float ta[UM][4], tb[UM][4];
          if (ok) {
#pragma unroll
            for (int i = 0; i < UM; ++i)
              if (u0 + i < u1) {
                const uint8_t* sa = st + (size_t)i * p.slot_bytes;
                mma_pair_terms<WT>(PL, sa, sa + p.half_bytes, u0 + i, ta[i], tb[i]);
              }
          }
          release_chunk(p, item, k, cps, n_gst, used, ring, full, issued_g, ok, lane);
          if (ch > 0) {
            ok = receive_sums(&turn[warp], n_rx, slot, lane, 4, acc, ok, p.status);
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = 0.0f;
          }
          if (ok) {
#pragma unroll
            for (int kk = 0; kk < UM; ++kk)
              if (u0 + kk < u1) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  acc[i] = __fadd_rn(acc[i], ta[kk][i]);
                  if constexpr (WT == B2_Q4_K) acc[i] = __fsub_rn(acc[i], tb[kk][i]);
                }
              }
          }
          if (ch + 1 < p.n_ch) pass_sums(&turn[grp * S + (ch + 1) % S], slot, lane, 4, acc);
        }
      }
      if (last_split) pair_epilogue(p, y, item, g, q, acc, ok);
    } else {
      constexpr int NB = MODE;
      const int g = lane & 7, j = lane >> 3;   // tile row g, unit residue j
      float acc[NB];
#pragma unroll
      for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
      for (int kc = 0; kc < my_chunks; ++kc) {
        if constexpr (!KS) {
          const int s = (int)(consumed % p.n_stages);
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (uint32_t)((consumed / p.n_stages) & 1), p.status, 1));
          const uint8_t* st = ring + (size_t)s * p.stage_bytes;
          const int u0 = kc * p.U, u1 = min(u0 + p.U, p.nu);
          if (ok) {
            // GM groups of 4 units at a time: all their terms, then all the
            // shuffles, then the adds in unit order (a warp issues in order,
            // so a fold right after its own terms would wait on them)
            constexpr int GM = ks_dp4a_groups(WT, NB);
            for (int ub = u0; ub < u1; ub += 4 * GM) {
              float pa[GM][NB], pb[GM][NB];
#pragma unroll
              for (int kk = 0; kk < GM; ++kk) {
                const int u = ub + 4 * kk + j;
                if (u < u1) {
                  dp4a_terms<WT, NB>(p, st + (size_t)(u - u0) * p.slot_bytes, act, u, g, pa[kk], pb[kk]);
                } else {
#pragma unroll
                  for (int t = 0; t < NB; ++t) pa[kk][t] = pb[kk][t] = 0.0f;
                }
              }
              float sa[GM][4][NB], sb[GM][4][NB];
#pragma unroll
              for (int kk = 0; kk < GM; ++kk)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                  for (int t = 0; t < NB; ++t) {
                    sa[kk][jj][t] = __shfl_sync(0xffffffffu, pa[kk][t], g + 8 * jj);
                    if constexpr (WT == B2_Q4_K) sb[kk][jj][t] = __shfl_sync(0xffffffffu, pb[kk][t], g + 8 * jj);
                  }
#pragma unroll
              for (int kk = 0; kk < GM; ++kk)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
                  if (ub + 4 * kk + jj < u1) {
#pragma unroll
                    for (int t = 0; t < NB; ++t) {
                      acc[t] = __fadd_rn(acc[t], sa[kk][jj][t]);
                      if constexpr (WT == B2_Q4_K) acc[t] = __fsub_rn(acc[t], sb[kk][jj][t]);
                    }
                  }
            }
          }
          __syncwarp();
          if (ok && issued < n_stages_total) {
            if (lane < p.ipt) {
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              issue_stage(p, item0, issued, nw, ring, full, lane);
            }
            ++issued;
          }
          ++consumed;
        } else {
          constexpr int GM = ks_dp4a_groups(WT, NB);
          const int ch = split + kc * S, k = ch / cps, sl = k % p.n_stages;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[sl], (uint32_t)((k / p.n_stages) & 1), p.status, 1));
          const uint8_t* st = ring + (size_t)sl * p.stage_bytes + (size_t)(ch - k * cps) * p.U * p.slot_bytes;
          const int u0 = ch * p.U, u1 = min(u0 + p.U, p.nu);
          float pa[GM][NB], pb[GM][NB];
#pragma unroll
          for (int kk = 0; kk < GM; ++kk) {
            const int u = u0 + 4 * kk + j;
            if (ok && u < u1) {
              dp4a_terms<WT, NB>(p, st + (size_t)(u - u0) * p.slot_bytes, act, u, g, pa[kk], pb[kk]);
            } else {
#pragma unroll
              for (int t = 0; t < NB; ++t) pa[kk][t] = pb[kk][t] = 0.0f;
            }
          }
          release_chunk(p, item, k, cps, n_gst, used, ring, full, issued_g, ok, lane);
          // every lane of row g gathers the row's unit terms before the sums
          // arrive, so only the adds remain on the ring's path
          float sa[GM][4][NB], sb[GM][4][NB];
#pragma unroll
          for (int kk = 0; kk < GM; ++kk)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
              for (int t = 0; t < NB; ++t) {
                sa[kk][jj][t] = __shfl_sync(0xffffffffu, pa[kk][t], g + 8 * jj);
                if constexpr (WT == B2_Q4_K) sb[kk][jj][t] = __shfl_sync(0xffffffffu, pb[kk][t], g + 8 * jj);
              }
          if (ch > 0) {
            ok = receive_sums(&turn[warp], n_rx, slot, lane, NB, acc, ok, p.status);
          } else {
#pragma unroll
            for (int t = 0; t < NB; ++t) acc[t] = 0.0f;
          }
          if (ok) {
#pragma unroll
            for (int kk = 0; kk < GM; ++kk)
#pragma unroll
              for (int jj = 0; jj < 4; ++jj)
                if (u0 + 4 * kk + jj < u1) {
#pragma unroll
                  for (int t = 0; t < NB; ++t) {
                    acc[t] = __fadd_rn(acc[t], sa[kk][jj][t]);
                    if constexpr (WT == B2_Q4_K) acc[t] = __fsub_rn(acc[t], sb[kk][jj][t]);
                  }
                }
          }
          if (ch + 1 < p.n_ch) pass_sums(&turn[grp * S + (ch + 1) % S], slot, lane, NB, acc);
        }
      }
      if (last_split) tile_epilogue<NB>(p, y, tl, g, j, acc, ok);
    }
  }
  // Copies still in flight after a failed wait: wait for them (bounded).
  if constexpr (KS) {
    const bool any_fail = __syncthreads_or(!ok);
    if (any_fail && my_items && split == 0 && lane == 0) {
      const int n_iss = *issued_g;
      for (int k = max(0, n_iss - p.n_stages); k < n_iss; ++k)
        mbar_wait_bounded(&full[k % p.n_stages], (uint32_t)((k / p.n_stages) & 1), nullptr, 0);
    }
  } else {
    if (!ok && lane == 0) {
      for (int64_t l = consumed; l < issued; ++l)
        mbar_wait_bounded(&full[l % p.n_stages], (uint32_t)((l / p.n_stages) & 1), nullptr, 0);
    }
  }
  if (p.peer.n) {
    // Every thread's peer stores are ordered before the CTA barrier; the
    // signalling thread's system-scope fence after it makes them all visible
    // before the count (the grid-barrier pattern).
    __syncthreads();
    if (threadIdx.x == 0) signal_peers(p);
  }
}

// Row-fold form for 1-2 tokens over few tiles per CTA.  The CTA's whole run
// of tiles (a contiguous range of the tiled matrix) is copied into shared
// memory before the grid dependency resolves; a CTA takes at most
// kRowsSmemCap bytes, so two fit on an SM and the next launch's weights
// stream while this launch computes.  After the activations are in place,
// all warps (16 for Q4_0 / Q8_0, 8 for the K-quants) compute unit terms of
// any (tile, unit) — lane (g, j) the
// term of row g and unit 4q + j, exactly as dp4a_terms forms it — into a
// [token][row][unit] table, and then one thread per (token, row) folds its
// row's terms in unit order: the reference's left fold, sumf = ((0 + p_0) +
// p_1) + ... (Q4_K: ((sumf + a_u) − b_u)), so the outputs are the same bits
// as gemv_kernel's.  The fold is one chain of nu adds per row; the terms,
// which are most of the work, are spread over every warp whatever the
// number of tiles.
// 16 warps for Q4_0 / Q8_0 (64 registers a thread, so two CTAs fit), 8 for
// the K-quants, whose unit terms take more registers.
__host__ __device__ constexpr int rows_threads(int type) { return type == B2_Q4_0 || type == B2_Q8_0 ? 512 : 256; }
constexpr int kRowsSmemCap = 112 * 1024;
constexpr int kRowsHdr = 128;   // the weights' and the activations' mbarriers

template <int WT, int NB>
__global__ void __launch_bounds__(rows_threads(WT), 2) gemv_rows_kernel(const GemvP p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NT = WT == B2_Q4_K ? 2 : 1;   // term tables: a (and b for Q4_K)
  uint64_t* wbar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* abar = wbar + 1;
  uint8_t* act = smem + kRowsHdr;
  uint8_t* wsm = act + p.act_region;
  float* terms = reinterpret_cast<float*>(wsm + p.rf_w_bytes);   // [NT][NB][rf_rows][rf_stride]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = p.n_tiles * blockIdx.x / gridDim.x, t1 = p.n_tiles * (blockIdx.x + 1) / gridDim.x;
  const int nt = (int)(t1 - t0);
  if (tid == 0) {
    mbar_init(wbar, 1);
    mbar_init(abar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // The weights do not depend on the previous kernel: one bulk copy per
  // tile, from different lanes so that they overlap.
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(wbar, (uint32_t)nt * (uint32_t)p.tile_bytes);
    __syncwarp();
    if (lane < nt)
      bulk_g2s(wsm + (size_t)lane * p.tile_bytes, p.wl[0] + (t0 + lane) * p.tile_bytes, (uint32_t)p.tile_bytes, wbar);
  }
  pdl_wait();
  bool ok = true;
  if (p.act_img) {
    if (tid == 0) {
      mbar_arrive_expect_tx(abar, p.act_bytes);
      bulk_g2s(act, p.act_img, p.act_bytes, abar);
    }
    ok = mbar_wait_bounded(abar, 0, p.status, 3);
  } else {
    ActImage ai;
    ai.img = act;
    ai.kq = p.kq;
    ai.nu = p.nu;
    ai.type = p.type;
    ai.n_act_tok = p.n_tok;
    ai.off_dx = p.off_dx;
    ai.off_bs = p.off_bs;
    quantize_image(p.x, p.x_stride, p.n_tok, ai, tid, rows_threads(WT));
  }
  if (ok) ok = mbar_wait_bounded(wbar, 0, p.status, 1);
  ok = __syncthreads_and(ok);
  const int stride = p.rf_stride, rows = p.rf_rows;
  if (ok) {
    if constexpr (WT == B2_Q4_0 || WT == B2_Q8_0) {
    // Terms, Q4_0 / Q8_0: item (tile i, unit u) per lane, all 8 rows of the
    // tile (unit_terms8), so a unit's activation codes are read once per
    // tile.  Lanes take consecutive units: slots 144 or 272 bytes apart (4
    // words mod 32) and table rows whose stride is 4 (mod 32) words, so
    // neither the loads nor the stores conflict on banks.
    const int n_items = nt * p.nu;
    for (int it = tid; it < n_items; it += rows_threads(WT)) {
      const int i = it / p.nu, u = it - i * p.nu;
      unit_terms8<WT, NB>(p, wsm + (size_t)i * p.tile_bytes + (size_t)u * p.slot_bytes, act, u,
                          terms + (size_t)i * 8 * stride + u, stride, rows * stride);
    }
    } else {
    // Terms, K-quants: quad q of tile i is (tile i, units 4q..4q+3); a table
    // row's stride is 4 (mod 32) words, so the 32 lanes' stores hit 32
    // banks.  Two quads per round (w and w + 8), whose loads and integer
    // work interleave.
    constexpr int NW = rows_threads(WT) / 32;
    const int nq = (p.nu + 3) >> 2, g = lane & 7, j = lane >> 3, n_w = nt * nq;
    int wi = 0, wq = warp;   // quad w0 = wi·nq + wq, kept without a division
    while (wq >= nq) {
      wq -= nq;
      ++wi;
    }
    for (int w0 = warp; w0 < n_w; w0 += 2 * NW) {
      float pa[2][NB], pb[2][NB];
      int i[2], u[2];
      i[0] = wi;
      u[0] = wq * 4 + j;
      i[1] = wi;
      int q1 = wq + NW;
      while (q1 >= nq) {
        q1 -= nq;
        ++i[1];
      }
      u[1] = q1 * 4 + j;
      wi = i[1];
      wq = q1 + NW;
      while (wq >= nq) {
        wq -= nq;
        ++wi;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int w = w0 + h * NW;
        if (w < n_w && u[h] < p.nu)
          dp4a_terms<WT, NB>(p, wsm + (size_t)i[h] * p.tile_bytes + (size_t)u[h] * p.slot_bytes, act, u[h], g,
                             pa[h], pb[h]);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (w0 + h * NW < n_w && u[h] < p.nu) {
#pragma unroll
          for (int t = 0; t < NB; ++t) {
            terms[((size_t)t * rows + i[h] * 8 + g) * stride + u[h]] = pa[h][t];
            if constexpr (NT == 2) terms[((size_t)(NB + t) * rows + i[h] * 8 + g) * stride + u[h]] = pb[h][t];
          }
        }
      }
    }
    }
  }
  __syncthreads();
  // The fold: thread (t, r) over row r's terms of token t, in unit order.
  const int t = tid / rows, r = tid - t * rows;
  const bool mine = ok && t < NB && r < nt * 8;
  float acc = 0.0f;
  if (mine) {
    const float* ta = terms + ((size_t)t * rows + r) * stride;
    const float* tb = terms + ((size_t)(NB + t) * rows + r) * stride;
    int u = 0;
    for (; u + 4 <= p.nu; u += 4) {
      const float4 a = *reinterpret_cast<const float4*>(ta + u);
      if constexpr (NT == 2) {
        const float4 b = *reinterpret_cast<const float4*>(tb + u);
        acc = __fsub_rn(__fadd_rn(acc, a.x), b.x);
        acc = __fsub_rn(__fadd_rn(acc, a.y), b.y);
        acc = __fsub_rn(__fadd_rn(acc, a.z), b.z);
        acc = __fsub_rn(__fadd_rn(acc, a.w), b.w);
      } else {
        acc = __fadd_rn(acc, a.x);
        acc = __fadd_rn(acc, a.y);
        acc = __fadd_rn(acc, a.z);
        acc = __fadd_rn(acc, a.w);
      }
    }
    for (; u < p.nu; ++u) {
      acc = __fadd_rn(acc, ta[u]);
      if constexpr (NT == 2) acc = __fsub_rn(acc, tb[u]);
    }
  }
  // rows r and r + 1 (r even) are neighbouring lanes of one warp: rows is a
  // multiple of 8
  const float other = __shfl_down_sync(0xffffffffu, acc, 1);
  if (mine) {
    const int64_t row = t0 * 8 + r;
    float* y = p.yl[0];
    if (p.epilogue == EPI_ROPE_KV || p.epilogue == EPI_SWIGLU) {
      if ((r & 1) == 0) emit_pair(p, y, t, row, acc, other);
    } else if (row < p.n_rows) {
      store_y(p, y, t, row, acc);
    }
  }
  if (!ok && tid == 0) {   // copies still in flight after a failed wait (bounded)
    mbar_wait_bounded(wbar, 0, nullptr, 0);
    if (p.act_img) mbar_wait_bounded(abar, 0, nullptr, 0);
  }
  if (p.peer.n) {
    __syncthreads();
    if (tid == 0) signal_peers(p);
  }
}

constexpr int kSmemCap = 227 * 1024;

template <int WT, int MODE, bool KS>
int set_attr() {
  B2_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<WT, MODE, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap));
  return B2_OK;
}

template <int WT>
int set_attr_all() {
  int rc = 0;
  B2_CUDA_TRY(cudaFuncSetAttribute(gemv_rows_kernel<WT, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemCap));
  B2_CUDA_TRY(cudaFuncSetAttribute(gemv_rows_kernel<WT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemCap));
  rc = set_attr<WT, 1, false>();
  if (!rc) rc = set_attr<WT, 2, false>();
  if (!rc) rc = set_attr<WT, 3, false>();
  if (!rc) rc = set_attr<WT, 1, true>();
  if (!rc) rc = set_attr<WT, 2, true>();
  if (!rc) rc = set_attr<WT, 3, true>();
  return rc;
}

template <int WT, int MODE, bool KS>
int launch_t(const GemvP& p, int grid, int nw, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(nw * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_kernel<WT, MODE, KS>, p));
  return B2_OK;
}

template <int WT, bool KS>
int launch_k(const GemvP& p, int grid, int nw, size_t smem, cudaStream_t s) {
  if (p.ipt == 2) return launch_t<WT, 3, KS>(p, grid, nw, smem, s);
  if (p.n_tok == 1) return launch_t<WT, 1, KS>(p, grid, nw, smem, s);
  return launch_t<WT, 2, KS>(p, grid, nw, smem, s);
}

template <int WT>
int launch_rows(const GemvP& p, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(rows_threads(WT));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.n_tok == 1) {
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_rows_kernel<WT, 1>, p));
  } else {
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_rows_kernel<WT, 2>, p));
  }
  return B2_OK;
}

template <int WT>
int launch_w(const GemvP& p, int grid, int nw, size_t smem, cudaStream_t s) {
  return p.S > 1 ? launch_k<WT, true>(p, grid, nw, smem, s) : launch_k<WT, false>(p, grid, nw, smem, s);
}

int launch_quantize_image(const float* x, int64_t x_stride, int n_tok, const ActImage& g, cudaStream_t s) {
  const bool k_quant = g.type == B2_Q4_K || g.type == B2_Q6_K;
  const int64_t work = (int64_t)n_tok * g.nu * (k_quant ? 32 : 2);   // threads wanted (Q8_0: 8 lanes per block, 4 rounds)
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

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

// Carve-up of the activation image for w at n_tok tokens: codes [n_tok][kq]
// in natural order (kq = k rounded up to 128, plus 16 bytes so that the
// token rows of one mma fragment load fall on different banks), fp32 unit
// scales [n_tok][nu], int16 block sums [n_tok][nu][nb].
ActImage gemv_act_image(const QMatrix& w, int n_tok, uint8_t* img) {
  ActImage g;
  g.img = img;
  g.type = w.type;
  g.nu = w.nu;
  g.n_act_tok = n_tok;
  g.kq = (int)((w.k + 127) / 128 * 128 + 16);
  const int bs_per_unit = w.type == B2_Q4_0 ? 1 : w.type == B2_Q4_K ? 8 : w.type == B2_Q6_K ? 16 : 0;
  const size_t qs_b = (size_t)n_tok * g.kq;
  const size_t dx_b = align_up((size_t)n_tok * w.nu * 4, 16);
  const size_t bs_b = align_up((size_t)n_tok * w.nu * bs_per_unit * 2, 16);
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
  B2_CHECK_ARG(w.data != nullptr && w.nu > 0 && w.splits == 1, "matrix");
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
  p.n_mat = a.n_mat;
  if (a.mat_ids) {
    B2_CHECK_ARG(a.n_mat >= 1 && a.n_mat <= kMaxMat && a.n_expert >= 1 && a.mat_stride > 0,
                 "grouped-expert GEMV: 1..64 matrices");
    B2_CHECK_ARG(a.n_tok <= kDp4aMaxTok && a.epilogue == EPI_STORE && !(a.peer && a.peer->n > 0) && !a.image_ready,
                 "grouped-expert GEMV: 1-2 tokens, plain store");
    p.wl[0] = w.data;
    p.yl[0] = a.y;
    p.mat_ids = a.mat_ids;
    p.n_expert = a.n_expert;
    p.mat_stride = a.mat_stride;
    p.y_mat_stride = a.y_mat_stride;
    p.x_mat_stride = a.x_mat_stride;
    B2_CHECK_ARG(a.x_mat_stride == 0 || !gemv_needs_image(w, a.n_tok),
                 "grouped-expert GEMV: per-expert inputs of at most 8192 values");
  } else if (a.n_mat == 1) {
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
  p.slot_bytes = w.slot_bytes;
  p.tile_bytes = w.tile_bytes;
  p.n_rows = w.n_rows;
  p.n_tiles = w.n_tiles;
  p.k = w.k;
  p.n_tok = a.n_tok;
  p.x = a.x;
  p.x_stride = a.x_stride;
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
  p.act_region = (uint32_t)align_up(ag.bytes, 128);
  // Small activations are quantized by each CTA itself (no extra kernel and
  // no dependency on a shared image between consecutive launches); large ones
  // once, into the image every CTA copies.
  const bool in_kernel = !a.image_ready && !gemv_needs_image(w, a.n_tok);
  p.act_img = in_kernel ? nullptr : a.act_img;
  if (a.epilogue == EPI_ROPE_KV) p.rope = *a.rope;
  // Geometry.  One CTA per SM over a contiguous run of items: 8-row tiles
  // for 1-2 tokens, tile pairs for 3..8 (one rows-as-M mma covers 16 rows x
  // 8 tokens).  With more than kKsMaxItems items per CTA every warp folds
  // whole items (up to 8 warps, 16 with pairs); with fewer, the CTA runs one
  // group of S warps per item and the S warps split the item's units in
  // chunks of U (KS), so that up to 16 warps stream and compute even when
  // the CTA has one or two items.  Each warp's ring gets an equal share of
  // the shared memory left after the activations; with small activations
  // and at most 8 warps that is about 110 KB in all, so that two CTAs fit
  // on an SM and the next launch's weights stream while this one finishes.
  p.tpm = w.n_tiles;
  const int sms = sm_count();
  const bool pairs = a.n_tok > kDp4aMaxTok;
  // Row-fold form: 1-2 tokens of one matrix, where a CTA's run of tiles fits
  // in kRowsSmemCap with the activations and the terms table; one CTA per
  // SM, or two where one SM's share does not fit.
  for (int per_sm = 1; per_sm <= 2 && !pairs && a.n_mat == 1 && !a.mat_ids; ++per_sm) {
    const int rgrid = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)per_sm * sms, w.n_tiles));
    const int64_t max_tiles = (w.n_tiles + rgrid - 1) / rgrid;
    const int64_t rows = max_tiles * 8;
    const size_t stride = align_up((size_t)w.nu, 32) + 4;
    const size_t wbytes = align_up((size_t)max_tiles * (size_t)w.tile_bytes, 128);
    const size_t tbytes = (size_t)(w.type == B2_Q4_K ? 2 : 1) * a.n_tok * rows * stride * 4;
    const size_t rsmem = kRowsHdr + p.act_region + wbytes + tbytes;
    if (a.n_tok * rows <= rows_threads(w.type) && rsmem <= kRowsSmemCap) {
      p.rf_rows = (int)rows;
      p.rf_stride = (int)stride;
      p.rf_w_bytes = (uint32_t)wbytes;
      if (!in_kernel && !a.image_ready) {
        const int qrc = launch_quantize_image(a.x, a.x_stride, a.n_tok, ag, s);
        if (qrc) return qrc;
      }
      switch (w.type) {
        case B2_Q4_0: return launch_rows<B2_Q4_0>(p, rgrid, rsmem, s);
        case B2_Q8_0: return launch_rows<B2_Q8_0>(p, rgrid, rsmem, s);
        case B2_Q4_K: return launch_rows<B2_Q4_K>(p, rgrid, rsmem, s);
        case B2_Q6_K: return launch_rows<B2_Q6_K>(p, rgrid, rsmem, s);
      }
    }
  }
  p.ipt = pairs ? 2 : 1;
  const int64_t n_items = pairs ? (w.n_tiles + 1) / 2 : p.tpm * p.n_mat;
  int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, n_items));
  int64_t per_cta = (n_items + grid - 1) / grid;
  if (p.x_mat_stride) {   // n_mat sets of CTAs, each over one matrix's tiles
    const int cpm = (int)std::max<int64_t>(1, std::min<int64_t>(sms / p.n_mat, p.tpm));
    grid = cpm * p.n_mat;
    per_cta = (p.tpm + cpm - 1) / cpm;
  }
  const int gran = pairs ? 1 : 4;   // units that one step of the fold takes
  int S = 1, nw, U = 0;
  if (per_cta <= kKsMaxItems) {
    const int64_t n_gran = (w.nu + gran - 1) / gran;
    S = (int)std::min<int64_t>(kMaxWarps / per_cta, n_gran);
    if (S >= 2) {
      const int64_t per_warp = (n_gran + S - 1) / S;
      U = gran * (int)std::min<int64_t>(pairs ? kKsPairUnits : ks_dp4a_groups(w.type, a.n_tok), per_warp);
      S = (int)std::min<int64_t>(S, (w.nu + U - 1) / U);   // every warp gets a chunk
    }
    if (S < 2) S = 1;
  }
  const size_t item_slot = (size_t)p.ipt * w.slot_bytes, item_bytes = (size_t)p.ipt * w.tile_bytes;
  // Split items: the group's stages hold the whole item where it fits the
  // group's share of shared memory, else as many whole chunk rounds (S
  // chunks of U units) as fit twice; where not even that fits, the chunk and
  // then the number of warps shrink.
  size_t cap = 0, fixed = 0;
  int Ug = 0;
  while (S > 1) {
    nw = (int)per_cta * S;
    p.tok_bytes = (uint32_t)per_cta * 32 * 4 * 4;
    cap = in_kernel && a.n_mat == 1 && nw <= 8 ? (size_t)110 * 1024 : (size_t)kSmemCap;
    fixed = kHdrBytes + p.tok_bytes + p.act_region;
    const size_t share_g = fixed < cap ? (cap - fixed) / per_cta : 0;
    const int n_ch = (w.nu + U - 1) / U;
    if ((size_t)n_ch * U * item_slot <= share_g) {
      Ug = n_ch * U;   // the whole item in one stage
      break;
    }
    const int fit = (int)(share_g / 2 / item_slot);   // units per stage with two stages
    if (fit >= S * U) {
      Ug = fit / (S * U) * (S * U);
      break;
    }
    const int u_fit = fit / S / gran * gran;
    if (u_fit >= gran) {
      U = u_fit;
      Ug = S * U;
      break;
    }
    --S;
  }
  if (S > 1) {
    S = (int)std::min<int64_t>(S, (w.nu + U - 1) / U);   // every warp gets a chunk
    nw = (int)per_cta * S;
  } else {
    S = 1;
    nw = (int)std::max<int64_t>(1, std::min<int64_t>(pairs ? 16 : 8, per_cta));
    p.tok_bytes = 0;
    cap = in_kernel && a.n_mat == 1 && nw <= 8 ? (size_t)110 * 1024 : (size_t)kSmemCap;
    fixed = kHdrBytes + p.act_region;
  }
  p.S = S;
  if (fixed >= cap || (S == 1 && fixed + (size_t)nw * item_slot > cap)) {
    set_error("gemv: shared memory too small for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  const int n_rings = S > 1 ? (int)per_cta : nw;   // rings: one per group (split items) or per warp
  const size_t share = (cap - fixed) / n_rings;
  if (S == 1) {
    const int64_t items_per_warp = (per_cta + nw - 1) / nw;
    if (item_bytes <= share && (items_per_warp <= 1 || item_bytes * 2 <= share)) {
      U = w.nu;   // whole items
    } else {
      U = (int)std::max<size_t>(1, std::min<size_t>(w.nu, share / 2 / item_slot));
      if (!pairs && U < w.nu) U = std::max(4, U / 4 * 4);   // the dp4a fold takes units four at a time
    }
    Ug = U;
  }
  const size_t stage = (size_t)Ug * item_slot;
  if (stage > share) {
    set_error("gemv: no stage of unit slots fits for n_tok=%d k=%lld", a.n_tok, (long long)w.k);
    return B2_ERR_UNSUPPORTED;
  }
  p.U = U;
  p.Ug = Ug;
  p.n_ch = (w.nu + U - 1) / U;
  p.n_stages = (int)std::max<size_t>(1, std::min<size_t>(kMaxStages, share / stage));
  p.half_bytes = (uint32_t)((size_t)Ug * w.slot_bytes);
  p.stage_bytes = (uint32_t)stage;
  const size_t smem = fixed + (size_t)n_rings * p.n_stages * stage;
  if (!in_kernel && !a.image_ready) {
    const int qrc = launch_quantize_image(a.x, a.x_stride, a.n_tok, ag, s);
    if (qrc) return qrc;
  }
  switch (w.type) {
    case B2_Q4_0: return launch_w<B2_Q4_0>(p, grid, nw, smem, s);
    case B2_Q8_0: return launch_w<B2_Q8_0>(p, grid, nw, smem, s);
    case B2_Q4_K: return launch_w<B2_Q4_K>(p, grid, nw, smem, s);
    case B2_Q6_K: return launch_w<B2_Q6_K>(p, grid, nw, smem, s);
  }
  set_error("gemv: unsupported weight type %d", w.type);
  return B2_ERR_UNSUPPORTED;
}

}  // namespace b2
