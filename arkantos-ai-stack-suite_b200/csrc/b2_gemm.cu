// Prefill GEMM for Q4_K weights on the 5th-generation tensor cores:
// Y[t][r] = Σ_super-blocks of W row r · Q8_K(X[t]) — the reference's
// matmul_quantized (Singularity/src/core/cortex_a5_engine.cpp:997-1027) with
// ggml's Q4_K x Q8_K dot, for many tokens at once.
//
// Exactness.  Per 256-weight super-block the reference adds
//   (d·dx)·isum  then subtracts  (dmin·dx)·msum,
// isum = Σ_j sc_j Σ_k q·y and msum = Σ_j m_j·bsum_j exact integers.  Here the
// integer sums come from tcgen05.mma kind::f16 with fp32 accumulation in
// TMEM on operands that are exact small integers in fp16: A = sc_j·q (<= 945)
// and B = the Q8_K codes (|y| <= 127).  Every product and every partial sum
// of a half super-block (<= 15.4e6 < 2^24) is an exact fp32 integer, so the
// tensor core's summation order cannot change it; the halves are added in
// fp32 (the correctly rounded exact isum, i.e. (float)isum).  msum comes from
// one more K=16 MMA: A = (m_0..m_7, m_0..m_7), B = (64·bh_j, bl_j) with
// bsum_j = 64·bh_j + bl_j, all exact.  The epilogue then applies the
// reference's own sequence per super-block with explicitly rounded fp32
// operations, so Y is bit-identical to the reference-order CPU matmul.
//
// Structure (one CTA per 128 weight rows x 64 tokens, 10 warps):
//   warp 0   TMA producer: per super-block the 16 Q4_K row tiles (1-D bulk
//            copies of the tile layout), the four 64-k activation sub-tiles
//            and the msum operand; the tile's activation scales once.
//   warp 1   allocates TMEM (512 columns: two buffers of isum-half-0,
//            isum-half-1, msum x 64 tokens) and issues the MMAs from one
//            thread; tcgen05.commit releases operand stages and hands a
//            finished super-block to the epilogue.
//   warps 2-5  dequantize one row each into canonical K-major fp16 tiles
//            (8x8 core matrices, no swizzle) and publish d, dmin.
//   warps 6-9  epilogue: tcgen05.ld of their 32 TMEM lanes (rows), the
//            per-super-block fp32 update for 64 tokens in registers, then Y.
// Every wait is bounded; an expired wait records a status code and the
// thread proceeds (results are then garbage, the kernel still ends).
#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kMT = 128;            // weight rows per CTA (MMA M)
constexpr int kNT = 64;             // tokens per CTA (MMA N)
constexpr int kSubK = 64;           // k per A/B sub-tile (4 MMAs of K=16)
constexpr int kRaw = 3, kARing = 4, kBRing = 4;
constexpr int kRawStage = 16 * 1152;          // 16 eight-row Q4_K tiles, one super-block
constexpr int kASub = kMT * kSubK * 2;        // 16 KB
constexpr int kBSub = kNT * kSubK * 2;        // 8 KB
constexpr int kAm = kMT * 16 * 2;             // 4 KB
constexpr int kBm = kNT * 16 * 2;             // 2 KB
constexpr int kThreads = 10 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kBufCols = 192;                 // isum0 | isum1 | msum, 64 columns each

struct GemmP {
  const uint8_t* w;          // Q4_K tile layout
  int64_t tile_bytes;
  int nu, S, L, slot_bytes;
  int64_t n_rows;
  int n_tok;
  const uint8_t* bimg;       // activation codes, fp16, [tok tile][k/64][8 KB]
  const uint8_t* bmimg;      // msum operand, fp16, [tok tile][nsb][2 KB]
  const float* dximg;        // activation scales [tok tile][nsb][64]
  float* y;                  // [n_tok][n_rows]
  int* status;
};

// ---- tcgen05 / UMMA helpers ----------------------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored as 128 contiguous bytes; lbo = byte stride between
// core matrices along K, sbo = along M/N.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;   // descriptor version (sm_100)
  return d;                 // base offset 0, lbo mode 0, layout type 0 (no swizzle)
}
// Instruction descriptor: kind::f16, A and B fp16 K-major, D fp32, M=128, N=kNT.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kNT >> 3) << 17) |
                            ((uint32_t)(kMT >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Ring wait helpers: the n-th use (n >= 0) of a slot waits for parity n & 1
// of its full barrier; a producer's n-th refill (n >= 1) waits for parity
// (n - 1) & 1 of the empty barrier.  After one wait in the CTA has expired
// (the shared abort flag), every later wait returns false at once, so a lost
// transfer costs one bounded wait, not one per pipeline stage.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, int* status, int code, int* abort_flag) {
  if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
  if (mbar_wait_bounded(bar, parity, status, code)) return true;
  *reinterpret_cast<volatile int*>(abort_flag) = 1;
  return false;
}
__device__ __forceinline__ bool wait_full(uint64_t* bar, int64_t use, int* status, int code, int* abort_flag) {
  return ring_wait(bar, (uint32_t)(use & 1), status, code, abort_flag);
}
__device__ __forceinline__ bool wait_empty(uint64_t* bar, int64_t use, int* status, int code, int* abort_flag) {
  return use == 0 || ring_wait(bar, (uint32_t)((use - 1) & 1), status, code, abort_flag);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return (uint32_t)f2h_rn(a) | ((uint32_t)f2h_rn(b) << 16);
}

// ---- activation image ---------------------------------------------------------------------
// x fp32 [n_tok][k] -> Q8_K codes as fp16 in the canonical B layout, the msum
// operand and the scales; tokens n_tok..(padded) are zero.  One warp per
// (token, super-block), 8 values per lane.
__global__ void gemm_act_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, int n_tok_pad, int nsb,
                                uint8_t* __restrict__ bimg, uint8_t* __restrict__ bmimg, float* __restrict__ dximg) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)n_tok_pad * nsb;
  const int nss = nsb * 4;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < total;
       i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(i / nsb), sb = (int)(i - (int64_t)t * nsb);
    int8_t q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int bs = 0;
    float d = 0.0f;
    if (t < n_tok) {   // warp-uniform
      const float4* src = reinterpret_cast<const float4*>(x + t * x_stride + (int64_t)sb * 256 + lane * 8);
      const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
      const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
      d = quant_q8_k_lane(v, q, &bs);
    }
    const int tt = t / kNT, tr = t % kNT;
    // codes: k = sb*256 + 8*lane .. +7 -> sub-tile sb*4 + lane/8, k block lane%8
    uint8_t* bsub = bimg + ((int64_t)tt * nss + sb * 4 + lane / 8) * kBSub;
    *reinterpret_cast<uint4*>(bsub + (tr / 8) * 1024 + (lane % 8) * 128 + (tr % 8) * 16) =
        make_uint4(pack_h2(q[0], q[1]), pack_h2(q[2], q[3]), pack_h2(q[4], q[5]), pack_h2(q[6], q[7]));
    // msum operand: bsum_j (32 values) = 64*bh + bl, bl in [0, 64)
    const int b32 = bs + __shfl_xor_sync(0xffffffffu, bs, 2);
    if ((lane & 3) == 0) {
      const int j = lane / 4;
      const int bh = b32 >> 6, bl = b32 - 64 * bh;
      uint8_t* bm = bmimg + ((int64_t)tt * nsb + sb) * kBm + (tr / 8) * 256 + (tr % 8) * 16;
      reinterpret_cast<uint16_t*>(bm)[j] = f2h_rn((float)(64 * bh));
      reinterpret_cast<uint16_t*>(bm + 128)[j] = f2h_rn((float)bl);
    }
    if (lane == 0) dximg[((int64_t)tt * nsb + sb) * kNT + tr] = d;
  }
}

// ---- the GEMM ------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) gemm_q4k_kernel(const GemmP p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nsb = p.nu;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* raw_full = bars;                 // [3]
  uint64_t* raw_empty = raw_full + kRaw;     // [3]
  uint64_t* a_full = raw_empty + kRaw;       // [4]
  uint64_t* a_empty = a_full + kARing;       // [4]
  uint64_t* b_full = a_empty + kARing;       // [4]
  uint64_t* b_empty = b_full + kBRing;       // [4]
  uint64_t* am_full = b_empty + kBRing;      // [2]
  uint64_t* am_empty = am_full + 2;          // [2]
  uint64_t* bm_full = am_empty + 2;          // [2]
  uint64_t* bm_empty = bm_full + 2;          // [2]
  uint64_t* acc_full = bm_empty + 2;         // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* sc_full = acc_empty + 2;         // [2]
  uint64_t* sc_empty = sc_full + 2;          // [2]
  uint64_t* dx_bar = sc_empty + 2;           // [1]
  uint64_t* mma_done = dx_bar + 1;           // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 496);
  int* abort_flag = reinterpret_cast<int*>(smem + 500);
  uint8_t* raw = smem + 512;
  uint8_t* As = raw + kRaw * kRawStage;
  uint8_t* Bs = As + kARing * kASub;
  uint8_t* Ams = Bs + kBRing * kBSub;
  uint8_t* Bms = Ams + 2 * kAm;
  float* scl = reinterpret_cast<float*>(Bms + 2 * kBm);      // [2][128][2] d, dmin
  float* dxs = scl + 2 * kMT * 2;                             // [nsb][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_blk = blockIdx.x, tok_tile = blockIdx.y;
  const int64_t r0 = (int64_t)row_blk * kMT;
  const int tile0 = row_blk * (kMT / 8);
  const int n_tiles_total = (int)((p.n_rows + 7) / 8);
  const int tiles_here = min(kMT / 8, n_tiles_total - tile0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRaw; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 128);
    }
    for (int i = 0; i < kARing; ++i) {
      mbar_init(&a_full[i], 128);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kBRing; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&am_full[i], 128);
      mbar_init(&am_empty[i], 1);
      mbar_init(&bm_full[i], 1);
      mbar_init(&bm_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
      mbar_init(&sc_full[i], 128);
      mbar_init(&sc_empty[i], 128);
    }
    mbar_init(dx_bar, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {   // TMEM: 512 columns, address to shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      pdl_wait();   // the activation image comes from the previous kernel
      mbar_arrive_expect_tx(dx_bar, (uint32_t)(nsb * kNT * 4));
      bulk_g2s(dxs, p.dximg + (int64_t)tok_tile * nsb * kNT, (uint32_t)(nsb * kNT * 4), dx_bar);
      int n_raw = 0, n_b = 0, n_bm = 0;   // copies issued per ring, in order
      for (int s = 0; s < nsb; ++s) {
        const int rs = s % kRaw;
        if (!wait_empty(&raw_empty[rs], s / kRaw, p.status, 20, abort_flag)) break;
        mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(tiles_here * 1152));
        // unit s of tile t: slot (i = s % L) * S + (w = s / L) of the tile layout
        const int wr = s / p.L, ii = s - wr * p.L;
        for (int t = 0; t < tiles_here; ++t)
          bulk_g2s(raw + rs * kRawStage + t * 1152,
                   p.w + (int64_t)(tile0 + t) * p.tile_bytes + (int64_t)(ii * p.S + wr) * p.slot_bytes, 1152,
                   &raw_full[rs]);
        ++n_raw;
        bool ok = true;
        for (int ss = 0; ss < 4 && ok; ++ss) {
          const int idx = s * 4 + ss, bsl = idx % kBRing;
          ok = wait_empty(&b_empty[bsl], idx / kBRing, p.status, 21, abort_flag);
          if (!ok) break;
          mbar_arrive_expect_tx(&b_full[bsl], kBSub);
          bulk_g2s(Bs + bsl * kBSub, p.bimg + ((int64_t)tok_tile * nsb * 4 + idx) * kBSub, kBSub, &b_full[bsl]);
          ++n_b;
        }
        const int ms = s % 2;
        if (!ok || !wait_empty(&bm_empty[ms], s / 2, p.status, 22, abort_flag)) break;
        mbar_arrive_expect_tx(&bm_full[ms], kBm);
        bulk_g2s(Bms + ms * kBm, p.bmimg + ((int64_t)tok_tile * nsb + s) * kBm, kBm, &bm_full[ms]);
        ++n_bm;
      }
      // Before the CTA may exit, every copy it issued has landed: wait for the
      // last phase of each ring slot (immediate when the consumers saw them).
      mbar_wait_bounded(dx_bar, 0, p.status, 23);
      for (int u = max(0, n_raw - kRaw); u < n_raw; ++u) mbar_wait_bounded(&raw_full[u % kRaw], (u / kRaw) & 1, p.status, 23);
      for (int u = max(0, n_b - kBRing); u < n_b; ++u) mbar_wait_bounded(&b_full[u % kBRing], (u / kBRing) & 1, p.status, 23);
      for (int u = max(0, n_bm - 2); u < n_bm; ++u) mbar_wait_bounded(&bm_full[u % 2], (u / 2) & 1, p.status, 23);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int s = 0; s < nsb; ++s) {
        const int b = s & 1;
        if (!wait_empty(&acc_empty[b], s / 2, p.status, 30, abort_flag)) break;
        tc_fence_after();
        bool ok = true;
        for (int ss = 0; ss < 4; ++ss) {
          const int idx = s * 4 + ss, asl = idx % kARing, bsl = idx % kBRing;
          ok = wait_full(&a_full[asl], idx / kARing, p.status, 31, abort_flag) &&
               wait_full(&b_full[bsl], idx / kBRing, p.status, 32, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t acc = tmem + b * kBufCols + (ss / 2) * kNT;
          const uint32_t abase = smem_u32(As + asl * kASub), bbase = smem_u32(Bs + bsl * kBSub);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(acc, smem_desc(abase + kk * 256, 128, 1024), smem_desc(bbase + kk * 256, 128, 1024),
                     ((ss & 1) | kk) != 0);
          umma_commit(&a_empty[asl]);
          umma_commit(&b_empty[bsl]);
        }
        const int ms = s % 2;
        if (!ok || !wait_full(&am_full[ms], s / 2, p.status, 33, abort_flag) ||
            !wait_full(&bm_full[ms], s / 2, p.status, 34, abort_flag))
          break;
        tc_fence_after();
        umma_f16(tmem + b * kBufCols + 2 * kNT, smem_desc(smem_u32(Ams + ms * kAm), 128, 256),
                 smem_desc(smem_u32(Bms + ms * kBm), 128, 256), 0u);
        umma_commit(&am_empty[ms]);
        umma_commit(&bm_empty[ms]);
        umma_commit(&acc_full[b]);
      }
      // every MMA issued has completed before TMEM is released
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status, 35);
    }
  } else if (warp < 6) {
    // ---------------- dequantize: thread = one weight row ----------------
    const int r = (warp - 2) * 32 + lane;
    const int tl = r >> 3, g = r & 7;
    const bool live = r0 + r < p.n_rows;
    for (int s = 0; s < nsb; ++s) {
      const int rs = s % kRaw;
      wait_full(&raw_full[rs], s / kRaw, p.status, 40, abort_flag);
      uint32_t qw[32];
      uint32_t s0 = 0, s1 = 0, s2 = 0, dd = 0;
      if (live) {
        const uint8_t* unit = raw + rs * kRawStage + tl * 1152;
        const uint4 meta = *reinterpret_cast<const uint4*>(unit + 1024 + 16 * g);
        dd = meta.x;
        s0 = meta.y;
        s1 = meta.z;
        s2 = meta.w;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(unit + 128 * g + 16 * ((c + g) & 7));
          qw[4 * c] = v.x;
          qw[4 * c + 1] = v.y;
          qw[4 * c + 2] = v.z;
          qw[4 * c + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) qw[c] = 0;
      }
      mbar_arrive(&raw_empty[rs]);
      // 6-bit scales and mins
      int sc[8], mn[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[j] = (int)((s0 >> (8 * j)) & 63);
        mn[j] = (int)((s1 >> (8 * j)) & 63);
        sc[j + 4] = (int)(((s2 >> (8 * j)) & 0x0F) | (((s0 >> (8 * j + 6)) & 3) << 4));
        mn[j + 4] = (int)(((s2 >> (8 * j + 4)) & 0x0F) | (((s1 >> (8 * j + 6)) & 3) << 4));
      }
      // d, dmin for the epilogue
      const int sl2 = s % 2;
      wait_empty(&sc_empty[sl2], s / 2, p.status, 41, abort_flag);
      scl[(sl2 * kMT + r) * 2] = h2f((uint16_t)(dd & 0xFFFFu));
      scl[(sl2 * kMT + r) * 2 + 1] = h2f((uint16_t)(dd >> 16));
      mbar_arrive(&sc_full[sl2]);
      // A sub-tiles: sub-step ss = qs chunk pair ss: k 0..31 low nibbles (scale
      // sc[2ss]), k 32..63 high nibbles (scale sc[2ss+1]) of its 32 bytes
#pragma unroll
      for (int ss = 0; ss < 4; ++ss) {
        const int idx = s * 4 + ss, asl = idx % kARing;
        wait_empty(&a_empty[asl], idx / kARing, p.status, 42, abort_flag);
        uint8_t* arow = As + asl * kASub + (r >> 3) * 1024 + (r & 7) * 16;
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) {
          const int hi = kb >> 2, scv = sc[2 * ss + hi];
          const uint32_t w0 = qw[8 * ss + 2 * (kb & 3)], w1 = qw[8 * ss + 2 * (kb & 3) + 1];
          const uint32_t n0 = hi ? (w0 >> 4) & 0x0F0F0F0Fu : w0 & 0x0F0F0F0Fu;
          const uint32_t n1 = hi ? (w1 >> 4) & 0x0F0F0F0Fu : w1 & 0x0F0F0F0Fu;
          uint4 o;
          o.x = pack_h2((float)(((n0 >> 0) & 0xFF) * scv), (float)(((n0 >> 8) & 0xFF) * scv));
          o.y = pack_h2((float)(((n0 >> 16) & 0xFF) * scv), (float)(((n0 >> 24) & 0xFF) * scv));
          o.z = pack_h2((float)(((n1 >> 0) & 0xFF) * scv), (float)(((n1 >> 8) & 0xFF) * scv));
          o.w = pack_h2((float)(((n1 >> 16) & 0xFF) * scv), (float)(((n1 >> 24) & 0xFF) * scv));
          *reinterpret_cast<uint4*>(arow + kb * 128) = o;
        }
        fence_async_smem();
        mbar_arrive(&a_full[asl]);
      }
      // msum operand: (m_0..m_7 | m_0..m_7)
      const int ms = s % 2;
      wait_empty(&am_empty[ms], s / 2, p.status, 43, abort_flag);
      uint8_t* am = Ams + ms * kAm + (r >> 3) * 256 + (r & 7) * 16;
      const uint4 mv = make_uint4(pack_h2((float)mn[0], (float)mn[1]), pack_h2((float)mn[2], (float)mn[3]),
                                  pack_h2((float)mn[4], (float)mn[5]), pack_h2((float)mn[6], (float)mn[7]));
      *reinterpret_cast<uint4*>(am) = mv;
      *reinterpret_cast<uint4*>(am + 128) = mv;
      fence_async_smem();
      mbar_arrive(&am_full[ms]);
    }
  } else {
    // ---------------- epilogue: thread = one weight row (TMEM lane) ----------------
    const int qt = warp & 3;                   // TMEM lane quarter of this warp
    const int r = qt * 32 + lane;
    float out[kNT];
#pragma unroll
    for (int t = 0; t < kNT; ++t) out[t] = 0.0f;
    ring_wait(dx_bar, 0, p.status, 50, abort_flag);
    for (int s = 0; s < nsb; ++s) {
      const int b = s & 1, sl2 = s % 2;
      wait_full(&acc_full[b], s / 2, p.status, 51, abort_flag);
      tc_fence_after();
      wait_full(&sc_full[sl2], s / 2, p.status, 52, abort_flag);
      const float d = scl[(sl2 * kMT + r) * 2], dmin = scl[(sl2 * kMT + r) * 2 + 1];
      mbar_arrive(&sc_empty[sl2]);
      const uint32_t tbase = tmem + ((uint32_t)(qt * 32) << 16) + b * kBufCols;
#pragma unroll
      for (int c = 0; c < kNT / 16; ++c) {
        uint32_t a0[16], a1[16], am[16];
        tmem_ld16(tbase + c * 16, a0);
        tmem_ld16(tbase + kNT + c * 16, a1);
        tmem_ld16(tbase + 2 * kNT + c * 16, am);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float dx = dxs[s * kNT + c * 16 + t];
          const float isum = __fadd_rn(__uint_as_float(a0[t]), __uint_as_float(a1[t]));
          const float msum = __uint_as_float(am[t]);
          float o = out[c * 16 + t];
          o = __fadd_rn(o, __fmul_rn(__fmul_rn(d, dx), isum));
          o = __fsub_rn(o, __fmul_rn(__fmul_rn(dmin, dx), msum));
          out[c * 16 + t] = o;
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    const int64_t row = r0 + r;
    if (row < p.n_rows) {
#pragma unroll
      for (int t = 0; t < kNT; ++t) {
        const int tok = tok_tile * kNT + t;
        if (tok < p.n_tok) p.y[(int64_t)tok * p.n_rows + row] = out[t];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

size_t gemm_smem_bytes(int nsb) {
  return 512 + (size_t)kRaw * kRawStage + (size_t)kARing * kASub + (size_t)kBRing * kBSub + 2 * kAm + 2 * kBm +
         (size_t)2 * kMT * 2 * 4 + (size_t)nsb * kNT * 4;
}

}  // namespace

size_t gemm_act_image_bytes(const QMatrix& w, int n_tok) {
  const int nsb = w.nu;
  const int tiles = (n_tok + kNT - 1) / kNT;
  return (size_t)tiles * nsb * (4 * kBSub + kBm + kNT * 4);
}

int launch_gemm(const QMatrix& w, const float* x, int64_t x_stride, int n_tok, float* y, uint8_t* img, int* status,
                cudaStream_t s) {
  B2_CHECK_ARG(w.type == B2_Q4_K, "the tensor-core GEMM takes Q4_K weights");
  B2_CHECK_ARG(n_tok >= 1 && x && y && img, "gemm arguments");
  B2_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && x_stride % 4 == 0, "x alignment");
  const int nsb = w.nu;
  const size_t smem = gemm_smem_bytes(nsb);
  B2_CHECK_ARG(smem <= 227 * 1024, "k too large for the GEMM's shared memory");
  const int tiles = (n_tok + kNT - 1) / kNT;
  uint8_t* bimg = img;
  uint8_t* bmimg = bimg + (size_t)tiles * nsb * 4 * kBSub;
  float* dximg = reinterpret_cast<float*>(bmimg + (size_t)tiles * nsb * kBm);
  {
    cudaLaunchConfig_t cfg = {};
    const int64_t warps = (int64_t)tiles * kNT * nsb;
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((warps * 32 + 255) / 256, 8 * sm_count())));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_act_kernel, x, x_stride, n_tok, tiles * kNT, nsb, bimg, bmimg, dximg));
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    B2_CUDA_TRY(cudaFuncSetAttribute(gemm_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_set[dev] = true;
  }
  GemmP p = {};
  p.w = w.data;
  p.tile_bytes = w.tile_bytes;
  p.nu = w.nu;
  p.S = w.splits;
  p.L = w.ulen;
  p.slot_bytes = w.slot_bytes;
  p.n_rows = w.n_rows;
  p.n_tok = n_tok;
  p.bimg = bimg;
  p.bmimg = bmimg;
  p.dximg = dximg;
  p.y = y;
  p.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((w.n_rows + kMT - 1) / kMT), (unsigned)tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_q4k_kernel, p));
  return B2_OK;
}

}  // namespace b2
