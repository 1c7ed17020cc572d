// Prefill GEMMs for Q4_K and Q8_0 weights on the 5th-generation tensor cores:
// Y[t][r] = Σ_(super-)blocks of W row r · Q8(X[t]) — the reference's
// matmul_quantized (Singularity/src/core/cortex_a5_engine.cpp:997-1027) with
// ggml's Q4_K x Q8_K dot, or the Q8_0 x Q8_0 dot, for many tokens at once.
// The Q4_K kernel comes first; the Q8_0 kernel (integer MMAs) follows it.
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
// Structure (one CTA per 128 weight rows x 64 tokens, 18 warps):
//   warp 0   TMA producer: per super-block the 16 Q4_K row tiles (1-D bulk
//            copies of the tile layout), the four 64-k activation sub-tiles
//            and the msum operand; the tile's activation scales once.
//   warp 1   allocates TMEM (512 columns: two accumulator buffers of
//            isum-half-0 | isum-half-1 | msum x 64 tokens, a ring of three A
//            sub-tiles and two msum A operands) and issues the MMAs from one
//            thread, A from TMEM and B from shared memory (128-byte swizzled);
//            tcgen05.commit releases stages and hands a finished super-block
//            to the epilogue.
//   warps 2-9  dequantize: warp w serves TMEM lanes 32*(w%4).. (one weight
//            row per lane) and k-half (w-2)/4 of every 64-k sub-step; the
//            values sc*q are formed with integer ops and one packed fp16
//            subtract (1024 + v, exact below 1024) and stored into the A ring
//            with tcgen05.st; they also publish d, dmin and the msum operand.
//   warps 10-17  epilogue: warp w reads TMEM lanes 32*(w%4).. (rows) for
//            token half (w-10)/4 and keeps the per-super-block fp32 update
//            for its 32 tokens in registers (scalar, explicitly rounded
//            operations), then Y.
// Every wait is bounded; an expired wait records a status code and the
// thread proceeds (results are then garbage, the kernel still ends).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "b2_common.cuh"
#include "b2_quant.cuh"

namespace b2 {
namespace {

constexpr int kMT = 128;            // weight rows per CTA (MMA M)
constexpr int kNT = 64;             // tokens per CTA (MMA N)
constexpr int kSubK = 64;           // k per A/B sub-tile (4 MMAs of K=16)
constexpr int kRaw = 4, kARing = 3, kBGroups = 3;   // B ring: groups of the 4 sub-tiles of a super-block
constexpr int kRawStage = 16 * 1152;          // 16 eight-row Q4_K tiles, one super-block
constexpr int kBSub = kNT * kSubK * 2;        // 8 KB: 64 token rows x 128 B, 128-byte swizzled
constexpr int kBGroup = 4 * kBSub;            // one super-block of B sub-tiles, one copy

constexpr int kBm = kNT * 16 * 2;             // 2 KB
constexpr int kDqWarps = 8, kEpWarps = 8;
constexpr int kThreads = (2 + kDqWarps + kEpWarps) * 32;
constexpr int kDqThreads = kDqWarps * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kBufCols = 192;                 // isum0 | isum1 | msum, 64 columns each
constexpr int kAcols = 32;                    // one A sub-tile in TMEM: 128 lanes x 64 fp16
constexpr int kAcol0 = 2 * kBufCols;          // the A ring after the two accumulator buffers
constexpr int kAmCol0 = kAcol0 + kARing * kAcols;   // two msum A operands (8 columns each)

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
// K-major, 128-byte swizzle: rows of 128 bytes (64 fp16 of k), 16-byte chunk
// c of row n stored at chunk c ^ (n % 8); 8-row groups 1024 bytes apart
// (SBO); the atom starts 1024-byte aligned.  A K=16 step advances the start
// address by 32 bytes (the hardware applies the swizzle to the address).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                    // LBO (unused for swizzled K-major): 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;          // SBO: 8 rows x 128 bytes
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // layout type: 128-byte swizzle
  return d;
}
// Byte offset of (row n, k) in a 128-byte-swizzled K-major tile of 64-wide k.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int n, int k) {
  return (uint32_t)n * 128u + ((uint32_t)((k >> 3) ^ (n & 7)) << 4) + (uint32_t)(k & 7) * 2u;
}

// Instruction descriptor: kind::f16, A and B fp16 K-major, D fp32, M=128, N=kNT.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kNT >> 3) << 17) |
                            ((uint32_t)(kMT >> 4) << 24);

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM loads and stores are asynchronous on their registers until the
// matching wait: each helper issues the access and its wait in one asm block,
// so no register can be read or reused in between.
// Three 8-column loads (isum0, isum1, msum of 8 tokens) of this warp's lanes.
__device__ __forceinline__ void tmem_ld8x3(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t (&a)[8], uint32_t (&b)[8],
                                           uint32_t (&c)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%24];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%25];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%26];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
        "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]),
        "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]), "=r"(c[7])
      : "r"(t0), "r"(t1), "r"(t2)
      : "memory");
}
// 8 columns of this warp's lanes, completed before return.
__device__ __forceinline__ void tmem_st8_sync(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
// 16 columns of this warp's lanes, completed before return.
__device__ __forceinline__ void tmem_st16_sync(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// D = A x B with A from TMEM (128 lanes = rows, K=16 fp16 in 8 columns), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, p;\n\t}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(accumulate), "r"(kIdesc));
}

// Four 4-bit values (the low nibbles of the bytes of w) times sc as two
// fp16x2 words: each 16-bit lane gets 0x6400 + n*sc = fp16(1024 + n*sc)
// (exact, n*sc <= 945 < 1024), minus 1024 in fp16 = fp16(n*sc) exactly.
__device__ __forceinline__ void nib4_to_h2(uint32_t w, uint32_t sc, uint32_t& h01, uint32_t& h23) {
  const uint32_t m = w & 0x0F0F0F0Fu;
  const uint32_t x0 = __byte_perm(m, 0u, 0x4140) * sc + 0x64006400u;   // bytes 0, 1 -> 16-bit lanes
  const uint32_t x1 = __byte_perm(m, 0u, 0x4342) * sc + 0x64006400u;   // bytes 2, 3
  const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  const __half2 r0 = __hsub2(*reinterpret_cast<const __half2*>(&x0), k1024);
  const __half2 r1 = __hsub2(*reinterpret_cast<const __half2*>(&x1), k1024);
  h01 = *reinterpret_cast<const uint32_t*>(&r0);
  h23 = *reinterpret_cast<const uint32_t*>(&r1);
}

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

// 3-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
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
    *reinterpret_cast<uint4*>(bsub + sw128_offset(tr, (lane % 8) * 8)) =
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
__global__ void __launch_bounds__(kThreads, 1) gemm_q4k_kernel(const GemmP p, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the B ring needs 1024-byte alignment (128-byte swizzle atoms)
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int nsb = p.nu;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* raw_full = bars;                 // [kRaw]
  uint64_t* raw_empty = raw_full + kRaw;     // [kRaw]
  uint64_t* a_full = raw_empty + kRaw;       // [kARing]  A sub-tile written into TMEM
  uint64_t* a_empty = a_full + kARing;       // [kARing]  ... and read by its MMAs
  uint64_t* b_full = a_empty + kARing;       // [kBGroups]
  uint64_t* b_empty = b_full + kBGroups;     // [kBGroups]
  uint64_t* am_full = b_empty + kBGroups;    // [2]
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
  uint8_t* Bs = smem + 1024;
  uint8_t* raw = Bs + kBGroups * kBGroup;
  uint8_t* Bms = raw + kRaw * kRawStage;
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
      mbar_init(&raw_empty[i], kDqThreads);
    }
    for (int i = 0; i < kARing; ++i) {
      mbar_init(&a_full[i], kDqThreads);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kBGroups; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&am_full[i], kDqThreads);
      mbar_init(&am_empty[i], 1);
      mbar_init(&bm_full[i], 1);
      mbar_init(&bm_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpWarps * 32);
      mbar_init(&sc_full[i], kDqThreads);
      mbar_init(&sc_empty[i], kEpWarps * 32);
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
        // unit s of the CTA's 16 tiles: slot (i = s % L) * S + (w = s / L), one 3-D copy
        // (tiles past the matrix are zero-filled and still counted)
        mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)kRawStage);
        const int wr = s / p.L, ii = s - wr * p.L;
        tma_load_3d(raw + rs * kRawStage, &wmap, 0, ii * p.S + wr, tile0, &raw_full[rs]);
        ++n_raw;
        const int bg = s % kBGroups;
        if (!wait_empty(&b_empty[bg], s / kBGroups, p.status, 21, abort_flag)) break;
        mbar_arrive_expect_tx(&b_full[bg], kBGroup);
        bulk_g2s(Bs + bg * kBGroup, p.bimg + ((int64_t)tok_tile * nsb * 4 + s * 4) * kBSub, kBGroup, &b_full[bg]);
        ++n_b;
        const int ms = s % 2;
        if (!wait_empty(&bm_empty[ms], s / 2, p.status, 22, abort_flag)) break;
        mbar_arrive_expect_tx(&bm_full[ms], kBm);
        bulk_g2s(Bms + ms * kBm, p.bmimg + ((int64_t)tok_tile * nsb + s) * kBm, kBm, &bm_full[ms]);
        ++n_bm;
      }
      // Before the CTA may exit, every copy it issued has landed: wait for the
      // last phase of each ring slot (immediate when the consumers saw them).
      mbar_wait_bounded(dx_bar, 0, p.status, 23);
      for (int u = max(0, n_raw - kRaw); u < n_raw; ++u) mbar_wait_bounded(&raw_full[u % kRaw], (u / kRaw) & 1, p.status, 23);
      for (int u = max(0, n_b - kBGroups); u < n_b; ++u)
        mbar_wait_bounded(&b_full[u % kBGroups], (u / kBGroups) & 1, p.status, 23);
      for (int u = max(0, n_bm - 2); u < n_bm; ++u) mbar_wait_bounded(&bm_full[u % 2], (u / 2) & 1, p.status, 23);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int s = 0; s < nsb; ++s) {
        const int b = s & 1;
        if (!wait_empty(&acc_empty[b], s / 2, p.status, 30, abort_flag)) break;
        tc_fence_after();
        const int bg = s % kBGroups;
        bool ok = wait_full(&b_full[bg], s / kBGroups, p.status, 32, abort_flag);
        for (int ss = 0; ss < 4 && ok; ++ss) {
          const int idx = s * 4 + ss, asl = idx % kARing;
          ok = wait_full(&a_full[asl], idx / kARing, p.status, 31, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t acc = tmem + b * kBufCols + (ss / 2) * kNT;
          const uint32_t abase = tmem + kAcol0 + asl * kAcols, bbase = smem_u32(Bs + bg * kBGroup + ss * kBSub);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ts(acc, abase + kk * 8, smem_desc_sw128(bbase + kk * 32), ((ss & 1) | kk) != 0);
          umma_commit(&a_empty[asl]);
        }
        if (ok) umma_commit(&b_empty[bg]);
        const int ms = s % 2;
        if (!ok || !wait_full(&am_full[ms], s / 2, p.status, 33, abort_flag) ||
            !wait_full(&bm_full[ms], s / 2, p.status, 34, abort_flag))
          break;
        tc_fence_after();
        umma_f16_ts(tmem + b * kBufCols + 2 * kNT, tmem + kAmCol0 + ms * 8, smem_desc(smem_u32(Bms + ms * kBm), 128, 256),
                    0u);
        umma_commit(&am_empty[ms]);
        umma_commit(&bm_empty[ms]);
        umma_commit(&acc_full[b]);
      }
      // every MMA issued has completed before TMEM is released
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status, 35);
    }
  } else if (warp < 2 + kDqWarps) {
    // ---------------- dequantize: lane = weight row of the warp's TMEM lane quarter ----------------
    const int qd = warp & 3, kh = (warp - 2) >> 2;   // lane quarter, k-half of each sub-step
    const int r = qd * 32 + lane;
    const int tl = r >> 3, g = r & 7;
    const bool live = r0 + r < p.n_rows;
    const uint32_t tlane = (uint32_t)(qd * 32) << 16;
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
      if (kh == 0) {
        scl[(sl2 * kMT + r) * 2] = h2f((uint16_t)(dd & 0xFFFFu));
        scl[(sl2 * kMT + r) * 2 + 1] = h2f((uint16_t)(dd >> 16));
      }
      mbar_arrive(&sc_full[sl2]);
      // A sub-tile ss (k 64ss..64ss+63 of the super-block) = qs bytes
      // 32ss..32ss+31: k-half 0 the low nibbles (scale sc[2ss]), k-half 1 the
      // high nibbles (sc[2ss+1]); 16 TMEM columns of fp16 pairs per half.
#pragma unroll
      for (int ss = 0; ss < 4; ++ss) {
        const int idx = s * 4 + ss, asl = idx % kARing;
        const uint32_t scv = (uint32_t)sc[2 * ss + kh];
        uint32_t h[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t w = kh ? (qw[8 * ss + i] >> 4) : qw[8 * ss + i];
          nib4_to_h2(w, scv, h[2 * i], h[2 * i + 1]);
        }
        wait_empty(&a_empty[asl], idx / kARing, p.status, 42, abort_flag);
        tc_fence_after();
        tmem_st16_sync(tmem + tlane + kAcol0 + asl * kAcols + kh * 16, h);
        tc_fence_before();
        mbar_arrive(&a_full[asl]);
      }
      // msum operand: (m_0..m_7 | m_0..m_7)
      const int ms = s % 2;
      wait_empty(&am_empty[ms], s / 2, p.status, 43, abort_flag);
      if (kh == 0) {   // warp-uniform: warps 2-5 store the 8 columns of their lanes
        uint32_t mv[8];
        mv[0] = mv[4] = pack_h2((float)mn[0], (float)mn[1]);
        mv[1] = mv[5] = pack_h2((float)mn[2], (float)mn[3]);
        mv[2] = mv[6] = pack_h2((float)mn[4], (float)mn[5]);
        mv[3] = mv[7] = pack_h2((float)mn[6], (float)mn[7]);
        tc_fence_after();
        tmem_st8_sync(tmem + tlane + kAmCol0 + ms * 8, mv);
        tc_fence_before();
      }
      mbar_arrive(&am_full[ms]);
    }
  } else {
    // ---------------- epilogue: thread = one weight row (TMEM lane), 32 of the 64 tokens ----------------
    constexpr int NE = kNT / 2;                // tokens per epilogue thread
    const int qt = warp & 3;                   // TMEM lane quarter of this warp
    const int eh = (warp - 2 - kDqWarps) >> 2; // token half
    const int r = qt * 32 + lane;
    float2 out[NE / 2];
#pragma unroll
    for (int t = 0; t < NE / 2; ++t) out[t] = make_float2(0.0f, 0.0f);
    ring_wait(dx_bar, 0, p.status, 50, abort_flag);
    for (int s = 0; s < nsb; ++s) {
      const int b = s & 1, sl2 = s % 2;
      wait_full(&acc_full[b], s / 2, p.status, 51, abort_flag);
      tc_fence_after();
      wait_full(&sc_full[sl2], s / 2, p.status, 52, abort_flag);
      const float d = scl[(sl2 * kMT + r) * 2], dmin = scl[(sl2 * kMT + r) * 2 + 1];
      mbar_arrive(&sc_empty[sl2]);
      const uint32_t tbase = tmem + ((uint32_t)(qt * 32) << 16) + b * kBufCols + eh * NE;
      const float2* dx2 = reinterpret_cast<const float2*>(dxs + s * kNT + eh * NE);
      // 8 tokens per step
#pragma unroll
      for (int c = 0; c < NE / 8; ++c) {
        uint32_t a0[8], a1[8], am[8];
        tmem_ld8x3(tbase + c * 8, tbase + kNT + c * 8, tbase + 2 * kNT + c * 8, a0, a1, am);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 dx = dx2[c * 4 + t];
          const float i0 = __fadd_rn(__uint_as_float(a0[2 * t]), __uint_as_float(a1[2 * t]));
          const float i1 = __fadd_rn(__uint_as_float(a0[2 * t + 1]), __uint_as_float(a1[2 * t + 1]));
          float2 o = out[c * 4 + t];
          o.x = __fadd_rn(o.x, __fmul_rn(__fmul_rn(d, dx.x), i0));
          o.y = __fadd_rn(o.y, __fmul_rn(__fmul_rn(d, dx.y), i1));
          o.x = __fsub_rn(o.x, __fmul_rn(__fmul_rn(dmin, dx.x), __uint_as_float(am[2 * t])));
          o.y = __fsub_rn(o.y, __fmul_rn(__fmul_rn(dmin, dx.y), __uint_as_float(am[2 * t + 1])));
          out[c * 4 + t] = o;
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    const int64_t row = r0 + r;
    if (row < p.n_rows) {
#pragma unroll
      for (int t = 0; t < NE / 2; ++t) {
        const int tok = tok_tile * kNT + eh * NE + 2 * t;
        if (tok < p.n_tok) p.y[(int64_t)tok * p.n_rows + row] = out[t].x;
        if (tok + 1 < p.n_tok) p.y[(int64_t)(tok + 1) * p.n_rows + row] = out[t].y;
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

// ---- Q8_0 weights: the integer tensor-core path ----------------------------------------------
// Per 32-weight block the reference adds (d_w·d_x)·sumi with sumi the exact
// int32 dot of the codes (Singularity/tests/test_and_bench_a5.cpp:205-221).
// A repacked Q8_0 slot is already two K-major 8x16-byte core matrices of the
// tile's 8 rows (codes 0-15 at +0, 16-31 at +128, the fp16 scales at +256),
// so a TMA copy of one slot per tile gives tcgen05.mma kind::i8 its A operand
// as loaded: no dequantization.  One K=32 MMA per block writes that block's
// sumi (int32) into its own 64 TMEM columns; the accumulators start at
// 0x4B400000, so the result read back as fp32 is 12582912 + sumi exactly
// (|sumi| <= 2^19) and one subtraction recovers (float)sumi.  The epilogue
// then applies acc + (d_w·d_x)·sumi block by block in order, two tokens per
// instruction with fma.rn.f32x2: a·b as fma(a, b, -0), a + b as fma(a, 1, b)
// and the subtraction as fma(x, 1, -12582912) each round exactly as the
// scalar operation, so Y is bit-identical to the reference-order matmul.
// The constants 1, -0 and -12582912 arrive as kernel parameters: with
// literal operands the compiler may turn such an fma back into a multiply or
// an add and fuse the pair into one fma (one rounding instead of two), which
// was measured to break the reference's rounding.
//
// Structure (one CTA per 128 weight rows x 64 tokens, 10 warps, two CTAs per
// SM so one's start-up and tail overlap the other's epilogue): warp 0 issues
// the copies of a group of 2 blocks per stage (16 slot tiles per block, the
// codes and scales of the activations); warp 1 owns 256 TMEM columns (two
// buffers of 2 blocks x 64 columns) and issues the MMAs; warps 2-9 are the
// epilogue, warp w reading TMEM lanes 32*(w%4).. for tokens 32*((w-2)/4)..,
// and re-seeding the columns it has read before handing the buffer back.
constexpr int kQ8G = 2;                             // blocks per group (one TMEM buffer)
constexpr int kQ8Stages = 6;
constexpr int kQ8A = (kMT / 8) * 272;               // 16 slots of one block
constexpr int kQ8B = kNT * 32;                      // 64 tokens x 32 codes, core-matrix order
constexpr int kQ8Dx = kNT * 4;
constexpr int kQ8Stage = kQ8G * (kQ8A + kQ8B + kQ8Dx);
constexpr int kQ8EpWarps = 8;
constexpr int kQ8Threads = (2 + kQ8EpWarps) * 32;
constexpr uint32_t kQ8TmemCols = 2 * kQ8G * kNT;
constexpr uint32_t kQ8Seed = 0x4B400000u;           // 12582912.0f
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kNT >> 3) << 17) |
                              ((uint32_t)(kMT >> 4) << 24);   // s32 D, s8 A and B, K-major, M=128, N=kNT

struct GemmQ8P {
  int nb, S, L;
  int64_t n_rows;
  int n_tok;
  const uint8_t* bimg;       // activation codes [tok tile][nb][kQ8B]
  const float* dximg;        // activation scales [tok tile][nb][kNT]
  float* y;                  // [n_tok][n_rows]
  int* status;
  float one, nzero, nseed;   // 1, -0, -12582912: opaque to the compiler (see above)
};

__device__ __forceinline__ void umma_i8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, p;\n\t}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(kIdescI8));
}
// 32 columns of this warp's lanes, loaded before return.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
// The same 32-bit value into 32 columns of this warp's lanes, completed before return.
__device__ __forceinline__ void tmem_fill32_sync(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr), "r"(v)
      : "memory");
}
// (d0, d1) = (a0·b0 + c0, a1·b1 + c1), each lane one correctly rounded fma.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// x fp32 [n_tok][k] -> Q8_0 codes in the B core-matrix order and the scales
// (as fp32 of the fp16 scale); padded tokens are zero.  One warp per (token,
// block), one value per lane, quantized like ref_quantize_row_q8_0.
__global__ void gemm_act_q8_0_kernel(const float* __restrict__ x, int64_t x_stride, int n_tok, int n_tok_pad, int nb,
                                     uint8_t* __restrict__ bimg, float* __restrict__ dximg) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)n_tok_pad * nb;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < total;
       i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(i / nb), b = (int)(i - (int64_t)t * nb);
    uint32_t c = 0;
    uint16_t d16 = 0;
    if (t < n_tok) c = (uint8_t)quant_q8_0_lane(x[t * x_stride + (int64_t)b * 32 + lane], &d16);   // warp-uniform
    const uint32_t w = c | (__shfl_down_sync(0xffffffffu, c, 1) << 8) | (__shfl_down_sync(0xffffffffu, c, 2) << 16) |
                       (__shfl_down_sync(0xffffffffu, c, 3) << 24);
    const int tt = t / kNT, tr = t % kNT;
    uint8_t* blk = bimg + ((int64_t)tt * nb + b) * kQ8B;
    if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(blk + (tr / 8) * 256 + (lane / 16) * 128 + (tr % 8) * 16 + (lane % 16)) = w;
    if (lane == 0) dximg[((int64_t)tt * nb + b) * kNT + tr] = h2f(d16);
  }
}

__global__ void __launch_bounds__(kQ8Threads, 2)
    gemm_q8_0_kernel(const GemmQ8P p, const __grid_constant__ CUtensorMap wmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int nb = p.nb, ng = (nb + kQ8G - 1) / kQ8G;
  uint64_t* st_full = reinterpret_cast<uint64_t*>(smem);   // [kQ8Stages]
  uint64_t* st_empty = st_full + kQ8Stages;                 // [kQ8Stages] MMA commit + every epilogue thread
  uint64_t* acc_full = st_empty + kQ8Stages;                // [2]
  uint64_t* acc_empty = acc_full + 2;                       // [2] every epilogue thread (seeded)
  uint64_t* mma_done = acc_empty + 2;                       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 496);
  int* abort_flag = reinterpret_cast<int*>(smem + 500);
  uint8_t* stages = smem + 1024;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_blk = blockIdx.x, tok_tile = blockIdx.y;
  const int64_t r0 = (int64_t)row_blk * kMT;
  const int tile0 = row_blk * (kMT / 8);
  constexpr int kEpThreads = kQ8EpWarps * 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQ8Stages; ++i) {
      mbar_init(&st_full[i], 1);
      mbar_init(&st_empty[i], 1 + kEpThreads);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpThreads);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kQ8TmemCols)
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
      int issued = 0;
      for (int g = 0; g < ng; ++g) {
        const int st = g % kQ8Stages, b0 = g * kQ8G, gb = min(kQ8G, nb - b0);
        if (!wait_empty(&st_empty[st], g / kQ8Stages, p.status, 60, abort_flag)) break;
        uint8_t* sp = stages + st * kQ8Stage;
        mbar_arrive_expect_tx(&st_full[st], (uint32_t)(gb * (kQ8A + kQ8B + kQ8Dx)));
        for (int j = 0; j < gb; ++j) {
          const int u = b0 + j, wr = u / p.L, ii = u - wr * p.L;
          tma_load_3d(sp + j * kQ8A, &wmap, 0, ii * p.S + wr, tile0, &st_full[st]);
        }
        const int64_t blk0 = (int64_t)tok_tile * nb + b0;
        bulk_g2s(sp + kQ8G * kQ8A, p.bimg + blk0 * kQ8B, (uint32_t)(gb * kQ8B), &st_full[st]);
        bulk_g2s(sp + kQ8G * (kQ8A + kQ8B), p.dximg + blk0 * kNT, (uint32_t)(gb * kQ8Dx), &st_full[st]);
        ++issued;
      }
      // every copy issued has landed before the CTA may exit
      for (int u = max(0, issued - kQ8Stages); u < issued; ++u)
        mbar_wait_bounded(&st_full[u % kQ8Stages], (u / kQ8Stages) & 1, p.status, 61);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      for (int g = 0; g < ng; ++g) {
        const int b = g & 1, st = g % kQ8Stages, gb = min(kQ8G, nb - g * kQ8G);
        // phase u of acc_empty[b] completes when the epilogue has seeded the buffer for use u
        if (!wait_full(&acc_empty[b], g / 2, p.status, 62, abort_flag)) break;
        tc_fence_after();
        if (!wait_full(&st_full[st], g / kQ8Stages, p.status, 63, abort_flag)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(stages + st * kQ8Stage), sb = sa + kQ8G * kQ8A;
        for (int j = 0; j < gb; ++j)
          umma_i8_ss(tmem + b * (kQ8G * kNT) + j * kNT, smem_desc(sa + j * kQ8A, 128, 272), smem_desc(sb + j * kQ8B, 128, 256),
                     1u);
        umma_commit(&st_empty[st]);
        umma_commit(&acc_full[b]);
      }
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status, 64);
    }
  } else {
    // ---------------- epilogue: thread = one weight row (TMEM lane), 32 tokens ----------------
    constexpr int NE = kNT / 2;
    const int qt = warp & 3, eh = (warp - 2) >> 2;
    const int r = qt * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(qt * 32) << 16) + eh * NE;
    // seed both buffers, then hand them to the MMA issuer
#pragma unroll
    for (int c = 0; c < 2 * kQ8G; ++c) tmem_fill32_sync(tl + c * kNT, kQ8Seed);
    tc_fence_before();
    mbar_arrive(&acc_empty[0]);
    mbar_arrive(&acc_empty[1]);
    float2 out[NE / 2];
#pragma unroll
    for (int t = 0; t < NE / 2; ++t) out[t] = make_float2(0.0f, 0.0f);
    const float2 one2 = make_float2(p.one, p.one), nz2 = make_float2(p.nzero, p.nzero),
                 nseed2 = make_float2(p.nseed, p.nseed);
    const int dw_off = (r >> 3) * 272 + 256 + (r & 7) * 2;
    for (int g = 0; g < ng; ++g) {
      const int b = g & 1, st = g % kQ8Stages, gb = min(kQ8G, nb - g * kQ8G);
      wait_full(&acc_full[b], g / 2, p.status, 65, abort_flag);
      tc_fence_after();
      wait_full(&st_full[st], g / kQ8Stages, p.status, 66, abort_flag);   // complete already: orders the smem reads
      const uint8_t* sp = stages + st * kQ8Stage;
#pragma unroll
      for (int j = 0; j < kQ8G; ++j) {
        if (j < gb) {
          const float dw = h2f(*reinterpret_cast<const uint16_t*>(sp + j * kQ8A + dw_off));
          const float2 dw2 = make_float2(dw, dw);
          const float4* dx4 = reinterpret_cast<const float4*>(sp + kQ8G * (kQ8A + kQ8B) + j * kQ8Dx) + eh * (NE / 4);
          uint32_t v[NE];
          tmem_ld32(tl + b * (kQ8G * kNT) + j * kNT, v);
#pragma unroll
          for (int q4 = 0; q4 < NE / 4; ++q4) {
            const float4 dx = dx4[q4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int t2 = q4 * 2 + h;
              const float2 sumi =
                  fma2(make_float2(__uint_as_float(v[2 * t2]), __uint_as_float(v[2 * t2 + 1])), one2, nseed2);
              const float2 dd = fma2(dw2, h ? make_float2(dx.z, dx.w) : make_float2(dx.x, dx.y), nz2);
              out[t2] = fma2(fma2(dd, sumi, nz2), one2, out[t2]);
            }
          }
        }
      }
      mbar_arrive(&st_empty[st]);
#pragma unroll
      for (int c = 0; c < kQ8G; ++c) tmem_fill32_sync(tl + b * (kQ8G * kNT) + c * kNT, kQ8Seed);
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    const int64_t row = r0 + r;
    if (row < p.n_rows) {
#pragma unroll
      for (int t = 0; t < NE / 2; ++t) {
        const int tok = tok_tile * kNT + eh * NE + 2 * t;
        if (tok < p.n_tok) p.y[(int64_t)tok * p.n_rows + row] = out[t].x;
        if (tok + 1 < p.n_tok) p.y[(int64_t)(tok + 1) * p.n_rows + row] = out[t].y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kQ8TmemCols) : "memory");
  }
}

size_t gemm_q8_0_smem_bytes() { return 1024 + 1024 + (size_t)kQ8Stages * kQ8Stage; }

size_t gemm_smem_bytes(int nsb) {
  return 1024 + 1024 + (size_t)kBGroups * kBGroup + (size_t)kRaw * kRawStage + 2 * kBm +
         (size_t)2 * kMT * 2 * 4 + (size_t)nsb * kNT * 4;
}

// The weight tensor map: the tile layout as [tiles][slots][slot_bytes / 8 x
// 8 bytes], boxes of 16 tiles x 1 slot (one unit of a CTA's 128 rows).
int make_weight_map(const QMatrix& w, CUtensorMap* map) {
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess || !fn) {
      set_error("gemm: cuTensorMapEncodeTiled unavailable");
      return B2_ERR_CUDA;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  const cuuint64_t dims[3] = {(cuuint64_t)w.slot_bytes / 8, (cuuint64_t)w.splits * w.ulen, (cuuint64_t)w.n_tiles};
  const cuuint64_t strides[2] = {(cuuint64_t)w.slot_bytes, (cuuint64_t)w.tile_bytes};
  const cuuint32_t box[3] = {(cuuint32_t)w.slot_bytes / 8, 1, kMT / 8};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(w.data), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gemm: weight tensor map rejected (CUresult %d)", (int)r);
    return B2_ERR_CUDA;
  }
  return B2_OK;
}

}  // namespace

size_t gemm_act_image_bytes(const QMatrix& w, int n_tok) {
  const int tiles = (n_tok + kNT - 1) / kNT;
  if (w.type == B2_Q8_0) return (size_t)tiles * w.nu * (kQ8B + kQ8Dx);
  return (size_t)tiles * w.nu * (4 * kBSub + kBm + kNT * 4);
}

namespace {
int launch_gemm_q8_0(const QMatrix& w, const float* x, int64_t x_stride, int n_tok, float* y, uint8_t* img,
                     int* status, cudaStream_t s) {
  const int nb = w.nu;
  const int tiles = (n_tok + kNT - 1) / kNT;
  uint8_t* bimg = img;
  float* dximg = reinterpret_cast<float*>(bimg + (size_t)tiles * nb * kQ8B);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  {
    cudaLaunchConfig_t cfg = {};
    const int64_t warps = (int64_t)tiles * kNT * nb;
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((warps * 32 + 255) / 256, 8 * sm_count())));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_act_q8_0_kernel, x, x_stride, n_tok, tiles * kNT, nb, bimg, dximg));
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = gemm_q8_0_smem_bytes();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    B2_CUDA_TRY(cudaFuncSetAttribute(gemm_q8_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[dev] = true;
  }
  GemmQ8P p = {};
  p.nb = nb;
  p.S = w.splits;
  p.L = w.ulen;
  p.n_rows = w.n_rows;
  p.n_tok = n_tok;
  p.bimg = bimg;
  p.dximg = dximg;
  p.y = y;
  p.status = status;
  p.one = 1.0f;
  p.nzero = -0.0f;
  p.nseed = -12582912.0f;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((w.n_rows + kMT - 1) / kMT), (unsigned)tiles);
  cfg.blockDim = dim3(kQ8Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap wmap;
  const int mrc = make_weight_map(w, &wmap);
  if (mrc) return mrc;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_q8_0_kernel, p, wmap));
  return B2_OK;
}
}  // namespace

int launch_gemm(const QMatrix& w, const float* x, int64_t x_stride, int n_tok, float* y, uint8_t* img, int* status,
                cudaStream_t s) {
  B2_CHECK_ARG(w.type == B2_Q4_K || w.type == B2_Q8_0, "the tensor-core GEMM takes Q4_K or Q8_0 weights");
  B2_CHECK_ARG(n_tok >= 1 && x && y && img, "gemm arguments");
  B2_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && x_stride % 4 == 0, "x alignment");
  if (w.type == B2_Q8_0) return launch_gemm_q8_0(w, x, x_stride, n_tok, y, img, status, s);
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
  CUtensorMap wmap;
  const int mrc = make_weight_map(w, &wmap);
  if (mrc) return mrc;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_q4k_kernel, p, wmap));
  return B2_OK;
}

}  // namespace b2
