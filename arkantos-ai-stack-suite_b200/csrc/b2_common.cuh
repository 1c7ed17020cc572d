// Shared device helpers for the sm_100a kernels: fp16 conversion, PDL
// (programmatic dependent launch) controls, mbarriers and bulk async copies.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_internal.hpp"

namespace b2 {

constexpr int kSMs = 148;

// ---- programmatic dependent launch ------------------------------------------
// Blocks until every grid this one depends on has finished and its writes are
// visible.  Weight streaming may start before it; activations are read after.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream start launching its CTAs.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches kern with programmatic stream serialization when PDL is on.
template <typename K, typename... Args>
int launch_pdl(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...));
  return B2_OK;
}

// ---- mbarrier -----------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after kMbarWaitNs of wall time (each try_wait itself
// suspends for a hardware-chosen interval, so the bound is on the clock, not
// on the number of polls), records the failure in *status and returns false.
// Every wait in these kernels is bounded so a lost transfer ends the kernel
// with an error code instead of hanging the GPU.
constexpr uint64_t kMbarWaitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > kMbarWaitNs) break;
  }
  if (status) atomicExch(status, code);
  return false;
}

// ---- peer flags (system scope: written and read across GPUs) -------------------------
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Waits until flags[0..n) all reach `target`, for at most kPeerWaitNs of
// wall time; on expiry records `code` in *status and returns false (the
// caller then proceeds on whatever the buffers hold, so a lost peer ends the
// step with an error status instead of hanging the GPU).
constexpr uint64_t kPeerWaitNs = 2000000000ull;
constexpr int kPeerWaitStatus = 3;   // status code of an expired exchange wait
__device__ __forceinline__ bool wait_peer_flags(const unsigned long long* flags, int n, unsigned long long target,
                                                int* status, int code) {
  // after one expiry in this step the others give up at once (a lost peer
  // costs one wait, not one per phase)
  if (status && *reinterpret_cast<volatile int*>(status) != 0) return false;
  const uint64_t t0 = globaltimer_ns();
  for (int j = 0; j < n; ++j) {
    while (ld_acquire_sys_u64(flags + j) < target) {
      if (globaltimer_ns() - t0 > kPeerWaitNs) {
        if (status) atomicExch(status, code);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// The exchange wait of a consumer kernel (one thread), its wall time added to
// in.wait_ns by the grid's first CTA: the time a rank spends waiting for its
// peers' partials.
__device__ __forceinline__ bool peer_wait(const PeerIn& in, int* status, int code) {
  const uint64_t t0 = globaltimer_ns();
  const bool ok = wait_peer_flags(in.flags, in.n, *in.epoch, status, code);
  if (in.wait_ns && blockIdx.x == 0 && blockIdx.y == 0)
    atomicAdd(in.wait_ns, (unsigned long long)(globaltimer_ns() - t0));
  return ok;
}

// ---- bulk async copy (1-D TMA, global -> shared, completes on an mbarrier) ----
// Both addresses 16-byte aligned, size a multiple of 16 bytes.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of a global range (no data returned).
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

// ---- loads ----------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h_rn(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Nibble bytes n in [0,15] -> signed bytes n-8, four lanes at once, with no
// carry across bytes ((n + 120) never exceeds 135).
__device__ __forceinline__ int nib_lo_s8(uint32_t v) { return (int)((((v & 0x0F0F0F0Fu) + 0x78787878u)) ^ 0x80808080u); }
__device__ __forceinline__ int nib_hi_s8(uint32_t v) {
  return (int)(((((v >> 4) & 0x0F0F0F0Fu) + 0x78787878u)) ^ 0x80808080u);
}

// exp(x) in fp32: Cody-Waite reduction x = n·ln2 + r (|r| <= ln2/2, ln2 split
// into a 16-bit head so n·ln2_hi is exact), the degree-7 Taylor polynomial of
// e^r by Horner's rule (truncation < 0.2 ulp), then scaling by 2^n built
// from exponent bits.  Every step is one IEEE-rounded operation written as an
// explicit intrinsic, so the result is the same bits as the oracle's C copy
// of this algorithm on any conforming fp32 unit.
__device__ __forceinline__ float b2_expf(float x) {
  if (!(x == x)) return x;
  if (x > 88.7228394f) return __int_as_float(0x7f800000);
  if (x < -103.972084f) return 0.0f;
  const float t = __fmul_rn(x, 1.44269502f);
  const float n = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
  float r = __fsub_rn(x, __fmul_rn(n, 0.693145751953125f));
  r = __fsub_rn(r, __fmul_rn(n, 1.42860677e-06f));
  float p = 1.98412698e-04f;
  p = __fadd_rn(__fmul_rn(p, r), 1.38888889e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 8.33333333e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 4.16666667e-02f);
  p = __fadd_rn(__fmul_rn(p, r), 1.66666667e-01f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  int ni = (int)n;
  float s2 = 1.0f;
  if (ni > 127) {
    ni -= 1;
    s2 = 2.0f;
  } else if (ni < -126) {
    ni += 64;
    s2 = 5.42101086e-20f;   // 2^-64
  }
  const float s1 = __int_as_float((ni + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

// exp(x) in fp32 with the results of the host C library's expf (glibc 2.28+,
// the table-driven algorithm published with ARM's optimized-routines):
// x·32/ln2 = k + r with k rounded to an integer through the 1.5·2^52 shift,
// 2^(k/32) from a 32-entry table of 2^(i/32) (rounded to double, with the
// exponent field pre-biased by i·2^47), 2^(r/32) by a cubic, all in double,
// then one rounding to float.  r is formed with one fused multiply-add, the
// form the library's FMA build evaluates; the whole float range was compared
// against the host library bit for bit.  The reference's CPU path
// (ref_softmax_f32, Singularity/tests/test_and_bench_a5.cpp:260-278, and the
// SiLU of the forward) calls expf, so kernels that must reproduce it bit for
// bit use this.
__constant__ static const unsigned long long kExp2Tab32[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};
// tab: kExp2Tab32 itself, or a copy of it in shared memory (exp_table_to_smem):
// the lanes of a warp index the table with different k, which the constant
// cache serves one address at a time and shared memory in one access.
__device__ __forceinline__ float b2_expf_ref(float x, const unsigned long long* tab) {
  if (!(x == x)) return x;
  if (x > 88.7228394f) return __int_as_float(0x7f800000);
  if (x < -103.972084f) return 0.0f;
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0, shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32768.0, c1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
               c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
  double kd = __dadd_rn(__dmul_rn(inv_ln2_n, xd), shift);
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, shift);
  const double r = __fma_rn(inv_ln2_n, xd, -kd);
  const double s = __longlong_as_double((long long)(tab[ki & 31] + (ki << 47)));
  const double z = __dadd_rn(__dmul_rn(c0, r), c1);
  const double r2 = __dmul_rn(r, r);
  double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
  y = __dadd_rn(__dmul_rn(z, r2), y);
  return __double2float_rn(__dmul_rn(y, s));
}

// silu(g)·u in the reference's order: (g / (1 + expf(-g))) · u.
__device__ __forceinline__ float b2_expf_ref(float x) { return b2_expf_ref(x, kExp2Tab32); }
// Copies the table into tab[32] of shared memory (threads tid of n); the
// caller synchronizes before the first use.
__device__ __forceinline__ void exp_table_to_smem(unsigned long long* tab, int tid, int n) {
  for (int i = tid; i < 32; i += n) tab[i] = kExp2Tab32[i];
}
__device__ __forceinline__ float silu_mul_ref(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, b2_expf_ref(-g))), u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace b2
