// Decode attention without any device allocation, for callers that cannot
// allocate device memory while they run: hosts that hand the library a fixed
// device-memory budget at start-up, and real-time decode loops that must not
// take an allocation's latency or risk its failure in the middle of a turn.
//
// The attention's scratch (scores, exponentials, chunk maxima) lives in one file-scope
// __device__ array of B2_NOALLOC_SCRATCH_BYTES; every GPU that loads the
// library holds that array until the process exits.  The caller still passes q, the caches and out.
// The array's device address is taken with cudaGetSymbolAddress the first
// time the entry point runs on a device (with that device current), so that
// first call should come before any stream capture.  A call on a stream that
// is not capturing looks the address up again, so a device reset
// (cudaDeviceReset, which reloads the module) between calls is picked up; a
// call under capture uses the address seen last, and a reset between that
// lookup and the capture leaves it stale.  All calls share the array: calls
// whose work overlaps on the GPU (different streams, or other threads) race
// on it and must be serialized by the caller.
#include <mutex>

#include "b2_common.cuh"
#include "b2_layers.hpp"

namespace b2 {
namespace {

constexpr size_t kScratchBytes = (size_t)B2_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_scratch on the current device: looked up on every
// call outside stream capture, cached for calls under capture.
int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("attn_decode_noalloc: device ordinal %d beyond %d", dev, kMaxDevices);
    return B2_ERR_UNSUPPORTED;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  B2_CUDA_TRY(cudaStreamIsCapturing(stream, &cap));
  std::lock_guard<std::mutex> lock(g_mu);
  if (cap == cudaStreamCaptureStatusNone || !g_addr[dev]) {
    void* p = nullptr;
    B2_CUDA_TRY(cudaGetSymbolAddress(&p, g_scratch));
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_attn_decode_noalloc(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                      const int32_t* pos, const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv,
                                      int head_dim, int cap, float* out, void* stream) {
  B2_CHECK_ARG(q && k_cache && v_cache && pos && seq && out && cap > 0 && n_seq > 0, "attn_decode_noalloc arguments");
  B2_CHECK_ARG(n_kv > 0 && n_head % n_kv == 0, "n_head must be a multiple of n_kv");
  if (n_q < 1 || n_q > B2_NOALLOC_MAX_QUERIES) {
    set_error("attn_decode_noalloc: n_q=%d outside [1, %d]", n_q, B2_NOALLOC_MAX_QUERIES);
    return B2_ERR_INVALID;
  }
  const size_t sc_bytes = attn_scratch_floats(n_q, n_head, n_kv, cap) * sizeof(float);
  if (sc_bytes > kScratchBytes) {
    set_error("attn_decode_noalloc: %d queries x %d heads x %d positions need %zu scratch bytes, "
              "more than the %zu built in",
              n_q, n_head, cap, sc_bytes, kScratchBytes);
    return B2_ERR_INVALID;
  }
  void* base = nullptr;
  const int rc = scratch_address(static_cast<cudaStream_t>(stream), &base);
  if (rc) return rc;
  // every value the kernels read is written earlier in the same call
  return launch_attention(q, n_q, n_head, n_kv, head_dim, pos, seq, k_cache, B2_F16, v_cache, B2_F16, nullptr, n_seq,
                          cap, static_cast<float*>(base), out, static_cast<cudaStream_t>(stream));
}
