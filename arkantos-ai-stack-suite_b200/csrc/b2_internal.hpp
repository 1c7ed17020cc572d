// Host-side internals shared by the library's translation units: error
// reporting, block formats and the repacked quantized-matrix descriptor.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "../../include/b2gguf.h"

namespace b2 {

// ---- error reporting ----------------------------------------------------------
// Thread-local message for b2_last_error(); every failing C-ABI call sets it.
void set_error(const char* fmt, ...);
const char* last_error();

#define B2_CUDA_TRY(expr)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) {                                                                \
      ::b2::set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(e_));   \
      return e_ == cudaErrorMemoryAllocation ? B2_ERR_OOM : B2_ERR_CUDA;                    \
    }                                                                                       \
  } while (0)

#define B2_CHECK_ARG(cond, msg)                        \
  do {                                                 \
    if (!(cond)) {                                     \
      ::b2::set_error("invalid argument: %s", msg);    \
      return B2_ERR_INVALID;                           \
    }                                                  \
  } while (0)

// ---- block formats (GGUF; ids and sizes as ggml) --------------------------------
constexpr int QK4_0 = 32, QK8_0 = 32, QK_K = 256;
struct __attribute__((packed)) BlockQ4_0 { uint16_t d; uint8_t qs[16]; };
struct __attribute__((packed)) BlockQ8_0 { uint16_t d; int8_t qs[32]; };
struct __attribute__((packed)) BlockQ4_K { uint16_t d; uint16_t dmin; uint8_t scales[12]; uint8_t qs[128]; };
struct __attribute__((packed)) BlockQ6_K { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; };
struct __attribute__((packed)) BlockQ8_K { float d; int8_t qs[256]; int16_t bsums[16]; };
static_assert(sizeof(BlockQ4_0) == 18 && sizeof(BlockQ8_0) == 34, "block sizes");
static_assert(sizeof(BlockQ4_K) == 144 && sizeof(BlockQ6_K) == 210 && sizeof(BlockQ8_K) == 292, "k-quant sizes");

size_t row_bytes(int type, int64_t k);
int block_elems(int type);
bool is_weight_type(int type);
// The activation format the reference's CPU dot pairs with each weight type:
// Q8_0 for Q4_0/Q8_0, Q8_K for Q4_K/Q6_K.
inline int act_type_for(int wtype) { return (wtype == B2_Q4_K || wtype == B2_Q6_K) ? B2_Q8_K : B2_Q8_0; }

// ---- repacked quantized matrix (device) -----------------------------------------
// W is [n_rows x k] in GGUF blocks along k.  On upload the columns are split
// into n_chunks chunks of kc columns (kc a multiple of 256, kp = n_chunks*kc
// >= k, the tail zero-padded), and the block bytes are split into planes so
// every (row, chunk) piece is 16-byte aligned and a whole multiple of 16
// bytes — one cp.async.bulk each:
//   Q4_0  plane0 = nibbles   (16 B / 32 cols)       plane1 = fp16 d per 32 cols
//   Q8_0  plane0 = int8 q    (32 B / 32 cols)       plane1 = fp16 d per 32 cols
//   Q4_K  plane0 = the 144 B GGUF super-blocks as-is (d, dmin, scales, qs)
//   Q6_K  plane0 = ql|qh|scales (208 B / 256 cols)  plane1 = fp16 d per 256 cols
// plane0 row r, chunk c at r*p0_row + c*p0_chunk; plane1 at r*p1_row + c*p1_chunk
// (p1_chunk padded up to 16 B).  Bytes are bit-identical to the GGUF input.
struct QMatrix {
  int type = 0;
  int64_t n_rows = 0, k = 0, kp = 0;
  int kc = 0, n_chunks = 0;
  uint8_t* plane0 = nullptr;
  uint8_t* plane1 = nullptr;
  int64_t p0_row = 0, p0_chunk = 0, p1_row = 0, p1_chunk = 0;
  int device = 0;
  bool owns = true;
};

// Chooses kc / n_chunks / plane strides for a matrix shape.
void plan_qmatrix(QMatrix& m);
// Repacks GGUF rows [r0, r1) into host plane buffers laid out as in QMatrix.
void repack_rows_host(const QMatrix& m, const uint8_t* gguf, int64_t r0, int64_t r1, uint8_t* p0, uint8_t* p1);

// ---- planar quantized activations (device) ---------------------------------------
// B token rows of kp values: qs [B][kp] int8 (zero beyond k), d [B][kp/32]
// (Q8_0, as fp32 converted exactly from the fp16 scale) or [B][kp/256] (Q8_K,
// fp32), bsum [B][kp/16] int16 (Q8_K only).
struct ActQ {
  int type = 0;
  int n_tok = 0;
  int64_t kp = 0;
  int8_t* qs = nullptr;
  float* d = nullptr;
  int16_t* bsum = nullptr;
};

// ---- kernel launchers (device pointers, async) ------------------------------------
// Epilogue applied to each output value y[t][r].
enum Epilogue : int {
  EPI_STORE = 0,       // y = W·x
  EPI_ACCUM = 1,       // y += W·x (residual add)
  EPI_SWIGLU = 2,      // rows (2i, 2i+1) are (gate_i, up_i): y[i] = silu(gate)·up
};

// Tensor-parallel exchange over peer memory (CUDA IPC mappings over NVLink).
// A row-split projection (attention-out, FFN-down, the vocabulary-sharded
// head) on rank r stores its outputs into slot r of every rank's gather
// buffer; its last CTA then raises the phase's epoch in every rank's flag r.
// The consumer on each rank waits until all flags reach the epoch and sums the
// slots in rank order — a fixed-order allreduce with no library collective.
constexpr int kMaxTp = 8;
struct PeerOut {
  int n = 0;                                   // ranks (0: plain local store)
  float* dst[kMaxTp] = {};                     // per rank: this rank's slot in its gather buffer
  unsigned long long* flag[kMaxTp] = {};       // per rank: this rank's flag word of the phase
  unsigned int* done = nullptr;                // local: CTAs of the launch that have stored
  unsigned long long* epoch = nullptr;         // local: epochs of the phase so far
};
struct PeerIn {
  int n = 0;                                   // ranks (0: no exchange)
  const float* parts = nullptr;                // local gather buffer, slot j at parts + j * slot
  int64_t slot = 0;                            // elements between slots
  const unsigned long long* flags = nullptr;   // local flags of the phase [n]
  const unsigned long long* epoch = nullptr;   // local epoch counter of the phase
};

struct GemvArgs {
  const QMatrix* w;
  const float* x;       // fp32 [n_tok][x_stride] when act == nullptr (quantized in-kernel)
  int64_t x_stride;
  const ActQ* act;      // pre-quantized activations, or nullptr
  int n_tok;
  float* y;             // [n_tok][y_stride]
  int64_t y_stride;
  int epilogue;
  int64_t row_begin, row_end;   // rows of W to compute (TP slices, tests); end<=n_rows
  int* status;          // device status word (bounded waits), may be nullptr
  const PeerOut* peer = nullptr;   // tensor-parallel exchange of the outputs (EPI_STORE only)
};
int launch_gemv(const GemvArgs& a, cudaStream_t s);
// Sets the large dynamic shared-memory limit of every GEMV instantiation on
// the current device (done outside graph capture).
int prepare_gemv_kernels();
int launch_quantize_act(int act_type, const float* x, int64_t x_stride, int n_tok, int64_t k, ActQ& out,
                        cudaStream_t s);
int launch_act_to_blocks(const ActQ& a, int64_t k, void* blocks, cudaStream_t s);
int launch_block_dots(const QMatrix& w, const ActQ& a, int64_t row, int32_t* out_i, int32_t* out_m,
                      cudaStream_t s);
int launch_dequantize(const QMatrix& w, float* dst, cudaStream_t s);

// Multiprocessor count of the current device (cached per device).
int sm_count();

// Programmatic dependent launch between this library's kernels (per thread).
bool pdl_enabled();
void set_pdl(bool on);

// ---- host helpers (b2_host.cpp) -----------------------------------------------------
uint16_t host_f32_to_f16(float f);
float host_f16_to_f32(uint16_t h);
int quantize_weights(int type, const float* src, int64_t n_rows, int64_t k, void* dst, int n_threads);
int synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float std_dev, float* out, int n_threads);
void rope_table(float theta, int head_dim, int p0, int n_pos, float* out);

}  // namespace b2
