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

// ---- tiled quantized matrix (device) ---------------------------------------------
// W is [n_rows x k] in GGUF units along k: 32-weight blocks (Q4_0, Q8_0) or
// 256-weight super-blocks (Q4_K, Q6_K), nu units per row.  On upload the rows
// are grouped into tiles of 8 (the last tile zero-padded); a tile is nu unit
// slots in unit order, slot u carrying unit u of the tile's 8 rows, so any
// run of a tile's units is one contiguous bulk copy.  Within a slot the 8
// rows' unit bytes are moved into planes, row g of each plane at g * (plane
// row bytes); planes of 64 or 128 B per row have row g's 16-byte chunks
// rotated by g, so per-row shared-memory reads hit distinct banks.  Bytes
// are those of the GGUF input.
//   Q4_0  144 B: qs 8x16 @0,  d 8x2 @128
//   Q8_0  272 B: qs[0:16] 8x16 @0, qs[16:32] 8x16 @128, d 8x2 @256
//   Q4_K 1152 B: qs 8x128 @0 (rotated), d|dmin|scales 8x16 @1024
//   Q6_K 1680 B: ql 8x128 @0 (rotated), qh 8x64 @1024 (rotated), scales 8x16 @1536, d 8x2 @1664
// (splits/ulen describe the slot order: S ranges of L units, slot i*S + w =
// unit w*L + i; the layout uploaded here is S = 1, L = nu, i.e. unit order.)
#if defined(__CUDACC__)
#define B2_HD __host__ __device__
#else
#define B2_HD
#endif
struct QMatrix {
  int type = 0;
  int64_t n_rows = 0, k = 0;
  int nu = 0, splits = 1, ulen = 0;      // units per row, S, L
  int slot_bytes = 0;                    // one unit of the tile's 8 rows
  int64_t n_tiles = 0, tile_bytes = 0;   // tiles of 8 rows, S*L*slot_bytes each
  uint8_t* data = nullptr;
  int device = 0;
  bool owns = true;
  int64_t bytes() const { return n_tiles * tile_bytes; }
};

B2_HD inline int unit_elems(int type) { return (type == B2_Q4_K || type == B2_Q6_K) ? 256 : 32; }
B2_HD inline int gguf_unit_bytes(int type) {
  return type == B2_Q4_0 ? 18 : type == B2_Q8_0 ? 34 : type == B2_Q4_K ? 144 : type == B2_Q6_K ? 210 : 0;
}
B2_HD inline int tile_slot_bytes(int type) {
  return type == B2_Q4_0 ? 144 : type == B2_Q8_0 ? 272 : type == B2_Q4_K ? 1152 : type == B2_Q6_K ? 1680 : 0;
}
// Slot-order ranges per row of the uploaded layout: one (units in order).
B2_HD inline int tile_splits(int type, int64_t k) { return 1; }
// Byte offset of (tile, unit u) in the matrix data.
B2_HD inline int64_t slot_offset(const QMatrix& m, int64_t tile, int u) {
  const int w = u / m.ulen, i = u - w * m.ulen;
  return tile * m.tile_bytes + (int64_t)(i * m.splits + w) * m.slot_bytes;
}

B2_HD inline void copy_bytes(uint8_t* d, const uint8_t* s, int n) {
  for (int i = 0; i < n; ++i) d[i] = s[i];
}
// Moves row g's GGUF unit into its slot, and back.
B2_HD inline void unit_to_slot(int type, const uint8_t* src, int g, uint8_t* slot) {
  switch (type) {
    case B2_Q4_0: copy_bytes(slot + 128 + 2 * g, src, 2); copy_bytes(slot + 16 * g, src + 2, 16); break;
    case B2_Q8_0:
      copy_bytes(slot + 256 + 2 * g, src, 2);
      copy_bytes(slot + 16 * g, src + 2, 16);
      copy_bytes(slot + 128 + 16 * g, src + 18, 16);
      break;
    case B2_Q4_K:
      copy_bytes(slot + 1024 + 16 * g, src, 16);
      for (int c = 0; c < 8; ++c) copy_bytes(slot + 128 * g + 16 * ((c + g) & 7), src + 16 + 16 * c, 16);
      break;
    case B2_Q6_K:
      for (int c = 0; c < 8; ++c) copy_bytes(slot + 128 * g + 16 * ((c + g) & 7), src + 16 * c, 16);
      for (int c = 0; c < 4; ++c) copy_bytes(slot + 1024 + 64 * g + 16 * ((c + g) & 3), src + 128 + 16 * c, 16);
      copy_bytes(slot + 1536 + 16 * g, src + 192, 16);
      copy_bytes(slot + 1664 + 2 * g, src + 208, 2);
      break;
    default: break;
  }
}
B2_HD inline void slot_to_unit(int type, const uint8_t* slot, int g, uint8_t* dst) {
  switch (type) {
    case B2_Q4_0: copy_bytes(dst, slot + 128 + 2 * g, 2); copy_bytes(dst + 2, slot + 16 * g, 16); break;
    case B2_Q8_0:
      copy_bytes(dst, slot + 256 + 2 * g, 2);
      copy_bytes(dst + 2, slot + 16 * g, 16);
      copy_bytes(dst + 18, slot + 128 + 16 * g, 16);
      break;
    case B2_Q4_K:
      copy_bytes(dst, slot + 1024 + 16 * g, 16);
      for (int c = 0; c < 8; ++c) copy_bytes(dst + 16 + 16 * c, slot + 128 * g + 16 * ((c + g) & 7), 16);
      break;
    case B2_Q6_K:
      for (int c = 0; c < 8; ++c) copy_bytes(dst + 16 * c, slot + 128 * g + 16 * ((c + g) & 7), 16);
      for (int c = 0; c < 4; ++c) copy_bytes(dst + 128 + 16 * c, slot + 1024 + 64 * g + 16 * ((c + g) & 3), 16);
      copy_bytes(dst + 192, slot + 1536 + 16 * g, 16);
      copy_bytes(dst + 208, slot + 1664 + 2 * g, 2);
      break;
    default: break;
  }
}

// Fills the tile geometry of m from type, n_rows and k.
void plan_qmatrix(QMatrix& m);
// Repacks into host buffer `out` the tiles [t0, t1); row r's GGUF bytes are
// at rows[r] (rows past n_rows are zero).
void repack_tiles_host(const QMatrix& m, const uint8_t* const* rows, int64_t t0, int64_t t1, uint8_t* out);
// Pinned, double-buffered staging for weight uploads: the host threads
// repack one slab while the previous slab is copied to the device on the
// stager's stream.  One stager serves a whole model load (pinning memory is
// costly); finish() waits for every copy issued.
struct UploadStager {
  uint8_t* h[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaStream_t stream = nullptr;
  size_t bytes = 0;   // per buffer
  int next = 0;
  UploadStager() = default;
  UploadStager(const UploadStager&) = delete;
  UploadStager& operator=(const UploadStager&) = delete;
  ~UploadStager();
  int init(size_t per_buffer);
  int finish();
};
// Plans m (type, n_rows, k set), allocates m.data on the current device and
// uploads the repacked tiles; rows[r] points at row r's GGUF bytes.  With a
// stager the copies may still be in flight on return (the stager's finish()
// completes them); without one the call stages through its own and waits.
int upload_tiles(QMatrix& m, const uint8_t* const* rows, UploadStager* st = nullptr);

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
  EPI_ROPE_KV = 3,     // fused Q/K/V rows: RoPE on q and k, q to q_out, k and v into the fp16 KV cache
};

// Per-sequence KV bookkeeping, read by kernels from device memory (a null
// state array means every sequence is in the plain layout, slot = position).  Logical
// position p lives in physical slot p when p < n_keep (the pinned prefix),
// otherwise in n_keep + (ring_head + p − n_keep) mod (cap − n_keep): the
// slots after the prefix form a ring, so dropping the oldest positions
// after the prefix (Milda's KV shift) only advances ring_head.
struct KvSeqState {
  int32_t n_keep;
  int32_t ring_head;
};
B2_HD inline int64_t kv_slot(const KvSeqState& st, int p, int cap) {
  const int ring = cap - st.n_keep;
  if (p < st.n_keep || ring <= 0) return p;
  const int r = (st.ring_head + (p - st.n_keep)) % ring;
  return st.n_keep + r;
}

// The QKV projection's fused epilogue (EPI_ROPE_KV): output row r of token t
// is dim r % hd of head r / hd (n_head query heads, then n_kv key heads, then
// n_kv value heads).  Pairs (2i, 2i+1) of q and k rows are rotated by the
// token's position (rope: [position][hd] cos, sin pairs) exactly as
// rope_kv_kernel does; q goes to q_out [t][n_head*hd], k and v to the cache
// slot of (seq[t], pos[t]) in fp16 (RNE).  A token whose sequence or position
// is outside the cache gets a zero q and stores nothing.
struct RopeKvEpi {
  const int32_t* pos = nullptr;
  const int32_t* seq = nullptr;
  const float* rope = nullptr;
  float* q_out = nullptr;
  uint16_t* kc = nullptr;
  uint16_t* vc = nullptr;
  const KvSeqState* st = nullptr;   // may be null (plain layout)
  int n_head = 0, n_kv = 0, hd = 0, n_seq = 0, cap = 0;
};

// Where a GEMV's quantized activations live: the image carve-up of
// gemv_act_image(w, n_tok) — codes [n_act_tok][kq] in natural order, fp32
// scales per (token, unit), int16 block sums per (token, unit).  Producers
// other than the GEMV's own quantizer (the fused RMSNorm, the attention's
// last CTAs) write it through the same store helpers.
struct ActImage {
  uint8_t* img = nullptr;
  int kq = 0, nu = 0, type = 0, n_act_tok = 0;
  uint32_t off_dx = 0, off_bs = 0, bytes = 0;
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
  unsigned long long* wait_ns = nullptr;       // accumulated wall time of the waits (CTA 0), or null
};

struct GemvArgs {
  const QMatrix* w;
  const float* x;       // fp32 [n_tok][x_stride], 16-byte aligned
  int64_t x_stride;
  int n_tok;
  // Device scratch of gemv_act_image_bytes(w, n_tok) bytes: x quantized into
  // the image the GEMV's CTAs copy into shared memory (written by a quantize
  // kernel launched first).
  uint8_t* act_img;
  float* y;             // [n_tok][y_stride]
  int64_t y_stride;
  int epilogue;
  int* status;          // device status word (bounded waits), may be nullptr
  const PeerOut* peer = nullptr;   // tensor-parallel exchange of the outputs (EPI_STORE only)
  const RopeKvEpi* rope = nullptr; // EPI_ROPE_KV targets
  bool image_ready = false;        // act_img already holds x quantized (x is not read)
  // Several matrices of w's type and shape over the same x in one launch
  // (1-2 tokens, plain store): wlist[i] -> ylist[i]; w = wlist[0].
  int n_mat = 1;
  const QMatrix* const* wlist = nullptr;
  float* const* ylist = nullptr;
  // Grouped experts (1-2 tokens, plain store): matrix i is expert mat_ids[i]
  // (device) of a stack of n_expert matrices shaped like w, mat_stride bytes
  // apart from w->data; its output is y + i·y_mat_stride.
  const int32_t* mat_ids = nullptr;
  int n_expert = 0;
  int64_t mat_stride = 0, y_mat_stride = 0;
  int64_t x_mat_stride = 0;   // matrix i reads x + i·x_mat_stride (0: all read x)
};
int launch_gemv(const GemvArgs& a, cudaStream_t s);
size_t gemv_act_image_bytes(const QMatrix& w, int n_tok);
bool gemv_needs_image(const QMatrix& w, int n_tok);
// The image carve-up the GEMV over w expects for n_tok tokens, at img.
ActImage gemv_act_image(const QMatrix& w, int n_tok, uint8_t* img);

// Tensor-core prefill GEMM (Q4_K weights, any number of tokens), summation
// order identical to the reference's per-row vec_dot.  `img` is device
// scratch of gemm_act_image_bytes(w, n_tok) bytes; y fp32 [n_tok][n_rows].
size_t gemm_act_image_bytes(const QMatrix& w, int n_tok);
int launch_gemm(const QMatrix& w, const float* x, int64_t x_stride, int n_tok, float* y, uint8_t* img, int* status,
                cudaStream_t s);
// Sets the large dynamic shared-memory limit of every GEMV instantiation on
// the current device (done outside graph capture).
int prepare_gemv_kernels();
int launch_quantize_act(int act_type, const float* x, int64_t x_stride, int n_tok, int64_t k, ActQ& out,
                        cudaStream_t s);
int launch_act_to_blocks(const ActQ& a, int64_t k, void* blocks, cudaStream_t s);
int launch_block_dots(const QMatrix& w, const ActQ& a, int64_t row, int32_t* out_i, int32_t* out_m,
                      cudaStream_t s);
int launch_dequantize(const QMatrix& w, float* dst, cudaStream_t s);
// The exchange's bounded wait on its own: *status = kPeerWaitStatus when the
// flags did not all reach `target` within the wait bound.
int launch_flag_wait(const unsigned long long* flags, int n, unsigned long long target, int* status,
                     cudaStream_t s);

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
