// C ABI: device utilities, host format helpers, the GGUF tensor upload and the
// single-op entry points.  Every function is noexcept and maps failures to a
// status code with a message for b2_last_error().
#include <string.h>

#include <new>
#include <thread>
#include <vector>

#include <cuda_profiler_api.h>

#include "b2_common.cuh"
#include "b2_layers.hpp"

struct b2_qmatrix {
  b2::QMatrix m;
};

namespace b2 {
namespace {

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Stream-ordered planar activation buffer for n_tok rows of kp values.
int alloc_act(ActQ& a, int type, int n_tok, int64_t kp, cudaStream_t s) {
  a.type = type;
  a.n_tok = n_tok;
  a.kp = kp;
  const size_t nq = (size_t)n_tok * kp;
  const size_t nd = (size_t)n_tok * (type == B2_Q8_0 ? kp / 32 : kp / 256);
  const size_t nb = type == B2_Q8_K ? (size_t)n_tok * (kp / 16) : 0;
  void* base = nullptr;
  const size_t bytes = (nq + 15) / 16 * 16 + nd * 4 + nb * 2 + 64;
  B2_CUDA_TRY(cudaMallocAsync(&base, bytes, s));
  a.qs = static_cast<int8_t*>(base);
  a.d = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + (nq + 15) / 16 * 16);
  a.bsum = nb ? reinterpret_cast<int16_t*>(a.d + nd) : nullptr;
  return B2_OK;
}

void free_act(ActQ& a, cudaStream_t s) {
  if (a.qs) cudaFreeAsync(a.qs, s);
  a.qs = nullptr;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

int b2_abi_version(void) { return B2_ABI_VERSION; }
const char* b2_last_error(void) { return b2::last_error(); }

int b2_device_count(int* n) {
  B2_CHECK_ARG(n, "n");
  B2_CUDA_TRY(cudaGetDeviceCount(n));
  return B2_OK;
}
int b2_set_device(int device) {
  B2_CUDA_TRY(cudaSetDevice(device));
  return B2_OK;
}
int b2_get_device(int* device) {
  B2_CHECK_ARG(device, "device");
  B2_CUDA_TRY(cudaGetDevice(device));
  return B2_OK;
}
int b2_malloc(void** dptr, size_t bytes) {
  B2_CHECK_ARG(dptr, "dptr");
  B2_CUDA_TRY(cudaMalloc(dptr, bytes ? bytes : 1));
  return B2_OK;
}
int b2_free(void* dptr) {
  B2_CUDA_TRY(cudaFree(dptr));
  return B2_OK;
}
int b2_host_alloc(void** hptr, size_t bytes) {
  B2_CHECK_ARG(hptr, "hptr");
  B2_CUDA_TRY(cudaMallocHost(hptr, bytes ? bytes : 1));
  return B2_OK;
}
int b2_host_free(void* hptr) {
  B2_CUDA_TRY(cudaFreeHost(hptr));
  return B2_OK;
}
int b2_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  B2_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
  return B2_OK;
}
int b2_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  B2_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
  return B2_OK;
}
int b2_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  B2_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
  return B2_OK;
}
int b2_memset(void* dst, int value, size_t bytes, void* stream) {
  B2_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, as_stream(stream)));
  return B2_OK;
}
int b2_stream_create(void** stream) {
  B2_CHECK_ARG(stream, "stream");
  cudaStream_t s;
  B2_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return B2_OK;
}
int b2_stream_destroy(void* stream) {
  B2_CUDA_TRY(cudaStreamDestroy(as_stream(stream)));
  return B2_OK;
}
int b2_stream_synchronize(void* stream) {
  B2_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  return B2_OK;
}
int b2_device_synchronize(void) {
  B2_CUDA_TRY(cudaDeviceSynchronize());
  return B2_OK;
}
int b2_event_create(void** event) {
  B2_CHECK_ARG(event, "event");
  cudaEvent_t e;
  B2_CUDA_TRY(cudaEventCreate(&e));
  *event = e;
  return B2_OK;
}
int b2_event_destroy(void* event) {
  B2_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return B2_OK;
}
int b2_event_record(void* event, void* stream) {
  B2_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), as_stream(stream)));
  return B2_OK;
}
int b2_event_elapsed_ms(void* start, void* stop, float* ms) {
  B2_CHECK_ARG(ms, "ms");
  B2_CUDA_TRY(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)));
  return B2_OK;
}
int b2_graph_capture_begin(void* stream) {
  B2_CHECK_ARG(stream, "graph capture needs a created stream");
  B2_CUDA_TRY(cudaStreamBeginCapture(as_stream(stream), cudaStreamCaptureModeThreadLocal));
  return B2_OK;
}
int b2_graph_capture_end(void* stream, void** graph_exec) {
  B2_CHECK_ARG(stream && graph_exec, "graph_capture_end arguments");
  cudaGraph_t g = nullptr;
  B2_CUDA_TRY(cudaStreamEndCapture(as_stream(stream), &g));
  cudaGraphExec_t e = nullptr;
  const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  B2_CUDA_TRY(err);
  *graph_exec = e;
  return B2_OK;
}
int b2_graph_launch(void* graph_exec, void* stream) {
  B2_CUDA_TRY(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), as_stream(stream)));
  return B2_OK;
}
int b2_graph_destroy(void* graph_exec) {
  B2_CUDA_TRY(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)));
  return B2_OK;
}
int b2_profiler_range(int start) {
  B2_CUDA_TRY(start ? cudaProfilerStart() : cudaProfilerStop());
  return B2_OK;
}

int b2_set_pdl(int enabled) {
  b2::set_pdl(enabled != 0);
  return B2_OK;
}

// ---- host format helpers -------------------------------------------------------------
size_t b2_row_bytes(int type, int64_t k) { return b2::row_bytes(type, k); }

int b2_quantize_weights(int type, const float* src, int64_t n_rows, int64_t k, void* dst, int n_threads) {
  B2_CHECK_ARG(src && dst && n_rows >= 0 && k > 0, "quantize_weights arguments");
  try {
    return b2::quantize_weights(type, src, n_rows, k, dst, n_threads);
  } catch (...) {
    b2::set_error("quantize_weights: host exception");
    return B2_ERR_OOM;
  }
}

int b2_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float std_dev, float* out, int n_threads) {
  B2_CHECK_ARG(out && n >= 0, "synth_normal arguments");
  try {
    return b2::synth_normal(seed, offset, n, mean, std_dev, out, n_threads);
  } catch (...) {
    b2::set_error("synth_normal: host exception");
    return B2_ERR_OOM;
  }
}

int b2_rope_table(float theta, int head_dim, int p0, int n_pos, float* out) {
  B2_CHECK_ARG(out && head_dim > 0 && (head_dim % 2) == 0 && n_pos >= 0, "rope_table arguments");
  b2::rope_table(theta, head_dim, p0, n_pos, out);
  return B2_OK;
}

// ---- GGUF tensor upload ----------------------------------------------------------------
int b2_qmatrix_upload(int type, const void* gguf_bytes, int64_t n_rows, int64_t k, b2_qmatrix** out) {
  B2_CHECK_ARG(out && gguf_bytes && n_rows > 0 && k > 0, "qmatrix_upload arguments");
  B2_CHECK_ARG(b2::is_weight_type(type), "weight type must be Q4_0, Q8_0, Q4_K or Q6_K");
  B2_CHECK_ARG(k % b2::block_elems(type) == 0, "k must be a multiple of the block size");
  *out = nullptr;
  b2_qmatrix* h = new (std::nothrow) b2_qmatrix;
  if (!h) {
    set_error("qmatrix_upload: host allocation");
    return B2_ERR_OOM;
  }
  QMatrix& m = h->m;
  m.type = type;
  m.n_rows = n_rows;
  m.k = k;
  std::vector<const uint8_t*> rows((size_t)n_rows);
  const size_t rb = b2::row_bytes(type, k);
  for (int64_t r = 0; r < n_rows; ++r) rows[(size_t)r] = static_cast<const uint8_t*>(gguf_bytes) + (size_t)r * rb;
  const int rc = upload_tiles(m, rows.data());
  if (rc != B2_OK) {
    delete h;
    return rc;
  }
  *out = h;
  return B2_OK;
}

int b2_qmatrix_free(b2_qmatrix* h) {
  if (!h) return B2_OK;
  if (h->m.owns && h->m.data) cudaFree(h->m.data);
  delete h;
  return B2_OK;
}

int b2_qmatrix_device_bytes(const b2_qmatrix* h, int64_t* bytes) {
  B2_CHECK_ARG(h && bytes, "qmatrix_device_bytes arguments");
  *bytes = h->m.bytes();
  return B2_OK;
}

int b2_qmatrix_dequantize(const b2_qmatrix* h, float* dst, void* stream) {
  B2_CHECK_ARG(h && dst, "qmatrix_dequantize arguments");
  return launch_dequantize(h->m, dst, as_stream(stream));
}

// ---- single ops ---------------------------------------------------------------------------
int b2_quantize_act(int act_type, const float* x, int n_tok, int64_t k, void* blocks, void* stream) {
  B2_CHECK_ARG(x && blocks && n_tok > 0 && k > 0, "quantize_act arguments");
  B2_CHECK_ARG(act_type == B2_Q8_0 || act_type == B2_Q8_K, "act_type must be Q8_0 or Q8_K");
  const int64_t be = act_type == B2_Q8_0 ? 32 : 256;
  B2_CHECK_ARG(k % be == 0, "k must be a multiple of the block size");
  cudaStream_t s = as_stream(stream);
  ActQ a;
  int rc = alloc_act(a, act_type, n_tok, (k + 255) / 256 * 256, s);
  if (rc != B2_OK) return rc;
  rc = launch_quantize_act(act_type, x, k, n_tok, k, a, s);
  if (rc == B2_OK) rc = launch_act_to_blocks(a, k, blocks, s);
  free_act(a, s);
  return rc;
}

int b2_gemv_multi(const b2_qmatrix* const* w, int n_mat, const float* x, int n_tok, float* const* y, void* stream) {
  B2_CHECK_ARG(w && x && y && n_mat >= 1 && n_mat <= 64 && n_tok >= 1 && n_tok <= 2, "gemv_multi arguments");
  std::vector<const QMatrix*> ws((size_t)n_mat);
  for (int i = 0; i < n_mat; ++i) {
    B2_CHECK_ARG(w[i] && y[i], "gemv_multi: null matrix or output");
    ws[(size_t)i] = &w[i]->m;
  }
  GemvArgs a = {};
  a.w = ws[0];
  a.x = x;
  a.x_stride = w[0]->m.k;
  a.n_tok = n_tok;
  a.y = y[0];
  a.y_stride = w[0]->m.n_rows;
  a.epilogue = EPI_STORE;
  a.n_mat = n_mat;
  a.wlist = ws.data();
  a.ylist = y;
  cudaStream_t s = as_stream(stream);
  if (!gemv_needs_image(w[0]->m, n_tok)) return launch_gemv(a, s);
  B2_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&a.act_img), gemv_act_image_bytes(w[0]->m, n_tok), s));
  const int rc = launch_gemv(a, s);
  const cudaError_t e = cudaFreeAsync(a.act_img, s);
  if (rc) return rc;
  B2_CUDA_TRY(e);
  return B2_OK;
}

int b2_gemv(const b2_qmatrix* w, const float* x, int n_tok, float* y, void* stream) {
  B2_CHECK_ARG(w && x && y, "gemv arguments");
  GemvArgs a = {};
  a.w = &w->m;
  a.x = x;
  a.x_stride = w->m.k;
  a.n_tok = n_tok;
  a.y = y;
  a.y_stride = w->m.n_rows;
  a.epilogue = EPI_STORE;
  B2_CHECK_ARG(n_tok >= 1 && n_tok <= 8, "n_tok must be in [1, 8]");
  cudaStream_t s = as_stream(stream);
  // Small activations are quantized inside the GEMV: no scratch, so a
  // captured sequence of GEMVs is kernels only and keeps its programmatic
  // (PDL) edges.  Larger ones get stream-ordered scratch for the image.
  if (!gemv_needs_image(w->m, n_tok)) return launch_gemv(a, s);
  B2_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&a.act_img), gemv_act_image_bytes(w->m, n_tok), s));
  const int rc = launch_gemv(a, s);
  const cudaError_t e = cudaFreeAsync(a.act_img, s);
  if (rc) return rc;
  B2_CUDA_TRY(e);
  return B2_OK;
}

int b2_moe_route(const float* logits, int32_t n_tok, int32_t n_expert, int32_t n_used, int32_t norm_weights,
                 int32_t* ids, float* weights, void* stream) {
  return launch_moe_route(logits, n_tok, n_expert, n_used, norm_weights, ids, weights, as_stream(stream));
}

int b2_moe_gemv(const b2_qmatrix* experts, int32_t n_expert, const float* x, int32_t x_per_expert, int32_t n_tok,
                const int32_t* ids, int32_t n_used, float* y, void* stream) {
  B2_CHECK_ARG(experts && x && ids && y && n_expert >= 1 && n_tok >= 1 && n_used >= 1 && n_used <= 64,
               "moe_gemv arguments (1 <= n_used <= 64)");
  const QMatrix& st = experts->m;
  B2_CHECK_ARG(st.n_rows % n_expert == 0 && (st.n_rows / n_expert) % 8 == 0,
               "moe_gemv: the stack holds n_expert matrices of a multiple of 8 rows each");
  // expert 0 of the stack; expert e is e whole tile runs further
  QMatrix e0 = st;
  e0.n_rows = st.n_rows / n_expert;
  e0.n_tiles = e0.n_rows / 8;
  e0.owns = false;
  GemvArgs a = {};
  a.w = &e0;
  a.x_stride = st.k;
  a.n_tok = 1;
  a.y_stride = e0.n_rows;
  a.epilogue = EPI_STORE;
  a.n_mat = n_used;
  a.n_expert = n_expert;
  a.mat_stride = e0.n_tiles * e0.tile_bytes;
  a.y_mat_stride = e0.n_rows;
  cudaStream_t s = as_stream(stream);
  const bool img = gemv_needs_image(e0, 1);
  if (img) B2_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&a.act_img), gemv_act_image_bytes(e0, 1), s));
  int rc = B2_OK;
  // One launch per token over its experts; with per-expert inputs each
  // expert's CTAs quantize their own input (inputs of up to 8192 values),
  // else one launch per (token, expert).
  const bool split = x_per_expert && img;
  const int per = split ? 1 : n_used;
  if (x_per_expert && !img) a.x_mat_stride = st.k;
  a.n_mat = per;
  for (int t = 0; t < n_tok && rc == B2_OK; ++t)
    for (int j = 0; j < n_used && rc == B2_OK; j += per) {
      a.x = x + ((int64_t)t * (x_per_expert ? n_used : 1) + (x_per_expert ? j : 0)) * st.k;
      a.mat_ids = ids + (int64_t)t * n_used + j;
      a.y = y + ((int64_t)t * n_used + j) * e0.n_rows;
      rc = launch_gemv(a, s);
    }
  if (img) {
    const cudaError_t e = cudaFreeAsync(a.act_img, s);
    if (rc) return rc;
    B2_CUDA_TRY(e);
  }
  return rc;
}

int b2_moe_combine(const float* y, const float* weights, int32_t n_tok, int32_t n_used, int32_t n, float* out,
                   void* stream) {
  return launch_moe_combine(y, weights, n_tok, n_used, n, out, as_stream(stream));
}

int b2_gemm_workspace_bytes(const b2_qmatrix* w, int n_tok, size_t* bytes) {
  B2_CHECK_ARG(w && bytes && n_tok >= 1, "gemm_workspace_bytes arguments");
  *bytes = gemm_act_image_bytes(w->m, n_tok);
  return B2_OK;
}

int b2_gemm(const b2_qmatrix* w, const float* x, int n_tok, float* y, void* workspace, size_t workspace_bytes,
            int* status, void* stream) {
  B2_CHECK_ARG(w && x && y && n_tok >= 1, "gemm arguments");
  B2_CHECK_ARG(w->m.type == B2_Q4_K || w->m.type == B2_Q8_0, "b2_gemm takes Q4_K or Q8_0 weights");
  cudaStream_t s = as_stream(stream);
  const size_t need = gemm_act_image_bytes(w->m, n_tok);
  if (workspace) {
    B2_CHECK_ARG(workspace_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0,
                 "gemm workspace too small or not 16-byte aligned");
    return launch_gemm(w->m, x, w->m.k, n_tok, y, static_cast<uint8_t*>(workspace), status, s);
  }
  uint8_t* img = nullptr;
  B2_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&img), need, s));
  const int rc = launch_gemm(w->m, x, w->m.k, n_tok, y, img, status, s);
  const cudaError_t e = cudaFreeAsync(img, s);
  if (rc) return rc;
  B2_CUDA_TRY(e);
  return B2_OK;
}

namespace {
// Per-thread device staging for the host-buffer entry points, grown on demand
// and kept, so a call does no allocation once warm.
struct HostStage {
  void* dev = nullptr;
  size_t bytes = 0;
  int device = -1;
  ~HostStage() {
    if (dev) cudaFree(dev);
  }
};
thread_local HostStage g_stage;
int stage_reserve(size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (g_stage.dev && (g_stage.bytes < bytes || g_stage.device != dev)) {
    cudaFree(g_stage.dev);
    g_stage.dev = nullptr;
  }
  if (!g_stage.dev) {
    B2_CUDA_TRY(cudaMalloc(&g_stage.dev, bytes));
    g_stage.bytes = bytes;
    g_stage.device = dev;
  }
  return B2_OK;
}
}  // namespace

int b2_gemv_host(const b2_qmatrix* w, const float* x_host, int n_tok, float* y_host) {
  B2_CHECK_ARG(w && x_host && y_host && n_tok >= 1 && n_tok <= 8, "gemv_host arguments");
  const size_t xb = (size_t)n_tok * w->m.k * 4, yb = (size_t)n_tok * w->m.n_rows * 4;
  const size_t xoff = (xb + 255) / 256 * 256;
  int rc = stage_reserve(xoff + yb);
  if (rc != B2_OK) return rc;
  cudaStream_t s = 0;
  float* xd = static_cast<float*>(g_stage.dev);
  float* yd = reinterpret_cast<float*>(static_cast<uint8_t*>(g_stage.dev) + xoff);
  B2_CUDA_TRY(cudaMemcpyAsync(xd, x_host, xb, cudaMemcpyHostToDevice, s));
  rc = b2_gemv(w, xd, n_tok, yd, s);
  if (rc != B2_OK) return rc;
  B2_CUDA_TRY(cudaMemcpyAsync(y_host, yd, yb, cudaMemcpyDeviceToHost, s));
  B2_CUDA_TRY(cudaStreamSynchronize(s));
  return B2_OK;
}

int b2_gemm_host(const b2_qmatrix* w, const float* x_host, int n_tok, float* y_host) {
  B2_CHECK_ARG(w && x_host && y_host && n_tok >= 1, "gemm_host arguments");
  const size_t xb = (size_t)n_tok * w->m.k * 4, yb = (size_t)n_tok * w->m.n_rows * 4;
  const size_t xoff = (xb + 255) / 256 * 256, soff = xoff + (yb + 255) / 256 * 256;
  int rc = stage_reserve(soff + 256);
  if (rc != B2_OK) return rc;
  cudaStream_t s = 0;
  uint8_t* base = static_cast<uint8_t*>(g_stage.dev);
  float* xd = reinterpret_cast<float*>(base);
  float* yd = reinterpret_cast<float*>(base + xoff);
  int* st = reinterpret_cast<int*>(base + soff);
  B2_CUDA_TRY(cudaMemsetAsync(st, 0, sizeof(int), s));
  B2_CUDA_TRY(cudaMemcpyAsync(xd, x_host, xb, cudaMemcpyHostToDevice, s));
  rc = b2_gemm(w, xd, n_tok, yd, nullptr, 0, st, s);
  if (rc != B2_OK) return rc;
  int code = 0;
  B2_CUDA_TRY(cudaMemcpyAsync(y_host, yd, yb, cudaMemcpyDeviceToHost, s));
  B2_CUDA_TRY(cudaMemcpyAsync(&code, st, sizeof(int), cudaMemcpyDeviceToHost, s));
  B2_CUDA_TRY(cudaStreamSynchronize(s));
  return code ? B2_ERR_TIMEOUT : B2_OK;
}

int b2_block_dots(const b2_qmatrix* w, int64_t row, const float* x, int32_t* out_i, int32_t* out_m, void* stream) {
  B2_CHECK_ARG(w && x && out_i && row >= 0 && row < w->m.n_rows, "block_dots arguments");
  B2_CHECK_ARG(w->m.type != B2_Q4_K || out_m, "Q4_K needs out_m");
  cudaStream_t s = as_stream(stream);
  ActQ a;
  int rc = alloc_act(a, act_type_for(w->m.type), 1, (w->m.k + 255) / 256 * 256, s);
  if (rc != B2_OK) return rc;
  rc = launch_quantize_act(a.type, x, w->m.k, 1, w->m.k, a, s);
  if (rc == B2_OK) rc = launch_block_dots(w->m, a, row, out_i, out_m, s);
  free_act(a, s);
  return rc;
}

int b2_embed(int type, const void* table, int n_vocab, int n_embd, const int32_t* tokens, int n_tok, float* out,
             void* stream) {
  B2_CHECK_ARG(table && tokens && out && n_vocab > 0 && n_embd > 0 && n_tok > 0, "embed arguments");
  B2_CHECK_ARG(type == B2_F32 || type == B2_F16 || b2::is_weight_type(type), "embedding type");
  B2_CHECK_ARG(n_embd % b2::block_elems(type) == 0, "n_embd must be a multiple of the block size");
  return launch_embed(tokens, n_tok, n_vocab, type, static_cast<const uint8_t*>(table),
                      (int64_t)b2::row_bytes(type, n_embd), n_embd, out, as_stream(stream));
}

int b2_rmsnorm(float* x, const float* delta, const float* w, float* out, int n_rows, int n, float eps, void* stream) {
  B2_CHECK_ARG(x && w && out && n_rows > 0 && n > 0, "rmsnorm arguments");
  return launch_add_rmsnorm(x, delta, w, out, n_rows, n, eps, as_stream(stream));
}

int64_t b2_kv_row_bytes(int type, int head_dim) {
  return kv_type_ok(type) && head_dim > 0 ? kv_row_bytes(type, head_dim) : 0;
}

int b2_rope_kv_store_typed(const float* qkv, int n_tok, int n_seq, int n_head, int n_kv, int head_dim,
                           const int32_t* pos, const int32_t* seq, const float* rope, float* q_out, void* k_cache,
                           int type_k, void* v_cache, int type_v, int cap, void* stream) {
  B2_CHECK_ARG(qkv && pos && seq && rope && q_out && k_cache && v_cache && n_tok > 0 && n_seq > 0 && cap > 0,
               "rope_kv_store arguments");
  B2_CHECK_ARG(head_dim % 32 == 0 && n_head > 0 && n_kv > 0, "head shape (head_dim a multiple of 32)");
  return launch_rope_kv(qkv, n_tok, n_head, n_kv, head_dim, pos, seq, rope, q_out, k_cache, type_k, v_cache, type_v,
                        nullptr, n_seq, cap, as_stream(stream));
}

int b2_rope_kv_store(const float* qkv, int n_tok, int n_seq, int n_head, int n_kv, int head_dim, const int32_t* pos,
                     const int32_t* seq, const float* rope, float* q_out, uint16_t* k_cache, uint16_t* v_cache, int cap,
                     void* stream) {
  return b2_rope_kv_store_typed(qkv, n_tok, n_seq, n_head, n_kv, head_dim, pos, seq, rope, q_out, k_cache, B2_F16,
                                v_cache, B2_F16, cap, stream);
}

int b2_attn_decode_typed(const float* q, const void* k_cache, int type_k, const void* v_cache, int type_v,
                         const int32_t* pos, const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv,
                         int head_dim, int cap, float* out, void* stream) {
  B2_CHECK_ARG(q && k_cache && v_cache && pos && seq && out && n_q > 0 && n_seq > 0 && cap > 0,
               "attn_decode arguments");
  B2_CHECK_ARG(n_kv > 0 && n_head % n_kv == 0, "n_head must be a multiple of n_kv");
  B2_CHECK_ARG(kv_type_ok(type_k) && kv_type_ok(type_v), "KV cache types must be B2_F16, B2_Q8_0 or B2_Q4_0");
  cudaStream_t s = as_stream(stream);
  // scores, exponentials and chunk maxima (no initialisation needed)
  void* scratch = nullptr;
  B2_CUDA_TRY(cudaMallocAsync(&scratch, attn_scratch_floats(n_q, n_head, n_kv, cap) * 4, s));
  const int rc = launch_attention(q, n_q, n_head, n_kv, head_dim, pos, seq, k_cache, type_k, v_cache, type_v, nullptr,
                                  n_seq, cap, static_cast<float*>(scratch), out, s);
  cudaFreeAsync(scratch, s);
  return rc;
}

int b2_attn_decode(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                   const int32_t* seq, int n_q, int n_seq, int n_head, int n_kv, int head_dim, int cap, float* out,
                   void* stream) {
  return b2_attn_decode_typed(q, k_cache, B2_F16, v_cache, B2_F16, pos, seq, n_q, n_seq, n_head, n_kv, head_dim, cap,
                              out, stream);
}

int b2_kv_shift_k_typed(void* k_cache, int type_k, int seq, int n_kv, int head_dim, int cap, int p_begin, int p_end,
                        int delta, float theta, void* stream) {
  B2_CHECK_ARG(k_cache && seq >= 0 && p_begin >= 0 && p_end <= cap && head_dim % 32 == 0 && head_dim <= 2 * kRotPairs,
               "kv_shift_k arguments");
  B2_CHECK_ARG(kv_type_ok(type_k), "KV cache type must be B2_F16, B2_Q8_0 or B2_Q4_0");
  RotTable cs;
  rope_table(theta, head_dim, delta, 1, cs.cs);
  const KvSeqState st{0, 0};
  return launch_kv_shift(k_cache, type_k, n_kv, head_dim, seq, st, cap, p_begin, p_end, cs, as_stream(stream));
}

int b2_kv_shift_k(uint16_t* k_cache, int seq, int n_kv, int head_dim, int cap, int p_begin, int p_end, int delta,
                  float theta, void* stream) {
  return b2_kv_shift_k_typed(k_cache, B2_F16, seq, n_kv, head_dim, cap, p_begin, p_end, delta, theta, stream);
}

int b2_flag_wait(const uint64_t* flags, int n, uint64_t target, int* status, void* stream) {
  B2_CHECK_ARG(flags && status && n > 0, "flag_wait arguments");
  return launch_flag_wait(reinterpret_cast<const unsigned long long*>(flags), n, (unsigned long long)target, status,
                          as_stream(stream));
}

}  // extern "C"
