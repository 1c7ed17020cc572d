// The llama.cpp-shaped engine behind the C ABI: model load (GGUF -> repacked
// device shards), context (fp16 KV ring per sequence, step buffers), decode
// (one CUDA graph per step shape), KV shift / removal, greedy argmax, and
// tensor parallelism over NVLink peer memory.
//
// Mirrors the calls Milda and Sutra make (Milda/src/engine.cpp:703-1292,
// 1521-1548, 1642-1675, 1962-2117; Sutra/src/llm_backends.cpp:2395-2760) and
// the forward order of Singularity's forward_token
// (Singularity/src/core/cortex_a5_engine.cpp:1029-1293).
//
// Tensor parallelism (tp ranks, one process per GPU): Q/K/V and gate/up are
// split by output rows (heads / FFN features), O and down by input columns,
// the output head by vocabulary rows.  Shard boundaries fall on quantization
// block boundaries, so each rank quantizes its activation slice exactly as
// the full vector would be quantized.  The O / down partial outputs and the
// head's logit shards are exchanged without a library collective: each
// rank's GEMV stores its outputs straight into its slot of every rank's
// gather buffer (CUDA IPC mappings over NVLink) and raises a per-phase epoch
// flag; the next kernel on each rank waits for all flags and sums the slots
// in rank order, so every rank holds bit-identical activations and the
// result does not depend on timing.  NCCL is used once per context, to
// exchange the IPC handles.
#include <math.h>
#include <stdlib.h>
#include <nccl.h>
#include <string.h>

#include <memory>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "b2_gguf.hpp"
#include "b2_internal.hpp"
#include "b2_layers.hpp"
#include "b2_sampler.hpp"

namespace b2 {

int write_synthetic_llama(const b2_llama_hparams& hp, const char* path, int n_threads);

namespace {

constexpr int kStepMax = 8;          // tokens per device step (GEMV batch)
constexpr int kResWords = 32;        // ids, top-1/margin pairs, status (3*kStepMax+1, padded)

struct DevQ {
  QMatrix m;
  ~DevQ() {
    if (m.data) cudaFree(m.data);
  }
};

// Uploads rows given by pointers to their first byte (all rows k values of
// `type` starting at the slice's first column).
int upload_rows(DevQ& q, int type, int64_t k, const std::vector<const uint8_t*>& rows, UploadStager* st) {
  q.m.type = type;
  q.m.n_rows = (int64_t)rows.size();
  q.m.k = k;
  return upload_tiles(q.m, rows.data(), st);
}

struct Layer {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  DevQ wqkv, wo, wgu, wdown;
};

}  // namespace
}  // namespace b2

struct b2_model {
  int device = 0;
  int tp_rank = 0, tp_size = 1;
  ncclComm_t comm = nullptr;
  b2::GgufFile gguf;
  int n_layer = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, n_vocab = 0, head_dim = 0, n_ctx_train = 0;
  int nh_l = 0, nkv_l = 0, ff_l = 0, v_l = 0;   // per-rank shares
  float eps = 1e-5f, theta = 10000.0f;
  int wtype = 0, embd_type = 0, out_type = 0;
  std::vector<std::unique_ptr<b2::Layer>> layers;
  uint8_t* embd = nullptr;
  int64_t embd_row_bytes = 0;
  float* out_norm = nullptr;
  b2::DevQ head;
  int64_t device_bytes = 0;
  ~b2_model();
};

b2_model::~b2_model() {
  if (device >= 0) cudaSetDevice(device);
  for (auto& l : layers) {
    if (l->attn_norm) cudaFree(l->attn_norm);
    if (l->ffn_norm) cudaFree(l->ffn_norm);
  }
  layers.clear();
  if (embd) cudaFree(embd);
  if (out_norm) cudaFree(out_norm);
  if (comm) ncclCommDestroy(comm);
}

struct b2_context {
  b2_model* model = nullptr;
  int n_ctx = 0, n_seq = 0;
  cudaStream_t stream = nullptr;
  // KV ring per layer: [n_seq][nkv_l][n_ctx] rows of the cache types
  // (kv_row_bytes: fp16, or Q8_0 codes + block scales)
  std::vector<uint8_t*> kc, vc;
  int type_k = B2_F16, type_v = B2_F16;
  b2::KvSeqState* st_d = nullptr;
  std::vector<b2::KvSeqState> st;
  std::vector<int> n_past;
  float* rope = nullptr;        // [n_ctx][head_dim]
  // step inputs (device + pinned host staging)
  // [tok | pos | seq] x kStepMax in one allocation: one H2D copy per step
  int32_t *in_d = nullptr, *tok_d = nullptr, *pos_d = nullptr, *seq_d = nullptr;
  int32_t* in_h = nullptr;      // [2 slots][3][kStepMax] pinned, then res_h
  int32_t* res_h = nullptr;     // [kResWords] pinned copy of res
  cudaEvent_t in_ev[2] = {nullptr, nullptr};
  int in_slot = 0;
  // step buffers
  float *x = nullptr, *delta = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *h = nullptr;
  float *logits = nullptr, *scores = nullptr, *top = nullptr;   // scores: the attention's scratch for kStepMax queries
  uint32_t* argmax_scr = nullptr;     // vocabulary-slice partials and arrival counters of the argmax
  // [ids kStepMax | top-1, margin 2*kStepMax | status] in one allocation: one
  // D2H copy returns a step's greedy result and the device-wait status
  int32_t* res = nullptr;
  unsigned long long* wait_ns = nullptr;   // exchange waits' wall time (tensor parallelism)
  int32_t* ids = nullptr;
  int* status = nullptr;
  // device-side greedy loop: [n_ctx][kStepMax] generated ids, per-row counts
  int32_t *gen_out = nullptr, *gen_count = nullptr;
  uint8_t* act_img = nullptr;   // quantized activations of the GEMV being run
  // Prefill through the tensor-core GEMMs: chunks of up to pf_cap tokens,
  // buffers allocated at the first long enough prompt.
  bool prefill_gemm = true;
  int pf_cap = 0;
  int32_t* pf_in = nullptr;     // [tok | pos | seq] x pf_cap
  int32_t* pf_in_h = nullptr;   // pinned staging of pf_in
  cudaEvent_t pf_ev = nullptr;  // the staging's last copy
  float *pf_x = nullptr, *pf_xn = nullptr, *pf_delta = nullptr, *pf_qkv = nullptr, *pf_q = nullptr;
  float *pf_att = nullptr, *pf_gu = nullptr, *pf_h = nullptr, *pf_scores = nullptr;
  float* pf_gather = nullptr;   // [tp][cap][n_embd]: the ranks' partial projections (tensor parallelism)
  uint8_t* pf_ws = nullptr;     // GEMM activation images
  // last decode
  int last_n = 0;
  bool last_logits = false;
  // graphs per (n_tok, with_logits)
  cudaGraphExec_t graphs[b2::kStepMax + 1][2] = {};
  cudaGraphExec_t gen_graphs[b2::kStepMax + 1] = {};
  cudaGraphExec_t samp_graphs[b2::kStepMax + 1] = {};   // device loop with the sampler chain
  // sampler chain (allocated at the first sampler on this context)
  b2::SamplerDev** samp_d = nullptr;          // [kStepMax] the rows' samplers during a sampled loop
  unsigned long long* samp_keys = nullptr;   // candidate keys of the selecting CTAs
  bool use_graph = true;
  b2_abort_callback abort_cb = nullptr;
  void* abort_user = nullptr;
  b2_eval_callback eval_cb = nullptr;
  void* eval_user = nullptr;
  std::vector<void*> allocs;
  // tensor-parallel exchange (tp > 1): one IPC-exported allocation per rank
  // [parts: 2 phases x tp slots x kStepMax x n_embd][logits: tp x kStepMax x v_l]
  // [flags: 3 phases x tp][epochs: 3][done counters: 3]
  uint8_t* xbuf = nullptr;
  std::vector<uint8_t*> peer_xbuf;   // per rank (own = xbuf)
  size_t x_parts = 0, x_logits = 0, x_flags = 0, x_epoch = 0, x_done = 0;   // byte offsets
  ~b2_context();
};

// One sampler chain (llama_sampler of Milda's chain) bound to a context:
// its parameters and initial state on the host, its state on the context's
// device.
struct b2_sampler {
  b2_context* ctx = nullptr;
  b2::SamplerDev host;                 // parameters + the fresh state
  b2::SamplerDev* dev = nullptr;       // device state
  b2::SamplerDev** self = nullptr;     // device array { dev } for single-row sampling
};

b2_context::~b2_context() {
  if (model) cudaSetDevice(model->device);
  for (auto& row : graphs)
    for (auto& g : row)
      if (g) cudaGraphExecDestroy(g);
  for (auto& g : gen_graphs)
    if (g) cudaGraphExecDestroy(g);
  for (auto& g : samp_graphs)
    if (g) cudaGraphExecDestroy(g);
  for (size_t j = 0; j < peer_xbuf.size(); ++j)
    if (peer_xbuf[j] && peer_xbuf[j] != xbuf) cudaIpcCloseMemHandle(peer_xbuf[j]);
  if (xbuf) cudaFree(xbuf);
  for (void* p : allocs) cudaFree(p);
  if (in_h) cudaFreeHost(in_h);
  if (pf_in_h) cudaFreeHost(pf_in_h);
  if (pf_ev) cudaEventDestroy(pf_ev);
  for (auto& e : in_ev)
    if (e) cudaEventDestroy(e);
  if (stream) cudaStreamDestroy(stream);
}

namespace b2 {
namespace {

template <typename T>
int dalloc(b2_context* c, T** p, size_t count) {
  void* v = nullptr;
  B2_CUDA_TRY(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 16)));
  c->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return B2_OK;
}

int upload_f32(const GgufTensor* t, int64_t n, float** out) {
  std::vector<float> v((size_t)n);
  if (t->type == B2_F32) {
    memcpy(v.data(), t->data, (size_t)n * 4);
  } else if (t->type == B2_F16) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(t->data);
    for (int64_t i = 0; i < n; ++i) v[i] = host_f16_to_f32(h[i]);
  } else {
    set_error("norm tensor %s: type %d not F32/F16", t->name.c_str(), t->type);
    return B2_ERR_FORMAT;
  }
  B2_CUDA_TRY(cudaMalloc(out, (size_t)n * 4));
  B2_CUDA_TRY(cudaMemcpy(*out, v.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  return B2_OK;
}

#define B2_NCCL_TRY(expr)                                                         \
  do {                                                                            \
    ncclResult_t r_ = (expr);                                                     \
    if (r_ != ncclSuccess) {                                                      \
      ::b2::set_error("%s: %s", #expr, ncclGetErrorString(r_));                   \
      return B2_ERR_NCCL;                                                         \
    }                                                                             \
  } while (0)

int load_model(b2_model* m, const char* path, const b2_model_params* p) {
  if (p->device >= 0) B2_CUDA_TRY(cudaSetDevice(p->device));
  cudaGetDevice(&m->device);
  m->tp_rank = p->tp_rank;
  m->tp_size = p->tp_size;
  std::string err;
  if (!m->gguf.open(path, &err)) {
    set_error("model load: %s", err.c_str());
    return B2_ERR_FORMAT;
  }
  const GgufFile& g = m->gguf;
  // The forward implemented here is Llama's (adjacent-pair RoPE, no
  // projection biases).  Any other architecture, or a Llama file carrying
  // biases, would load and silently compute the wrong function: refuse it.
  {
    const std::string arch = g.get_str("general.architecture", "");
    if (arch != "llama") {
      set_error("model load: architecture '%s' unsupported (llama only)", arch.c_str());
      return B2_ERR_UNSUPPORTED;
    }
    for (const GgufTensor& t : g.tensors)
      if (t.name.size() > 5 && t.name.compare(t.name.size() - 5, 5, ".bias") == 0) {
        set_error("model load: bias tensor %s unsupported", t.name.c_str());
        return B2_ERR_UNSUPPORTED;
      }
  }
  m->n_layer = (int)g.get_int(".block_count", 0);
  m->n_embd = (int)g.get_int(".embedding_length", 0);
  m->n_ff = (int)g.get_int(".feed_forward_length", 0);
  m->n_head = (int)g.get_int(".attention.head_count", 0);
  m->n_head_kv = (int)g.get_int(".attention.head_count_kv", m->n_head);
  m->n_ctx_train = (int)g.get_int(".context_length", 0);
  m->eps = (float)g.get_float(".layer_norm_rms_epsilon", 1e-5);
  m->theta = (float)g.get_float(".rope.freq_base", 10000.0);
  const GgufTensor* te = g.tensor("token_embd.weight");
  const GgufTensor* tn = g.tensor("output_norm.weight");
  const GgufTensor* to = g.tensor("output.weight");
  if (!to) to = te;   // tied head (Singularity/src/core/cortex_a5_engine.cpp:650-654)
  if (m->n_layer <= 0 || m->n_embd <= 0 || m->n_head <= 0 || !te || !tn || m->n_embd % m->n_head) {
    set_error("model load: missing llama hyper-parameters or tensors");
    return B2_ERR_FORMAT;
  }
  m->n_vocab = (int)te->ne[1];
  m->head_dim = m->n_embd / m->n_head;
  const int tp = m->tp_size, r = m->tp_rank;
  if (tp < 1 || r < 0 || r >= tp || m->n_head % tp || m->n_head_kv % tp || m->n_ff % tp || m->n_vocab % tp ||
      (int)to->ne[1] != m->n_vocab) {
    set_error("model load: heads / ffn / vocab not divisible by tp=%d", tp);
    return B2_ERR_UNSUPPORTED;
  }
  if (m->head_dim != 64 && m->head_dim != 128) {
    set_error("model load: head_dim %d unsupported (64 or 128)", m->head_dim);
    return B2_ERR_UNSUPPORTED;
  }
  m->nh_l = m->n_head / tp;
  m->nkv_l = m->n_head_kv / tp;
  m->ff_l = m->n_ff / tp;
  m->v_l = m->n_vocab / tp;
  const int hd = m->head_dim, d = m->n_embd;
  if (tp > 1) {
    if (!p->nccl_id) {
      set_error("model load: tp_size > 1 needs an NCCL unique id");
      return B2_ERR_INVALID;
    }
    ncclUniqueId id;
    memcpy(&id, p->nccl_id, sizeof id);
    // NCCL only carries the IPC-handle exchange here: no NVLink multicast
    // (NVLS) objects are wanted, unless the user asked for them.
    setenv("NCCL_NVLS_ENABLE", "0", 0);
    B2_NCCL_TRY(ncclCommInitRank(&m->comm, tp, id, r));
  }
  // Embedding table (replicated, GGUF bytes as-is) and output norm.
  m->embd_type = te->type;
  m->embd_row_bytes = (int64_t)row_bytes(te->type, d);
  B2_CUDA_TRY(cudaMalloc(&m->embd, te->bytes));
  B2_CUDA_TRY(cudaMemcpy(m->embd, te->data, te->bytes, cudaMemcpyHostToDevice));
  m->device_bytes += (int64_t)te->bytes;
  int rc = upload_f32(tn, d, &m->out_norm);
  if (rc) return rc;
  // One pinned double-buffered stager for every weight matrix: repacking on
  // the host overlaps the copies of the previous slab.
  UploadStager stager;
  // Output head: vocabulary rows [r*v_l, (r+1)*v_l).
  m->out_type = to->type;
  if (!is_weight_type(to->type)) {
    set_error("model load: output head type %d unsupported", to->type);
    return B2_ERR_UNSUPPORTED;
  }
  {
    std::vector<const uint8_t*> rows;
    const size_t rb = row_bytes(to->type, d);
    for (int64_t i = 0; i < m->v_l; ++i) rows.push_back(to->data + (size_t)(r * (int64_t)m->v_l + i) * rb);
    if ((rc = upload_rows(m->head, to->type, d, rows, &stager))) return rc;
  }
  for (int l = 0; l < m->n_layer; ++l) {
    auto L = std::make_unique<Layer>();
    const std::string b = "blk." + std::to_string(l) + ".";
    auto T = [&](const char* n) { return g.tensor(b + n); };
    const GgufTensor *an = T("attn_norm.weight"), *fn = T("ffn_norm.weight"), *wq = T("attn_q.weight"),
                     *wk = T("attn_k.weight"), *wv = T("attn_v.weight"), *wo = T("attn_output.weight"),
                     *wg = T("ffn_gate.weight"), *wu = T("ffn_up.weight"), *wd = T("ffn_down.weight");
    if (!an || !fn || !wq || !wk || !wv || !wo || !wg || !wu || !wd) {
      set_error("model load: layer %d tensors missing", l);
      return B2_ERR_FORMAT;
    }
    if (wq->type != wk->type || wq->type != wv->type || wg->type != wu->type) {
      set_error("model load: layer %d mixes quantization types within fused projections", l);
      return B2_ERR_UNSUPPORTED;
    }
    if (l == 0) m->wtype = wq->type;
    if ((rc = upload_f32(an, d, &L->attn_norm)) || (rc = upload_f32(fn, d, &L->ffn_norm))) return rc;
    // Q/K/V rows of this rank's heads, concatenated.
    {
      std::vector<const uint8_t*> rows;
      const size_t rb = row_bytes(wq->type, d);
      for (int64_t i = 0; i < (int64_t)m->nh_l * hd; ++i) rows.push_back(wq->data + ((int64_t)r * m->nh_l * hd + i) * rb);
      for (int64_t i = 0; i < (int64_t)m->nkv_l * hd; ++i) rows.push_back(wk->data + ((int64_t)r * m->nkv_l * hd + i) * rb);
      for (int64_t i = 0; i < (int64_t)m->nkv_l * hd; ++i) rows.push_back(wv->data + ((int64_t)r * m->nkv_l * hd + i) * rb);
      if ((rc = upload_rows(L->wqkv, wq->type, d, rows, &stager))) return rc;
    }
    // O: all rows, input columns of this rank's heads.
    {
      const int64_t k_all = (int64_t)m->n_head * hd, k_l = (int64_t)m->nh_l * hd;
      if (k_l % block_elems(wo->type)) {
        set_error("model load: attention-out shard not block aligned");
        return B2_ERR_UNSUPPORTED;
      }
      std::vector<const uint8_t*> rows;
      const size_t rb = row_bytes(wo->type, k_all), off = row_bytes(wo->type, r * k_l);
      for (int64_t i = 0; i < d; ++i) rows.push_back(wo->data + i * rb + off);
      if ((rc = upload_rows(L->wo, wo->type, k_l, rows, &stager))) return rc;
    }
    // gate/up interleaved (gate_i, up_i) for this rank's FFN features.
    {
      std::vector<const uint8_t*> rows;
      const size_t rb = row_bytes(wg->type, d);
      for (int64_t i = 0; i < m->ff_l; ++i) {
        rows.push_back(wg->data + ((int64_t)r * m->ff_l + i) * rb);
        rows.push_back(wu->data + ((int64_t)r * m->ff_l + i) * rb);
      }
      if ((rc = upload_rows(L->wgu, wg->type, d, rows, &stager))) return rc;
    }
    // down: all rows, input columns of this rank's FFN features.
    {
      if (m->ff_l % block_elems(wd->type)) {
        set_error("model load: ffn-down shard not block aligned");
        return B2_ERR_UNSUPPORTED;
      }
      std::vector<const uint8_t*> rows;
      const size_t rb = row_bytes(wd->type, m->n_ff), off = row_bytes(wd->type, (int64_t)r * m->ff_l);
      for (int64_t i = 0; i < d; ++i) rows.push_back(wd->data + i * rb + off);
      if ((rc = upload_rows(L->wdown, wd->type, m->ff_l, rows, &stager))) return rc;
    }
    for (const DevQ* q : {&L->wqkv, &L->wo, &L->wgu, &L->wdown}) m->device_bytes += q->m.bytes();
    m->device_bytes += 2 * d * 4;
    m->layers.push_back(std::move(L));
  }
  m->device_bytes += m->head.m.bytes();
  const int frc = stager.finish();   // every upload has landed
  if (frc == B2_OK && !p->keep_page_cache) m->gguf.release_pages();
  return frc;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Collective over the model's ranks (every rank creates its contexts in the
// same order): allocates the exchange buffer, exports it, gathers every
// rank's IPC handle through NCCL and maps the peers' buffers.
int setup_exchange(b2_context* c) {
  b2_model* m = c->model;
  const int tp = m->tp_size, r = m->tp_rank;
  if (tp > kMaxTp) {
    set_error("context: tensor parallelism over %d ranks, at most %d", tp, kMaxTp);
    return B2_ERR_UNSUPPORTED;
  }
  c->x_parts = 0;
  c->x_logits = align256(c->x_parts + (size_t)2 * tp * kStepMax * m->n_embd * 4);
  c->x_flags = align256(c->x_logits + (size_t)tp * kStepMax * m->v_l * 4);
  c->x_epoch = align256(c->x_flags + (size_t)3 * tp * 8);
  c->x_done = align256(c->x_epoch + 3 * 8);
  const size_t bytes = align256(c->x_done + 3 * 4);
  B2_CUDA_TRY(cudaMalloc(&c->xbuf, bytes));
  B2_CUDA_TRY(cudaMemset(c->xbuf, 0, bytes));
  cudaIpcMemHandle_t h;
  B2_CUDA_TRY(cudaIpcGetMemHandle(&h, c->xbuf));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  uint8_t* dh = nullptr;
  B2_CUDA_TRY(cudaMalloc(&dh, (size_t)tp * 64));
  std::vector<cudaIpcMemHandle_t> all(tp);
  int rc = B2_OK;
  {
    cudaError_t e = cudaMemcpyAsync(dh + (size_t)r * 64, &h, 64, cudaMemcpyHostToDevice, c->stream);
    ncclResult_t nr = e == cudaSuccess ? ncclAllGather(dh + (size_t)r * 64, dh, 64, ncclChar, m->comm, c->stream)
                                       : ncclSuccess;
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaMemcpyAsync(all.data(), dh, (size_t)tp * 64,
                                                                    cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(dh);
    if (nr != ncclSuccess) {
      set_error("context: IPC handle exchange: %s", ncclGetErrorString(nr));
      return B2_ERR_NCCL;
    }
    B2_CUDA_TRY(e);
  }
  c->logits = reinterpret_cast<float*>(c->xbuf + c->x_logits);   // [tp][n][v_l], filled by the ranks' heads
  c->peer_xbuf.assign(tp, nullptr);
  for (int j = 0; j < tp; ++j) {
    if (j == r) {
      c->peer_xbuf[j] = c->xbuf;
      continue;
    }
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, all[j], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      set_error("context: mapping rank %d's exchange buffer: %s (needs peer access between the GPUs)", j,
                cudaGetErrorString(e));
      rc = B2_ERR_CUDA;
      break;
    }
    c->peer_xbuf[j] = static_cast<uint8_t*>(p);
  }
  return rc;
}

// Exchange descriptors of one phase (0 attention-out, 1 FFN-down, 2 head
// logits of an n-token step).
PeerOut peer_out(const b2_context* c, int phase, int n) {
  const b2_model* m = c->model;
  const int tp = m->tp_size, r = m->tp_rank;
  PeerOut o;
  o.n = tp;
  for (int j = 0; j < tp; ++j) {
    uint8_t* base = c->peer_xbuf[j];
    if (phase < 2)
      o.dst[j] = reinterpret_cast<float*>(base + c->x_parts) + ((size_t)phase * tp + r) * kStepMax * m->n_embd;
    else
      o.dst[j] = reinterpret_cast<float*>(base + c->x_logits) + (size_t)r * n * m->v_l;
    o.flag[j] = reinterpret_cast<unsigned long long*>(base + c->x_flags) + (size_t)phase * tp + r;
  }
  o.done = reinterpret_cast<unsigned int*>(c->xbuf + c->x_done) + phase;
  o.epoch = reinterpret_cast<unsigned long long*>(c->xbuf + c->x_epoch) + phase;
  return o;
}

PeerIn peer_in(const b2_context* c, int phase) {
  const b2_model* m = c->model;
  const int tp = m->tp_size;
  PeerIn in;
  in.n = tp;
  in.parts = reinterpret_cast<const float*>(c->xbuf + c->x_parts) + (size_t)phase * tp * kStepMax * m->n_embd;
  in.slot = (int64_t)kStepMax * m->n_embd;
  in.flags = reinterpret_cast<const unsigned long long*>(c->xbuf + c->x_flags) + (size_t)phase * tp;
  in.epoch = reinterpret_cast<const unsigned long long*>(c->xbuf + c->x_epoch) + phase;
  in.wait_ns = c->wait_ns;
  return in;
}

int create_context(b2_context* c, b2_model* m, const b2_context_params* p) {
  B2_CUDA_TRY(cudaSetDevice(m->device));
  c->model = m;
  c->n_ctx = p->n_ctx;
  c->n_seq = p->n_seq_max;
  c->use_graph = p->use_graph != 0;
  c->prefill_gemm = p->prefill_gemm != 0;
  B2_CUDA_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  const int hd = m->head_dim, d = m->n_embd;
  c->type_k = p->type_k;
  c->type_v = p->type_v;
  const size_t rows = (size_t)c->n_seq * m->nkv_l * c->n_ctx;
  const size_t kb = rows * kv_row_bytes(c->type_k, hd), vb = rows * kv_row_bytes(c->type_v, hd);
  c->kc.resize(m->n_layer);
  c->vc.resize(m->n_layer);
  int rc;
  for (int l = 0; l < m->n_layer; ++l) {
    if ((rc = dalloc(c, &c->kc[l], kb)) || (rc = dalloc(c, &c->vc[l], vb))) return rc;
    B2_CUDA_TRY(cudaMemset(c->kc[l], 0, kb));
    B2_CUDA_TRY(cudaMemset(c->vc[l], 0, vb));
  }
  c->st.assign(c->n_seq, KvSeqState{0, 0});
  c->n_past.assign(c->n_seq, 0);
  if ((rc = dalloc(c, &c->st_d, c->n_seq))) return rc;
  B2_CUDA_TRY(cudaMemcpy(c->st_d, c->st.data(), c->n_seq * sizeof(KvSeqState), cudaMemcpyHostToDevice));
  std::vector<float> rope((size_t)c->n_ctx * hd);
  rope_table(m->theta, hd, 0, c->n_ctx, rope.data());
  if ((rc = dalloc(c, &c->rope, rope.size()))) return rc;
  B2_CUDA_TRY(cudaMemcpy(c->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice));
  if ((rc = dalloc(c, &c->in_d, 3 * kStepMax))) return rc;
  c->tok_d = c->in_d;
  c->pos_d = c->in_d + kStepMax;
  c->seq_d = c->in_d + 2 * kStepMax;
  B2_CUDA_TRY(cudaMallocHost(&c->in_h, (2 * 3 * kStepMax + kResWords) * sizeof(int32_t)));
  c->res_h = c->in_h + 2 * 3 * kStepMax;
  for (auto& e : c->in_ev) B2_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  if ((rc = prepare_gemv_kernels())) return rc;
  const int T = kStepMax;
  if ((rc = dalloc(c, &c->x, (size_t)T * d)) || (rc = dalloc(c, &c->delta, (size_t)T * d)) ||
      (rc = dalloc(c, &c->xn, (size_t)T * d)) ||
      (rc = dalloc(c, &c->qkv, (size_t)T * (m->nh_l + 2 * m->nkv_l) * hd)) ||
      (rc = dalloc(c, &c->q, (size_t)T * m->nh_l * hd)) || (rc = dalloc(c, &c->att, (size_t)T * m->nh_l * hd)) ||
      (rc = dalloc(c, &c->h, (size_t)T * m->ff_l)) ||
      (m->tp_size == 1 && (rc = dalloc(c, &c->logits, (size_t)T * m->n_vocab))) ||
      (rc = dalloc(c, &c->scores, attn_scratch_floats(T, m->nh_l, m->nkv_l, c->n_ctx))) || (rc = dalloc(c, &c->res, kResWords)) ||
      (rc = dalloc(c, &c->gen_out, (size_t)c->n_ctx * T)) || (rc = dalloc(c, &c->gen_count, T)))
    return rc;
  {
    size_t img = gemv_act_image_bytes(m->head.m, T);
    const Layer& L0 = *m->layers[0];
    for (const DevQ* q : {&L0.wqkv, &L0.wo, &L0.wgu, &L0.wdown})
      for (int n = 1; n <= T; ++n) img = std::max(img, gemv_act_image_bytes(q->m, n));
    if ((rc = dalloc(c, &c->act_img, img))) return rc;
  }
  static_assert(kStepMax <= kArgmaxTok, "argmax scratch sized for the step");
  if ((rc = dalloc(c, &c->argmax_scr, argmax_scratch_words()))) return rc;
  B2_CUDA_TRY(cudaMemset(c->argmax_scr, 0, argmax_scratch_words() * sizeof(uint32_t)));
  c->ids = c->res;
  c->top = reinterpret_cast<float*>(c->res + kStepMax);
  c->status = c->res + 3 * kStepMax;
  B2_CUDA_TRY(cudaMemset(c->res, 0, kResWords * 4));
  if (m->tp_size > 1) {
    if ((rc = dalloc(c, &c->wait_ns, 1))) return rc;
    B2_CUDA_TRY(cudaMemset(c->wait_ns, 0, sizeof(unsigned long long)));
    return setup_exchange(c);
  }
  return B2_OK;
}

// One device step over n tokens already staged in tok_d/pos_d/seq_d.  With
// `feed`, the step ends by writing its argmax ids back as the next tokens.
int enqueue_step(b2_context* c, int n, bool with_logits, bool feed = false, bool sampled = false) {
  b2_model* m = c->model;
  cudaStream_t s = c->stream;
  const int d = m->n_embd, hd = m->head_dim;
  int rc = launch_embed(c->tok_d, n, m->n_vocab, m->embd_type, m->embd, m->embd_row_bytes, d, c->x, s);
  if (rc) return rc;
  const bool tp = m->tp_size > 1;
  PeerOut out_o, out_down, out_head;
  PeerIn in_o, in_down, in_head;
  if (tp) {
    out_o = peer_out(c, 0, n);
    out_down = peer_out(c, 1, n);
    out_head = peer_out(c, 2, n);
    in_o = peer_in(c, 0);
    in_down = peer_in(c, 1);
    in_head = peer_in(c, 2);
  }
  auto gemv = [&](const DevQ& w, const float* x, int64_t xs, float* y, int64_t ys, int epi,
                  const PeerOut* peer = nullptr) {
    GemvArgs a = {};
    a.w = &w.m;
    a.x = x;
    a.x_stride = xs;
    a.n_tok = n;
    a.y = y;
    a.y_stride = ys;
    a.epilogue = epi;
    a.status = c->status;
    a.act_img = c->act_img;
    a.peer = peer;
    return launch_gemv(a, s);
  };
  // cb_eval-style tap (eager steps only).
  auto tap = [&](const char* name, int layer, const float* p, int64_t count) -> int {
    if (!c->eval_cb) return B2_OK;
    B2_CUDA_TRY(cudaStreamSynchronize(s));
    c->eval_cb(name, layer, p, count, c->eval_user);
    return B2_OK;
  };
  if ((rc = tap("embed", -1, c->x, (int64_t)n * d))) return rc;
  // Fused form (no evaluation taps): each RMSNorm writes the next GEMV's
  // quantized activation image, and the QKV GEMV's epilogue applies RoPE and
  // stores K/V into the cache.  Same operations, fewer launches.
  const bool fuse = !c->eval_cb && add_rmsnorm_q_supported(d, m->layers[0]->wqkv.m.type);
  // Residual add + RMSNorm, then the GEMV over its output (fused or not).
  auto norm_gemv = [&](const float* delta, const float* nw, const PeerIn* in, const DevQ& w, float* y, int64_t ys,
                       int epi, const RopeKvEpi* rk) -> int {
    GemvArgs a = {};
    a.w = &w.m;
    a.x = c->xn;
    a.x_stride = d;
    a.n_tok = n;
    a.y = y;
    a.y_stride = ys;
    a.epilogue = epi;
    a.status = c->status;
    a.act_img = c->act_img;
    a.rope = rk;
    int r;
    if (fuse) {
      const ActImage im = gemv_act_image(w.m, n, c->act_img);
      if ((r = launch_add_rmsnorm_q(c->x, delta, nw, nullptr, n, d, m->eps, im, s, in, c->status))) return r;
      a.image_ready = true;
    } else if ((r = launch_add_rmsnorm(c->x, delta, nw, c->xn, n, d, m->eps, s, in, c->status))) {
      return r;
    }
    return launch_gemv(a, s);
  };
  const int qkv_w = (m->nh_l + 2 * m->nkv_l) * hd;
  // The QKV GEMV's RoPE epilogue stores fp16 K/V; a Q8_0 cache is written by
  // the RoPE + store kernel, which quantizes each 32-value block.
  const bool f16_kv = c->type_k == B2_F16 && c->type_v == B2_F16;
  for (int l = 0; l < m->n_layer; ++l) {
    Layer& L = *m->layers[l];
    if (fuse && !f16_kv) {
      if ((rc = norm_gemv(l ? c->delta : nullptr, L.attn_norm, tp && l ? &in_down : nullptr, L.wqkv, c->qkv, qkv_w,
                          EPI_STORE, nullptr)) ||
          (rc = launch_rope_kv(c->qkv, n, m->nh_l, m->nkv_l, hd, c->pos_d, c->seq_d, c->rope, c->q, c->kc[l],
                               c->type_k, c->vc[l], c->type_v, c->st_d, c->n_seq, c->n_ctx, s)))
        return rc;
    } else if (fuse) {
      RopeKvEpi rk;
      rk.pos = c->pos_d;
      rk.seq = c->seq_d;
      rk.rope = c->rope;
      rk.q_out = c->q;
      rk.kc = reinterpret_cast<uint16_t*>(c->kc[l]);
      rk.vc = reinterpret_cast<uint16_t*>(c->vc[l]);
      rk.st = c->st_d;
      rk.n_head = m->nh_l;
      rk.n_kv = m->nkv_l;
      rk.hd = hd;
      rk.n_seq = c->n_seq;
      rk.cap = c->n_ctx;
      if ((rc = norm_gemv(l ? c->delta : nullptr, L.attn_norm, tp && l ? &in_down : nullptr, L.wqkv, nullptr, 0,
                          EPI_ROPE_KV, &rk)))
        return rc;
    } else {
      if ((rc = launch_add_rmsnorm(c->x, l ? c->delta : nullptr, L.attn_norm, c->xn, n, d, m->eps, s,
                                   tp && l ? &in_down : nullptr, c->status)))
        return rc;
      if ((rc = tap("attn_norm", l, c->xn, (int64_t)n * d))) return rc;
      if ((rc = gemv(L.wqkv, c->xn, d, c->qkv, qkv_w, EPI_STORE))) return rc;
      if ((rc = tap("qkv", l, c->qkv, (int64_t)n * qkv_w))) return rc;
      if ((rc = launch_rope_kv(c->qkv, n, m->nh_l, m->nkv_l, hd, c->pos_d, c->seq_d, c->rope, c->q, c->kc[l],
                               c->type_k, c->vc[l], c->type_v, c->st_d, c->n_seq, c->n_ctx, s)))
        return rc;
      if ((rc = tap("q_rope", l, c->q, (int64_t)n * m->nh_l * hd))) return rc;
    }
    if ((rc = launch_attention(c->q, n, m->nh_l, m->nkv_l, hd, c->pos_d, c->seq_d, c->kc[l], c->type_k, c->vc[l],
                               c->type_v, c->st_d, c->n_seq, c->n_ctx, c->scores, c->att, s, c->status)))
      return rc;
    if ((rc = tap("attn_out", l, c->att, (int64_t)n * m->nh_l * hd))) return rc;
    {
      GemvArgs a = {};
      a.w = &L.wo.m;
      a.x = c->att;
      a.x_stride = (int64_t)m->nh_l * hd;
      a.n_tok = n;
      a.y = c->delta;
      a.y_stride = d;
      a.epilogue = EPI_STORE;
      a.status = c->status;
      a.act_img = c->act_img;
      a.peer = tp ? &out_o : nullptr;
      if ((rc = launch_gemv(a, s))) return rc;
    }
    if (!tp && (rc = tap("attn_proj", l, c->delta, (int64_t)n * d))) return rc;
    if (fuse) {
      if ((rc = norm_gemv(c->delta, L.ffn_norm, tp ? &in_o : nullptr, L.wgu, c->h, m->ff_l, EPI_SWIGLU, nullptr)))
        return rc;
    } else {
      if ((rc = launch_add_rmsnorm(c->x, c->delta, L.ffn_norm, c->xn, n, d, m->eps, s, tp ? &in_o : nullptr,
                                   c->status)))
        return rc;
      if ((rc = tap("ffn_norm", l, c->xn, (int64_t)n * d))) return rc;
      if ((rc = gemv(L.wgu, c->xn, d, c->h, m->ff_l, EPI_SWIGLU))) return rc;
    }
    if ((rc = tap("ffn_act", l, c->h, (int64_t)n * m->ff_l))) return rc;
    if ((rc = gemv(L.wdown, c->h, m->ff_l, c->delta, d, EPI_STORE, tp ? &out_down : nullptr))) return rc;
    if (!tp && (rc = tap("ffn_out", l, c->delta, (int64_t)n * d))) return rc;
  }
  if (fuse && with_logits) {
    // the head GEMV reads the image; its rows of x are still completed in place
    GemvArgs a = {};
    a.w = &m->head.m;
    a.n_tok = n;
    a.y = c->logits;
    a.y_stride = m->v_l;
    a.epilogue = EPI_STORE;
    a.status = c->status;
    a.act_img = c->act_img;
    a.peer = tp ? &out_head : nullptr;
    a.image_ready = true;
    const ActImage im = gemv_act_image(m->head.m, n, c->act_img);
    if ((rc = launch_add_rmsnorm_q(c->x, c->delta, m->out_norm, c->xn, n, d, m->eps, im, s,
                                   tp ? &in_down : nullptr, c->status)))
      return rc;
    if ((rc = launch_gemv(a, s))) return rc;
  } else {
    if ((rc = launch_add_rmsnorm(c->x, c->delta, m->out_norm, c->xn, n, d, m->eps, s, tp ? &in_down : nullptr,
                                 c->status)))
      return rc;
    if ((rc = tap("result_norm", -1, c->xn, (int64_t)n * d))) return rc;
    if (!with_logits) return B2_OK;
    if ((rc = gemv(m->head, c->xn, d, c->logits, m->v_l, EPI_STORE, tp ? &out_head : nullptr))) return rc;
  }
  GreedyFeed f;
  if (feed) {
    f.tok = c->tok_d;
    f.pos = c->pos_d;
    f.out = c->gen_out;
    f.count = c->gen_count;
    f.cap = c->n_ctx;
  }
  if (!sampled)
    return launch_argmax(c->logits, n, m->n_vocab, m->v_l, c->ids, c->top, s, f, tp ? &in_head : nullptr, c->status,
                         c->argmax_scr);
  // the argmax (which also waits for the ranks' head shards), then the
  // rows' sampler chains, which feed the next step
  if ((rc = launch_argmax(c->logits, n, m->n_vocab, m->v_l, c->ids, c->top, s, GreedyFeed{}, tp ? &in_head : nullptr,
                          c->status, c->argmax_scr)))
    return rc;
  return launch_sample(c->logits, n, 0, n, m->n_vocab, m->v_l, c->samp_d, c->ids, f, c->samp_keys, s);
}

int run_step(b2_context* c, int n, bool with_logits, bool feed = false, bool sampled = false) {
  if (!c->use_graph || c->eval_cb) return enqueue_step(c, n, with_logits, feed, sampled);
  cudaGraphExec_t& g = sampled ? c->samp_graphs[n] : feed ? c->gen_graphs[n] : c->graphs[n][with_logits ? 1 : 0];
  if (!g) {
    B2_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(c, n, with_logits, feed, sampled);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    B2_CUDA_TRY(e);
    const cudaError_t ei = cudaGraphInstantiate(&g, graph, 0);
    cudaGraphDestroy(graph);
    B2_CUDA_TRY(ei);
  }
  B2_CUDA_TRY(cudaGraphLaunch(g, c->stream));
  return B2_OK;
}

int check_status(b2_context* c) {
  int st = 0;
  B2_CUDA_TRY(cudaMemcpyAsync(&st, c->status, 4, cudaMemcpyDeviceToHost, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (st != 0) {
    cudaMemsetAsync(c->status, 0, 4, c->stream);
    set_error("device wait timed out (status %d)", st);
    return B2_ERR_TIMEOUT;
  }
  return B2_OK;
}

// ---- prefill through the tensor-core GEMMs ------------------------------------------------
// A long prompt's tokens (all but the last kStepMax of a b2_decode call) go
// through the layers in chunks of up to pf_cap tokens: every projection is
// one tensor-core GEMM over the chunk (Q4_K or Q8_0 weights, the reference's
// row order), RoPE + KV store, the split-K attention and SwiGLU run as in the
// unfused decode step.  Only the KV cache leaves a chunk: the tokens that
// need logits take the decode step afterwards.
constexpr int kPrefillMin = 64;              // tokens worth a GEMM pass
constexpr int kPrefillCapMax = 512;
constexpr size_t kPrefillBudget = (size_t)384 << 20;

bool gemm_type(int t) { return t == B2_Q4_K || t == B2_Q8_0; }

bool prefill_eligible(const b2_context* c) {
  const b2_model* m = c->model;
  if (!c->prefill_gemm || c->eval_cb) return false;
  for (const auto& L : m->layers)
    if (!gemm_type(L->wqkv.m.type) || !gemm_type(L->wo.m.type) || !gemm_type(L->wgu.m.type) ||
        !gemm_type(L->wdown.m.type))
      return false;
  return true;
}

int prefill_alloc(b2_context* c) {
  if (c->pf_cap) return B2_OK;
  b2_model* m = c->model;
  const int d = m->n_embd, hd = m->head_dim, qkv_w = (m->nh_l + 2 * m->nkv_l) * hd, nq = m->nh_l * hd;
  const size_t per_tok = 4 * ((size_t)3 * d + qkv_w + 2 * (size_t)nq + 3 * (size_t)m->ff_l +
                              attn_scratch_floats(1, m->nh_l, m->nkv_l, c->n_ctx) + 3);
  const int cap = (int)std::max<size_t>(kPrefillMin, std::min<size_t>(kPrefillCapMax, kPrefillBudget / per_tok));
  size_t ws = 0;
  for (const auto& L : m->layers)
    for (const DevQ* q : {&L->wqkv, &L->wo, &L->wgu, &L->wdown}) ws = std::max(ws, gemm_act_image_bytes(q->m, cap));
  const size_t n_before = c->allocs.size();
  int rc;
  if ((rc = dalloc(c, &c->pf_in, (size_t)3 * cap)) || (rc = dalloc(c, &c->pf_x, (size_t)cap * d)) ||
      (rc = dalloc(c, &c->pf_xn, (size_t)cap * d)) || (rc = dalloc(c, &c->pf_delta, (size_t)cap * d)) ||
      (rc = dalloc(c, &c->pf_qkv, (size_t)cap * qkv_w)) || (rc = dalloc(c, &c->pf_q, (size_t)cap * nq)) ||
      (rc = dalloc(c, &c->pf_att, (size_t)cap * nq)) || (rc = dalloc(c, &c->pf_gu, (size_t)cap * 2 * m->ff_l)) ||
      (rc = dalloc(c, &c->pf_h, (size_t)cap * m->ff_l)) ||
      (rc = dalloc(c, &c->pf_scores, attn_scratch_floats(cap, m->nh_l, m->nkv_l, c->n_ctx))) ||
      (rc = dalloc(c, &c->pf_ws, ws)) ||
      (m->tp_size > 1 && (rc = dalloc(c, &c->pf_gather, (size_t)m->tp_size * cap * d)))) {
    // A context short of memory keeps none of the chunk buffers: free the
    // ones this call took (nothing has been enqueued on them).
    for (size_t i = n_before; i < c->allocs.size(); ++i) cudaFree(c->allocs[i]);
    c->allocs.resize(n_before);
    c->pf_in = nullptr;
    c->pf_x = c->pf_xn = c->pf_delta = c->pf_qkv = c->pf_q = c->pf_att = c->pf_gu = c->pf_h = nullptr;
    c->pf_scores = nullptr;
    c->pf_ws = nullptr;
    c->pf_gather = nullptr;
    return rc;
  }
  B2_CUDA_TRY(cudaMallocHost(&c->pf_in_h, (size_t)3 * cap * sizeof(int32_t)));
  B2_CUDA_TRY(cudaEventCreateWithFlags(&c->pf_ev, cudaEventDisableTiming));
  c->pf_cap = cap;
  return B2_OK;
}

// Under tensor parallelism the attention-out and FFN-down GEMMs of a chunk
// give each rank a partial over its input columns: the ranks gather all
// partials (NCCL all-gather) and each sums them in rank order, the order of
// the decode step's exchange.
int prefill_reduce(b2_context* c, int nt) {
  b2_model* m = c->model;
  if (m->tp_size == 1) return B2_OK;
  const size_t n = (size_t)nt * m->n_embd;
  B2_NCCL_TRY(ncclAllGather(c->pf_delta, c->pf_gather, n, ncclFloat, m->comm, c->stream));
  return launch_rank_sum(c->pf_gather, m->tp_size, (int64_t)n, c->pf_delta, c->stream);
}

// One chunk of nt tokens staged in pf_in: the layers up to the KV cache.
int enqueue_prefill_chunk(b2_context* c, int nt) {
  b2_model* m = c->model;
  cudaStream_t s = c->stream;
  const int d = m->n_embd, hd = m->head_dim, nq = m->nh_l * hd;
  const int32_t *tok = c->pf_in, *pos = c->pf_in + c->pf_cap, *seq = c->pf_in + 2 * c->pf_cap;
  int rc = launch_embed(tok, nt, m->n_vocab, m->embd_type, m->embd, m->embd_row_bytes, d, c->pf_x, s);
  for (int l = 0; l < m->n_layer && rc == B2_OK; ++l) {
    const Layer& L = *m->layers[l];
    if ((rc = launch_add_rmsnorm(c->pf_x, l ? c->pf_delta : nullptr, L.attn_norm, c->pf_xn, nt, d, m->eps, s,
                                 nullptr, c->status)) ||
        (rc = launch_gemm(L.wqkv.m, c->pf_xn, d, nt, c->pf_qkv, c->pf_ws, c->status, s)) ||
        (rc = launch_rope_kv(c->pf_qkv, nt, m->nh_l, m->nkv_l, hd, pos, seq, c->rope, c->pf_q, c->kc[l], c->type_k,
                             c->vc[l], c->type_v, c->st_d, c->n_seq, c->n_ctx, s)) ||
        (rc = launch_attention(c->pf_q, nt, m->nh_l, m->nkv_l, hd, pos, seq, c->kc[l], c->type_k, c->vc[l],
                               c->type_v, c->st_d, c->n_seq, c->n_ctx, c->pf_scores, c->pf_att, s, c->status)) ||
        (rc = launch_gemm(L.wo.m, c->pf_att, nq, nt, c->pf_delta, c->pf_ws, c->status, s)) ||
        (rc = prefill_reduce(c, nt)) ||
        (rc = launch_add_rmsnorm(c->pf_x, c->pf_delta, L.ffn_norm, c->pf_xn, nt, d, m->eps, s, nullptr,
                                 c->status)) ||
        (rc = launch_gemm(L.wgu.m, c->pf_xn, d, nt, c->pf_gu, c->pf_ws, c->status, s)) ||
        (rc = launch_swiglu_pairs(c->pf_gu, nt, m->ff_l, c->pf_h, s)) ||
        (rc = launch_gemm(L.wdown.m, c->pf_h, m->ff_l, nt, c->pf_delta, c->pf_ws, c->status, s)) ||
        (rc = prefill_reduce(c, nt)))
      break;
  }
  return rc;
}

// Tokens [0, np) of a validated decode call through the GEMM chunks.
int prefill_gemm_tokens(b2_context* c, const int32_t* tokens, const std::vector<int32_t>& pv,
                        const std::vector<int32_t>& sv, int np) {
  int rc = prefill_alloc(c);
  if (rc) return rc;
  const int cap = c->pf_cap;
  for (int j0 = 0; j0 < np; j0 += cap) {
    if (c->abort_cb && c->abort_cb(c->abort_user)) return B2_ABORTED;
    const int nt = std::min(cap, np - j0);
    B2_CUDA_TRY(cudaEventSynchronize(c->pf_ev));   // the staging's previous copy has been read
    for (int i = 0; i < nt; ++i) {
      c->pf_in_h[i] = tokens[j0 + i];
      c->pf_in_h[cap + i] = pv[j0 + i];
      c->pf_in_h[2 * cap + i] = sv[j0 + i];
    }
    B2_CUDA_TRY(cudaMemcpyAsync(c->pf_in, c->pf_in_h, (size_t)3 * cap * 4, cudaMemcpyHostToDevice, c->stream));
    B2_CUDA_TRY(cudaEventRecord(c->pf_ev, c->stream));
    if ((rc = enqueue_prefill_chunk(c, nt))) return rc;
  }
  return B2_OK;
}

int decode(b2_context* c, const int32_t* tokens, const int32_t* pos, const int32_t* seq, int n, int want_logits) {
  b2_model* m = c->model;
  B2_CUDA_TRY(cudaSetDevice(m->device));
  B2_CHECK_ARG(tokens && n > 0, "decode arguments");
  // Validate: every token appends to its sequence at the next position.
  std::vector<int> next(c->n_past);
  std::vector<int32_t> pv(n), sv(n);
  for (int i = 0; i < n; ++i) {
    const int s = seq ? seq[i] : 0;
    if (s < 0 || s >= c->n_seq) {
      set_error("decode: sequence id %d out of range", s);
      return B2_ERR_INVALID;
    }
    const int p = pos ? pos[i] : next[s];
    if (p != next[s]) {
      set_error("decode: token %d of sequence %d at position %d, expected %d", i, s, p, next[s]);
      return B2_ERR_INVALID;
    }
    if (p >= c->n_ctx) return B2_NO_KV_SLOT;
    next[s] = p + 1;
    pv[i] = p;
    sv[i] = s;
  }
  // A long prompt: all but the last kStepMax tokens through the GEMM chunks
  // (no logits are asked of them), the rest through the decode step.
  int i0 = 0;
  c->last_n = 0;
  c->last_logits = false;
  {
    const int np = n - std::min(n, kStepMax);
    if (want_logits != 1 && np >= kPrefillMin && prefill_eligible(c)) {
      const int rc = prefill_gemm_tokens(c, tokens, pv, sv, np);
      if (rc == B2_ERR_OOM && c->pf_cap == 0) {
        // no room for the chunk buffers: this context keeps the decode step
        // for long prompts (nothing was enqueued)
        cudaGetLastError();
        c->prefill_gemm = false;
      } else if (rc) {
        return rc;
      } else {
        i0 = np;
      }
    }
  }
  // Steps of up to kStepMax tokens; a step never holds two tokens of one
  // sequence out of order (they are consecutive and written before the
  // step's attention reads them).
  while (i0 < n) {
    if (c->abort_cb && c->abort_cb(c->abort_user)) return B2_ABORTED;
    const int k = std::min(kStepMax, n - i0);
    const bool last = i0 + k == n;
    const bool with_logits = want_logits == 1 || (want_logits == 2 && last);
    // Two pinned staging slots: a slot is rewritten only after the copies
    // that read it two steps ago have completed.
    const int slot = c->in_slot;
    c->in_slot ^= 1;
    B2_CUDA_TRY(cudaEventSynchronize(c->in_ev[slot]));
    int32_t* hs = c->in_h + slot * 3 * kStepMax;
    for (int i = 0; i < k; ++i) {
      hs[i] = tokens[i0 + i];
      hs[kStepMax + i] = pv[i0 + i];
      hs[2 * kStepMax + i] = sv[i0 + i];
    }
    B2_CUDA_TRY(cudaMemcpyAsync(c->in_d, hs, 3 * kStepMax * 4, cudaMemcpyHostToDevice, c->stream));
    B2_CUDA_TRY(cudaEventRecord(c->in_ev[slot], c->stream));
    int rc = run_step(c, k, with_logits);
    if (rc) return rc;
    c->last_n = k;
    c->last_logits = with_logits;
    i0 += k;
  }
  for (int s = 0; s < c->n_seq; ++s) c->n_past[s] = next[s];
  return B2_OK;
}

// Greedy generation with the loop on the device: step t feeds every row the
// argmax of step t-1 (step 0 feeds `first`), so consecutive steps are graph
// replays with no host round trip.  The ids come back in one copy at the end.
int generate(b2_context* c, const int32_t* first, const int32_t* seq, int n, int n_steps, int32_t* out,
             b2_sampler* const* samplers = nullptr) {
  b2_model* m = c->model;
  B2_CUDA_TRY(cudaSetDevice(m->device));
  B2_CHECK_ARG(first && out && n > 0 && n <= kStepMax && n_steps >= 0, "generate arguments");
  std::vector<int32_t> sv(n);
  std::vector<char> used(c->n_seq, 0);
  for (int i = 0; i < n; ++i) {
    const int s = seq ? seq[i] : i;
    if (s < 0 || s >= c->n_seq || used[s]) {
      set_error("generate: sequence id %d out of range or repeated", s);
      return B2_ERR_INVALID;
    }
    used[s] = 1;
    sv[i] = s;
    if (first[i] < 0 || first[i] >= m->n_vocab) {
      set_error("generate: token %d outside the vocabulary", first[i]);
      return B2_ERR_INVALID;
    }
    if (c->n_past[s] + n_steps > c->n_ctx) return B2_NO_KV_SLOT;
  }
  if (samplers) {
    std::vector<SamplerDev*> sp(kStepMax, nullptr);
    for (int i = 0; i < n; ++i) {
      if (!samplers[i] || samplers[i]->ctx != c) {
        set_error("generate: row %d has no sampler of this context", i);
        return B2_ERR_INVALID;
      }
      for (int j = 0; j < i; ++j)
        if (samplers[j] == samplers[i]) {
          set_error("generate: rows %d and %d share one sampler", j, i);
          return B2_ERR_INVALID;
        }
      sp[i] = samplers[i]->dev;
    }
    B2_CUDA_TRY(cudaMemcpyAsync(c->samp_d, sp.data(), kStepMax * sizeof(SamplerDev*), cudaMemcpyHostToDevice,
                                c->stream));
  }
  if (n_steps == 0) return B2_OK;
  const int slot = c->in_slot;
  c->in_slot ^= 1;
  B2_CUDA_TRY(cudaEventSynchronize(c->in_ev[slot]));
  int32_t* hs = c->in_h + slot * 3 * kStepMax;
  for (int i = 0; i < n; ++i) {
    hs[i] = first[i];
    hs[kStepMax + i] = c->n_past[sv[i]];
    hs[2 * kStepMax + i] = sv[i];
  }
  B2_CUDA_TRY(cudaMemcpyAsync(c->in_d, hs, 3 * kStepMax * 4, cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaEventRecord(c->in_ev[slot], c->stream));
  B2_CUDA_TRY(cudaMemsetAsync(c->gen_count, 0, n * 4, c->stream));
  int done = 0, rc = B2_OK;
  for (; done < n_steps; ++done) {
    if (c->abort_cb && c->abort_cb(c->abort_user)) {
      rc = B2_ABORTED;
      break;
    }
    if ((rc = run_step(c, n, true, true, samplers != nullptr))) return rc;
  }
  if (done > 0) {
    B2_CUDA_TRY(cudaMemcpyAsync(out, c->gen_out, (size_t)done * n * 4, cudaMemcpyDeviceToHost, c->stream));
    c->last_n = n;
    c->last_logits = true;
  }
  const int st = check_status(c);
  if (st) return st;
  for (int i = 0; i < n; ++i) c->n_past[sv[i]] += done;
  return rc;
}

// Milda's shift (seq_rm [p0,p1) then seq_add(p1, end, -(p1-p0))), applied
// when the add arrives.  Fast path: p0 is the start of the ring (the pinned
// prefix length) — rotate the kept K in place and advance the ring head.
// Otherwise rows are compacted with the same rotation.
int kv_shift(b2_context* c, int s, int p0, int p1) {
  b2_model* m = c->model;
  const int n_past = c->n_past[s];
  const int nd = p1 - p0;
  if (nd <= 0) return B2_OK;
  KvSeqState& st = c->st[s];
  const bool fresh = st.ring_head == 0 && st.n_keep == 0;
  if (fresh) st.n_keep = p0;
  RotTable cs;
  rope_table(m->theta, m->head_dim, -nd, 1, cs.cs);
  int rc = B2_OK;
  if (p0 == st.n_keep) {
    for (int l = 0; l < m->n_layer && !rc; ++l)
      rc = launch_kv_shift(c->kc[l], c->type_k, m->nkv_l, m->head_dim, s, st, c->n_ctx, p1, n_past, cs, c->stream);
    const int ring = c->n_ctx - st.n_keep;
    st.ring_head = ring > 0 ? (st.ring_head + nd) % ring : 0;
  } else {
    for (int l = 0; l < m->n_layer && !rc; ++l)
      rc = launch_kv_compact(c->kc[l], c->type_k, c->vc[l], c->type_v, m->nkv_l, m->head_dim, s, st, c->n_ctx, p0,
                             p1, n_past - p1, cs, c->stream);
  }
  if (rc) return rc;
  c->n_past[s] = n_past - nd;
  B2_CUDA_TRY(cudaMemcpyAsync(c->st_d + s, &st, sizeof(KvSeqState), cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return B2_OK;
}

// Sequence-state snapshot (llama_state_seq_get_data / set_data): the
// sequence's K and V rows of this rank's KV heads in logical position order
// (rows in the cache types' storage), behind a header that names the shape
// and cache types they belong to.
struct SeqStateHeader {
  char magic[8];          // "B2KVSEQ"
  uint32_t version;       // 2
  int32_t n_layer, n_kv, head_dim, n_pos, type_k, tp_rank, tp_size, type_v;
  int32_t reserved[5];
};
constexpr uint32_t kSeqVersion = 2;
static_assert(sizeof(SeqStateHeader) == 64, "snapshot header size");
constexpr char kSeqMagic[8] = {'B', '2', 'K', 'V', 'S', 'E', 'Q', 0};

size_t seq_state_bytes(const b2_context* c, int n_pos) {
  const b2_model* m = c->model;
  return sizeof(SeqStateHeader) + (size_t)m->n_layer * m->nkv_l * n_pos *
                                      (size_t)(kv_row_bytes(c->type_k, m->head_dim) +
                                               kv_row_bytes(c->type_v, m->head_dim));
}

// Copies logical positions [0, n_pos) of sequence s between the cache and
// host memory: per layer K then V, each [n_kv][n_pos] rows.  The ring
// maps a position range to at most three contiguous slot runs; each run is
// one strided copy over the KV heads.
int seq_state_copy(b2_context* c, int s, int n_pos, uint8_t* host, bool to_host) {
  const b2_model* m = c->model;
  const KvSeqState st = to_host ? c->st[s] : KvSeqState{0, 0};
  const size_t krow = kv_row_bytes(c->type_k, m->head_dim), vrow = kv_row_bytes(c->type_v, m->head_dim);
  const size_t cap = (size_t)c->n_ctx;
  for (int l = 0; l < m->n_layer; ++l)
    for (int kv = 0; kv < 2; ++kv) {
      const size_t row = kv ? vrow : krow;
      uint8_t* base = (kv ? c->vc[l] : c->kc[l]) + (size_t)s * m->nkv_l * cap * row;
      uint8_t* h = host + (size_t)l * m->nkv_l * n_pos * (krow + vrow) + (kv ? (size_t)m->nkv_l * n_pos * krow : 0);
      for (int p = 0; p < n_pos;) {
        const int64_t slot = kv_slot(st, p, c->n_ctx);
        int len = 1;
        while (p + len < n_pos && kv_slot(st, p + len, c->n_ctx) == slot + len) ++len;
        uint8_t* dev = base + (size_t)slot * row;
        uint8_t* hp = h + (size_t)p * row;
        if (to_host)
          B2_CUDA_TRY(cudaMemcpy2DAsync(hp, (size_t)n_pos * row, dev, cap * row, (size_t)len * row, m->nkv_l,
                                        cudaMemcpyDeviceToHost, c->stream));
        else
          B2_CUDA_TRY(cudaMemcpy2DAsync(dev, cap * row, hp, (size_t)n_pos * row, (size_t)len * row, m->nkv_l,
                                        cudaMemcpyHostToDevice, c->stream));
        p += len;
      }
    }
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return B2_OK;
}

// Pending middle removals per sequence (seq_rm waiting for its seq_add).
struct Pending {
  int p0 = -1, p1 = -1;
};
thread_local std::vector<std::pair<const b2_context*, std::vector<Pending>>> g_pending;
std::vector<Pending>& pending_for(const b2_context* c) {
  for (auto& e : g_pending)
    if (e.first == c) return e.second;
  g_pending.push_back({c, std::vector<Pending>(c->n_seq)});
  return g_pending.back().second;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

int b2_gguf_write_synthetic_llama(const b2_llama_hparams* hp, const char* path, int n_threads) {
  B2_CHECK_ARG(hp && path, "synthetic llama arguments");
  return write_synthetic_llama(*hp, path, n_threads);
}

void b2_model_default_params(b2_model_params* p) {
  if (!p) return;
  p->device = -1;
  p->tp_rank = 0;
  p->tp_size = 1;
  p->nccl_id = nullptr;
  p->keep_page_cache = 0;
}

int b2_nccl_unique_id(void* out) {
  B2_CHECK_ARG(out, "out");
  ncclUniqueId id;
  B2_NCCL_TRY(ncclGetUniqueId(&id));
  memcpy(out, &id, sizeof id);
  return B2_OK;
}

int b2_model_load(const char* path, const b2_model_params* params, b2_model** out) {
  B2_CHECK_ARG(path && out, "model_load arguments");
  *out = nullptr;
  b2_model_params p;
  b2_model_default_params(&p);
  if (params) p = *params;
  b2_model* m = new (std::nothrow) b2_model;
  if (!m) return B2_ERR_OOM;
  int rc;
  try {
    rc = load_model(m, path, &p);
  } catch (const std::bad_alloc&) {
    set_error("model load: host out of memory");
    rc = B2_ERR_OOM;
  }
  if (rc) {
    delete m;
    return rc;
  }
  *out = m;
  return B2_OK;
}

int b2_model_free(b2_model* m) {
  delete m;
  return B2_OK;
}

int b2_model_info(const b2_model* m, int32_t* out, int32_t n) {
  B2_CHECK_ARG(m && out, "model_info arguments");
  const int32_t v[12] = {m->n_layer, m->n_embd,   m->n_ff,        m->n_head,  m->n_head_kv, m->n_vocab,
                         m->head_dim, m->n_ctx_train, m->wtype, m->out_type, m->tp_rank,  m->tp_size};
  for (int i = 0; i < n && i < 12; ++i) out[i] = v[i];
  return B2_OK;
}

int b2_model_device_bytes(const b2_model* m, int64_t* bytes) {
  B2_CHECK_ARG(m && bytes, "model_device_bytes arguments");
  *bytes = m->device_bytes;
  return B2_OK;
}

void b2_context_default_params(b2_context_params* p) {
  if (!p) return;
  p->n_ctx = 4096;
  p->n_seq_max = 1;
  p->use_graph = 1;
  p->prefill_gemm = 1;
  p->type_k = B2_F16;
  p->type_v = B2_F16;
}

int b2_context_create(b2_model* m, const b2_context_params* params, b2_context** out) {
  B2_CHECK_ARG(m && out, "context_create arguments");
  *out = nullptr;
  b2_context_params p;
  b2_context_default_params(&p);
  if (params) p = *params;
  B2_CHECK_ARG(p.n_ctx > 0 && p.n_seq_max > 0, "n_ctx and n_seq_max must be positive");
  B2_CHECK_ARG(kv_type_ok(p.type_k) && kv_type_ok(p.type_v), "type_k / type_v must be B2_F16, B2_Q8_0 or B2_Q4_0");
  b2_context* c = new (std::nothrow) b2_context;
  if (!c) return B2_ERR_OOM;
  int rc;
  try {
    rc = create_context(c, m, &p);
  } catch (const std::bad_alloc&) {
    rc = B2_ERR_OOM;
  }
  if (rc) {
    delete c;
    return rc;
  }
  *out = c;
  return B2_OK;
}

int b2_context_free(b2_context* c) {
  for (auto it = g_pending.begin(); it != g_pending.end(); ++it)
    if (it->first == c) {
      g_pending.erase(it);
      break;
    }
  delete c;
  return B2_OK;
}

int b2_context_stream(b2_context* c, void** stream) {
  B2_CHECK_ARG(c && stream, "context_stream arguments");
  *stream = c->stream;
  return B2_OK;
}

int b2_decode(b2_context* c, const int32_t* tokens, const int32_t* pos, const int32_t* seq, int32_t n_tokens,
              int32_t want_logits) {
  B2_CHECK_ARG(c, "context");
  for (const auto& p : pending_for(c))
    if (p.p0 >= 0) {
      set_error("decode: a KV removal is waiting for its position shift (b2_kv_seq_add)");
      return B2_ERR_INVALID;
    }
  return decode(c, tokens, pos, seq, n_tokens, want_logits);
}

int b2_generate(b2_context* c, const int32_t* first, const int32_t* seq, int32_t n, int32_t n_steps, int32_t* out) {
  B2_CHECK_ARG(c, "context");
  for (const auto& p : pending_for(c))
    if (p.p0 >= 0) {
      set_error("generate: a KV removal is waiting for its position shift (b2_kv_seq_add)");
      return B2_ERR_INVALID;
    }
  return generate(c, first, seq, n, n_steps, out);
}

void b2_sampler_default_params(b2_sampler_params* p) {
  if (!p) return;
  // Milda's configuration defaults (Milda/include/milda/engine.hpp:79-84) and
  // its penalty window of 64 (Milda/src/engine.cpp:1354-1355)
  p->penalty_last_n = 64;
  p->penalty_repeat = 1.08f;
  p->penalty_freq = 0.0f;
  p->penalty_present = 0.0f;
  p->top_k = 40;
  p->top_p = 0.90f;
  p->min_p = 0.05f;
  p->temperature = 0.75f;
  p->seed = 42u;
}

int b2_sampler_create(b2_context* c, const b2_sampler_params* p, b2_sampler** out) {
  B2_CHECK_ARG(c && p && out, "sampler_create arguments");
  *out = nullptr;
  B2_CHECK_ARG(p->penalty_last_n >= 0 && p->penalty_last_n <= kSampRing, "penalty_last_n must be in [0, 256]");
  B2_CHECK_ARG(p->temperature <= 0.0f || (p->top_k >= 1 && p->top_k <= kSampTopKMax),
               "a sampling chain (temperature > 0) needs top_k in [1, 256] on the device");
  B2_CHECK_ARG(p->penalty_repeat > 0.0f, "penalty_repeat must be positive");
  if (c->model->n_vocab > kSampParts * kSampSlice) {
    set_error("sampler: vocabularies of up to %d entries are sampled on the device", kSampParts * kSampSlice);
    return B2_ERR_UNSUPPORTED;
  }
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  if (!c->samp_d) {
    int rc;
    if ((rc = dalloc(c, &c->samp_d, kStepMax)) || (rc = dalloc(c, &c->samp_keys, sampler_scratch_keys()))) return rc;
  }
  b2_sampler* sm = new (std::nothrow) b2_sampler;
  if (!sm) return B2_ERR_OOM;
  sm->ctx = c;
  SamplerDev& h = sm->host;
  memset(&h, 0, sizeof h);
  h.last_n = p->penalty_last_n;
  h.rep = p->penalty_repeat;
  h.freq = p->penalty_freq;
  h.pres = p->penalty_present;
  h.top_k = p->top_k;
  h.top_p = p->top_p;
  h.min_p = p->min_p;
  h.logf_min_p = p->min_p > 0.0f ? logf(p->min_p) : 0.0f;
  h.temp = p->temperature;
  h.seed = p->seed;
  sampler_init_state(&h);
  if (cudaMalloc(&sm->dev, sizeof(SamplerDev)) != cudaSuccess ||
      cudaMalloc(&sm->self, sizeof(SamplerDev*)) != cudaSuccess) {
    cudaFree(sm->dev);
    delete sm;
    set_error("sampler_create: device allocation failed");
    return B2_ERR_OOM;
  }
  B2_CUDA_TRY(cudaMemcpyAsync(sm->dev, &h, sizeof h, cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaMemcpyAsync(sm->self, &sm->dev, sizeof(SamplerDev*), cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  *out = sm;
  return B2_OK;
}

int b2_sampler_free(b2_sampler* sm) {
  if (!sm) return B2_OK;
  cudaSetDevice(sm->ctx->model->device);
  cudaStreamSynchronize(sm->ctx->stream);
  cudaFree(sm->dev);
  cudaFree(sm->self);
  delete sm;
  return B2_OK;
}

int b2_sampler_reset(b2_sampler* sm) {
  B2_CHECK_ARG(sm, "sampler");
  B2_CUDA_TRY(cudaSetDevice(sm->ctx->model->device));
  SamplerDev& h = sm->host;
  sampler_init_state(&h);
  B2_CUDA_TRY(cudaMemcpyAsync(sm->dev, &h, sizeof h, cudaMemcpyHostToDevice, sm->ctx->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(sm->ctx->stream));
  return B2_OK;
}

int b2_sampler_accept(b2_sampler* sm, int32_t token) {
  B2_CHECK_ARG(sm && token >= 0 && token < kSampParts * kSampSlice, "sampler_accept arguments");
  B2_CUDA_TRY(cudaSetDevice(sm->ctx->model->device));
  return launch_sampler_accept(sm->dev, token, sm->ctx->stream);
}

int b2_sampler_sample(b2_sampler* sm, int32_t idx, int32_t* token) {
  B2_CHECK_ARG(sm && token, "sampler_sample arguments");
  b2_context* c = sm->ctx;
  B2_CHECK_ARG(c->last_logits, "the last decode computed no logits");
  if (idx < 0) idx += c->last_n;
  B2_CHECK_ARG(idx >= 0 && idx < c->last_n, "logits row out of range");
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  const b2_model* m = c->model;
  int rc = launch_sample(c->logits, c->last_n, idx, 1, m->n_vocab, m->v_l, sm->self, c->ids, GreedyFeed{},
                         c->samp_keys, c->stream);
  if (rc) return rc;
  B2_CUDA_TRY(cudaMemcpyAsync(c->res_h, c->ids + idx, 4, cudaMemcpyDeviceToHost, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  *token = c->res_h[0];
  return check_status(c);
}

int b2_sampler_sample_logits(b2_sampler* sm, const float* logits, int32_t n_vocab, int32_t* token) {
  B2_CHECK_ARG(sm && logits && token && n_vocab > 0, "sampler_sample_logits arguments");
  b2_context* c = sm->ctx;
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  int rc = launch_sample(logits, 1, 0, 1, n_vocab, n_vocab, sm->self, c->ids, GreedyFeed{}, c->samp_keys, c->stream);
  if (rc) return rc;
  B2_CUDA_TRY(cudaMemcpyAsync(c->res_h, c->ids, 4, cudaMemcpyDeviceToHost, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  *token = c->res_h[0];
  return B2_OK;
}

int b2_generate_sampled(b2_context* c, b2_sampler* const* samplers, const int32_t* first, const int32_t* seq,
                        int32_t n, int32_t n_steps, int32_t* out) {
  B2_CHECK_ARG(c && samplers, "generate_sampled arguments");
  for (const auto& p : pending_for(c))
    if (p.p0 >= 0) {
      set_error("generate: a KV removal is waiting for its position shift (b2_kv_seq_add)");
      return B2_ERR_INVALID;
    }
  return generate(c, first, seq, n, n_steps, out, samplers);
}

int b2_get_logits(b2_context* c, int32_t i, float* out, int64_t n) {
  B2_CHECK_ARG(c && out, "get_logits arguments");
  B2_CHECK_ARG(c->last_logits, "the last decode computed no logits");
  if (i < 0) i += c->last_n;
  B2_CHECK_ARG(i >= 0 && i < c->last_n, "logits row out of range");
  b2_model* m = c->model;
  B2_CUDA_TRY(cudaSetDevice(m->device));
  const int64_t cnt = std::min<int64_t>(n, m->n_vocab);
  const int64_t vl = m->v_l;
  // gathered layout [tp][n_tok][v_l]
  for (int r = 0; r < m->tp_size && r * vl < cnt; ++r) {
    const int64_t len = std::min<int64_t>(vl, cnt - r * vl);
    B2_CUDA_TRY(cudaMemcpyAsync(out + r * vl, c->logits + ((int64_t)r * c->last_n + i) * vl, len * 4,
                                cudaMemcpyDeviceToHost, c->stream));
  }
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return check_status(c);
}

int b2_get_argmax(b2_context* c, int32_t* ids, float* top1, float* margin, int32_t n) {
  B2_CHECK_ARG(c && ids, "get_argmax arguments");
  B2_CHECK_ARG(c->last_logits, "the last decode computed no logits");
  B2_CHECK_ARG(n >= c->last_n, "output arrays shorter than the last batch");
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  int32_t* r = c->res_h;
  B2_CUDA_TRY(cudaMemcpyAsync(r, c->res, kResWords * 4, cudaMemcpyDeviceToHost, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  const float* top = reinterpret_cast<const float*>(r + kStepMax);
  for (int i = 0; i < c->last_n; ++i) {
    ids[i] = r[i];
    if (top1) top1[i] = top[2 * i];
    if (margin) margin[i] = top[2 * i + 1];
  }
  if (r[3 * kStepMax] != 0) return check_status(c);
  return B2_OK;
}

int b2_context_exchange_wait_ns(b2_context* c, uint64_t* ns, int32_t reset) {
  B2_CHECK_ARG(c && ns, "context_exchange_wait_ns arguments");
  *ns = 0;
  if (!c->wait_ns) return B2_OK;
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  unsigned long long v = 0;
  B2_CUDA_TRY(cudaMemcpyAsync(&v, c->wait_ns, sizeof v, cudaMemcpyDeviceToHost, c->stream));
  if (reset) B2_CUDA_TRY(cudaMemsetAsync(c->wait_ns, 0, sizeof v, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  *ns = v;
  return B2_OK;
}

int b2_get_last_rows(b2_context* c, int32_t* n) {
  B2_CHECK_ARG(c && n, "get_last_rows arguments");
  *n = c->last_logits ? c->last_n : 0;
  return B2_OK;
}

int b2_synchronize_context(b2_context* c) {
  B2_CHECK_ARG(c, "context");
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return check_status(c);
}

int b2_kv_clear(b2_context* c) {
  B2_CHECK_ARG(c, "context");
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  for (int s = 0; s < c->n_seq; ++s) {
    c->st[s] = KvSeqState{0, 0};
    c->n_past[s] = 0;
  }
  for (auto& p : pending_for(c)) p = Pending{};
  B2_CUDA_TRY(cudaMemcpyAsync(c->st_d, c->st.data(), c->n_seq * sizeof(KvSeqState), cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  return B2_OK;
}

int b2_kv_seq_rm(b2_context* c, int32_t seq, int32_t p0, int32_t p1) {
  B2_CHECK_ARG(c && seq >= 0 && seq < c->n_seq, "kv_seq_rm arguments");
  const int n_past = c->n_past[seq];
  if (p0 < 0) p0 = 0;
  if (p1 < 0 || p1 > n_past) p1 = n_past;
  if (p0 >= p1) return B2_OK;
  if (p1 == n_past) {   // suffix: truncate
    c->n_past[seq] = p0;
    return B2_OK;
  }
  pending_for(c)[seq] = Pending{p0, p1};
  return B2_OK;
}

int b2_kv_seq_add(b2_context* c, int32_t seq, int32_t p0, int32_t p1, int32_t delta) {
  B2_CHECK_ARG(c && seq >= 0 && seq < c->n_seq, "kv_seq_add arguments");
  Pending& pd = pending_for(c)[seq];
  if (p1 < 0) p1 = c->n_past[seq];
  if (pd.p0 < 0 || p0 != pd.p1 || p1 != c->n_past[seq] || delta != -(pd.p1 - pd.p0)) {
    set_error("kv_seq_add: only the shift that closes a preceding kv_seq_rm gap is supported");
    return B2_ERR_UNSUPPORTED;
  }
  B2_CUDA_TRY(cudaSetDevice(c->model->device));
  const int rc = kv_shift(c, seq, pd.p0, pd.p1);
  pd = Pending{};
  return rc;
}

int b2_kv_seq_pos_max(b2_context* c, int32_t seq, int32_t* pos) {
  B2_CHECK_ARG(c && pos && seq >= 0 && seq < c->n_seq, "kv_seq_pos_max arguments");
  *pos = c->n_past[seq] - 1;
  return B2_OK;
}

int b2_n_ctx(const b2_context* c, int32_t* n_ctx) {
  B2_CHECK_ARG(c && n_ctx, "n_ctx arguments");
  *n_ctx = c->n_ctx;
  return B2_OK;
}

int b2_memory_can_shift(const b2_context* c, int32_t* can_shift) {
  B2_CHECK_ARG(c && can_shift, "memory_can_shift arguments");
  *can_shift = 1;   // the ring cache re-rotates K in place (fp16 or Q8_0) for any shift
  return B2_OK;
}

int b2_state_seq_get_size(b2_context* c, int32_t seq, size_t* size) {
  B2_CHECK_ARG(c && size && seq >= 0 && seq < c->n_seq, "state_seq_get_size arguments");
  *size = seq_state_bytes(c, c->n_past[seq]);
  return B2_OK;
}

int b2_state_seq_get_data(b2_context* c, int32_t seq, void* dst, size_t size, size_t* written) {
  B2_CHECK_ARG(c && dst && seq >= 0 && seq < c->n_seq, "state_seq_get_data arguments");
  if (written) *written = 0;
  for (const auto& p : pending_for(c))
    if (p.p0 >= 0) {
      set_error("state_seq_get_data: a KV removal is waiting for its position shift (b2_kv_seq_add)");
      return B2_ERR_INVALID;
    }
  const b2_model* m = c->model;
  const int n_pos = c->n_past[seq];
  const size_t need = seq_state_bytes(c, n_pos);
  if (size < need) {
    set_error("state_seq_get_data: %zu bytes given, the state of sequence %d takes %zu", size, seq, need);
    return B2_ERR_INVALID;
  }
  B2_CUDA_TRY(cudaSetDevice(m->device));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  SeqStateHeader h = {};
  memcpy(h.magic, kSeqMagic, 8);
  h.version = kSeqVersion;
  h.n_layer = m->n_layer;
  h.n_kv = m->nkv_l;
  h.head_dim = m->head_dim;
  h.n_pos = n_pos;
  h.type_k = c->type_k;
  h.type_v = c->type_v;
  h.tp_rank = m->tp_rank;
  h.tp_size = m->tp_size;
  memcpy(dst, &h, sizeof h);
  const int rc = seq_state_copy(c, seq, n_pos, static_cast<uint8_t*>(dst) + sizeof h, true);
  if (rc) return rc;
  if (written) *written = need;
  return check_status(c);
}

int b2_state_seq_set_data(b2_context* c, int32_t seq, const void* src, size_t size, size_t* read) {
  B2_CHECK_ARG(c && src && seq >= 0 && seq < c->n_seq, "state_seq_set_data arguments");
  if (read) *read = 0;
  const b2_model* m = c->model;
  SeqStateHeader h;
  if (size < sizeof h) {
    set_error("state_seq_set_data: %zu bytes, shorter than the header", size);
    return B2_ERR_FORMAT;
  }
  memcpy(&h, src, sizeof h);
  if (memcmp(h.magic, kSeqMagic, 8) != 0 || h.version != kSeqVersion) {
    set_error("state_seq_set_data: not a sequence-state snapshot of this library");
    return B2_ERR_FORMAT;
  }
  if (h.n_layer != m->n_layer || h.n_kv != m->nkv_l || h.head_dim != m->head_dim || h.type_k != c->type_k ||
      h.type_v != c->type_v || h.tp_rank != m->tp_rank || h.tp_size != m->tp_size) {
    set_error("state_seq_set_data: snapshot of another model shape, cache type or rank (%d layers, %d kv heads, "
              "hd %d, K/V types %d/%d, rank %d/%d)", h.n_layer, h.n_kv, h.head_dim, h.type_k, h.type_v, h.tp_rank,
              h.tp_size);
    return B2_ERR_FORMAT;
  }
  if (h.n_pos < 0 || h.n_pos > c->n_ctx) {
    set_error("state_seq_set_data: %d positions, the context holds %d", h.n_pos, c->n_ctx);
    return B2_NO_KV_SLOT;
  }
  const size_t need = seq_state_bytes(c, h.n_pos);
  if (size < need) {
    set_error("state_seq_set_data: %zu bytes, the snapshot declares %zu", size, need);
    return B2_ERR_FORMAT;
  }
  B2_CUDA_TRY(cudaSetDevice(m->device));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  // The restored sequence starts a fresh ring: positions in slots 0..n_pos-1.
  pending_for(c)[seq] = Pending{};
  const int rc = seq_state_copy(c, seq, h.n_pos, const_cast<uint8_t*>(static_cast<const uint8_t*>(src)) + sizeof h,
                                false);
  if (rc) return rc;
  c->st[seq] = KvSeqState{0, 0};
  c->n_past[seq] = h.n_pos;
  B2_CUDA_TRY(cudaMemcpyAsync(c->st_d + seq, &c->st[seq], sizeof(KvSeqState), cudaMemcpyHostToDevice, c->stream));
  B2_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (read) *read = need;
  return B2_OK;
}

int b2_set_eval_callback(b2_context* c, b2_eval_callback cb, void* user) {
  B2_CHECK_ARG(c, "context");
  c->eval_cb = cb;
  c->eval_user = user;
  return B2_OK;
}

int b2_set_abort_callback(b2_context* c, b2_abort_callback cb, void* user) {
  B2_CHECK_ARG(c, "context");
  c->abort_cb = cb;
  c->abort_user = user;
  return B2_OK;
}

}  // extern "C"
