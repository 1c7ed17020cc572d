// Synthetic Llama-architecture GGUF files: the tensors and metadata the
// engines load (names as Singularity/src/core/cortex_a5_engine.cpp:579-648
// binds them), weights drawn from the seeded normal generator and quantized
// with the library's GGUF quantizers, norms set to 1.  Used to stand in for
// the real model files on benchmark shapes.
#include <fcntl.h>
#include <string.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "b2_gguf.hpp"
#include "b2_internal.hpp"

namespace b2 {
namespace {

uint64_t tensor_seed(uint64_t seed, uint64_t index) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ull + (index + 1) * 0xBF58476D1CE4E5B9ull;
  z ^= z >> 31;
  z *= 0x94D049BB133111EBull;
  return z ^ (z >> 29);
}

bool write_all(int fd, const uint8_t* p, size_t n, off_t off) {
  while (n > 0) {
    const ssize_t w = pwrite(fd, p, n, off);
    if (w <= 0) return false;
    p += w;
    n -= (size_t)w;
    off += w;
  }
  return true;
}

}  // namespace

int write_synthetic_llama(const b2_llama_hparams& hp, const char* path, int n_threads) {
  const int d = hp.n_embd, ff = hp.n_ff, nh = hp.n_head, nkv = hp.n_head_kv, V = hp.n_vocab;
  if (d <= 0 || ff <= 0 || nh <= 0 || nkv <= 0 || V <= 0 || hp.n_layer <= 0 || d % nh || nh % nkv) {
    set_error("synthetic llama: inconsistent shapes");
    return B2_ERR_INVALID;
  }
  const int hd = d / nh;
  auto ok_type = [](int t, int64_t k) { return is_weight_type(t) && k % block_elems(t) == 0; };
  const int out_type = hp.out_type < 0 ? hp.embd_type : hp.out_type;
  if (!ok_type(hp.wtype, d) || !ok_type(hp.wtype, ff) || !(ok_type(hp.embd_type, d) || hp.embd_type == B2_F32) ||
      !(ok_type(out_type, d) || out_type == B2_F32)) {
    set_error("synthetic llama: unsupported type / shape combination");
    return B2_ERR_UNSUPPORTED;
  }
  GgufWriter w;
  w.add_str("general.architecture", "llama");
  w.add_str("general.name", "b2-synthetic-llama");
  w.add_u32("general.alignment", 32);
  w.add_u32("llama.block_count", (uint32_t)hp.n_layer);
  w.add_u32("llama.context_length", (uint32_t)hp.n_ctx_train);
  w.add_u32("llama.embedding_length", (uint32_t)d);
  w.add_u32("llama.feed_forward_length", (uint32_t)ff);
  w.add_u32("llama.attention.head_count", (uint32_t)nh);
  w.add_u32("llama.attention.head_count_kv", (uint32_t)nkv);
  w.add_u32("llama.rope.dimension_count", (uint32_t)hd);
  w.add_u32("llama.vocab_size", (uint32_t)V);
  w.add_f32("llama.attention.layer_norm_rms_epsilon", hp.rms_eps);
  w.add_f32("llama.rope.freq_base", hp.rope_theta);
  struct Spec {
    int type;
    bool norm;
  };
  std::vector<Spec> specs;
  w.add_tensor("token_embd.weight", hp.embd_type, d, V, 2);
  specs.push_back({hp.embd_type, false});
  w.add_tensor("output_norm.weight", B2_F32, d, 1, 1);
  specs.push_back({B2_F32, true});
  if (hp.out_type >= 0) {
    w.add_tensor("output.weight", hp.out_type, d, V, 2);
    specs.push_back({hp.out_type, false});
  }
  for (int l = 0; l < hp.n_layer; ++l) {
    const std::string b = "blk." + std::to_string(l) + ".";
    w.add_tensor(b + "attn_norm.weight", B2_F32, d, 1, 1);
    specs.push_back({B2_F32, true});
    w.add_tensor(b + "attn_q.weight", hp.wtype, d, (int64_t)nh * hd, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "attn_k.weight", hp.wtype, d, (int64_t)nkv * hd, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "attn_v.weight", hp.wtype, d, (int64_t)nkv * hd, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "attn_output.weight", hp.wtype, (int64_t)nh * hd, d, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "ffn_norm.weight", B2_F32, d, 1, 1);
    specs.push_back({B2_F32, true});
    w.add_tensor(b + "ffn_gate.weight", hp.wtype, d, ff, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "ffn_up.weight", hp.wtype, d, ff, 2);
    specs.push_back({hp.wtype, false});
    w.add_tensor(b + "ffn_down.weight", hp.wtype, ff, d, 2);
    specs.push_back({hp.wtype, false});
  }
  const int fd = ::open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) {
    set_error("synthetic llama: cannot create %s", path);
    return B2_ERR_IO;
  }
  int rc = B2_OK;
  try {
    std::vector<uint8_t> hdr(w.header_bytes());
    w.write_header(hdr.data());
    if (!write_all(fd, hdr.data(), hdr.size(), 0)) rc = B2_ERR_IO;
    std::vector<float> vals;
    std::vector<uint8_t> q;
    for (size_t i = 0; rc == B2_OK && i < w.tensors.size(); ++i) {
      const auto& t = w.tensors[i];
      const off_t off = (off_t)w.tensor_file_offset(i);
      if (specs[i].norm) {
        vals.assign((size_t)t.ne0, 1.0f);
        if (!write_all(fd, reinterpret_cast<const uint8_t*>(vals.data()), vals.size() * 4, off)) rc = B2_ERR_IO;
        continue;
      }
      const uint64_t ts = tensor_seed(hp.seed, i);
      const size_t rb = row_bytes(t.type, t.ne0);
      // Row slabs of ~64 MB of fp32 keep host memory bounded for large tensors.
      const int64_t slab = std::max<int64_t>(1, (int64_t)(16u << 20) / t.ne0);
      for (int64_t r0 = 0; rc == B2_OK && r0 < t.ne1; r0 += slab) {
        const int64_t r1 = std::min<int64_t>(t.ne1, r0 + slab);
        const int64_t n = (r1 - r0) * t.ne0;
        vals.resize((size_t)n);
        synth_normal(ts, (uint64_t)(r0 * t.ne0), n, 0.0f, hp.w_std, vals.data(), n_threads);
        if (t.type == B2_F32) {
          if (!write_all(fd, reinterpret_cast<const uint8_t*>(vals.data()), (size_t)n * 4, off + (off_t)(r0 * rb)))
            rc = B2_ERR_IO;
          continue;
        }
        q.resize((size_t)(r1 - r0) * rb);
        rc = quantize_weights(t.type, vals.data(), r1 - r0, t.ne0, q.data(), n_threads);
        if (rc == B2_OK && !write_all(fd, q.data(), q.size(), off + (off_t)(r0 * rb))) rc = B2_ERR_IO;
      }
    }
    // Pad the file to the aligned end of the last tensor.
    if (rc == B2_OK && ftruncate(fd, (off_t)w.total_bytes()) != 0) rc = B2_ERR_IO;
  } catch (...) {
    rc = B2_ERR_OOM;
  }
  ::close(fd);
  if (rc == B2_ERR_IO) set_error("synthetic llama: write to %s failed", path);
  return rc;
}

}  // namespace b2
