// Milda's llama.cpp call sequence replayed through include/b2gguf.h, compiled
// as C++ (the engines' host language) and linked to libb2gguf.so: model load
// (Milda/src/engine.cpp:897-934), context (:1180-1236), chunked prefill of
// the system prompt (decode_tokens_chunked, :1521-1548), the pinned system
// state (:1487-1492), a turn's greedy decode loop with llama_get_logits_ith
// (:1962-2117), the in-place KV shift (shift_kv_cache_in_place, :1642-1675),
// and clear_conversation in both of its forms (:1677-1720): suffix removal
// back to the system prompt, and clear + restore of the pinned state.  The
// two forms must give bit-identical logits for the next turn.  The sequence
// runs twice: with an fp16 cache and greedy picks, then with Milda's default
// configuration, a Q8_0 K and V cache (engine.hpp:85-86) and the sampler
// chain rebuild_sampler builds (:1321-1384), sampled on the device and
// accepted again after each draw (:1970, :2029), reset with the conversation
// (:1693).
//
// Usage: milda_sequence MODEL_PATH   (writes a small synthetic model there)
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "b2gguf.h"

namespace {

#define CHECK(expr)                                                                       \
  do {                                                                                    \
    const int rc_ = (expr);                                                               \
    if (rc_ != B2_OK) {                                                                   \
      std::fprintf(stderr, "%s:%d: %s -> %d: %s\n", __FILE__, __LINE__, #expr, rc_,       \
                   b2_last_error());                                                      \
      return 1;                                                                           \
    }                                                                                     \
  } while (0)

#define EXPECT(cond)                                                                      \
  do {                                                                                    \
    if (!(cond)) {                                                                        \
      std::fprintf(stderr, "%s:%d: expected %s\n", __FILE__, __LINE__, #cond);            \
      return 1;                                                                           \
    }                                                                                     \
  } while (0)

struct Lcg {
  uint64_t s;
  int32_t next(int32_t n) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return (int32_t)((s >> 33) % (uint64_t)n);
  }
};

int32_t argmax(const std::vector<float>& v) {
  return (int32_t)(std::max_element(v.begin(), v.end()) - v.begin());
}

// decode_tokens_chunked: llama_batch_get_one over chunks of n_batch tokens,
// logits of the last token of each chunk.
int decode_chunked(b2_context* ctx, const int32_t* tokens, int32_t count, int32_t n_batch) {
  for (int32_t off = 0; off < count;) {
    const int32_t step = std::min(n_batch, count - off);
    const int rc = b2_decode(ctx, tokens + off, nullptr, nullptr, step, 2);
    if (rc != B2_OK) return rc;
    off += step;
  }
  return B2_OK;
}

int run_sequence(b2_model* model, int32_t n_vocab, bool milda_defaults) {
  b2_context_params cp;
  b2_context_default_params(&cp);
  cp.n_ctx = 160;
  cp.n_seq_max = 1;
  if (milda_defaults) {
    cp.type_k = B2_Q8_0;
    cp.type_v = B2_Q8_0;
  }
  b2_context* ctx = nullptr;
  CHECK(b2_context_create(model, &cp, &ctx));
  int32_t n_ctx = 0;
  CHECK(b2_n_ctx(ctx, &n_ctx));
  EXPECT(n_ctx == 160);
  b2_sampler* sampler = nullptr;
  if (milda_defaults) {
    b2_sampler_params sp;
    b2_sampler_default_params(&sp);
    EXPECT(sp.top_k == 40 && sp.penalty_last_n == 64);
    CHECK(b2_sampler_create(ctx, &sp, &sampler));
  }

  // system prompt, prefilled in chunks, then its state pinned
  Lcg rng{12345};
  std::vector<int32_t> sys(70);
  for (auto& t : sys) t = rng.next(n_vocab);
  const int32_t n_keep = (int32_t)sys.size();
  CHECK(decode_chunked(ctx, sys.data(), n_keep, 32));
  size_t st_size = 0, written = 0;
  CHECK(b2_state_seq_get_size(ctx, 0, &st_size));
  std::vector<uint8_t> pinned(st_size);
  CHECK(b2_state_seq_get_data(ctx, 0, pinned.data(), pinned.size(), &written));
  EXPECT(written == st_size);

  // a turn: user prompt, then the decode loop; the context fills up and the
  // in-place shift makes room, as generate_turn does
  std::vector<float> logits(n_vocab);
  std::vector<int32_t> user(24);
  for (auto& t : user) t = rng.next(n_vocab);
  CHECK(decode_chunked(ctx, user.data(), (int32_t)user.size(), 32));
  CHECK(b2_get_logits(ctx, -1, logits.data(), n_vocab));
  int32_t n_past = n_keep + (int32_t)user.size();
  int shifts = 0;
  for (int step = 0; step < 120; ++step) {
    int32_t tok = 0;
    if (sampler) {
      CHECK(b2_sampler_sample(sampler, -1, &tok));
      CHECK(b2_sampler_accept(sampler, tok));
      EXPECT(tok >= 0 && tok < n_vocab);
    } else {
      tok = argmax(logits);
    }
    if (n_past + 1 >= n_ctx) {   // shift_kv_cache_in_place
      int32_t can_shift = 0;
      CHECK(b2_memory_can_shift(ctx, &can_shift));
      EXPECT(can_shift == 1);
      const int32_t removable = n_past - n_keep;
      const int32_t n_discard = std::clamp(std::max(1, removable / 2), 1, removable);
      CHECK(b2_kv_seq_rm(ctx, 0, n_keep, n_keep + n_discard));
      CHECK(b2_kv_seq_add(ctx, 0, n_keep + n_discard, -1, -n_discard));
      n_past -= n_discard;
      int32_t pmax = 0;
      CHECK(b2_kv_seq_pos_max(ctx, 0, &pmax));
      EXPECT(pmax == n_past - 1);
      ++shifts;
    }
    CHECK(b2_decode(ctx, &tok, nullptr, nullptr, 1, 1));
    ++n_past;
    if (!sampler) CHECK(b2_get_logits(ctx, -1, logits.data(), n_vocab));
  }
  EXPECT(shifts >= 2);

  // clear_conversation, form 1: remove everything after the system prompt
  if (sampler) CHECK(b2_sampler_reset(sampler));
  std::vector<int32_t> user2(19);
  for (auto& t : user2) t = rng.next(n_vocab);
  CHECK(b2_kv_seq_rm(ctx, 0, n_keep, -1));
  CHECK(decode_chunked(ctx, user2.data(), (int32_t)user2.size(), 32));
  std::vector<float> via_rm(n_vocab);
  CHECK(b2_get_logits(ctx, -1, via_rm.data(), n_vocab));
  int32_t first_rm = -1;
  if (sampler) CHECK(b2_sampler_sample(sampler, -1, &first_rm));

  // form 2: clear the cache and restore the pinned system state
  size_t read = 0;
  if (sampler) CHECK(b2_sampler_reset(sampler));
  CHECK(b2_kv_clear(ctx));
  CHECK(b2_state_seq_set_data(ctx, 0, pinned.data(), pinned.size(), &read));
  EXPECT(read == pinned.size());
  int32_t pmax = 0;
  CHECK(b2_kv_seq_pos_max(ctx, 0, &pmax));
  EXPECT(pmax == n_keep - 1);
  CHECK(decode_chunked(ctx, user2.data(), (int32_t)user2.size(), 32));
  std::vector<float> via_restore(n_vocab);
  CHECK(b2_get_logits(ctx, -1, via_restore.data(), n_vocab));
  EXPECT(std::memcmp(via_rm.data(), via_restore.data(), n_vocab * sizeof(float)) == 0);
  if (sampler) {   // the reset chain draws the same first token of the turn
    int32_t first_restore = -1;
    CHECK(b2_sampler_sample(sampler, -1, &first_restore));
    EXPECT(first_restore == first_rm);
  }

  // a fresh context that prefills the same conversation from scratch agrees too
  b2_context* fresh = nullptr;
  CHECK(b2_context_create(model, &cp, &fresh));
  CHECK(decode_chunked(fresh, sys.data(), n_keep, 32));
  CHECK(decode_chunked(fresh, user2.data(), (int32_t)user2.size(), 32));
  std::vector<float> via_fresh(n_vocab);
  CHECK(b2_get_logits(fresh, -1, via_fresh.data(), n_vocab));
  EXPECT(std::memcmp(via_rm.data(), via_fresh.data(), n_vocab * sizeof(float)) == 0);

  if (sampler) CHECK(b2_sampler_free(sampler));
  CHECK(b2_context_free(fresh));
  CHECK(b2_context_free(ctx));
  std::printf("milda sequence ok (%s): %d shifts, %zu-byte pinned state, next-turn logits identical\n",
              milda_defaults ? "Q8_0 KV cache, sampler chain" : "fp16 KV cache, greedy", shifts, pinned.size());
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s MODEL_PATH\n", argv[0]);
    return 2;
  }
  b2_llama_hparams hp = {};
  hp.n_layer = 2;
  hp.n_embd = 256;
  hp.n_ff = 512;
  hp.n_head = 4;
  hp.n_head_kv = 2;
  hp.n_vocab = 512;
  hp.n_ctx_train = 256;
  hp.rms_eps = 1e-5f;
  hp.rope_theta = 10000.0f;
  hp.wtype = B2_Q4_K;
  hp.embd_type = B2_Q8_0;
  hp.out_type = B2_Q6_K;
  hp.seed = 77;
  hp.w_std = 0.02f;
  CHECK(b2_gguf_write_synthetic_llama(&hp, argv[1], 4));

  // initialize(): model, context, n_ctx
  b2_model_params mp;
  b2_model_default_params(&mp);
  mp.device = 0;
  b2_model* model = nullptr;
  if (b2_model_load(argv[1], &mp, &model) != B2_OK || model == nullptr) {
    std::fprintf(stderr, "model load failed: %s\n", b2_last_error());
    return 1;
  }
  int32_t info[12];
  CHECK(b2_model_info(model, info, 12));
  const int32_t n_vocab = info[5];
  EXPECT(info[0] == 2 && n_vocab == 512);
  if (run_sequence(model, n_vocab, false) != 0 || run_sequence(model, n_vocab, true) != 0) return 1;
  CHECK(b2_model_free(model));
  std::printf("milda sequence ok\n");
  return 0;
}
