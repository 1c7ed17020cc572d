// On-device sampler chain (b2_sampler.cu): the chain Milda builds in
// rebuild_sampler (Milda/src/engine.cpp:1321-1384) from llama.cpp's samplers
// — penalties, then greedy, or top-k, top-p, min-p, temperature and dist —
// with its state (the penalty window, the mt19937 generator) in device memory
// so that a decode loop samples without copying logits to the host.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_internal.hpp"
#include "b2_layers.hpp"

namespace b2 {

constexpr int kSampRing = 256;      // largest penalty window (penalty_last_n)
constexpr int kSampTopKMax = 256;   // largest top_k on the device
constexpr int kSampSlice = 2048;    // vocabulary entries per selecting CTA
constexpr int kSampParts = 64;      // selecting CTAs per row at most
constexpr int kMtN = 624;           // mt19937 state words

// One sampler chain instance in device memory: its parameters, then its state.
struct SamplerDev {
  int32_t last_n;        // penalty window (0: no penalties)
  float rep, freq, pres; // repeat / frequency / presence penalties
  int32_t top_k;         // candidates kept (greedy: 1)
  float top_p, min_p;    // top-p (>= 1: off), min-p (<= 0: off)
  float logf_min_p;      // logf(min_p), the host C library's value
  float temp;            // <= 0: greedy
  uint32_t seed;
  int32_t ring_len, ring_head;   // accepted tokens in the window, oldest slot
  int32_t ring[kSampRing];
  int32_t mti;                   // next mt19937 word (kMtN: twist first)
  uint32_t mt[kMtN];
};

// Candidate keys per context: [kStepMax rows][kSampParts][kSampTopKMax].
constexpr size_t sampler_scratch_keys() { return (size_t)8 * kSampParts * kSampTopKMax; }

// Samples rows row0 .. row0+n-1 of the logits (gather layout of the greedy
// argmax: v_local entries per shard, n_tok rows) with samplers sps[0..n)
// (a device array of device pointers), accepts each sampled token into its
// sampler (as llama_sampler_sample does) and writes it to ids[i]; with a feed
// it also becomes the next step's token of row row0 + i.  Two launches.
int launch_sample(const float* logits, int n_tok, int row0, int n, int n_vocab, int v_local, SamplerDev* const* sps,
                  int32_t* ids, const GreedyFeed& feed, unsigned long long* keys, cudaStream_t s);
// Pushes `token` into the penalty window of sampler sp (llama_sampler_accept).
int launch_sampler_accept(SamplerDev* sp, int32_t token, cudaStream_t s);
// The state of a fresh (or reset) chain: empty window, mt19937 seeded.
void sampler_init_state(SamplerDev* h);

}  // namespace b2
