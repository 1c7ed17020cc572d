"""Generates tests/golden/libstdcxx_sampler.npz: what the GNU C++ library's
std::mt19937 and std::discrete_distribution produce, the two pieces of
llama.cpp's dist sampler (llama_sampler_init_dist) that Milda's chain ends
with (Milda/src/engine.cpp:1380-1381).  llama.cpp builds the distribution
from the candidates' float probabilities and draws it with a std::mt19937
seeded by the sampler's seed; this script compiles the same construction
with the image's g++ and records

  * the first 8 outputs of std::mt19937(seed) for a few seeds, and its
    10000th output for the default seed (the C++ standard fixes it at
    4123659995);
  * 64 draws of std::discrete_distribution<int>(w.begin(), w.end()) with one
    std::mt19937(seed) per weight vector, for weight vectors with ties,
    tiny and dominant weights, one weight, and 40-entry softmax outputs.

    python tests/golden/make_sampler_golden.py
"""
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

SRC = r"""
#include <cstdio>
#include <cstdint>
#include <random>
#include <vector>
int main() {
  unsigned n_seeds; std::scanf("%u", &n_seeds);
  for (unsigned i = 0; i < n_seeds; ++i) {
    unsigned seed; std::scanf("%u", &seed);
    std::mt19937 g(seed);
    for (int k = 0; k < 8; ++k) std::printf("%u ", (unsigned)g());
    std::printf("\n");
  }
  { std::mt19937 g; unsigned v = 0; for (int k = 0; k < 10000; ++k) v = g(); std::printf("%u\n", v); }
  unsigned n_cases; std::scanf("%u", &n_cases);
  for (unsigned c = 0; c < n_cases; ++c) {
    unsigned seed, n; std::scanf("%u %u", &seed, &n);
    std::vector<float> w(n);
    for (unsigned k = 0; k < n; ++k) { unsigned bits; std::scanf("%u", &bits); float f; __builtin_memcpy(&f, &bits, 4); w[k] = f; }
    std::mt19937 g(seed);
    std::discrete_distribution<int> d(w.begin(), w.end());
    for (int k = 0; k < 64; ++k) std::printf("%d ", d(g));
    std::printf("\n");
  }
  return 0;
}
"""


def softmax32(x):
    x = np.asarray(x, np.float32)
    e = np.exp(x - x.max()).astype(np.float32)
    return (e / e.sum(dtype=np.float32)).astype(np.float32)


def main():
    rng = np.random.default_rng(11)
    seeds = [0, 1, 42, 5489, 123456789, 4294967295]
    cases = [
        (42, np.array([0.5, 0.5], np.float32)),
        (7, np.array([1.0], np.float32)),
        (3, np.array([1e-30, 1.0, 1e-30], np.float32)),
        (9, np.array([0.25] * 4, np.float32)),
        (42, softmax32(np.sort(rng.standard_normal(40) * 2)[::-1])),
        (1234, softmax32(np.sort(rng.standard_normal(40) * 0.3)[::-1])),
        (77, softmax32(np.sort(rng.standard_normal(256) * 4)[::-1])),
        (5, rng.random(17).astype(np.float32)),
    ]
    lines = [str(len(seeds))] + [str(s) for s in seeds] + [str(len(cases))]
    for seed, w in cases:
        lines.append(f"{seed} {w.size} " + " ".join(str(int(b)) for b in w.view(np.uint32)))
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "stdlib_dist")
        src = os.path.join(td, "stdlib_dist.cpp")
        with open(src, "w") as f:
            f.write(SRC)
        subprocess.run(["g++", "-O2", "-std=c++17", "-w", src, "-o", exe], check=True)
        out = subprocess.run([exe], input="\n".join(lines) + "\n", capture_output=True, text=True,
                             check=True).stdout.split("\n")
    mt_first = np.array([[int(v) for v in out[i].split()] for i in range(len(seeds))], np.uint32)
    mt_10000 = np.uint32(int(out[len(seeds)]))
    draws = np.array([[int(v) for v in out[len(seeds) + 1 + c].split()] for c in range(len(cases))], np.int32)
    w_all = np.zeros((len(cases), max(w.size for _, w in cases)), np.float32)
    for c, (_, w) in enumerate(cases):
        w_all[c, :w.size] = w
    np.savez_compressed(os.path.join(HERE, "libstdcxx_sampler.npz"), seeds=np.array(seeds, np.uint32),
                        mt_first=mt_first, mt_10000=mt_10000, case_seed=np.array([s for s, _ in cases], np.uint32),
                        case_n=np.array([w.size for _, w in cases], np.int32), weights=w_all, draws=draws)
    print("wrote libstdcxx_sampler.npz:", mt_first.shape, draws.shape, "mt19937 10000th", int(mt_10000))


if __name__ == "__main__":
    main()
