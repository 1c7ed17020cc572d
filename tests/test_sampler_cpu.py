"""The oracle's sampler chain (Milda's rebuild_sampler chain of llama.cpp
samplers) on CPU: its std::mt19937 and std::discrete_distribution are pinned
against the GNU C++ library (tests/golden/libstdcxx_sampler.npz, made by
tests/golden/make_sampler_golden.py) and the C++ standard's check value; the
chain's stages are checked on small hand-made cases."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "libstdcxx_sampler.npz")


def test_mt19937_matches_the_standard_and_libstdcxx():
    g = np.load(GOLDEN)
    assert int(g["mt_10000"]) == 4123659995                 # C++ [rand.predef]: mt19937's 10000th output
    assert int(O.mt19937(5489, 10000)[-1]) == 4123659995
    for s, row in zip(g["seeds"], g["mt_first"]):
        assert np.array_equal(O.mt19937(int(s), 8), row), f"seed {s}"


def test_discrete_distribution_matches_libstdcxx():
    g = np.load(GOLDEN)
    for c in range(len(g["case_seed"])):
        n = int(g["case_n"][c])
        s = O.Sampler(seed=int(g["case_seed"][c]))
        got = [s.draw(g["weights"][c, :n]) for _ in range(64)]
        assert np.array_equal(got, g["draws"][c]), f"case {c}"


def greedy(**kw):
    args = dict(last_n=0, repeat=1.0, top_k=40, top_p=1.0, min_p=0.0, temperature=0.0)
    args.update(kw)
    return O.Sampler(**args)


def test_greedy_and_penalties():
    logits = np.array([1.0, 3.0, 3.0, -2.0], np.float32)
    assert greedy().sample(logits) == 1                       # first of equal maxima
    s = greedy(last_n=4, repeat=2.0)
    s.accept(1)
    assert s.sample(logits) == 2                              # 3/2 < 3: token 2 wins
    s = greedy(last_n=4, repeat=2.0)
    for t in (1, 2):
        s.accept(t)
    assert s.sample(logits) == 1                              # both halved: first again
    s = greedy(last_n=2, repeat=10.0)
    for t in (1, 0, 3):                                       # token 1 falls out of a window of 2
        s.accept(t)
    assert s.sample(logits) == 1
    s = greedy(last_n=4, repeat=1.0, present=5.0)
    s.accept(1)
    assert s.sample(logits) == 2


def test_sampling_stages():
    logits = np.array([0.0, 5.0, 4.9, -30.0, 1.0], np.float32)
    # top_k 1 keeps only the largest logit whatever the seed
    for seed in range(5):
        assert O.Sampler(last_n=0, top_k=1, top_p=1.0, min_p=0.0, temperature=1.0, seed=seed).sample(logits) == 1
    # min_p prunes everything below the largest + log(p)
    s = O.Sampler(last_n=0, top_k=5, top_p=1.0, min_p=0.5, temperature=1.0, seed=3)
    assert {s.sample(logits) for _ in range(200)} == {1, 2}
    # top_p small enough keeps the top candidate only
    s = O.Sampler(last_n=0, top_k=5, top_p=0.3, min_p=0.0, temperature=1.0, seed=3)
    assert {s.sample(logits) for _ in range(50)} == {1}
    # the same seed gives the same tokens; reset restarts the generator
    a = O.Sampler(last_n=0, top_k=5, top_p=1.0, min_p=0.0, temperature=3.0, seed=9)
    first = [a.sample(logits) for _ in range(30)]
    a.reset()
    assert [a.sample(logits) for _ in range(30)] == first
    assert len(set(first)) > 1
