"""The on-device sampler chain against the oracle's, through the C ABI.

Milda's chain (rebuild_sampler, Milda/src/engine.cpp:1321-1384): penalties
over the last accepted tokens, then greedy, or top_k, top_p, min_p,
temperature and dist with a seeded std::mt19937.  Every draw must give the
oracle's token, step after step (the generators advance together), over
vocabularies of 7 to 128256 entries, across the generator's twist, with
Milda's second accept after each draw, and in the device-resident sampled
generation loop against a host loop over the same logits."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")

CHAINS = {
    "milda": dict(),
    "greedy_penalty": dict(temperature=0.0, penalty_repeat=1.3),
    "top_k_1": dict(top_k=1, temperature=1.0),
    "wide": dict(top_k=256, top_p=1.0, min_p=0.0, temperature=1.7, penalty_last_n=0),
    "present_freq": dict(penalty_freq=0.25, penalty_present=0.5, temperature=1.2, top_p=0.97, seed=7),
    "hot_top_p": dict(temperature=2.5, top_p=0.5, min_p=0.0, seed=123456789),
}


def oracle_sampler(p: "b2.SamplerParams") -> O.Sampler:
    return O.Sampler(last_n=p.penalty_last_n, repeat=p.penalty_repeat, freq=p.penalty_freq,
                     present=p.penalty_present, top_k=p.top_k, top_p=p.top_p, min_p=p.min_p,
                     temperature=p.temperature, seed=p.seed)


@pytest.fixture(scope="module")
def ctx(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("s") / "tiny.gguf")
    b2.write_synthetic_llama(path, 1, 256, 512, 4, 2, 512, b2.Q8_0, embd_type=b2.Q8_0, out_type=b2.Q8_0, seed=4)
    m = b2.Model(path)
    c = b2.Context(m, n_ctx=96, n_seq=2)
    yield c
    del c, m


@pytest.mark.parametrize("chain", sorted(CHAINS))
@pytest.mark.parametrize("n_vocab", [7, 1000, 32000, 128256])
def test_sampler_matches_oracle(ctx, chain, n_vocab):
    rng = np.random.default_rng(n_vocab)
    gs = b2.Sampler(ctx, **CHAINS[chain])
    os_ = oracle_sampler(gs.params)
    steps = 24 if n_vocab > 32000 else 40
    for step in range(steps):
        # logits with many near-ties among the leaders and repeats of recent tokens
        x = (rng.standard_normal(n_vocab) * 2.0).astype(np.float32)
        x[rng.integers(0, n_vocab, 8)] = np.float32(x.max())
        buf = b2.DeviceBuffer.from_array(x)
        got = gs.sample_logits(buf.ptr, n_vocab)
        want = os_.sample(x)
        assert got == want, f"{chain} vocab {n_vocab} step {step}: device {got}, oracle {want}"
        gs.accept(got)            # Milda accepts the sampled token once more
        os_.accept(want)


def test_sampler_crosses_the_generator_twist(ctx):
    """A draw takes two generator words, so 312 draws use one state of 624
    words; 700 draws cross two twists.  Reset re-seeds both generators."""
    rng = np.random.default_rng(5)
    gs = b2.Sampler(ctx, temperature=1.5, top_k=50, top_p=1.0, min_p=0.0, penalty_last_n=0, seed=2024)
    os_ = oracle_sampler(gs.params)
    x = (rng.standard_normal(300) * 0.5).astype(np.float32)
    buf = b2.DeviceBuffer.from_array(x)
    got = [gs.sample_logits(buf.ptr, 300) for _ in range(700)]
    want = [os_.sample(x) for _ in range(700)]
    assert got == want
    gs.reset()
    os_.reset()
    assert [gs.sample_logits(buf.ptr, 300) for _ in range(20)] == [os_.sample(x) for _ in range(20)]


def test_generate_sampled_matches_host_loop(ctx):
    """Two rows through b2_generate_sampled (no logits leave the device)
    against the host loop b2_decode -> b2_get_logits -> the oracle's chain;
    both accept each drawn token once, as llama_sampler_sample does."""
    rng = np.random.default_rng(1)
    nv = 512
    prompts = [rng.integers(0, nv, 6).tolist(), rng.integers(0, nv, 9).tolist()]
    seeds = [11, 12]
    # device loop
    ctx.kv_clear()
    firsts = []
    for s, pr in enumerate(prompts):
        ctx.decode(pr, pos=np.arange(len(pr)), seq=np.full(len(pr), s), want_logits=2)
        firsts.append(int(ctx.argmax()[0][-1]))
    sams = [b2.Sampler(ctx, seed=sd, temperature=1.1) for sd in seeds]
    # the feed of step 0 is `firsts`; continue at each row's next position
    ids = ctx.generate_sampled(sams, firsts, 20, seq=[0, 1])
    # host loop over the same prefix
    ctx.kv_clear()
    for s, pr in enumerate(prompts):
        ctx.decode(pr, pos=np.arange(len(pr)), seq=np.full(len(pr), s), want_logits=2)
    ors = [oracle_sampler(s.params) for s in sams]
    tok = list(firsts)
    pos = [len(p) for p in prompts]
    for step in range(20):
        ctx.decode(tok, pos=pos, seq=[0, 1], want_logits=1)
        for r in range(2):
            t = ors[r].sample(ctx.logits(r))
            assert t == int(ids[step, r]), f"step {step} row {r}"
            tok[r] = t
        pos = [p + 1 for p in pos]


def test_sampler_sample_host_api(ctx):
    """b2_sampler_sample over the context's last logits equals the oracle's
    draw over b2_get_logits."""
    rng = np.random.default_rng(2)
    ctx.kv_clear()
    gs = b2.Sampler(ctx, seed=99)
    os_ = oracle_sampler(gs.params)
    tok, pos = int(rng.integers(0, 512)), 0
    for step in range(12):
        ctx.decode([tok], pos=[pos], seq=[0], want_logits=1)
        t = gs.sample(-1)
        assert t == os_.sample(ctx.logits(0)), f"step {step}"
        gs.accept(t)
        os_.accept(t)
        tok, pos = t, pos + 1


def test_sampler_greedy_equals_argmax_loop(ctx):
    ctx.kv_clear()
    ctx.decode([5, 6, 7], want_logits=2)
    g = ctx.generate([int(ctx.argmax()[0][-1])], 10)
    ctx.kv_clear()
    ctx.decode([5, 6, 7], want_logits=2)
    first = int(ctx.argmax()[0][-1])
    s = b2.Sampler(ctx, temperature=0.0, penalty_last_n=0)
    assert np.array_equal(ctx.generate_sampled([s], [first], 10), g)


def test_sampler_argument_errors(ctx):
    for kw in (dict(top_k=0, temperature=0.8), dict(top_k=300), dict(penalty_last_n=257),
               dict(penalty_repeat=0.0)):
        with pytest.raises(b2.B2Error):
            b2.Sampler(ctx, **kw)
    s = b2.Sampler(ctx)
    with pytest.raises(b2.B2Error):
        ctx.generate_sampled([s, s], [1, 2], 2, seq=[0, 1])          # one sampler for two rows
    with pytest.raises(b2.B2Error):
        s.accept(10 ** 6)
