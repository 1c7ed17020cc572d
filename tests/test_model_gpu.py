"""Model-level parity on the GPU through the C ABI.

The quantized forward of a random-weight model is chaotic: a last-ulp change
in any fp32 sum can move an activation across a Q8 rounding boundary and the
logits then differ by percent.  The GPU path computes every op in the
reference's order (sequential block sums per row, sequential attention sums,
the C library's expf), so the model is checked bit for bit against the
oracle's reference-order forward: logits of every step, greedy tokens,
batched sequences, long prompts through the tensor-core prefill and the
in-place KV shift."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def assert_same(got, want, what):
    if not np.array_equal(_bits(got), _bits(want)):
        rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
        raise AssertionError(f"{what}: logits differ (max |d|/rms {float(np.max(np.abs(got - want))) / rms:.2e}, "
                             f"{int(np.sum(got != want))} of {got.size})")


MODELS = {
    # name: (layers, d, ff, heads, kv heads, vocab, wtype, embd type, out type, theta)
    "q4_0_hd64": (2, 256, 768, 4, 2, 512, 2, 2, 2, 10000.0),
    "q4_k_hd128": (2, 512, 1024, 4, 1, 768, 12, 12, 14, 500000.0),
    "q8_0_hd64": (2, 256, 512, 4, 4, 256, 8, 8, 8, 10000.0),
}


@pytest.fixture(scope="module", params=sorted(MODELS))
def model_file(request, tmp_path_factory):
    L, d, ff, nh, nkv, V, wt, et, ot, theta = MODELS[request.param]
    path = str(tmp_path_factory.mktemp("m") / f"{request.param}.gguf")
    b2.write_synthetic_llama(path, L, d, ff, nh, nkv, V, wt, embd_type=et, out_type=ot, seed=11, rope_theta=theta)
    return path


def oracle_run(path, n_seq, n_ctx):
    m = O.Model(path)
    m.init_cache(n_seq, n_ctx)
    return m


@pytest.mark.parametrize("n_seq,prefill_gemm", [(1, True), (2, True), (1, False)])
def test_long_prompt_prefill_bit_exact(model_file, n_seq, prefill_gemm):
    """A prompt long enough for the tensor-core prefill: all but the last 8
    tokens of the call go through the GEMM chunks when the layers are Q4_K or
    Q8_0 (the Q4_0 model, and prefill_gemm off, keep the decode step).  The
    last token's logits and the greedy steps after it are bit-exact with the
    oracle's reference-order forward."""
    rng = np.random.default_rng(3)
    n_ctx = 192
    om = O.Model(model_file)
    om.init_cache(n_seq, n_ctx)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=n_ctx, n_seq=n_seq, prefill_gemm=prefill_gemm)
    per = 90 // n_seq
    toks = rng.integers(0, om.vocab, (per, n_seq))
    order = [(int(toks[p, s]), p, s) for p in range(per) for s in range(n_seq)]   # sequences interleaved
    n = len(order)
    ctx.decode([t for t, _, _ in order], pos=[p for _, p, _ in order], seq=[s for _, _, s in order],
               want_logits=2)
    got = ctx.logits(-1)
    for i, (t, p, s) in enumerate(order):
        want = om.forward(s, t, p, logits=(i == n - 1))
    assert_same(got, want, "long prompt")
    s_last, pos = order[-1][2], order[-1][1] + 1
    for step in range(3):
        tok = int(np.argmax(want))
        ctx.decode([tok], pos=[pos], seq=[s_last], want_logits=1)
        got = ctx.logits(0)
        want = om.forward(s_last, tok, pos)
        pos += 1
        assert_same(got, want, f"decode step {step} after the long prompt")


@pytest.mark.parametrize("use_graph", [True, False])
def test_prefill_and_greedy_decode_bit_exact(model_file, use_graph):
    rng = np.random.default_rng(0)
    om = oracle_run(model_file, 1, 128)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=128, n_seq=1, use_graph=use_graph)
    prompt = rng.integers(0, om.vocab, 19).tolist()
    ctx.decode(prompt, want_logits=2)
    got = ctx.logits(-1)
    for p, t in enumerate(prompt):
        want = om.forward(0, t, p, logits=(p == len(prompt) - 1))
    assert_same(got, want, "prefill")
    pos = len(prompt)
    for step in range(12):
        ids, top, margin = ctx.argmax()
        tok = int(ids[-1])                      # greedy pick of the last token of the step
        assert tok == int(np.argmax(want)), f"greedy token differs at step {step}"
        assert top[-1] == np.max(want)
        srt = np.sort(want)
        assert margin[-1] == np.float32(srt[-1] - srt[-2])
        ctx.decode([tok], want_logits=1)
        got = ctx.logits(0)
        want = om.forward(0, tok, pos)
        pos += 1
        assert_same(got, want, f"decode step {step}")


def test_batched_sequences_bit_exact(model_file):
    rng = np.random.default_rng(1)
    n_seq = 3
    om = oracle_run(model_file, n_seq, 64)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=n_seq)
    prompts = [rng.integers(0, om.vocab, n).tolist() for n in (5, 9, 3)]
    for s, pr in enumerate(prompts):
        ctx.decode(pr, pos=list(range(len(pr))), seq=[s] * len(pr), want_logits=2)
        for p, t in enumerate(pr):
            want = om.forward(s, t, p, logits=(p == len(pr) - 1))
        assert_same(ctx.logits(-1), want, f"prompt {s}")
    pos = [len(p) for p in prompts]
    for step in range(4):
        toks = rng.integers(0, om.vocab, n_seq).tolist()
        ctx.decode(toks, pos=pos, seq=list(range(n_seq)), want_logits=1)
        for s in range(n_seq):
            assert_same(ctx.logits(s), om.forward(s, toks[s], pos[s]), f"seq {s} step {step}")
        pos = [p + 1 for p in pos]


@pytest.mark.parametrize("n_keep", [0, 4])
def test_kv_shift_bit_exact(model_file, n_keep):
    """Milda's shift_kv_cache_in_place: seq_rm(n_keep, n_keep+n_discard) then
    seq_add(n_keep+n_discard, -1, -n_discard); later tokens see re-rotated K."""
    rng = np.random.default_rng(2)
    om = oracle_run(model_file, 1, 64)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=1)
    toks = rng.integers(0, om.vocab, 40).tolist()
    ctx.decode(toks, want_logits=2)
    for p, t in enumerate(toks):
        want = om.forward(0, t, p, logits=(p == 39))
    assert_same(ctx.logits(-1), want, "before shift")
    n_discard = 16
    ctx.kv_seq_rm(0, n_keep, n_keep + n_discard)
    ctx.kv_seq_add(0, n_keep + n_discard, -1, -n_discard)
    om.kv_shift(0, n_keep, n_keep + n_discard, 40)
    assert ctx.kv_pos_max(0) == 40 - n_discard - 1
    pos = 40 - n_discard
    for step in range(6):
        t = int(rng.integers(0, om.vocab))
        ctx.decode([t], want_logits=1)
        assert_same(ctx.logits(0), om.forward(0, t, pos), f"after shift step {step}")
        pos += 1
    # a second shift on the same ring (the pinned prefix stays fixed)
    ctx.kv_seq_rm(0, n_keep, n_keep + 8)
    ctx.kv_seq_add(0, n_keep + 8, -1, -8)
    om.kv_shift(0, n_keep, n_keep + 8, pos)
    pos -= 8
    for step in range(3):
        t = int(rng.integers(0, om.vocab))
        ctx.decode([t], want_logits=1)
        assert_same(ctx.logits(0), om.forward(0, t, pos), f"after second shift step {step}")
        pos += 1


def test_eval_callback_reports_intermediates(model_file):
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=16, n_seq=1)
    seen = []
    ctx.set_eval_callback(lambda name, layer, a: seen.append((name, layer, a.size)))
    ctx.decode([1, 2], want_logits=1)
    names = [s[0] for s in seen]
    assert names[0] == "embed" and names[-1] == "result_norm"
    assert ("attn_out", gm.n_layer - 1) in [(n, l) for n, l, _ in seen]
    ctx.set_eval_callback(None)
    ctx.decode([3], want_logits=1)


def test_decode_errors_and_truncation(model_file):
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=16, n_seq=1)
    ctx.decode(list(range(10)), want_logits=0)
    with pytest.raises(b2.B2Error):
        ctx.decode([1], pos=[3])                    # not the next position
    eight = np.zeros(8, np.int32)
    assert b2.lib.b2_decode(ctx.h, eight.ctypes.data, None, None, 8, 0) == b2.NO_KV_SLOT
    ctx.kv_seq_rm(0, 6, -1)                          # suffix removal (Milda excise)
    assert ctx.kv_pos_max(0) == 5
    ctx.decode([1, 2], want_logits=2)
    assert np.all(np.isfinite(ctx.logits(-1)))
    ctx.kv_clear()
    assert ctx.kv_pos_max(0) == -1


@pytest.mark.parametrize("use_graph", [True, False])
def test_device_greedy_generate_bit_exact(model_file, use_graph):
    """b2_generate feeds each row its own argmax on the device: ids equal the
    oracle's greedy continuation and the last step's logits are bit-exact."""
    rng = np.random.default_rng(3)
    n_seq, n_steps = 2, 9
    om = oracle_run(model_file, n_seq, 64)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=n_seq, use_graph=use_graph)
    prompts = [rng.integers(0, om.vocab, n).tolist() for n in (7, 4)]
    first, pos = [], []
    for s, pr in enumerate(prompts):
        ctx.decode(pr, pos=list(range(len(pr))), seq=[s] * len(pr), want_logits=2)
        for p, t in enumerate(pr):
            want = om.forward(s, t, p, logits=(p == len(pr) - 1))
        first.append(int(np.argmax(want)))
        pos.append(len(pr))
    # rows in the opposite order of the sequence ids
    got = ctx.generate(first[::-1], n_steps, seq=[1, 0])
    assert got.shape == (n_steps, n_seq)
    for s in range(n_seq):
        tok = first[s]
        for t in range(n_steps):
            want = om.forward(s, tok, pos[s] + t)
            tok = int(np.argmax(want))
            assert got[t, 1 - s] == tok, f"sequence {s} step {t}"
        assert_same(ctx.logits(1 - s), want, f"sequence {s} last step")
    # the context continues at the next positions
    assert ctx.kv_pos_max(0) == pos[0] + n_steps - 1
    ctx.decode([5], pos=[pos[0] + n_steps], seq=[0], want_logits=1)
    assert_same(ctx.logits(0), om.forward(0, 5, pos[0] + n_steps), "decode after generate")
    rc = b2.lib.b2_generate(ctx.h, np.array([1], np.int32).ctypes.data, None, 1, 64, np.zeros(64, np.int32).ctypes.data)
    assert rc == b2.NO_KV_SLOT
    with pytest.raises(b2.B2Error):
        ctx.generate([1, 2], 2, seq=[0, 0])          # repeated sequence


def test_state_snapshot_restore_bit_exact(model_file):
    """Milda pins its system prompt's state after the first prefill
    (llama_state_seq_get_data, Milda/src/engine.cpp:1487-1492) and restores
    it when partial removal is refused (:1701-1705): after clear + restore
    the next step's logits equal the ones computed before, bit for bit, in
    the same sequence or in another one; a snapshot taken after an in-place
    shift (ring cache) restores the shifted state."""
    rng = np.random.default_rng(5)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=2)
    assert ctx.n_ctx() == 64 and ctx.can_shift()
    prompt = rng.integers(0, gm.n_vocab, 21).tolist()
    ctx.decode(prompt, want_logits=0)
    snap = ctx.state_seq_get(0)
    ctx.decode([7], pos=[21], want_logits=1)
    ref = ctx.logits(0)
    ctx.decode([9, 10, 11], want_logits=0)              # the conversation moves on
    ctx.kv_clear()
    assert ctx.state_seq_set(0, snap) == len(snap)
    assert ctx.kv_pos_max(0) == 20
    ctx.decode([7], pos=[21], want_logits=1)
    assert_same(ctx.logits(0), ref, "restored into its own sequence")
    assert ctx.state_seq_set(1, snap) == len(snap)    # Sutra's prefix cache: into another sequence
    ctx.decode([7], pos=[21], seq=[1], want_logits=1)
    assert_same(ctx.logits(0), ref, "restored into another sequence")
    # shift, snapshot the ring, restore into the other sequence
    ctx.kv_seq_rm(0, 4, 12)
    ctx.kv_seq_add(0, 12, -1, -8)
    shifted = ctx.state_seq_get(0)
    ctx.decode([3], pos=[14], seq=[0], want_logits=1)
    ref2 = ctx.logits(0)
    ctx.state_seq_set(1, shifted)
    ctx.decode([3], pos=[14], seq=[1], want_logits=1)
    assert_same(ctx.logits(0), ref2, "shifted state restored")
    with pytest.raises(b2.B2Error):
        ctx.state_seq_set(0, b"B2KVSEQ\0" + snap[8:40])   # truncated
    with pytest.raises(b2.B2Error):
        ctx.state_seq_set(0, b"XXXXXXXX" + snap[8:])      # not a snapshot
    small = b2.Context(gm, n_ctx=16, n_seq=1)
    assert b2.lib.b2_state_seq_set_data(small.h, 0, snap, len(snap), None) == b2.NO_KV_SLOT


def test_abort_callback_stops_decode_and_generate(model_file):
    """llama_set_abort_callback (Sutra/src/llm_backends.cpp:3017): a callback
    that asks to stop ends b2_decode / b2_generate with status 2 (Sutra maps
    it to Cancelled), and the context stays usable."""
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=1)
    calls = []
    stop = {"now": False}
    ctx.set_abort_callback(lambda: calls.append(1) or stop["now"])
    ctx.decode([1, 2, 3], want_logits=2)
    assert calls, "the callback is polled"
    stop["now"] = True
    assert b2.lib.b2_decode(ctx.h, np.array([4], np.int32).ctypes.data, None, None, 1, 1) == b2.ABORTED
    out = np.zeros(4, np.int32)
    assert b2.lib.b2_generate(ctx.h, np.array([4], np.int32).ctypes.data, None, 1, 4, out.ctypes.data) == b2.ABORTED
    assert ctx.kv_pos_max(0) == 2
    ctx.set_abort_callback(None)
    ctx.decode([4], want_logits=1)
    assert np.all(np.isfinite(ctx.logits(0)))


def test_page_cache_release_keeps_results(model_file):
    """After the upload the model drops its file mapping and evicts the
    file's pages (Milda's eviction of offloaded tensor ranges); a model that
    keeps them computes the same logits, and the file loads again."""
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, 200, 9).tolist()
    out = []
    for keep in (False, True, False):
        gm = b2.Model(model_file, keep_page_cache=keep)
        ctx = b2.Context(gm, n_ctx=32, n_seq=1)
        ctx.decode(prompt, want_logits=2)
        out.append(ctx.logits(-1))
        del ctx, gm
    assert_same(out[0], out[1], "released vs kept page cache")
    assert_same(out[2], out[1], "reloaded after release")
