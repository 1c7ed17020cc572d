"""Quantized KV caches (Milda's default cache_type_k / cache_type_v is Q8_0,
Milda/include/milda/engine.hpp:85-86; Q4_0 is its other choice) on the GPU
against the oracle, through the C ABI.

Rows are stored with the reference's Q8_0 quantizer or ggml's Q4_0 one;
attention over a quantized K quantizes the query to Q8_0 and scores with the
reference's Q8_0·Q8_0 or Q4_0·Q8_0 block dot; a quantized V is dequantized
(exact) before the reference-order P·V;
the shift dequantizes, rotates and re-quantizes K.  Everything is checked bit
for bit: stored rows, attention outputs, shifted rows, and model logits over
prefill, greedy decode, batched sequences, the in-place and compacting KV
shifts and the sequence-state snapshot."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")

TYPES = [(b2.Q8_0, b2.Q8_0), (b2.F16, b2.Q8_0), (b2.Q8_0, b2.F16), (b2.Q4_0, b2.Q4_0), (b2.Q4_0, b2.Q8_0),
         (b2.F16, b2.Q4_0)]
CODE_BYTES = {b2.Q8_0: 32, b2.Q4_0: 16}   # per 32-value block


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _dev(a):
    return b2.DeviceBuffer.from_array(np.ascontiguousarray(a))


def row_bytes(t, hd):
    return int(b2.lib.b2_kv_row_bytes(t, hd))


def to_gpu_rows(t, rows, hd):
    """Oracle rows (fp16 bits, or ggml Q8_0 / Q4_0 blocks) -> the cache's
    rows (codes, then the block scales, zero padding)."""
    rows = np.ascontiguousarray(rows, np.uint8)
    if t == b2.F16:
        return rows
    nb, cb = hd // 32, CODE_BYTES[t]
    blk = rows.reshape(rows.shape[:-1] + (nb, 2 + cb))
    out = np.zeros(rows.shape[:-1] + (row_bytes(t, hd),), np.uint8)
    out[..., :nb * cb] = blk[..., 2:].reshape(rows.shape[:-1] + (nb * cb,))
    out[..., nb * cb:nb * cb + 2 * nb] = blk[..., :2].reshape(rows.shape[:-1] + (2 * nb,))
    return out


def to_oracle_rows(t, rows, hd):
    rows = np.ascontiguousarray(rows, np.uint8)
    if t == b2.F16:
        return rows
    nb, cb = hd // 32, CODE_BYTES[t]
    blk = np.zeros(rows.shape[:-1] + (nb, 2 + cb), np.uint8)
    blk[..., 2:] = rows[..., :nb * cb].reshape(rows.shape[:-1] + (nb, cb))
    blk[..., :2] = rows[..., nb * cb:nb * cb + 2 * nb].reshape(rows.shape[:-1] + (nb, 2))
    return blk.reshape(rows.shape[:-1] + (nb * (2 + cb),))


def random_cache(rng, t, n_seq, n_kv, cap, hd):
    """A cache [n_seq][n_kv][cap] of rows stored from random values."""
    x = rng.standard_normal((n_seq, n_kv, cap, hd), dtype=np.float32)
    return to_gpu_rows(t, O.kv_store_rows(t, x), hd)


def oracle_view(t, cache, s, n_pos, hd):
    """Sequence s of a cache as the oracle's [n_pos][n_kv · row] bytes."""
    c = to_oracle_rows(t, cache[s, :, :n_pos], hd)     # [n_kv][n_pos][orow]
    return np.ascontiguousarray(c.transpose(1, 0, 2)).reshape(n_pos, -1)


@pytest.mark.parametrize("kt,vt", TYPES)
@pytest.mark.parametrize("n_head,n_kv,hd", [(32, 8, 128), (32, 4, 64)])
def test_rope_kv_store_rows_bit_exact(kt, vt, n_head, n_kv, hd):
    rng = np.random.default_rng(hd + kt)
    n_tok, n_seq, cap, theta = 5, 3, 40, 10000.0
    qkv = rng.standard_normal((n_tok, (n_head + 2 * n_kv) * hd)).astype(np.float32)
    pos = np.array([0, 7, 39, 12, 3], np.int32)
    seq = np.array([0, 1, 2, 1, 0], np.int32)
    table = b2.rope_table(theta, hd, 0, cap)
    kc = np.zeros((n_seq, n_kv, cap, row_bytes(kt, hd)), np.uint8)
    vc = np.zeros((n_seq, n_kv, cap, row_bytes(vt, hd)), np.uint8)
    kd, vd, qo = _dev(kc), _dev(vc), b2.DeviceBuffer(n_tok * n_head * hd * 4)
    keep = [_dev(qkv), _dev(pos), _dev(seq), _dev(table)]
    b2.check(b2.lib.b2_rope_kv_store_typed(keep[0].ptr, n_tok, n_seq, n_head, n_kv, hd, keep[1].ptr, keep[2].ptr,
                                           keep[3].ptr, qo.ptr, kd.ptr, kt, vd.ptr, vt, cap, None))
    q = qo.download(np.float32).reshape(n_tok, -1)
    kg = kd.download(np.uint8).reshape(kc.shape)
    vg = vd.download(np.uint8).reshape(vc.shape)
    for i in range(n_tok):
        row = qkv[i]
        assert np.array_equal(_bits(q[i]), _bits(O.rope_pairs(row[:n_head * hd], table[pos[i]], hd, n_head)))
        k = O.rope_pairs(row[n_head * hd:(n_head + n_kv) * hd], table[pos[i]], hd, n_kv).reshape(n_kv, hd)
        v = row[(n_head + n_kv) * hd:].reshape(n_kv, hd)
        assert np.array_equal(to_oracle_rows(kt, kg[seq[i], :, pos[i]], hd), O.kv_store_rows(kt, k))
        assert np.array_equal(to_oracle_rows(vt, vg[seq[i], :, pos[i]], hd), O.kv_store_rows(vt, v))


@pytest.mark.parametrize("kt,vt", TYPES)
@pytest.mark.parametrize("n_q,n_pos,n_head,n_kv,hd", [
    (1, 1, 4, 2, 64), (3, 300, 32, 4, 64), (1, 4096, 32, 8, 128), (16, 4096, 32, 8, 128), (2, 129, 16, 8, 64),
    (5, 700, 8, 8, 128), (2, 2049, 32, 4, 64)])
def test_attn_decode_typed_matches_oracle(kt, vt, n_q, n_pos, n_head, n_kv, hd):
    if kt != vt and n_q * n_pos > 8192:
        pytest.skip("mixed types are covered at the smaller shapes")
    rng = np.random.default_rng(n_pos + 7 * kt + vt)
    cap = max(n_pos, 64)
    n_seq = n_q
    kc = random_cache(rng, kt, n_seq, n_kv, cap, hd)
    vc = random_cache(rng, vt, n_seq, n_kv, cap, hd)
    q = rng.standard_normal((n_q, n_head * hd)).astype(np.float32)
    pos = np.array([n_pos - 1 - (i * 37) % max(1, n_pos // 2) for i in range(n_q)], np.int32)
    seq = np.arange(n_q, dtype=np.int32)
    out = b2.DeviceBuffer(q.nbytes)
    keep = [_dev(q), _dev(kc), _dev(vc), _dev(pos), _dev(seq)]
    b2.check(b2.lib.b2_attn_decode_typed(keep[0].ptr, keep[1].ptr, kt, keep[2].ptr, vt, keep[3].ptr, keep[4].ptr,
                                         n_q, n_seq, n_head, n_kv, hd, cap, out.ptr, None))
    got = out.download(np.float32).reshape(n_q, -1)
    for i in range(n_q):
        n = int(pos[i]) + 1
        want = O.attn_decode_typed(q[i], oracle_view(kt, kc, seq[i], n, hd), kt, oracle_view(vt, vc, seq[i], n, hd),
                                   vt, n, n_head, n_kv, hd)
        assert np.array_equal(_bits(got[i]), _bits(want)), f"query {i}: not bit-exact with the oracle"


@pytest.mark.parametrize("kt", [b2.Q8_0, b2.Q4_0])
@pytest.mark.parametrize("delta", [-1024, 5])
def test_kv_shift_quantized_bit_exact(kt, delta):
    rng = np.random.default_rng(4)
    n_seq, n_kv, cap, hd, theta = 2, 8, 2048, 128, 500000.0
    kc = random_cache(rng, kt, n_seq, n_kv, cap, hd)
    kd = _dev(kc)
    p0, p1 = 512, 2048
    b2.check(b2.lib.b2_kv_shift_k_typed(kd.ptr, kt, 1, n_kv, hd, cap, p0, p1, delta, np.float32(theta), None))
    got = kd.download(np.uint8).reshape(kc.shape)
    assert np.array_equal(got[0], kc[0])
    assert np.array_equal(got[1, :, :p0], kc[1, :, :p0])
    want = O.kv_shift_k_typed(oracle_view(kt, kc, 1, cap, hd)[p0:p1], kt, p1 - p0, n_kv, hd, delta, theta)
    assert np.array_equal(oracle_view(kt, got, 1, cap, hd)[p0:p1], want)


# ---- model level ----------------------------------------------------------------------------

MODELS = {
    # name: (layers, d, ff, heads, kv heads, vocab, wtype, embd type, out type, theta)
    "q4_0_hd64": (2, 256, 768, 4, 2, 512, 2, 2, 2, 10000.0),
    "q4_k_hd128": (2, 512, 1024, 4, 1, 768, 12, 12, 14, 500000.0),
}


@pytest.fixture(scope="module", params=sorted(MODELS))
def model_file(request, tmp_path_factory):
    L, d, ff, nh, nkv, V, wt, et, ot, theta = MODELS[request.param]
    path = str(tmp_path_factory.mktemp("m") / f"{request.param}.gguf")
    b2.write_synthetic_llama(path, L, d, ff, nh, nkv, V, wt, embd_type=et, out_type=ot, seed=13, rope_theta=theta)
    return path


def assert_same(got, want, what):
    if not np.array_equal(_bits(got), _bits(want)):
        raise AssertionError(f"{what}: logits differ ({int(np.sum(got != want))} of {got.size})")


@pytest.mark.parametrize("kt,vt", TYPES)
def test_model_decode_q8_0_cache_bit_exact(model_file, kt, vt):
    """Prefill (through the tensor-core GEMMs where the layers allow) and
    greedy decode of two interleaved sequences over a Q8_0 cache: every
    step's logits equal the oracle's with the same cache types."""
    rng = np.random.default_rng(8)
    n_seq, n_ctx = 2, 160
    om = O.Model(model_file)
    om.set_kv_types(kt, vt)
    om.init_cache(n_seq, n_ctx)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=n_ctx, n_seq=n_seq, type_k=kt, type_v=vt)
    per = 45
    toks = rng.integers(0, om.vocab, (per, n_seq))
    order = [(int(toks[p, s]), p, s) for p in range(per) for s in range(n_seq)]
    ctx.decode([t for t, _, _ in order], pos=[p for _, p, _ in order], seq=[s for _, _, s in order],
               want_logits=2)
    got = ctx.logits(-1)
    for i, (t, p, s) in enumerate(order):
        want = om.forward(s, t, p, logits=(i == len(order) - 1))
    assert_same(got, want, "prompt")
    pos = per
    for step in range(4):
        tk = [int(rng.integers(0, om.vocab)) for _ in range(n_seq)]
        ctx.decode(tk, pos=[pos] * n_seq, seq=list(range(n_seq)), want_logits=1)
        for s in range(n_seq):
            assert_same(ctx.logits(s), om.forward(s, tk[s], pos), f"step {step} sequence {s}")
        pos += 1


@pytest.mark.parametrize("kvt", [b2.Q8_0, b2.Q4_0])
@pytest.mark.parametrize("n_keep", [0, 4])
def test_model_kv_shift_quantized_bit_exact(model_file, n_keep, kvt):
    """Milda's in-place shift over a Q8_0 cache: the ring path (n_keep 0)
    and the compacting path (n_keep 4) re-quantize the rotated K rows as the
    oracle does."""
    rng = np.random.default_rng(2)
    om = O.Model(model_file)
    om.set_kv_types(kvt, kvt)
    om.init_cache(1, 64)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=1, type_k=kvt, type_v=kvt)
    toks = rng.integers(0, om.vocab, 40).tolist()
    ctx.decode(toks, want_logits=2)
    for p, t in enumerate(toks):
        want = om.forward(0, t, p, logits=(p == 39))
    assert_same(ctx.logits(-1), want, "before shift")
    n_discard = 16
    ctx.kv_seq_rm(0, n_keep, n_keep + n_discard)
    ctx.kv_seq_add(0, n_keep + n_discard, -1, -n_discard)
    om.kv_shift(0, n_keep, n_keep + n_discard, 40)
    pos = 40 - n_discard
    for step in range(5):
        t = int(rng.integers(0, om.vocab))
        ctx.decode([t], want_logits=1)
        assert_same(ctx.logits(0), om.forward(0, t, pos), f"after shift step {step}")
        pos += 1


def test_state_snapshot_q8_0_cache(model_file):
    """A Q8_0 cache's snapshot restores bit for bit; a context with other
    cache types refuses it."""
    rng = np.random.default_rng(6)
    gm = b2.Model(model_file)
    ctx = b2.Context(gm, n_ctx=64, n_seq=2, type_k=b2.Q8_0, type_v=b2.Q8_0)
    prompt = rng.integers(0, gm.n_vocab, 17).tolist()
    ctx.decode(prompt, want_logits=0)
    snap = ctx.state_seq_get(0)
    ctx.decode([5], pos=[17], want_logits=1)
    ref = ctx.logits(0)
    ctx.kv_clear()
    assert ctx.state_seq_set(1, snap) == len(snap)
    ctx.decode([5], pos=[17], seq=[1], want_logits=1)
    assert_same(ctx.logits(0), ref, "restored")
    f16 = b2.Context(gm, n_ctx=64, n_seq=1)
    with pytest.raises(b2.B2Error):
        f16.state_seq_set(0, snap)
