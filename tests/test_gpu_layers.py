"""GPU layer ops against the oracle through the C ABI: residual add + RMSNorm,
RoPE + fp16 KV store, split-K decode attention (config-3 shapes) and the KV
shift's re-rotation.

Bit-exact: the residual add, RoPE outputs, fp16 K/V stores, the shifted K
rows, and the decode attention against the reference's order (orc_attn_decode:
sequential score dots, softmax with the C library's expf, sequential P·V).
RMSNorm is bit-exact with ggml's double-sum form and within 1e-5 of the
reference's sequential-fp32 scalar ref."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _dev(a):
    return b2.DeviceBuffer.from_array(np.ascontiguousarray(a))


@pytest.mark.parametrize("t", [0, 1, 2, 8, 12, 14])
def test_embed_rows_bit_exact(t):
    rng = np.random.default_rng(t)
    n_vocab, n_embd = 300, 512
    if t == 0:
        table = rng.standard_normal((n_vocab, n_embd)).astype(np.float32).view(np.uint8)
    elif t == 1:
        table = rng.standard_normal((n_vocab, n_embd)).astype(np.float16).view(np.uint8)
    else:
        table = b2.quantize_weights(t, (rng.standard_normal((n_vocab, n_embd)) * 0.02).astype(np.float32))
    toks = np.array(list(range(n_vocab)) + [-1, n_vocab, 7], np.int32)
    keep = [_dev(table), _dev(toks)]
    out = b2.DeviceBuffer(toks.size * n_embd * 4)
    b2.check(b2.lib.b2_embed(t, keep[0].ptr, n_vocab, n_embd, keep[1].ptr, toks.size, out.ptr, None))
    got = out.download(np.float32).reshape(toks.size, n_embd)
    want = O.dequantize(t, table.reshape(n_vocab, -1), n_embd)
    assert np.array_equal(_bits(got[:n_vocab]), _bits(want))
    assert np.array_equal(_bits(got[n_vocab]), _bits(want[0])) and np.array_equal(_bits(got[n_vocab + 1]), _bits(want[0]))


def test_rmsnorm_with_residual():
    rng = np.random.default_rng(0)
    n_rows, n = 8, 4096
    x = rng.standard_normal((n_rows, n)).astype(np.float32)
    dl = rng.standard_normal((n_rows, n)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    xd, dd, wd, od = _dev(x), _dev(dl), _dev(w), b2.DeviceBuffer(x.nbytes)
    b2.check(b2.lib.b2_rmsnorm(xd.ptr, dd.ptr, wd.ptr, od.ptr, n_rows, n, np.float32(1e-5), None))
    xs = xd.download(np.float32).reshape(n_rows, n)
    out = od.download(np.float32).reshape(n_rows, n)
    assert np.array_equal(_bits(xs), _bits(x + dl))
    for r in range(n_rows):
        # bit-exact with ggml's double-sum RMSNorm; within 1e-5 of the
        # reference's sequential-fp32 scalar ref
        assert np.array_equal(_bits(out[r]), _bits(O.rmsnorm_ggml(x[r] + dl[r], w, 1e-5)))
        want = O.rmsnorm(x[r] + dl[r], w, 1e-5)
        assert np.max(np.abs(out[r] - want) / np.maximum(np.abs(want), 1e-3)) < 1e-5


def _cache_to_oracle(cache, s, n_pos):
    """[n_seq][n_kv][cap][hd] -> oracle layout [pos][n_kv*hd] for one sequence."""
    c = cache[s, :, :n_pos, :]                     # [n_kv][n_pos][hd]
    return np.ascontiguousarray(c.transpose(1, 0, 2).reshape(n_pos, -1))


@pytest.mark.parametrize("n_head,n_kv,hd", [(32, 8, 128), (32, 4, 64), (4, 4, 64)])
def test_rope_kv_store_bit_exact(n_head, n_kv, hd):
    rng = np.random.default_rng(1)
    n_tok, cap, n_seq, theta = 5, 64, 3, 10000.0
    qkv = rng.standard_normal((n_tok, (n_head + 2 * n_kv) * hd)).astype(np.float32)
    pos = np.array([0, 7, 63, 12, 12], np.int32)
    seq = np.array([0, 1, 2, 0, 1], np.int32)
    table = b2.rope_table(theta, hd, 0, cap)
    kc = np.zeros((n_seq, n_kv, cap, hd), np.uint16)
    vc = np.zeros_like(kc)
    kd, vd, qo = _dev(kc), _dev(vc), b2.DeviceBuffer(n_tok * n_head * hd * 4)
    keep = [_dev(qkv), _dev(pos), _dev(seq), _dev(table)]
    b2.check(b2.lib.b2_rope_kv_store(keep[0].ptr, n_tok, n_seq, n_head, n_kv, hd, keep[1].ptr, keep[2].ptr,
                                     keep[3].ptr, qo.ptr, kd.ptr, vd.ptr, cap, None))
    q = qo.download(np.float32).reshape(n_tok, n_head * hd)
    kg = kd.download(np.uint16).reshape(kc.shape)
    vg = vd.download(np.uint16).reshape(vc.shape)
    for i in range(n_tok):
        row = qkv[i]
        qw = O.rope_pairs(row[:n_head * hd], table[pos[i]], hd, n_head)
        kw = O.rope_pairs(row[n_head * hd:(n_head + n_kv) * hd], table[pos[i]], hd, n_kv)
        assert np.array_equal(_bits(q[i]), _bits(qw))
        assert np.array_equal(kg[seq[i], :, pos[i], :].ravel(), O.fp32_to_fp16_bits(kw))
        assert np.array_equal(vg[seq[i], :, pos[i], :].ravel(), O.fp32_to_fp16_bits(row[(n_head + n_kv) * hd:]))


@pytest.mark.parametrize("n_q,n_pos,n_head,n_kv,hd", [
    (1, 1, 4, 2, 64), (3, 300, 32, 4, 64), (4, 1000, 32, 8, 128), (1, 4096, 32, 8, 128), (16, 513, 32, 8, 128),
    (16, 4096, 32, 8, 128), (2, 2049, 32, 4, 64), (5, 700, 8, 8, 128), (2, 129, 16, 8, 64)])
def test_attn_decode_matches_oracle(n_q, n_pos, n_head, n_kv, hd):
    rng = np.random.default_rng(n_pos)
    cap = max(n_pos, 64)
    n_seq = n_q
    kc = rng.standard_normal((n_seq, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((n_seq, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((n_q, n_head * hd)).astype(np.float32)
    # queries at different lengths in their own sequences
    pos = np.array([n_pos - 1 - (i * 37) % max(1, n_pos // 2) for i in range(n_q)], np.int32)
    seq = np.arange(n_q, dtype=np.int32)
    out = b2.DeviceBuffer(q.nbytes)
    keep = [_dev(q), _dev(kc), _dev(vc), _dev(pos), _dev(seq)]
    b2.check(b2.lib.b2_attn_decode(keep[0].ptr, keep[1].ptr, keep[2].ptr, keep[3].ptr, keep[4].ptr, n_q,
                                   n_seq, n_head, n_kv, hd, cap, out.ptr, None))
    got = out.download(np.float32).reshape(n_q, -1)
    for i in range(n_q):
        n = int(pos[i]) + 1
        want = O.attn_decode(q[i], _cache_to_oracle(kc, seq[i], n), _cache_to_oracle(vc, seq[i], n), n, n_head,
                             n_kv, hd)
        err = np.max(np.abs(got[i] - want)) / max(float(np.max(np.abs(want))), 1e-6)
        assert err < 1e-4, f"query {i}: rel err {err:.2e}"
        assert np.array_equal(_bits(got[i]), _bits(want)), f"query {i}: not bit-exact with the reference order"


@pytest.mark.parametrize("delta", [-1024, -16, 5])
def test_kv_shift_bit_exact(delta):
    rng = np.random.default_rng(3)
    n_seq, n_kv, cap, hd, theta = 2, 8, 4096, 128, 10000.0
    kc = rng.standard_normal((n_seq, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
    kd = _dev(kc)
    p0, p1 = 1024, 4096
    b2.check(b2.lib.b2_kv_shift_k(kd.ptr, 1, n_kv, hd, cap, p0, p1, delta, np.float32(theta), None))
    got = kd.download(np.uint16).reshape(kc.shape)
    assert np.array_equal(got[0], kc[0])                 # other sequence untouched
    assert np.array_equal(got[1, :, :p0], kc[1, :, :p0])  # positions outside the range untouched
    want = O.kv_shift_k(_cache_to_oracle(kc, 1, cap)[p0:p1], p1 - p0, n_kv, hd, delta, theta)
    assert np.array_equal(_cache_to_oracle(got, 1, cap)[p0:p1], want)


def test_out_of_range_queries_read_nothing():
    """Sequence ids outside [0, n_seq) and positions outside [0, cap) are
    bounds-checked in the kernels: zero outputs, nothing stored, valid
    neighbours unaffected."""
    rng = np.random.default_rng(9)
    n_seq, n_head, n_kv, hd, cap = 2, 8, 2, 64, 64
    kc = rng.standard_normal((n_seq, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((n_seq, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((4, n_head * hd)).astype(np.float32)
    pos = np.array([10, 5, cap, 7], np.int32)
    seq = np.array([0, n_seq, 1, -1], np.int32)
    out = b2.DeviceBuffer(q.nbytes)
    keep = [_dev(q), _dev(kc), _dev(vc), _dev(pos), _dev(seq)]
    b2.check(b2.lib.b2_attn_decode(keep[0].ptr, keep[1].ptr, keep[2].ptr, keep[3].ptr, keep[4].ptr, 4, n_seq, n_head,
                                   n_kv, hd, cap, out.ptr, None))
    got = out.download(np.float32).reshape(4, -1)
    assert np.all(got[1:] == 0.0)
    ref = O.attn_decode(q[0], _cache_to_oracle(kc, 0, 11), _cache_to_oracle(vc, 0, 11), 11, n_head, n_kv, hd)
    assert np.array_equal(_bits(got[0]), _bits(ref))
    qkv = rng.standard_normal((2, (n_head + 2 * n_kv) * hd)).astype(np.float32)
    kd, vd, qo = _dev(np.zeros_like(kc)), _dev(np.zeros_like(vc)), b2.DeviceBuffer(2 * n_head * hd * 4)
    keep = [_dev(qkv), _dev(np.array([3, 3], np.int32)), _dev(np.array([5, 0], np.int32)),
            _dev(b2.rope_table(10000.0, hd, 0, cap))]
    b2.check(b2.lib.b2_rope_kv_store(keep[0].ptr, 2, n_seq, n_head, n_kv, hd, keep[1].ptr, keep[2].ptr, keep[3].ptr,
                                     qo.ptr, kd.ptr, vd.ptr, cap, None))
    assert np.all(qo.download(np.float32).reshape(2, -1)[0] == 0.0)
    kg = kd.download(np.uint16).reshape(kc.shape)
    assert np.all(kg[1] == 0) and np.any(kg[0, :, 3] != 0)
