"""The allocation-free decode attention entry point, for callers that cannot
allocate device memory while they run (a fixed device-memory budget handed
to the library at start-up, or a real-time decode loop that must not pay an
allocation's latency).  It must give the same result as b2_attn_decode,
bit for bit, and the reference's order (the oracle) for the first query, on
two calls in a row, the second with new inputs over the shared static
scratch, and must refuse requests larger than its built-in scratch.  This
file is collected last."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")


def _dev(a):
    return b2.DeviceBuffer.from_array(np.ascontiguousarray(a))


def _run(fn, q, kc, vc, pos, seq, n_head, n_kv, hd, cap):
    bufs = [_dev(q), _dev(kc), _dev(vc), _dev(pos), _dev(seq)]
    out = b2.DeviceBuffer(q.nbytes)
    n_seq = kc.shape[0]
    rc = fn(bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr, bufs[4].ptr, q.shape[0], n_seq, n_head, n_kv, hd, cap,
            out.ptr, None)
    b2.check(rc, fn.__name__)
    return out.download(np.float32).reshape(q.shape)


@pytest.mark.parametrize("n_q,cap,n_head,n_kv,hd", [(4, 1000, 32, 8, 128), (16, 4096, 32, 8, 128), (3, 300, 32, 4, 64)])
def test_noalloc_attention_matches_allocating_entry_point_twice(n_q, cap, n_head, n_kv, hd):
    rng = np.random.default_rng(cap + n_q)
    for call in range(2):
        kc = rng.standard_normal((n_q, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
        vc = rng.standard_normal((n_q, n_kv, cap, hd)).astype(np.float16).view(np.uint16)
        q = rng.standard_normal((n_q, n_head * hd)).astype(np.float32)
        pos = rng.integers(0, cap, n_q).astype(np.int32)
        seq = np.arange(n_q, dtype=np.int32)
        want = _run(b2.lib.b2_attn_decode, q, kc, vc, pos, seq, n_head, n_kv, hd, cap)
        got = _run(b2.lib.b2_attn_decode_noalloc, q, kc, vc, pos, seq, n_head, n_kv, hd, cap)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {call} differs"
        # query 0 (sequence 0) against the reference's order
        ref = O.attn_decode(q[0], kc[0].transpose(1, 0, 2).reshape(cap, n_kv * hd), vc[0].transpose(1, 0, 2).reshape(
            cap, n_kv * hd), int(pos[0]) + 1, n_head, n_kv, hd)
        assert np.array_equal(got[0].view(np.uint32), ref.view(np.uint32)), f"call {call}: not the reference order"


def test_noalloc_attention_rejects_oversize_requests():
    n_q, n_head, n_kv, hd, cap = 64, 32, 8, 128, 8192      # 64·8·(8192·8 + 4·64)·4 bytes (~134 MB) > 32 MiB
    q = np.zeros((n_q, n_head * hd), np.float32)
    kc = np.zeros((1, n_kv, cap, hd), np.uint16)
    pos = np.zeros(n_q, np.int32)
    seq = np.zeros(n_q, np.int32)
    with pytest.raises(b2.B2Error, match="scratch"):
        _run(b2.lib.b2_attn_decode_noalloc, q, kc, kc, pos, seq, n_head, n_kv, hd, cap)
    q1 = np.zeros((65, n_head * hd), np.float32)   # more queries than B2_NOALLOC_MAX_QUERIES
    with pytest.raises(b2.B2Error):
        _run(b2.lib.b2_attn_decode_noalloc, q1, kc, kc, np.zeros(65, np.int32), np.zeros(65, np.int32),
             n_head, n_kv, hd, 256)
