"""Mixture-of-experts FFN pieces on the GPU against the oracle, through the C
ABI: routing (softmax, top-k, weights), the grouped expert GEMV with device
expert ids, and the weighted combination, checked bit for bit; then a whole
routed FFN (gate, up, SiLU·mul, down, combine) of a Qwen3-MoE-like layer
shape against the oracle composed from the same ops."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _dev(a):
    return b2.DeviceBuffer.from_array(np.ascontiguousarray(a))


@pytest.mark.parametrize("n_expert,n_used,norm", [(128, 8, 1), (8, 2, 1), (256, 8, 0), (60, 6, 1), (4, 4, 0)])
def test_moe_route_bit_exact(n_expert, n_used, norm):
    rng = np.random.default_rng(n_expert)
    n_tok = 9
    lg = (rng.standard_normal((n_tok, n_expert)) * 2).astype(np.float32)
    lg[1, :] = 0.5                                   # all equal: the lowest ids win
    lg[2, 5:9] = lg[2].max() + 1.0                   # a tie at the top
    ids_d, w_d = b2.DeviceBuffer(n_tok * n_used * 4), b2.DeviceBuffer(n_tok * n_used * 4)
    ld = _dev(lg)
    b2.check(b2.lib.b2_moe_route(ld.ptr, n_tok, n_expert, n_used, norm, ids_d.ptr, w_d.ptr, None))
    ids = ids_d.download(np.int32).reshape(n_tok, n_used)
    w = w_d.download(np.float32).reshape(n_tok, n_used)
    want_ids, want_w = O.moe_route(lg, n_used, bool(norm))
    assert np.array_equal(ids, want_ids)
    assert np.array_equal(_bits(w), _bits(want_w))
    assert list(ids[1]) == list(range(n_used))


def _stack(t, n_expert, rows, k, seed):
    w = b2.synth_normal(seed, n_expert * rows * k, std=0.02).reshape(n_expert * rows, k)
    return b2.quantize_weights(t, w)


@pytest.mark.parametrize("per_expert", [0, 1])
@pytest.mark.parametrize("t,n_expert,rows,k,n_used", [(b2.Q4_K, 16, 768, 2048, 8), (b2.Q8_0, 8, 512, 1024, 2),
                                                     (b2.Q4_0, 32, 256, 4096, 4), (b2.Q6_K, 6, 128, 768, 3),
                                                     (b2.Q4_K, 8, 256, 14336, 2)])
def test_moe_gemv_bit_exact(t, n_expert, rows, k, n_used, per_expert):
    """Each expert output equals b2_gemv with that expert's own matrix and
    the oracle's reference-order matmul of its GGUF rows, over one input per
    token (gate, up) or one per chosen expert (down; inputs over 8192 values
    take one launch per expert)."""
    rng = np.random.default_rng(rows + k + per_expert)
    n_tok = 3
    q = _stack(t, n_expert, rows, k, 7)
    stack = b2.QMatrix(t, q, n_expert * rows, k)
    x = rng.standard_normal((n_tok, n_used, k) if per_expert else (n_tok, k)).astype(np.float32)
    ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tok)]).astype(np.int32)
    xd, idd, yd = _dev(x), _dev(ids), b2.DeviceBuffer(n_tok * n_used * rows * 4)
    b2.check(b2.lib.b2_moe_gemv(stack.h, n_expert, xd.ptr, per_expert, n_tok, idd.ptr, n_used, yd.ptr, None))
    y = yd.download(np.float32).reshape(n_tok, n_used, rows)
    rb = O.row_bytes(t, k)
    qr = q.reshape(n_expert * rows, rb)
    for e in sorted(set(ids.ravel().tolist())):
        we = qr[e * rows:(e + 1) * rows]
        me = b2.QMatrix(t, we, rows, k)
        for tt in range(n_tok):
            for j in np.nonzero(ids[tt] == e)[0]:
                xin = x[tt, j] if per_expert else x[tt]
                own = me.gemv(xin)[0]
                ref = O.gemv(t, we, rows, k, xin)[0]
                assert np.array_equal(_bits(y[tt, j]), _bits(own)), f"expert {e} token {tt}: not b2_gemv's"
                assert np.array_equal(_bits(y[tt, j]), _bits(ref)), f"expert {e} token {tt}: not the oracle's"


def test_moe_combine_bit_exact():
    rng = np.random.default_rng(3)
    n_tok, n_used, n = 4, 8, 2048
    y = rng.standard_normal((n_tok, n_used, n)).astype(np.float32)
    w = rng.random((n_tok, n_used)).astype(np.float32)
    out = b2.DeviceBuffer(n_tok * n * 4)
    yd, wd = _dev(y), _dev(w)
    b2.check(b2.lib.b2_moe_combine(yd.ptr, wd.ptr, n_tok, n_used, n, out.ptr, None))
    got = out.download(np.float32).reshape(n_tok, n)
    for t in range(n_tok):
        assert np.array_equal(_bits(got[t]), _bits(O.moe_combine(y[t], w[t])))


def test_moe_ffn_layer_bit_exact():
    """A routed FFN of a Qwen3-MoE-like shape (d 2048, expert FFN 768, 128
    experts, 8 used), Q4_K experts: router logits -> route -> gate and up
    expert GEMVs -> SiLU·mul -> down expert GEMV -> combine, all on the
    device, against the oracle composed from the reference-order ops."""
    rng = np.random.default_rng(8)
    d, ff, n_expert, n_used, n_tok = 2048, 768, 128, 8, 2
    gate = _stack(b2.Q4_K, n_expert, ff, d, 21)
    up = _stack(b2.Q4_K, n_expert, ff, d, 22)
    down = _stack(b2.Q4_K, n_expert, d, ff, 23)
    router = b2.quantize_weights(b2.Q8_0, b2.synth_normal(24, n_expert * d, std=0.05).reshape(n_expert, d))
    mg, mu, md = (b2.QMatrix(b2.Q4_K, gate, n_expert * ff, d), b2.QMatrix(b2.Q4_K, up, n_expert * ff, d),
                  b2.QMatrix(b2.Q4_K, down, n_expert * d, ff))
    mr = b2.QMatrix(b2.Q8_0, router, n_expert, d)
    x = rng.standard_normal((n_tok, d)).astype(np.float32)
    # device
    xd = _dev(x)
    lgd = b2.DeviceBuffer(n_tok * n_expert * 4)
    mr.gemv_device(xd, n_tok, lgd)
    idd, wd = b2.DeviceBuffer(n_tok * n_used * 4), b2.DeviceBuffer(n_tok * n_used * 4)
    b2.check(b2.lib.b2_moe_route(lgd.ptr, n_tok, n_expert, n_used, 1, idd.ptr, wd.ptr, None))
    gd, ud = b2.DeviceBuffer(n_tok * n_used * ff * 4), b2.DeviceBuffer(n_tok * n_used * ff * 4)
    b2.check(b2.lib.b2_moe_gemv(mg.h, n_expert, xd.ptr, 0, n_tok, idd.ptr, n_used, gd.ptr, None))
    b2.check(b2.lib.b2_moe_gemv(mu.h, n_expert, xd.ptr, 0, n_tok, idd.ptr, n_used, ud.ptr, None))
    g = gd.download(np.float32).reshape(n_tok, n_used, ff)
    u = ud.download(np.float32).reshape(n_tok, n_used, ff)
    act = np.stack([[O.silu_mul(g[t, j], u[t, j]) for j in range(n_used)] for t in range(n_tok)])
    ad = _dev(act)
    ids = idd.download(np.int32).reshape(n_tok, n_used)
    # the down projection: expert j of token t over act[t, j] (an input per expert)
    dd = b2.DeviceBuffer(n_tok * n_used * d * 4)
    b2.check(b2.lib.b2_moe_gemv(md.h, n_expert, ad.ptr, 1, n_tok, idd.ptr, n_used, dd.ptr, None))
    outd = b2.DeviceBuffer(n_tok * d * 4)
    b2.check(b2.lib.b2_moe_combine(dd.ptr, wd.ptr, n_tok, n_used, d, outd.ptr, None))
    got = outd.download(np.float32).reshape(n_tok, d)
    # oracle
    lg = O.gemv(b2.Q8_0, router, n_expert, d, x)
    o_ids, o_w = O.moe_route(lg, n_used, True)
    assert np.array_equal(o_ids, ids)
    gr = gate.reshape(n_expert * ff, -1)
    ur = up.reshape(n_expert * ff, -1)
    dr = down.reshape(n_expert * d, -1)
    for t in range(n_tok):
        ys = []
        for j, e in enumerate(o_ids[t]):
            gg = O.gemv(b2.Q4_K, gr[e * ff:(e + 1) * ff], ff, d, x[t])[0]
            uu = O.gemv(b2.Q4_K, ur[e * ff:(e + 1) * ff], ff, d, x[t])[0]
            a = O.silu_mul(gg, uu)
            assert np.array_equal(_bits(a), _bits(act[t, j]))
            ys.append(O.gemv(b2.Q4_K, dr[e * d:(e + 1) * d], d, ff, a)[0])
        want = O.moe_combine(np.stack(ys), o_w[t])
        assert np.array_equal(_bits(got[t]), _bits(want)), f"token {t}"
