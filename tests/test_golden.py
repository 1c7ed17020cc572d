"""Golden-vector pins (CPU): the oracle and the library's host-side weight
quantizers against fixtures from gguf-py 0.19.0 and from the reference's own
scalar ops (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_oracle_dequant_matches_gguf_py_all_types():
    w = _load("weight_quant_gguf.npz")
    k = w["x"].shape[1]
    for t, key in ((O.Q4_0, "q4_0"), (O.Q8_0, "q8_0")):
        got = O.dequantize(t, w[key], k)
        assert np.array_equal(_bits(got), _bits(w[key + "_deq"])), key
    kq = _load("kquant_gguf.npz")
    for t, key in ((O.Q4_K, "q4_k"), (O.Q6_K, "q6_k")):
        k = kq[key + "_deq"].shape[1]
        got = O.dequantize(t, kq[key], k)
        assert np.array_equal(_bits(got), _bits(kq[key + "_deq"])), key


def test_oracle_matches_reference_scalar_fixture():
    g = {key: v for key, v in _load("singularity_ref_ops.npz").items()}
    x, k = g["x"], g["x"].shape[1]
    q8, q4 = g["q8_0"], g["q4_0"]
    assert np.array_equal(O.quantize_q8_0(x), q8)
    n = x.shape[0]
    for r in range(n):
        a = O.lib.orc_vec_dot_q4_0_q8_0(k, q4[r].ctypes.data, q8[(r + 1) % n].ctypes.data)
        assert _bits(a) == _bits(g["dot_q4_0_q8_0"][r])
        b = O.lib.orc_vec_dot_q8_0_q8_0(k, q8[r].ctypes.data, q8[(r + 1) % n].ctypes.data)
        assert _bits(b) == _bits(g["dot_q8_0_q8_0"][r])
        assert np.array_equal(_bits(O.rmsnorm(x[r], g["norm_w"], 1e-5)), _bits(g["rmsnorm"][r]))
        assert np.array_equal(_bits(O.softmax(x[r])), _bits(g["softmax"][r]))


def test_library_weight_quantizer_matches_gguf_py():
    b2 = pytest.importorskip("b2gguf")
    w = _load("weight_quant_gguf.npz")
    x = w["x"]
    assert np.array_equal(b2.quantize_weights(b2.Q4_0, x), w["q4_0"])
    assert np.array_equal(b2.quantize_weights(b2.Q8_0, x), w["q8_0"])


@pytest.mark.parametrize("qt", ["Q4_K", "Q6_K"])
def test_library_kquant_quantizer_round_trip(qt):
    b2 = pytest.importorskip("b2gguf")
    t = getattr(b2, qt)
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)
    q = b2.quantize_weights(t, x)
    deq = O.dequantize(t, q, 1024)
    err = np.sqrt(np.mean((deq - x) ** 2)) / np.sqrt(np.mean(x ** 2))
    # 4-bit affine (Q4_K) and 6-bit symmetric (Q6_K) encodings of N(0, 0.02)
    assert err < (0.12 if qt == "Q4_K" else 0.04), err
    # edge rows: zeros stay zero, constants stay close
    z = np.zeros((2, 256), np.float32)
    z[1] = 0.25
    dz = O.dequantize(t, b2.quantize_weights(t, z), 256)
    assert np.all(dz[0] == 0.0)
    assert np.max(np.abs(dz[1] - 0.25)) < 0.02


def test_oracle_q8_k_properties():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 512)).astype(np.float32)
    x[1] = 0.0
    x[2, :256] = np.tile([2.0, -2.0], 128)   # |max| tie: first element wins
    qb = O.quantize_q8_k(x).reshape(4, 2, 292)
    d = qb[..., 0:4].copy().view(np.float32)[..., 0]
    qs = qb[..., 4:260].copy().view(np.int8)
    bs = qb[..., 260:292].copy().view(np.int16)
    assert np.all(qb[1] == 0)
    assert np.array_equal(bs, qs.reshape(4, 2, 16, 16).astype(np.int32).sum(-1))
    assert qs[2, 0, 0] == -127 and d[2, 0] < 0   # first max is +2 -> iscale = -127/2
    deq = qs.astype(np.float32) * d[..., None]
    assert np.max(np.abs(deq.reshape(4, 512)[0] - x[0])) <= np.max(np.abs(x[0])) / 127 * 0.51 + 1e-6


def test_device_exp_accuracy_against_libm():
    """The shared exp (Cody-Waite + degree-7 Taylor) within 2 ulp of libm's expf."""
    xs = np.concatenate([np.linspace(-103.9, 88.7, 200001, dtype=np.float32),
                         np.random.default_rng(0).standard_normal(50000).astype(np.float32) * 10,
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.72, -87.3, -100.0], np.float32)])
    got = np.array([O.lib.orc_expf_dev(float(v)) for v in xs], np.float32)
    want = np.exp(xs.astype(np.float64)).astype(np.float32)
    fin = np.isfinite(want) & (want > 1.2e-38)
    ulp = np.abs(got[fin].view(np.int32).astype(np.int64) - want[fin].view(np.int32).astype(np.int64))
    assert int(ulp.max()) <= 2, int(ulp.max())
    # subnormal results: within 2 subnormal steps (2 x 2^-149) of libm
    sub = (want > 0) & (want <= 1.2e-38)
    assert sub.any() and float(np.max(np.abs(got[sub].astype(np.float64) - want[sub]))) <= 2 * 2.0 ** -149
    # past the range: 0 below the underflow bound, inf above the overflow bound, NaN passes through
    edges = np.array([-104.0, -150.0, -1e4, 88.73, 100.0, 1e4], np.float32)
    got_e = np.array([O.lib.orc_expf_dev(float(v)) for v in edges], np.float32)
    assert np.array_equal(got_e, np.array([0, 0, 0, np.inf, np.inf, np.inf], np.float32))
    assert np.isnan(O.lib.orc_expf_dev(float("nan")))


@pytest.mark.parametrize("t", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q6_K])
def test_device_order_gemv_close_to_reference_order(t):
    b2 = pytest.importorskip("b2gguf")
    rng = np.random.default_rng(t)
    n, k = 64, 4096
    q = b2.quantize_weights(t, (rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = rng.standard_normal((2, k)).astype(np.float32)
    a = O.gemv(t, q, n, k, x)
    b = O.gemv_dev(t, q, n, k, x)
    assert np.max(np.abs(a - b)) <= 1e-5 * np.max(np.abs(a))


def test_device_order_attention_close_to_reference_order():
    rng = np.random.default_rng(4)
    n_pos, nh, nkv, hd = 700, 8, 2, 128
    kc = rng.standard_normal((n_pos, nkv * hd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((n_pos, nkv * hd)).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    a = O.attn_decode(q, kc, vc, n_pos, nh, nkv, hd)
    b = O.attn_decode_dev(q, kc, vc, n_pos, nh, nkv, hd)
    assert np.max(np.abs(a - b)) <= 1e-5 * np.max(np.abs(a))
