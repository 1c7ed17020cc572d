"""GPU parity of the single ops against the CPU oracle, through the C ABI.

Bit-exact: activation codes and scales, integer block dots, dequantized
weights, and the GEMV outputs against the oracle's reference-order matmul
(orc_matmul: one vec_dot per row, blocks added in order, as the reference's
matmul_quantized).  The relative check |gpu − oracle| <= 1e-4 ·
max(|oracle|, rms(row)) is the reference's own tolerance, kept beside it."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")

TOL = 1e-4


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _rel_ok(got, want, tol=TOL):
    got = np.atleast_2d(got)
    want = np.atleast_2d(want)
    rms = np.sqrt(np.mean(want.astype(np.float64) ** 2, axis=-1, keepdims=True))
    bound = tol * np.maximum(np.abs(want), rms)
    err = np.abs(got - want)
    return bool(np.all(err <= bound)), float(np.max(err / np.maximum(bound / tol, 1e-30)))


def _edge_acts(k, rng, n=8):
    x = rng.standard_normal((n, k)).astype(np.float32)
    x[0] = 0.0
    x[1, :32] = np.tile([1.0, -1.0], 16)
    x[2] *= 1e-6
    x[3] *= 1e4
    x[4, 3] = 50.0
    return x


@pytest.mark.parametrize("k", [32, 256, 4096, 5632])
def test_quantize_act_q8_0_bit_exact(k):
    rng = np.random.default_rng(k)
    x = _edge_acts(k, rng)
    got = b2.quantize_act(b2.Q8_0, x)
    assert np.array_equal(got, O.quantize_q8_0(x))


@pytest.mark.parametrize("k", [256, 4096, 14336])
def test_quantize_act_q8_k_bit_exact(k):
    rng = np.random.default_rng(k + 1)
    x = _edge_acts(k, rng)
    x[5, :256] = np.tile([2.0, -2.0], 128)
    got = b2.quantize_act(b2.Q8_K, x)
    assert np.array_equal(got, O.quantize_q8_k(x))


def _weights(t, n, k, seed):
    w = b2.synth_normal(seed, n * k, std=0.02).reshape(n, k)
    return b2.quantize_weights(t, w)


TYPES = [b2.Q4_0, b2.Q8_0, b2.Q4_K, b2.Q6_K]


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k", [(7, 256), (33, 4096), (16, 5632), (3, 14336)])
def test_upload_dequantize_bit_exact(t, n, k):
    q = _weights(t, n, k, 11)
    m = b2.QMatrix(t, q, n, k)
    assert np.array_equal(_bits(m.dequantize()), _bits(O.dequantize(t, q, k)))


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("k", [256, 4096, 5632])
def test_block_dots_bit_exact(t, k):
    n = 5
    q = _weights(t, n, k, 12)
    m = b2.QMatrix(t, q, n, k)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(k).astype(np.float32)
    xq = O.quantize_act(t, x)[0]
    for row in (0, n - 1):
        got = m.block_dots(row, x)
        want = O.block_dots(t, q[row], xq, k)
        if t == b2.Q4_K:
            assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
        else:
            assert np.array_equal(got, want)


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k", [(1, 256), (100, 2048), (257, 4096), (64, 5632), (48, 14336)])
@pytest.mark.parametrize("n_tok", [1, 2, 3, 8])
def test_gemv_matches_oracle(t, n, k, n_tok):
    q = _weights(t, n, k, 21)
    m = b2.QMatrix(t, q, n, k)
    rng = np.random.default_rng(n * 7 + k + n_tok)
    x = rng.standard_normal((n_tok, k)).astype(np.float32)
    got = m.gemv(x)
    want = O.gemv(t, q, n, k, x)
    ok, worst = _rel_ok(got, want)
    assert ok, f"worst relative error {worst:.3e}"
    assert np.array_equal(_bits(got), _bits(want)), "not bit-exact with the reference order"


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k", [(6144, 4096), (2048, 14336)])
@pytest.mark.parametrize("n_tok", [1, 3, 8])
def test_gemv_many_items_per_cta(t, n, k, n_tok):
    """A few items per SM: the warps of a group split each item's units and
    pass the partial sums on in unit order, with several chunks per warp so
    that the stage rings wrap: bit-exact with the reference order."""
    q = _weights(t, n, k, 41)
    m = b2.QMatrix(t, q, n, k)
    x = np.random.default_rng(n + k + n_tok).standard_normal((n_tok, k)).astype(np.float32)
    got = m.gemv(x)
    assert np.array_equal(_bits(got), _bits(O.gemv(t, q, n, k, x))), "not bit-exact with the reference order"


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k,n_tok", [(9480, 1024, 1), (9480, 1024, 2), (19000, 1024, 3), (19000, 1024, 5),
                                       (18945, 2048, 7), (28672, 4096, 8)])
def test_gemv_whole_items(t, n, k, n_tok):
    """More than eight items per SM: every warp folds whole items (8-row
    tiles for 1-2 tokens; for 3..8 tokens tile pairs, the 16 rows of two
    tiles as the M of one rows-as-M mma, an odd tile count leaving the last
    pair one tile short).  Bit-exact with the reference order."""
    q = _weights(t, n, k, 43)
    m = b2.QMatrix(t, q, n, k)
    x = np.random.default_rng(n + k + n_tok).standard_normal((n_tok, k)).astype(np.float32)
    got = m.gemv(x)
    assert np.array_equal(_bits(got), _bits(O.gemv(t, q, n, k, x))), "not bit-exact with the reference order"


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("n,k,n_tok,n_mat", [(4096, 4096, 1, 5), (200, 2048, 2, 3), (8, 512, 1, 64),
                                             (1000, 1024, 2, 2), (2048, 14336, 1, 2)])
def test_gemv_multi_matches_single(t, n, k, n_tok, n_mat):
    """One launch over several matrices (distinct weights, shared x): every
    output bit-identical to that matrix's own GEMV, and in the reference order."""
    mats, qs = [], []
    for i in range(n_mat):
        q = _weights(t, n, k, 100 + i)
        qs.append(q)
        mats.append(b2.QMatrix(t, q, n, k))
    x = np.random.default_rng(n + k + n_mat).standard_normal((n_tok, k)).astype(np.float32)
    xd = b2.DeviceBuffer.from_array(x)
    ys = [b2.DeviceBuffer(n_tok * n * 4) for _ in range(n_mat)]
    b2.gemv_multi(mats, xd, n_tok, ys)
    for i in (0, n_mat // 2, n_mat - 1):
        got = ys[i].download(np.float32).reshape(n_tok, n)
        assert np.array_equal(_bits(got), _bits(mats[i].gemv(x))), f"matrix {i} differs from its own GEMV"
        assert np.array_equal(_bits(got), _bits(O.gemv(t, qs[i], n, k, x))), f"matrix {i}: not the reference order"


def test_gemv_multi_rejects_mixed_shapes_and_batches():
    a = b2.QMatrix(b2.Q4_0, _weights(b2.Q4_0, 64, 256, 1), 64, 256)
    c = b2.QMatrix(b2.Q4_0, _weights(b2.Q4_0, 72, 256, 2), 72, 256)
    xd = b2.DeviceBuffer.from_array(np.zeros((3, 256), np.float32))
    ys = [b2.DeviceBuffer(3 * 72 * 4) for _ in range(2)]
    with pytest.raises(Exception):
        b2.gemv_multi([a, c], xd, 1, ys)
    with pytest.raises(Exception):
        b2.gemv_multi([a, a], xd, 3, ys)


def test_gemv_config1_q4_0_4096():
    """Q4_0 GEMV 4096x4096, batch 1: W N(0,0.02) seed 0, x N(0,1) seed 1."""
    n = k = 4096
    q = _weights(b2.Q4_0, n, k, 0)
    x = b2.synth_normal(1, k).reshape(1, k)
    m = b2.QMatrix(b2.Q4_0, q, n, k)
    got = m.gemv(x)
    want = O.gemv(O.Q4_0, q, n, k, x)
    ok, worst = _rel_ok(got, want)
    assert ok, worst
    assert np.array_equal(_bits(got), _bits(want)), "not bit-exact with the reference order"


def test_gemv_device_entry_point_and_repeat():
    t, n, k = b2.Q4_K, 512, 4096
    q = _weights(t, n, k, 31)
    m = b2.QMatrix(t, q, n, k)
    x = np.random.default_rng(0).standard_normal((4, k)).astype(np.float32)
    xd = b2.DeviceBuffer.from_array(x)
    yd = b2.DeviceBuffer(4 * n * 4)
    outs = []
    for _ in range(3):
        m.gemv_device(xd, 4, yd)
        outs.append(yd.download(np.float32).reshape(4, n))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    assert np.array_equal(_bits(outs[0]), _bits(O.gemv(t, q, n, k, x)))


def test_reference_fuzz_replay_on_gpu():
    """The reference test's XorShift32 fuzz inputs (seed 0x13572468) through the
    GPU quantizer and GEMV: codes bit-exact, dots within the reference's own
    1e-4 relative error (Singularity/tests/test_and_bench_a5.cpp:518-600)."""
    from tests.xorshift import XorShift32, rel_error
    rng = XorShift32(0x13572468)
    rows, k = 64, 128
    x = np.array([[rng.next_f32() for _ in range(k)] for _ in range(rows)], np.float32)
    assert np.array_equal(b2.quantize_act(b2.Q8_0, x), O.quantize_q8_0(x))
    w = np.array([[rng.next_f32() for _ in range(k)] for _ in range(rows)], np.float32)
    for t in (b2.Q4_0, b2.Q8_0):
        q = b2.quantize_weights(t, w)
        m = b2.QMatrix(t, q, rows, k)
        got = m.gemv(x[:8])
        want = O.gemv(t, q, rows, k, x[:8])
        errs = [rel_error(a, b) for a, b in zip(got.ravel(), want.ravel())]
        assert max(errs) <= 1e-4
        assert np.array_equal(_bits(got), _bits(want))


def test_expired_flag_wait_reports_status_and_device_stays_usable():
    """The exchange's bounded wait, run on flags that nothing raises: the
    kernel gives up after its wall-clock bound (2 s), stores the expiry
    status and returns; the stream and the context keep working.  With the
    flags raised the same wait returns at once with no status."""
    import time

    flags = b2.DeviceBuffer.from_array(np.zeros(2, np.uint64))
    status = b2.DeviceBuffer.from_array(np.zeros(1, np.int32))
    t0 = time.perf_counter()
    b2.check(b2.lib.b2_flag_wait(flags.ptr, 2, 1, status.ptr, None), "flag_wait")
    b2.check(b2.lib.b2_stream_synchronize(None), "sync")
    waited = time.perf_counter() - t0
    assert int(status.download(np.int32)[0]) == 3          # B2_WAIT_EXPIRED
    assert 1.5 < waited < 30.0, waited
    flags.upload(np.array([1, 5], np.uint64))
    status.zero()
    t0 = time.perf_counter()
    b2.check(b2.lib.b2_flag_wait(flags.ptr, 2, 1, status.ptr, None), "flag_wait")
    b2.check(b2.lib.b2_stream_synchronize(None), "sync")
    assert int(status.download(np.int32)[0]) == 0
    assert time.perf_counter() - t0 < 1.0
    # the device still computes correctly
    rng = np.random.default_rng(9)
    n, k = 64, 256
    q = b2.quantize_weights(b2.Q8_0, (rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = rng.standard_normal((1, k)).astype(np.float32)
    y = b2.QMatrix(b2.Q8_0, q, n, k).gemv(x)
    assert np.array_equal(_bits(y), _bits(O.gemv(O.Q8_0, q, n, k, x)))
