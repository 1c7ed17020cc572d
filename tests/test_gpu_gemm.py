"""GPU parity of the tensor-core prefill GEMMs (b2_gemm, Q4_K and Q8_0
weights) against the oracle's reference-order matmul (orc_matmul: one
vec_dot per row, (super-)blocks added in order).  Bit-exact: the integer
block sums are exact on the tensor cores and the per-block fp32 updates
follow the reference's sequence.

Sizes the oracle finishes in seconds run whole; the 11008 x 4096 x 512
prefill shape is checked bit-exact on a seeded sample of rows (every token)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _weights(n, k, seed, qt=b2.Q4_K):
    w = b2.synth_normal(seed, n * k, std=0.02).reshape(n, k)
    return b2.quantize_weights(qt, w)


def _acts(n_tok, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_tok, k)).astype(np.float32)
    if n_tok >= 5:
        x[0] = 0.0
        x[1, :min(k, 256)] = np.tile([1.0, -1.0], 128)[:min(k, 256)]
        x[2] *= 1e-6
        x[3] *= 1e4
        x[4, 3] = 50.0
    return x


def _oracle(q, n, k, x, rows=None, qt=b2.Q4_K):
    rb = O.row_bytes(qt, k)
    if rows is not None:
        q = np.ascontiguousarray(q.reshape(n, rb)[rows])
        n = len(rows)
    xq = O.quantize_act(qt, x)
    return np.stack([O.matmul(qt, q, n, k, xq[t]) for t in range(x.shape[0])])


@pytest.mark.parametrize("n,k,n_tok", [(128, 256, 1), (8, 512, 3), (200, 4096, 70), (131, 4096, 64),
                                       (257, 11008, 65), (384, 14336, 9)])
def test_gemm_q4_k_bit_exact(n, k, n_tok):
    q = _weights(n, k, 21 + n)
    m = b2.QMatrix(b2.Q4_K, q, n, k)
    x = _acts(n_tok, k, n + k)
    got = m.gemm(x)
    want = _oracle(q, n, k, x)
    assert np.array_equal(_bits(got), _bits(want))


@pytest.mark.parametrize("n,k,n_tok", [(128, 32, 1), (8, 96, 3), (200, 4096, 70), (131, 160, 64),
                                       (257, 11008, 65), (384, 14336, 9), (16, 4096, 130)])
def test_gemm_q8_0_bit_exact(n, k, n_tok):
    q = _weights(n, k, 31 + n, b2.Q8_0)
    m = b2.QMatrix(b2.Q8_0, q, n, k)
    x = _acts(n_tok, k, n + k + 1)
    got = m.gemm(x)
    want = _oracle(q, n, k, x, qt=b2.Q8_0)
    assert np.array_equal(_bits(got), _bits(want))


@pytest.mark.parametrize("qt", [b2.Q4_K, b2.Q8_0])
def test_gemm_prefill_shape_sampled_rows(qt):
    n, k, n_tok = 11008, 4096, 512
    q = _weights(n, k, 5, qt)
    m = b2.QMatrix(qt, q, n, k)
    x = _acts(n_tok, k, 6)
    got = m.gemm(x)
    rows = np.sort(np.random.default_rng(7).choice(n, 48, replace=False))
    rows = np.concatenate([[0, 127, 128, n - 1], rows])
    want = _oracle(q, n, k, x, rows, qt)
    assert np.array_equal(_bits(got[:, rows]), _bits(want))


@pytest.mark.parametrize("qt", [b2.Q4_K, b2.Q8_0])
def test_gemm_matches_gemv_reference_order_within_tolerance(qt):
    """The decode GEMV sums in its tile order; the GEMM in the reference's.
    Both agree to 1e-4 relative (the stated fp32 reordering tolerance)."""
    n, k, n_tok = 96, 4096, 8
    q = _weights(n, k, 9, qt)
    m = b2.QMatrix(qt, q, n, k)
    x = _acts(n_tok, k, 10)
    a = m.gemm(x)
    g = m.gemv(x)
    rms = np.sqrt(np.mean(a.astype(np.float64) ** 2, axis=-1, keepdims=True))
    assert np.all(np.abs(a - g) <= 1e-4 * np.maximum(np.abs(a), rms))
