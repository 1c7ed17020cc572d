"""Model files on the host (no GPU): the library's GGUF writer read back by
gguf-py 0.19.0 and by the oracle's parser; the oracle forward on it."""
import numpy as np
import pytest

from oracle import oracle as O

b2 = pytest.importorskip("b2gguf")
gguf = pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("m") / "tiny_q4k.gguf")
    b2.write_synthetic_llama(path, n_layer=2, n_embd=256, n_ff=768, n_head=4, n_head_kv=2, n_vocab=512,
                             wtype=b2.Q4_K, out_type=b2.Q6_K, seed=5, rope_theta=500000.0)
    return path


def test_writer_metadata_and_tensors_read_by_gguf_py(tiny_gguf):
    r = gguf.GGUFReader(tiny_gguf)
    f = r.fields
    assert bytes(f["general.architecture"].parts[-1]).decode() == "llama"
    assert int(f["llama.block_count"].parts[-1][0]) == 2
    assert int(f["llama.attention.head_count_kv"].parts[-1][0]) == 2
    assert float(f["llama.rope.freq_base"].parts[-1][0]) == 500000.0
    names = {t.name: t for t in r.tensors}
    assert names["output.weight"].tensor_type.name == "Q6_K"
    assert names["blk.1.ffn_down.weight"].tensor_type.name == "Q4_K"
    assert list(names["blk.1.ffn_down.weight"].shape) == [768, 256]
    # gguf-py's dequantization and the oracle's agree bit for bit on the file's bytes
    for name, t in (("blk.0.attn_q.weight", O.Q4_K), ("output.weight", O.Q6_K)):
        raw = np.ascontiguousarray(names[name].data).view(np.uint8)
        k = int(names[name].shape[0])
        ref = gguf.dequantize(raw, names[name].tensor_type).reshape(-1, k)
        got = O.dequantize(t, raw, k)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert 0.015 < float(np.std(got)) < 0.025   # N(0, 0.02) weights


def test_oracle_parses_and_runs(tiny_gguf):
    m = O.Model(tiny_gguf)
    assert (m.n_layers, m.dim, m.hidden, m.n_heads, m.n_kv, m.vocab, m.head_dim) == (2, 256, 768, 4, 2, 512, 64)
    m.init_cache(1, 64)
    for p, t in enumerate([1, 7, 300]):
        lg = m.forward(0, t, p, logits=(p == 2))
    assert lg.shape == (512,) and np.all(np.isfinite(lg))


def test_writer_is_deterministic(tmp_path):
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    for p in (a, b):
        b2.write_synthetic_llama(p, 1, 64, 128, 2, 1, 64, b2.Q4_0, seed=3)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_oracle_layer_range_forward_composes(tiny_gguf):
    """Layer-range steps (the bounded CPU-timing samples) compose to the full forward."""
    a, b = O.Model(tiny_gguf), O.Model(tiny_gguf)
    a.init_cache(1, 16)
    b.init_cache(1, 16)
    for p, t in enumerate([3, 9, 411]):
        want = a.forward(0, t, p)
        b.forward_range(0, t, p, 0, 1)
        got = b.forward_range(0, t, p, 1, 2, logits=True)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    b.cache_fill(0x3C00)
    assert np.all(np.isfinite(b.forward(0, 5, 3)))


@pytest.mark.parametrize("gemm_projections", [False, True])
def test_oracle_projection_order_modes(tiny_gguf, gemm_projections):
    """The oracle's GPU-order mode computes a projection in the decode GEMV's
    tile order; with gemm_projections (the order of the tensor-core prefill)
    the same projection takes the reference's row order, while the rest of
    the forward stays in the GPU's order."""
    m = O.Model(tiny_gguf)
    m.set_device_order(True, gemm_projections=gemm_projections)
    m.init_cache(1, 16)
    taps = {}
    m.set_tap(lambda name, layer, a: taps.__setitem__((name, layer), a))
    m.forward(0, 7, 0, logits=False)
    names = {t.name: t for t in gguf.GGUFReader(tiny_gguf).tensors}
    wd = np.ascontiguousarray(names["blk.0.ffn_down.weight"].data).view(np.uint8)   # k = 768: three units
    xq = O.quantize_act(O.Q4_K, taps[("ffn_act", 0)][None, :])[0]
    ref = O.matmul(O.Q4_K, wd, 256, 768, xq)
    dev = O.matmul_dev(O.Q4_K, wd, 256, 768, xq)
    assert not np.array_equal(ref.view(np.uint32), dev.view(np.uint32))   # the two orders differ here
    want = ref if gemm_projections else dev
    assert np.array_equal(taps[("ffn_out", 0)].view(np.uint32), want.view(np.uint32))
