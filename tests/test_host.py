"""Host-side checks (no GPU): the library loads and exports every declared
entry point, and its host helpers agree with the oracle."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O

b2 = pytest.importorskip("b2gguf")


def test_library_exports_every_header_symbol():
    names = b2.header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(b2.lib, n)]
    assert not missing, missing
    assert b2.lib.b2_abi_version() == 1


def test_row_bytes():
    assert b2.row_bytes(b2.Q4_0, 4096) == 128 * 18
    assert b2.row_bytes(b2.Q8_0, 4096) == 128 * 34
    assert b2.row_bytes(b2.Q4_K, 4096) == 16 * 144
    assert b2.row_bytes(b2.Q6_K, 4096) == 16 * 210
    assert b2.row_bytes(b2.Q8_K, 4096) == 16 * 292


@pytest.mark.parametrize("theta,hd,p0,n", [(10000.0, 64, 0, 300), (500000.0, 128, 0, 64), (10000.0, 128, -1024, 3)])
def test_rope_table_matches_oracle(theta, hd, p0, n):
    a = b2.rope_table(theta, hd, p0, n)
    b = O.rope_table(theta, hd, p0, n)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_synth_normal_is_seeded_sliceable_and_normal():
    a = b2.synth_normal(7, 200000, std=0.02)
    b = b2.synth_normal(7, 200000, std=0.02)
    assert np.array_equal(a, b)
    c = b2.synth_normal(7, 1000, std=0.02, offset=12345)
    assert np.array_equal(c, a[12345:13345])
    assert abs(a.mean()) < 2e-4 and abs(a.std() - 0.02) < 2e-4
    assert not np.array_equal(a[:1000], b2.synth_normal(8, 1000, std=0.02))


def test_error_reporting_on_bad_arguments():
    with pytest.raises(b2.B2Error):
        b2.quantize_weights(b2.Q4_0, np.zeros((2, 33), np.float32))
    with pytest.raises(b2.B2Error):
        b2.quantize_weights(99, np.zeros((2, 32), np.float32))


def test_context_default_params():
    """llama_context_default_params' counterpart: 4096 positions, one
    sequence, graph replay and the tensor-core prefill on, fp16 K and V
    caches."""
    p = b2.ContextParams()
    b2.lib.b2_context_default_params(ctypes.byref(p))
    assert (p.n_ctx, p.n_seq_max, p.use_graph, p.prefill_gemm) == (4096, 1, 1, 1)
    assert (p.type_k, p.type_v) == (b2.F16, b2.F16)


def test_kv_row_bytes():
    """Cache rows: fp16 values, or Q8_0 / Q4_0 codes + block scales padded
    to a multiple of 16 bytes; other types are refused (0)."""
    assert b2.lib.b2_kv_row_bytes(b2.F16, 128) == 256
    assert b2.lib.b2_kv_row_bytes(b2.Q8_0, 128) == 144
    assert b2.lib.b2_kv_row_bytes(b2.Q8_0, 64) == 80
    assert b2.lib.b2_kv_row_bytes(b2.Q4_0, 128) == 80
    assert b2.lib.b2_kv_row_bytes(b2.Q4_0, 64) == 48
    assert b2.lib.b2_kv_row_bytes(b2.Q4_K, 128) == 0


def test_sampler_default_params_are_mildas():
    """Milda/include/milda/engine.hpp:79-84 and the window of 64
    (Milda/src/engine.cpp:1354-1355)."""
    p = b2.SamplerParams()
    b2.lib.b2_sampler_default_params(ctypes.byref(p))
    assert (p.penalty_last_n, p.top_k, p.seed) == (64, 40, 42)
    assert np.float32(p.penalty_repeat) == np.float32(1.08) and np.float32(p.temperature) == np.float32(0.75)
    assert np.float32(p.top_p) == np.float32(0.90) and np.float32(p.min_p) == np.float32(0.05)
    assert p.penalty_freq == 0.0 and p.penalty_present == 0.0


def test_new_entry_points_refuse_bad_arguments():
    """Argument checks run on the host before anything reaches a GPU."""
    assert b2.lib.b2_moe_route(None, 1, 8, 2, 1, None, None, None) == b2.ERR_INVALID
    fake = ctypes.c_void_p(16)                      # never dereferenced: the checks fail first
    assert b2.lib.b2_moe_route(fake, 1, 300, 8, 1, fake, fake, None) == b2.ERR_INVALID   # > 256 experts
    assert b2.lib.b2_moe_route(fake, 1, 8, 9, 1, fake, fake, None) == b2.ERR_INVALID     # n_used > n_expert
    assert b2.lib.b2_moe_combine(None, None, 1, 2, 8, None, None) == b2.ERR_INVALID
    assert b2.lib.b2_moe_gemv(None, 8, None, 0, 1, None, 2, None, None) == b2.ERR_INVALID
    assert b2.lib.b2_sampler_create(None, None, None) == b2.ERR_INVALID
    assert b2.lib.b2_sampler_accept(None, 1) == b2.ERR_INVALID
    assert b2.lib.b2_attn_decode_typed(None, None, b2.F16, None, b2.F16, None, None, 1, 1, 8, 8, 128, 64, None,
                                       None) == b2.ERR_INVALID
    assert b2.lib.b2_kv_shift_k_typed(None, b2.Q8_0, 0, 8, 128, 64, 0, 8, 1, 10000.0, None) == b2.ERR_INVALID
    ns = ctypes.c_uint64(7)
    assert b2.lib.b2_context_exchange_wait_ns(None, ctypes.byref(ns), 0) == b2.ERR_INVALID


def _write_small_llama(path):
    b2.write_synthetic_llama(str(path), 1, 64, 128, 2, 1, 64, b2.Q8_0, embd_type=b2.Q8_0, out_type=b2.Q8_0, seed=3)
    return path.read_bytes()


def _load_rc(path) -> int:
    h = ctypes.c_void_p()
    rc = b2.lib.b2_model_load(str(path).encode(), None, ctypes.byref(h))
    assert not h.value, "a refused model must not hand out a handle"
    return rc


def test_model_load_refuses_other_architectures(tmp_path):
    """A Qwen2 (or any non-Llama) file would load and compute the wrong
    function (NeoX RoPE, projection biases): the loader refuses it before any
    device work, as llama_model_load_from_file returns null on an unusable
    file (Milda/src/engine.cpp:920-934)."""
    raw = _write_small_llama(tmp_path / "llama.gguf")
    qwen = tmp_path / "qwen2.gguf"
    qwen.write_bytes(raw.replace(b"llama", b"qwen2"))     # architecture and its key prefix
    assert _load_rc(qwen) == -6
    assert "qwen2" in b2.lib.b2_last_error().decode()


def test_model_load_refuses_bias_tensors(tmp_path):
    raw = _write_small_llama(tmp_path / "llama.gguf")
    name = b"blk.0.ffn_up.weight"
    assert raw.count(name) == 1
    biased = tmp_path / "bias.gguf"
    biased.write_bytes(raw.replace(name, b"blk.0.ffn_up.w.bias"))   # same length: only the name changes
    assert _load_rc(biased) == -6
    assert "bias" in b2.lib.b2_last_error().decode()


@pytest.mark.parametrize("cut", [0, 3, 24, 200, "data"])
def test_model_load_refuses_truncated_or_corrupt_files(tmp_path, cut):
    raw = _write_small_llama(tmp_path / "llama.gguf")
    bad = tmp_path / "bad.gguf"
    if cut == "data":
        bad.write_bytes(raw[: len(raw) - 1000])          # tensor data cut short
    else:
        bad.write_bytes(raw[:cut])                       # header cut short
    assert _load_rc(bad) == -4
    bad.write_bytes(b"GGUX" + raw[4:])                   # wrong magic
    assert _load_rc(bad) == -4
    assert _load_rc(tmp_path / "missing.gguf") == -4
