"""Pins the CPU oracle to the reference's own scalar ops.

The reference's scalar refs (Singularity/tests/test_and_bench_a5.cpp:150-293)
are compiled from its sources into oracle/_ref by oracle/build_ref.sh.  This
replays the reference test's 10 000-iteration parity fuzz
(test_and_bench_a5.cpp:392-620: XorShift32 seed 0x13572468, inputs uniform in
[-2, 2], 64/128-element slices) with the oracle in place of the NEON kernels,
and asks for bit-identical results (the reference asks 1e-4 / ±1 LSB of its
NEON code)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.xorshift import XorShift32, rel_error

REF = O.load_reference()
needs_ref = pytest.mark.skipif(REF is None, reason="reference scalar ops not built (oracle/_ref)")


def _p(a):
    return a.ctypes.data


def _bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


@needs_ref
def test_xorshift_matches_reference_generator():
    n = 4096
    ref = np.zeros(n, np.float32)
    st = np.zeros(1, np.uint32)
    REF.sref_xorshift_fill(0x13572468, _p(ref), n, _p(st))
    rng = XorShift32(0x13572468)
    mine = np.array([rng.next_f32() for _ in range(n)], np.float32)
    assert np.array_equal(_bits(mine), _bits(ref))
    assert rng.state == int(st[0])


@needs_ref
def test_fp16_conversions_match_reference_all_halves():
    h = np.arange(65536, dtype=np.uint16)
    mine = np.array([O.lib.orc_fp16_to_fp32(int(v)) for v in h], np.float32)
    ref = np.array([REF.sref_fp16_to_fp32(int(v)) for v in h], np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(mine), nan)
    assert np.array_equal(_bits(mine)[~nan], _bits(ref)[~nan])
    # independent check of the RNE fp32->fp16 path against numpy's converter
    rng = np.random.default_rng(7)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(5000) * 1e-5).astype(np.float32),     # half subnormals
        (rng.standard_normal(2000) * 6e4).astype(np.float32),      # near overflow
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.0**-25, 2.0**-24 * 1.5,
                  np.inf, -np.inf], np.float32),
    ])
    got = O.fp32_to_fp16_bits(x)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


@needs_ref
def test_reference_fuzz_10000_iterations_bit_exact():
    N = 256
    rng = XorShift32(0x13572468)
    f_in = np.zeros(N, np.float32)
    f_w = np.zeros(N, np.float32)
    for i in range(N):
        f_in[i] = rng.next_f32()
        f_w[i] = rng.next_f32()
    cos_sin = np.zeros(64, np.float32)
    for i in range(0, 64, 2):
        ang = np.float32(i) * np.float32(0.1)
        cos_sin[i] = np.cos(ang, dtype=np.float32)
        cos_sin[i + 1] = np.sin(ang, dtype=np.float32)
    q8_a = O.quantize_q8_0(f_in)[0].copy()
    q8_b = O.quantize_q8_0(f_w)[0].copy()
    q4 = np.zeros((N // 32, 18), np.uint8)
    for b in range(N // 32):
        q4[b, 0:2] = q8_a[b * 34:b * 34 + 2]
        for j in range(16):
            q4[b, 2 + j] = rng.next_u32() & 0xFF
    q8_ref = np.zeros(2 * 34, np.uint8)
    out_o = np.zeros(64, np.float32)
    out_r = np.zeros(64, np.float32)
    max_err = {"q4q8": 0.0, "q8q8": 0.0, "rms": 0.0, "softmax": 0.0, "rope": 0.0}
    for it in range(10000):
        idx = it & (N - 1)
        f_in[idx] = rng.next_f32()
        f_w[idx] = rng.next_f32()
        blk = (it >> 5) & ((N >> 5) - 1)
        d16 = REF.sref_fp32_to_fp16(np.float32(0.05) + np.float32(0.01) * np.float32(it & 7))
        q4[blk, 0] = d16 & 0xFF
        q4[blk, 1] = d16 >> 8
        q4[blk, 2 + (it & 15)] = rng.next_u32() & 0xFF

        O.lib.orc_quantize_row_q8_0(_p(f_in), _p(q8_a), 64)
        REF.sref_quantize_row_q8_0(_p(f_in), _p(q8_ref), 64)
        assert np.array_equal(q8_a[:68], q8_ref), f"quantize_row_q8_0 differs at iter {it}"

        so = O.lib.orc_vec_dot_q4_0_q8_0(128, _p(q4), _p(q8_a))
        sr = REF.sref_vec_dot_q4_0_q8_0(128, _p(q4), _p(q8_a))
        assert _bits(so) == _bits(sr), f"vec_dot_q4_0_q8_0 iter {it}: {so} vs {sr}"
        max_err["q4q8"] = max(max_err["q4q8"], rel_error(so, sr))

        so = O.lib.orc_vec_dot_q8_0_q8_0(128, _p(q8_a), _p(q8_b))
        sr = REF.sref_vec_dot_q8_0_q8_0(128, _p(q8_a), _p(q8_b))
        assert _bits(so) == _bits(sr), f"vec_dot_q8_0_q8_0 iter {it}"

        O.lib.orc_rmsnorm(_p(f_in), _p(f_w), _p(out_o), 64, np.float32(1e-5))
        REF.sref_rmsnorm_f32(_p(f_in), _p(f_w), _p(out_r), 64, np.float32(1e-5))
        assert np.array_equal(_bits(out_o), _bits(out_r)), f"rmsnorm iter {it}"

        n = 64 if (it & 1) else 35
        O.lib.orc_softmax(_p(f_in), _p(out_o), n)
        REF.sref_softmax_f32(_p(f_in), _p(out_r), n)
        assert np.array_equal(_bits(out_o[:n]), _bits(out_r[:n])), f"softmax iter {it}"

        a = f_in[:64].copy()
        b = f_in[:64].copy()
        O.lib.orc_rope_pairs(_p(a), _p(cos_sin), 32, 2)
        REF.sref_rope_f32(_p(b), _p(cos_sin), 32, 2)
        assert np.array_equal(_bits(a), _bits(b)), f"rope iter {it}"
    assert max_err["q4q8"] == 0.0
