"""Generates the committed golden fixtures in tests/golden/.

Run here, where the third-party checkers exist:
  * gguf-py 0.19.0 (llama.cpp's Python GGUF package, installed in the image):
    its numpy Q4_0 / Q8_0 quantizers (bit-exact with ggml's reference
    quantizers) and its Q4_0 / Q8_0 / Q4_K / Q6_K dequantizers pin the block
    layouts and the weight quantizer;
  * the reference's own scalar ops, compiled from its sources by
    oracle/build_ref.sh (oracle/_ref/libsingularity_ref.so), pin the
    activation quantizer and the block dot products on the reference test's
    own XorShift32 inputs.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import gguf  # noqa: E402
from gguf import GGMLQuantizationType as T  # noqa: E402

from oracle import oracle as O  # noqa: E402
from tests.xorshift import XorShift32  # noqa: E402


def edge_rows(k: int, rng: np.random.Generator) -> np.ndarray:
    rows = [
        np.zeros(k, np.float32),                                   # all zero
        np.where(np.arange(k) == 5, 3.0, 0.0).astype(np.float32),   # single spike
        -np.abs(rng.standard_normal(k)).astype(np.float32),        # negative maxima
        np.tile(np.array([1.0, -1.0], np.float32), k // 2),         # |max| ties of opposite sign
        (rng.standard_normal(k) * 1e-6).astype(np.float32),        # tiny (fp16 subnormal scales)
        (rng.standard_normal(k) * 1e4).astype(np.float32),         # large
        np.full(k, 0.5, np.float32),                               # constant
        rng.uniform(-2, 2, k).astype(np.float32),
    ]
    return np.stack(rows)


def weight_quant_fixture() -> None:
    rng = np.random.default_rng(1234)
    k = 512
    x = np.concatenate([edge_rows(k, rng), (rng.standard_normal((8, k)) * 0.02).astype(np.float32)])
    q4 = gguf.quantize(x, T.Q4_0)
    q8 = gguf.quantize(x, T.Q8_0)
    np.savez_compressed(os.path.join(HERE, "weight_quant_gguf.npz"), x=x, q4_0=q4, q8_0=q8,
                        q4_0_deq=gguf.dequantize(q4, T.Q4_0), q8_0_deq=gguf.dequantize(q8, T.Q8_0))


def random_kquant_blocks(qtype: int, n_rows: int, n_sb: int, rng: np.random.Generator) -> np.ndarray:
    nb = 144 if qtype == T.Q4_K else 210
    raw = rng.integers(0, 256, (n_rows, n_sb, nb), dtype=np.uint8)
    d = (rng.uniform(1e-4, 2e-2, (n_rows, n_sb)) * rng.choice([-1, 1], (n_rows, n_sb))).astype(np.float16)
    if qtype == T.Q4_K:
        raw[..., 0:2] = np.abs(d).view(np.uint8).reshape(n_rows, n_sb, 2)
        dmin = rng.uniform(1e-4, 2e-2, (n_rows, n_sb)).astype(np.float16)
        raw[..., 2:4] = dmin.view(np.uint8).reshape(n_rows, n_sb, 2)
    else:
        raw[..., 208:210] = d.view(np.uint8).reshape(n_rows, n_sb, 2)
    return raw.reshape(n_rows, n_sb * nb)


def kquant_fixture() -> None:
    rng = np.random.default_rng(99)
    q4k = random_kquant_blocks(T.Q4_K, 8, 4, rng)
    q6k = random_kquant_blocks(T.Q6_K, 8, 4, rng)
    np.savez_compressed(os.path.join(HERE, "kquant_gguf.npz"), q4_k=q4k, q6_k=q6k,
                        q4_k_deq=gguf.dequantize(q4k, T.Q4_K), q6_k_deq=gguf.dequantize(q6k, T.Q6_K))


def reference_fixture() -> None:
    ref = O.load_reference()
    if ref is None:
        raise SystemExit("build the reference scalar ops first: bash oracle/build_ref.sh")
    rng = XorShift32(0x13572468)
    n_rows, k = 64, 128
    x = np.array([[rng.next_f32() for _ in range(k)] for _ in range(n_rows)], np.float32)
    x[0] = 0.0
    x[1, 7] = 1.5
    q8 = np.zeros((n_rows, k // 32 * 34), np.uint8)
    for r in range(n_rows):
        xr = np.ascontiguousarray(x[r])
        ref.sref_quantize_row_q8_0(xr.ctypes.data, q8[r].ctypes.data, k)
    q4 = np.zeros((n_rows, k // 32 * 18), np.uint8)
    for r in range(n_rows):
        for b in range(k // 32):
            q4[r, b * 18:b * 18 + 2] = q8[r, b * 34:b * 34 + 2]
            for j in range(16):
                q4[r, b * 18 + 2 + j] = rng.next_u32() & 0xFF
    dot44 = np.zeros(n_rows, np.float32)
    dot88 = np.zeros(n_rows, np.float32)
    for r in range(n_rows):
        dot44[r] = ref.sref_vec_dot_q4_0_q8_0(k, q4[r].ctypes.data, q8[(r + 1) % n_rows].ctypes.data)
        dot88[r] = ref.sref_vec_dot_q8_0_q8_0(k, q8[r].ctypes.data, q8[(r + 1) % n_rows].ctypes.data)
    w = np.array([rng.next_f32() for _ in range(k)], np.float32)
    rms = np.zeros_like(x)
    sm = np.zeros_like(x)
    for r in range(n_rows):
        xr = np.ascontiguousarray(x[r])
        ref.sref_rmsnorm_f32(xr.ctypes.data, w.ctypes.data, rms[r].ctypes.data, k, np.float32(1e-5))
        ref.sref_softmax_f32(xr.ctypes.data, sm[r].ctypes.data, k)
    np.savez_compressed(os.path.join(HERE, "singularity_ref_ops.npz"), x=x, q8_0=q8, q4_0=q4,
                        dot_q4_0_q8_0=dot44, dot_q8_0_q8_0=dot88, norm_w=w, rmsnorm=rms, softmax=sm)


if __name__ == "__main__":
    weight_quant_fixture()
    kquant_fixture()
    reference_fixture()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
