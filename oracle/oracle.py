"""ctypes wrapper over the CPU oracle (liboracle.so) and the reference's own
scalar ops built from its sources (_ref/libsingularity_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference arm, always as the checker or the timed
CPU baseline, never as the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libsingularity_ref.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 2, 8, 12, 14, 15
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q8_K: (256, 292),
         F32: (1, 4), F16: (1, 2)}

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float


def build() -> None:
    """Compile liboracle.so (and the reference shim when its sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "orc_fp16_to_fp32": (_f, [ctypes.c_uint16]),
        "orc_fp32_to_fp16": (ctypes.c_uint16, [_f]),
        "orc_fp32_to_fp16_row": (None, [_vp, _vp, ctypes.c_int64]),
        "orc_quantize_row_q8_0": (None, [_vp, _vp, _i]),
        "orc_quantize_row_q8_k": (None, [_vp, _vp, _i]),
        "orc_vec_dot_q4_0_q8_0": (_f, [_i, _vp, _vp]),
        "orc_vec_dot_q8_0_q8_0": (_f, [_i, _vp, _vp]),
        "orc_vec_dot_q4_k_q8_k": (_f, [_i, _vp, _vp]),
        "orc_vec_dot_q6_k_q8_k": (_f, [_i, _vp, _vp]),
        "orc_block_dots_q4_0_q8_0": (None, [_i, _vp, _vp, _vp]),
        "orc_block_dots_q8_0_q8_0": (None, [_i, _vp, _vp, _vp]),
        "orc_block_dots_q4_k_q8_k": (None, [_i, _vp, _vp, _vp, _vp]),
        "orc_block_dots_q6_k_q8_k": (None, [_i, _vp, _vp, _vp]),
        "orc_dequantize_row": (None, [_i, _vp, _vp, _i]),
        "orc_rmsnorm": (None, [_vp, _vp, _vp, _i, _f]),
        "orc_rmsnorm_ggml": (None, [_vp, _vp, _vp, _i, _f]),
        "orc_softmax": (None, [_vp, _vp, _i]),
        "orc_rope_pairs": (None, [_vp, _vp, _i, _i]),
        "orc_silu_mul": (None, [_vp, _vp, _i]),
        "orc_rope_table": (None, [_f, _i, _i, _i, _vp]),
        "orc_matmul": (None, [_i, _vp, ctypes.c_int64, _i, _vp, _vp, _i]),
        "orc_attn_decode": (None, [_vp, _vp, _vp, ctypes.c_int64, _i, _i, _i, _i, _vp]),
        "orc_kv_shift_k": (None, [_vp, ctypes.c_int64, _i, _i, _i, _i, _f]),
        "orc_kv_store_row": (None, [_i, _vp, _vp, _i]),
        "orc_kv_store_rows": (None, [_i, _vp, _vp, ctypes.c_int64, _i]),
        "orc_attn_decode_typed": (None, [_vp, _vp, _i, ctypes.c_size_t, _vp, _i, ctypes.c_size_t, _i, _i, _i, _i,
                                         _vp]),
        "orc_kv_shift_k_typed": (None, [_vp, _i, ctypes.c_size_t, _i, _i, _i, _i, _f]),
        "orc_model_set_kv_types": (_i, [_vp, _i, _i]),
        "orc_sampler_new": (_vp, [_i, _f, _f, _f, _i, _f, _f, _f, ctypes.c_uint32]),
        "orc_sampler_free": (None, [_vp]),
        "orc_sampler_reset": (None, [_vp]),
        "orc_sampler_accept": (None, [_vp, ctypes.c_int32]),
        "orc_sampler_sample": (ctypes.c_int32, [_vp, _vp, _i]),
        "orc_mt19937": (None, [ctypes.c_uint32, _vp, _i]),
        "orc_discrete_draw": (_i, [_vp, _vp, _i]),
        "orc_moe_route": (None, [_vp, _i, _i, _i, _vp, _vp]),
        "orc_moe_combine": (None, [_vp, _vp, _i, _i, _vp]),
        "orc_model_open": (_vp, [ctypes.c_char_p]),
        "orc_model_from_memory": (_vp, [_vp, ctypes.c_size_t]),
        "orc_model_free": (None, [_vp]),
        "orc_model_info": (_i, [_vp, _vp, _i]),
        "orc_model_init_cache": (_i, [_vp, _i, _i]),
        "orc_model_forward": (_i, [_vp, _i, ctypes.c_int32, _i, _vp, _i]),
        "orc_model_forward_layers": (_i, [_vp, _i, ctypes.c_int32, _i, _vp, _i, _i]),
        "orc_model_forward_range": (_i, [_vp, _i, ctypes.c_int32, _i, _i, _i, _vp, _i]),
        "orc_model_cache_fill": (None, [_vp, ctypes.c_uint16]),
        "orc_model_set_tp": (_i, [_vp, _i]),
        "orc_model_kv_shift": (_i, [_vp, _i, _i, _i, _i]),
        "orc_model_hidden": (_i, [_vp, _vp, _i]),
        "orc_model_set_tap": (None, [_vp, _vp, _vp]),
        "orc_model_set_device_order": (None, [_vp, _i]),
        "orc_expf_dev": (_f, [_f]),
        "orc_matmul_dev": (None, [_i, _vp, ctypes.c_int64, _i, _vp, _vp, _i, _i]),
        "orc_attn_decode_dev": (None, [_vp, _vp, _vp, ctypes.c_int64, _i, _i, _i, _i, _vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def row_bytes(t: int, k: int) -> int:
    bs, nb = BLOCK[t]
    return k // bs * nb


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of fp32 -> Q8_0 bytes with the reference's activation formula."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.reshape(-1, x.shape[-1])
    out = np.zeros((rows.shape[0], row_bytes(Q8_0, rows.shape[1])), np.uint8)
    for r in range(rows.shape[0]):
        xr = np.ascontiguousarray(rows[r])
        lib.orc_quantize_row_q8_0(_p(xr), _p(out[r]), rows.shape[1])
    return out


def quantize_q8_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.reshape(-1, x.shape[-1])
    out = np.zeros((rows.shape[0], row_bytes(Q8_K, rows.shape[1])), np.uint8)
    for r in range(rows.shape[0]):
        xr = np.ascontiguousarray(rows[r])
        lib.orc_quantize_row_q8_k(_p(xr), _p(out[r]), rows.shape[1])
    return out


def quantize_act(wtype: int, x: np.ndarray) -> np.ndarray:
    return quantize_q8_k(x) if wtype in (Q4_K, Q6_K) else quantize_q8_0(x)


def dequantize(t: int, w: np.ndarray, k: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1, row_bytes(t, k))
    out = np.zeros((w.shape[0], k), np.float32)
    for r in range(w.shape[0]):
        lib.orc_dequantize_row(t, _p(w[r]), _p(out[r]), k)
    return out


def matmul(wtype: int, w: np.ndarray, n_rows: int, k: int, xq: np.ndarray, n_threads: int = 8) -> np.ndarray:
    """y[r] = vec_dot(W row r, xq) for one activation row xq (bytes)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    y = np.zeros(n_rows, np.float32)
    lib.orc_matmul(wtype, _p(w), n_rows, k, _p(xq), _p(y), n_threads)
    return y


def gemv(wtype: int, w: np.ndarray, n_rows: int, k: int, x: np.ndarray, n_threads: int = 8) -> np.ndarray:
    """Full oracle GEMV: quantize each activation row, then matmul. x: [B, k]."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    xq = quantize_act(wtype, x)
    return np.stack([matmul(wtype, w, n_rows, k, xq[b], n_threads) for b in range(x.shape[0])])


def matmul_dev(wtype: int, w: np.ndarray, n_rows: int, k: int, xq: np.ndarray, swiglu: bool = False,
               n_threads: int = 8) -> np.ndarray:
    """The device GEMV's evaluation order for one activation row."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    y = np.zeros(n_rows, np.float32)
    lib.orc_matmul_dev(wtype, _p(w), n_rows, k, _p(xq), _p(y), 1 if swiglu else 0, n_threads)
    return y


def gemv_dev(wtype: int, w: np.ndarray, n_rows: int, k: int, x: np.ndarray, n_threads: int = 8) -> np.ndarray:
    x = np.atleast_2d(np.asarray(x, np.float32))
    xq = quantize_act(wtype, x)
    return np.stack([matmul_dev(wtype, w, n_rows, k, xq[b], False, n_threads) for b in range(x.shape[0])])


def attn_decode_dev(q, kc, vc, n_pos: int, n_heads: int, n_kv: int, hd: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.uint16)
    vc = np.ascontiguousarray(vc, np.uint16)
    out = np.zeros(n_heads * hd, np.float32)
    lib.orc_attn_decode_dev(_p(q), _p(kc), _p(vc), n_kv * hd, n_pos, n_heads, n_kv, hd, _p(out))
    return out


def block_dots(wtype: int, w_row: np.ndarray, xq: np.ndarray, k: int):
    w_row = np.ascontiguousarray(w_row, np.uint8)
    xq = np.ascontiguousarray(xq, np.uint8)
    if wtype == Q4_0:
        out = np.zeros(k // 32, np.int32)
        lib.orc_block_dots_q4_0_q8_0(k, _p(w_row), _p(xq), _p(out))
        return out
    if wtype == Q8_0:
        out = np.zeros(k // 32, np.int32)
        lib.orc_block_dots_q8_0_q8_0(k, _p(w_row), _p(xq), _p(out))
        return out
    if wtype == Q4_K:
        a = np.zeros(k // 256, np.int32)
        b = np.zeros(k // 256, np.int32)
        lib.orc_block_dots_q4_k_q8_k(k, _p(w_row), _p(xq), _p(a), _p(b))
        return a, b
    a = np.zeros(k // 256, np.int32)
    lib.orc_block_dots_q6_k_q8_k(k, _p(w_row), _p(xq), _p(a))
    return a


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib.orc_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def rmsnorm_ggml(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib.orc_rmsnorm_ggml(_p(x), _p(w), _p(out), x.size, eps)
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib.orc_softmax(_p(x), _p(out), x.size)
    return out


def rope_pairs(x: np.ndarray, cos_sin: np.ndarray, head_dim: int, n_heads: int) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    cs = np.ascontiguousarray(cos_sin, np.float32)
    lib.orc_rope_pairs(_p(x), _p(cs), head_dim, n_heads)
    return x


def silu_mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.array(a, np.float32, copy=True, order="C")
    b = np.ascontiguousarray(b, np.float32)
    lib.orc_silu_mul(_p(a), _p(b), a.size)
    return a


def rope_table(theta: float, head_dim: int, p0: int, n_pos: int) -> np.ndarray:
    out = np.zeros((n_pos, head_dim), np.float32)
    lib.orc_rope_table(theta, head_dim, p0, n_pos, _p(out))
    return out


def fp32_to_fp16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.shape, np.uint16)
    lib.orc_fp32_to_fp16_row(_p(x), _p(out), x.size)
    return out


def attn_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_pos: int, n_heads: int, n_kv: int, hd: int) -> np.ndarray:
    """q: [n_heads*hd] fp32; kc/vc: uint16 fp16 bits [n_pos, n_kv*hd]."""
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.uint16)
    vc = np.ascontiguousarray(vc, np.uint16)
    out = np.zeros(n_heads * hd, np.float32)
    lib.orc_attn_decode(_p(q), _p(kc), _p(vc), n_kv * hd, n_pos, n_heads, n_kv, hd, _p(out))
    return out


def kv_shift_k(kc: np.ndarray, n_pos: int, n_kv: int, hd: int, delta: int, theta: float) -> np.ndarray:
    kc = np.array(kc, np.uint16, copy=True, order="C")
    lib.orc_kv_shift_k(_p(kc), n_kv * hd, n_pos, n_kv, hd, delta, theta)
    return kc


def kv_store_rows(t: int, x: np.ndarray) -> np.ndarray:
    """Cache rows in type t's storage (F16 bits or Q8_0 blocks) as bytes:
    x [..., n] fp32 -> uint8 [..., row_bytes(t, n)]."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    out = np.zeros((rows.shape[0], row_bytes(t, n)), np.uint8)
    lib.orc_kv_store_rows(t, _p(rows), _p(out), rows.shape[0], n)
    return out.reshape(x.shape[:-1] + (out.shape[-1],))


def attn_decode_typed(q: np.ndarray, kc: np.ndarray, ktype: int, vc: np.ndarray, vtype: int, n_pos: int,
                      n_heads: int, n_kv: int, hd: int) -> np.ndarray:
    """q: [n_heads*hd] fp32; kc / vc: uint8 [n_pos, n_kv * row_bytes(type, hd)]."""
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.uint8).reshape(n_pos, -1)
    vc = np.ascontiguousarray(vc, np.uint8).reshape(n_pos, -1)
    out = np.zeros(n_heads * hd, np.float32)
    lib.orc_attn_decode_typed(_p(q), _p(kc), ktype, kc.shape[1], _p(vc), vtype, vc.shape[1], n_pos, n_heads, n_kv,
                              hd, _p(out))
    return out


def kv_shift_k_typed(kc: np.ndarray, ktype: int, n_pos: int, n_kv: int, hd: int, delta: int,
                     theta: float) -> np.ndarray:
    kc = np.array(kc, np.uint8, copy=True, order="C").reshape(n_pos, -1)
    lib.orc_kv_shift_k_typed(_p(kc), ktype, kc.shape[1], n_pos, n_kv, hd, delta, theta)
    return kc


def moe_route(logits: np.ndarray, n_used: int, norm: bool = True):
    """Per token (rows of logits): expert ids [n_tok, n_used], weights."""
    lg = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
    ids = np.zeros((lg.shape[0], n_used), np.int32)
    w = np.zeros((lg.shape[0], n_used), np.float32)
    for t in range(lg.shape[0]):
        lib.orc_moe_route(_p(lg[t]), lg.shape[1], n_used, 1 if norm else 0, _p(ids[t]), _p(w[t]))
    return ids, w


def moe_combine(y: np.ndarray, w: np.ndarray) -> np.ndarray:
    """y [n_used, n], w [n_used] -> out [n]."""
    y = np.ascontiguousarray(y, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(y.shape[1], np.float32)
    lib.orc_moe_combine(_p(y), _p(w), y.shape[0], y.shape[1], _p(out))
    return out


def mt19937(seed: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.uint32)
    lib.orc_mt19937(seed, _p(out), n)
    return out


class Sampler:
    """Milda's sampler chain over llama.cpp's samplers (orc_sampler)."""

    def __init__(self, last_n=64, repeat=1.08, freq=0.0, present=0.0, top_k=40, top_p=0.9, min_p=0.05,
                 temperature=0.75, seed=42):
        self.h = lib.orc_sampler_new(last_n, repeat, freq, present, top_k, top_p, min_p, temperature, seed)
        if not self.h:
            raise ValueError("oracle sampler parameters")

    def sample(self, logits: np.ndarray) -> int:
        x = np.ascontiguousarray(logits, np.float32)
        return int(lib.orc_sampler_sample(self.h, _p(x), x.size))

    def accept(self, tok: int) -> None:
        lib.orc_sampler_accept(self.h, tok)

    def reset(self) -> None:
        lib.orc_sampler_reset(self.h)

    def draw(self, p: np.ndarray) -> int:
        """One std::discrete_distribution draw over weights p."""
        x = np.ascontiguousarray(p, np.float32)
        return int(lib.orc_discrete_draw(self.h, _p(x), x.size))

    def __del__(self):
        if getattr(self, "h", None):
            lib.orc_sampler_free(self.h)
            self.h = None


class Model:
    """Oracle Llama forward over a GGUF file or buffer."""

    def __init__(self, path: str | None = None, buf: np.ndarray | None = None):
        self._buf = buf
        if path is not None:
            self.h = lib.orc_model_open(path.encode())
        else:
            assert buf is not None
            self.h = lib.orc_model_from_memory(_p(buf), buf.nbytes)
        if not self.h:
            raise RuntimeError("oracle: GGUF parse failed")
        info = np.zeros(12, np.int32)
        lib.orc_model_info(self.h, _p(info), 12)
        (self.n_layers, self.dim, self.hidden, self.n_heads, self.n_kv, self.vocab,
         self.head_dim, self.ctx_len, self.wtype, self.embd_type, self.out_type, _) = [int(v) for v in info]

    def set_device_order(self, on: bool = True, gemm_projections: bool = False) -> None:
        """GPU kernels' order (on), optionally with the projections in the
        reference's row order, as the tensor-core prefill GEMMs compute them."""
        lib.orc_model_set_device_order(self.h, (2 if gemm_projections else 1) if on else 0)

    def set_kv_types(self, ktype: int, vtype: int) -> None:
        """K and V cache types (F16 or Q8_0); an existing cache restarts empty."""
        if lib.orc_model_set_kv_types(self.h, ktype, vtype) != 0:
            raise ValueError(f"oracle: unsupported cache types {ktype}/{vtype}")

    def init_cache(self, n_seq: int, n_ctx: int) -> None:
        if lib.orc_model_init_cache(self.h, n_seq, n_ctx) != 0:
            raise MemoryError("oracle cache")

    def forward(self, seq: int, token: int, pos: int, logits: bool = True, n_threads: int = 8,
                n_layers: int | None = None):
        out = np.zeros(self.vocab, np.float32) if logits else None
        nl = self.n_layers if n_layers is None else n_layers
        rc = lib.orc_model_forward_layers(self.h, seq, token, pos, _p(out) if logits else None, n_threads, nl)
        if rc != 0:
            raise RuntimeError(f"oracle forward rc={rc}")
        return out

    def set_tp(self, tp: int) -> None:
        """The forward as `tp` tensor-parallel ranks compute it: attention-out
        and FFN-down as per-rank column-slice partials (each in the reference's
        block order, or the tile order in device-order mode) summed in rank
        order."""
        if lib.orc_model_set_tp(self.h, tp) != 0:
            raise ValueError(f"model does not split over {tp} ranks")

    def cache_fill(self, bits: int = 0x3C00) -> None:
        lib.orc_model_cache_fill(self.h, bits)

    def forward_range(self, seq: int, token: int, pos: int, l0: int, l1: int, logits: bool = False,
                      n_threads: int = 8):
        """Layers [l0, l1) from the current residual (embedding when l0 == 0)."""
        out = np.zeros(self.vocab, np.float32) if logits else None
        rc = lib.orc_model_forward_range(self.h, seq, token, pos, l0, l1, _p(out) if logits else None, n_threads)
        if rc != 0:
            raise RuntimeError(f"oracle forward rc={rc}")
        return out

    TAP = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_long,
                           ctypes.c_void_p)

    def set_tap(self, fn) -> None:
        """fn(name, layer, np.ndarray copy) after each op; None removes it."""
        if fn is None:
            self._tap = None
            lib.orc_model_set_tap(self.h, None, None)
            return
        def cb(name, layer, data, n, user):
            fn(name.decode(), layer, np.ctypeslib.as_array(data, shape=(n,)).copy())
        self._tap = self.TAP(cb)
        lib.orc_model_set_tap(self.h, ctypes.cast(self._tap, ctypes.c_void_p), None)

    def hidden(self) -> np.ndarray:
        out = np.zeros(self.dim, np.float32)
        lib.orc_model_hidden(self.h, _p(out), self.dim)
        return out

    def kv_shift(self, seq: int, p0: int, p1: int, n_past: int) -> None:
        if lib.orc_model_kv_shift(self.h, seq, p0, p1, n_past) != 0:
            raise RuntimeError("oracle kv shift")

    def __del__(self):
        if getattr(self, "h", None):
            lib.orc_model_free(self.h)
            self.h = None


def load_reference() -> ctypes.CDLL | None:
    """The reference's own scalar ops (built by build_ref.sh), or None."""
    if not os.path.exists(REF_PATH):
        return None
    r = ctypes.CDLL(REF_PATH)
    sig = {
        "sref_fp16_to_fp32": (_f, [ctypes.c_uint16]),
        "sref_fp32_to_fp16": (ctypes.c_uint16, [_f]),
        "sref_vec_dot_q4_0_q8_0": (_f, [_i, _vp, _vp]),
        "sref_vec_dot_q8_0_q8_0": (_f, [_i, _vp, _vp]),
        "sref_quantize_row_q8_0": (None, [_vp, _vp, _i]),
        "sref_rmsnorm_f32": (None, [_vp, _vp, _vp, _i, _f]),
        "sref_softmax_f32": (None, [_vp, _vp, _i]),
        "sref_rope_f32": (None, [_vp, _vp, _i, _i]),
        "sref_xorshift_fill": (None, [ctypes.c_uint32, _vp, _i, _vp]),
        "sref_rel_error": (_f, [_f, _f]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(r, name)
        fn.restype = res
        fn.argtypes = args
    return r
