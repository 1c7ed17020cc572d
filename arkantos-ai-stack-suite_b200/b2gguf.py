"""ctypes binding for libb2gguf.so (the C ABI declared in include/b2gguf.h).

There is no fallback: if the shared library is missing or fails to load,
importing this module raises.  Build it with `make -C arkantos-ai-stack-suite_b200`
(or __graft_entry__.build()).
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libb2gguf.so")
HEADER = os.path.join(ROOT, "include", "b2gguf.h")

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, Q8_K = 0, 1, 2, 8, 12, 14, 15
OK, NO_KV_SLOT, ABORTED = 0, 1, 2
ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_FORMAT, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_NCCL, ERR_IO = -1, -2, -3, -4, -5, -6, -7, -8

if not os.path.exists(LIB_PATH):
    raise ImportError(f"libb2gguf.so not built at {LIB_PATH}; run make -C {HERE}")

lib = ctypes.CDLL(LIB_PATH)

_vp, _i, _i64, _u64, _f, _sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64,
                                ctypes.c_float, ctypes.c_size_t)
_TYPES = {"void*": _vp, "const void*": _vp, "int": _i, "int64_t": _i64, "uint64_t": _u64, "float": _f,
          "size_t": _sz, "int32_t": ctypes.c_int32, "uint32_t": ctypes.c_uint32}


def header_functions() -> list[str]:
    """Names of every function declared in include/b2gguf.h."""
    with open(HEADER) as f:
        src = f.read()
    return re.findall(r"^B2_API\s+[\w\s\*]+?\b(b2_\w+)\s*\(", src, flags=re.M)


def _bind() -> None:
    # Every pointer is passed as c_void_p; integers and floats are typed so
    # ctypes converts them exactly.
    sig = {
        "b2_abi_version": (_i, []),
        "b2_last_error": (ctypes.c_char_p, []),
        "b2_device_count": (_i, [_vp]),
        "b2_set_device": (_i, [_i]),
        "b2_get_device": (_i, [_vp]),
        "b2_malloc": (_i, [_vp, _sz]),
        "b2_free": (_i, [_vp]),
        "b2_host_alloc": (_i, [_vp, _sz]),
        "b2_host_free": (_i, [_vp]),
        "b2_memcpy_h2d": (_i, [_vp, _vp, _sz, _vp]),
        "b2_memcpy_d2h": (_i, [_vp, _vp, _sz, _vp]),
        "b2_memcpy_d2d": (_i, [_vp, _vp, _sz, _vp]),
        "b2_memset": (_i, [_vp, _i, _sz, _vp]),
        "b2_stream_create": (_i, [_vp]),
        "b2_stream_destroy": (_i, [_vp]),
        "b2_stream_synchronize": (_i, [_vp]),
        "b2_device_synchronize": (_i, []),
        "b2_event_create": (_i, [_vp]),
        "b2_event_destroy": (_i, [_vp]),
        "b2_event_record": (_i, [_vp, _vp]),
        "b2_event_elapsed_ms": (_i, [_vp, _vp, _vp]),
        "b2_set_pdl": (_i, [_i]),
        "b2_profiler_range": (_i, [_i]),
        "b2_graph_capture_begin": (_i, [_vp]),
        "b2_graph_capture_end": (_i, [_vp, _vp]),
        "b2_graph_launch": (_i, [_vp, _vp]),
        "b2_graph_destroy": (_i, [_vp]),
        "b2_row_bytes": (_sz, [_i, _i64]),
        "b2_quantize_weights": (_i, [_i, _vp, _i64, _i64, _vp, _i]),
        "b2_synth_normal": (_i, [_u64, _u64, _i64, _f, _f, _vp, _i]),
        "b2_rope_table": (_i, [_f, _i, _i, _i, _vp]),
        "b2_qmatrix_upload": (_i, [_i, _vp, _i64, _i64, _vp]),
        "b2_qmatrix_free": (_i, [_vp]),
        "b2_qmatrix_device_bytes": (_i, [_vp, _vp]),
        "b2_qmatrix_dequantize": (_i, [_vp, _vp, _vp]),
        "b2_quantize_act": (_i, [_i, _vp, _i, _i64, _vp, _vp]),
        "b2_gemv": (_i, [_vp, _vp, _i, _vp, _vp]),
        "b2_gemm": (_i, [_vp, _vp, _i, _vp, _vp, _sz, _vp, _vp]),
        "b2_gemv_multi": (_i, [_vp, _i, _vp, _i, _vp, _vp]),
        "b2_moe_route": (_i, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _vp, _vp, _vp]),
        "b2_moe_gemv": (_i, [_vp, ctypes.c_int32, _vp, ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_int32, _vp,
                             _vp]),
        "b2_moe_combine": (_i, [_vp, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _vp, _vp]),
        "b2_gemm_workspace_bytes": (_i, [_vp, _i, _vp]),
        "b2_gemm_host": (_i, [_vp, _vp, _i, _vp]),
        "b2_gemv_host": (_i, [_vp, _vp, _i, _vp]),
        "b2_block_dots": (_i, [_vp, _i64, _vp, _vp, _vp, _vp]),
        "b2_gguf_write_synthetic_llama": (_i, [_vp, ctypes.c_char_p, _i]),
        "b2_embed": (_i, [_i, _vp, _i, _i, _vp, _i, _vp, _vp]),
        "b2_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _i, _i, _f, _vp]),
        "b2_rope_kv_store": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
        "b2_attn_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
        "b2_attn_decode_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
        "b2_kv_shift_k": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
        "b2_kv_row_bytes": (ctypes.c_int64, [_i, _i]),
        "b2_rope_kv_store_typed": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _vp]),
        "b2_attn_decode_typed": (_i, [_vp, _vp, _i, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
        "b2_kv_shift_k_typed": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
        "b2_model_default_params": (None, [_vp]),
        "b2_nccl_unique_id": (_i, [_vp]),
        "b2_model_load": (_i, [ctypes.c_char_p, _vp, _vp]),
        "b2_model_free": (_i, [_vp]),
        "b2_model_info": (_i, [_vp, _vp, _i]),
        "b2_model_device_bytes": (_i, [_vp, _vp]),
        "b2_context_default_params": (None, [_vp]),
        "b2_context_create": (_i, [_vp, _vp, _vp]),
        "b2_context_free": (_i, [_vp]),
        "b2_context_stream": (_i, [_vp, _vp]),
        "b2_decode": (_i, [_vp, _vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32]),
        "b2_get_logits": (_i, [_vp, ctypes.c_int32, _vp, _i64]),
        "b2_get_argmax": (_i, [_vp, _vp, _vp, _vp, ctypes.c_int32]),
        "b2_generate": (_i, [_vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp]),
        "b2_context_exchange_wait_ns": (_i, [_vp, _vp, ctypes.c_int32]),
        "b2_get_last_rows": (_i, [_vp, _vp]),
        "b2_sampler_default_params": (None, [_vp]),
        "b2_sampler_create": (_i, [_vp, _vp, _vp]),
        "b2_sampler_free": (_i, [_vp]),
        "b2_sampler_reset": (_i, [_vp]),
        "b2_sampler_accept": (_i, [_vp, ctypes.c_int32]),
        "b2_sampler_sample": (_i, [_vp, ctypes.c_int32, _vp]),
        "b2_sampler_sample_logits": (_i, [_vp, _vp, ctypes.c_int32, _vp]),
        "b2_generate_sampled": (_i, [_vp, _vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp]),
        "b2_synchronize_context": (_i, [_vp]),
        "b2_kv_clear": (_i, [_vp]),
        "b2_kv_seq_rm": (_i, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
        "b2_kv_seq_add": (_i, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
        "b2_kv_seq_pos_max": (_i, [_vp, ctypes.c_int32, _vp]),
        "b2_set_abort_callback": (_i, [_vp, _vp, _vp]),
        "b2_set_eval_callback": (_i, [_vp, _vp, _vp]),
        "b2_n_ctx": (_i, [_vp, _vp]),
        "b2_flag_wait": (_i, [_vp, _i, _u64, _vp, _vp]),
        "b2_memory_can_shift": (_i, [_vp, _vp]),
        "b2_state_seq_get_size": (_i, [_vp, ctypes.c_int32, _vp]),
        "b2_state_seq_get_data": (_i, [_vp, ctypes.c_int32, _vp, _sz, _vp]),
        "b2_state_seq_set_data": (_i, [_vp, ctypes.c_int32, _vp, _sz, _vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


_bind()


class B2Error(RuntimeError):
    def __init__(self, rc: int, what: str):
        msg = lib.b2_last_error()
        super().__init__(f"{what} failed rc={rc}: {msg.decode() if msg else ''}")
        self.rc = rc


def check(rc: int, what: str = "b2 call") -> int:
    if rc < 0:
        raise B2Error(rc, what)
    return rc


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data


# ---- device memory -----------------------------------------------------------------------
class PinnedArray:
    """Page-locked host memory (b2_host_alloc) viewed as a numpy array."""

    def __init__(self, shape, dtype=np.float32):
        self.nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = ctypes.c_void_p()
        check(lib.b2_host_alloc(ctypes.byref(p), max(self.nbytes, 1)), "host_alloc")
        self.p = p.value
        buf = (ctypes.c_uint8 * max(self.nbytes, 1)).from_address(self.p)
        self.array = np.frombuffer(buf, np.uint8, self.nbytes).view(dtype).reshape(shape)

    @classmethod
    def from_array(cls, a: np.ndarray) -> "PinnedArray":
        h = cls(a.shape, a.dtype)
        h.array[...] = a
        return h

    def __del__(self):
        if getattr(self, "p", None):
            self.array = None
            lib.b2_host_free(self.p)
            self.p = None


class DeviceBuffer:
    """Raw device allocation owned by Python."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib.b2_malloc(ctypes.byref(p), max(1, int(nbytes))), "b2_malloc")
        self.ptr = p.value
        self.nbytes = int(nbytes)

    @classmethod
    def from_array(cls, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        b.upload(a)
        return b

    def upload(self, a: np.ndarray, stream: int | None = None) -> None:
        a = np.ascontiguousarray(a)
        assert a.nbytes <= self.nbytes
        check(lib.b2_memcpy_h2d(self.ptr, ptr(a), a.nbytes, stream), "h2d")
        if stream is None:
            check(lib.b2_stream_synchronize(None), "sync")

    def download(self, dtype, count: int | None = None, stream: int | None = None) -> np.ndarray:
        dt = np.dtype(dtype)
        n = self.nbytes // dt.itemsize if count is None else int(count)
        out = np.empty(n, dt)
        check(lib.b2_memcpy_d2h(ptr(out), self.ptr, out.nbytes, stream), "d2h")
        check(lib.b2_stream_synchronize(stream), "sync")
        return out

    def zero(self) -> None:
        check(lib.b2_memset(self.ptr, 0, self.nbytes, None), "memset")

    def free(self) -> None:
        if getattr(self, "ptr", None):
            lib.b2_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Stream:
    def __init__(self):
        p = ctypes.c_void_p()
        check(lib.b2_stream_create(ctypes.byref(p)), "stream_create")
        self.h = p.value

    def synchronize(self) -> None:
        check(lib.b2_stream_synchronize(self.h), "stream_synchronize")

    def __del__(self):
        if getattr(self, "h", None):
            lib.b2_stream_destroy(self.h)


class Graph:
    """Captures the library calls made by fn(stream) once; launch() replays them."""

    def __init__(self, stream: Stream, fn):
        check(lib.b2_graph_capture_begin(stream.h), "graph_capture_begin")
        try:
            fn(stream.h)
        finally:
            e = ctypes.c_void_p()
            rc = lib.b2_graph_capture_end(stream.h, ctypes.byref(e))
        check(rc, "graph_capture_end")
        self.h = e.value
        self.stream = stream

    def launch(self) -> None:
        check(lib.b2_graph_launch(self.h, self.stream.h), "graph_launch")

    def __del__(self):
        if getattr(self, "h", None):
            lib.b2_graph_destroy(self.h)


def synchronize() -> None:
    check(lib.b2_device_synchronize(), "device_synchronize")


def device_count() -> int:
    n = ctypes.c_int(0)
    rc = lib.b2_device_count(ctypes.byref(n))
    return n.value if rc == 0 else 0


class Event:
    def __init__(self):
        p = ctypes.c_void_p()
        check(lib.b2_event_create(ctypes.byref(p)), "event_create")
        self.h = p.value

    def record(self, stream: int | None = None) -> None:
        check(lib.b2_event_record(self.h, stream), "event_record")

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        check(lib.b2_event_elapsed_ms(self.h, end.h, ctypes.byref(ms)), "event_elapsed")
        return ms.value

    def __del__(self):
        if getattr(self, "h", None):
            lib.b2_event_destroy(self.h)


# ---- host helpers ---------------------------------------------------------------------------
BLOCK = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q6_K: 256, Q8_K: 256, F32: 1, F16: 1}


def row_bytes(t: int, k: int) -> int:
    return int(lib.b2_row_bytes(t, k))


def quantize_weights(t: int, w: np.ndarray, n_threads: int = 8) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    out = np.empty((n, row_bytes(t, k)), np.uint8)
    check(lib.b2_quantize_weights(t, ptr(w), n, k, ptr(out), n_threads), "quantize_weights")
    return out


def synth_normal(seed: int, n: int, std: float = 1.0, mean: float = 0.0, offset: int = 0,
                 n_threads: int = 8) -> np.ndarray:
    out = np.empty(int(n), np.float32)
    check(lib.b2_synth_normal(seed, offset, int(n), mean, std, ptr(out), n_threads), "synth_normal")
    return out


def rope_table(theta: float, head_dim: int, p0: int, n_pos: int) -> np.ndarray:
    out = np.empty((n_pos, head_dim), np.float32)
    check(lib.b2_rope_table(theta, head_dim, p0, n_pos, ptr(out)), "rope_table")
    return out


# ---- quantized matrices and single ops --------------------------------------------------------
def gemv_multi(mats, x: "DeviceBuffer", n_tok: int, ys, stream: int | None = None) -> None:
    """Several GEMVs of one type and shape over the same device input in one
    launch (1-2 tokens): ys[i] = mats[i]·x, each bit-identical to gemv_device."""
    n = len(mats)
    hs = (ctypes.c_void_p * n)(*[m.h for m in mats])
    yp = (ctypes.c_void_p * n)(*[y.ptr for y in ys])
    check(lib.b2_gemv_multi(hs, n, x.ptr, n_tok, yp, stream), "gemv_multi")


class QMatrix:
    """A GGUF tensor uploaded to the current device in the repacked layout."""

    def __init__(self, qtype: int, gguf_bytes: np.ndarray, n_rows: int, k: int):
        gguf_bytes = np.ascontiguousarray(gguf_bytes, np.uint8)
        assert gguf_bytes.nbytes == n_rows * row_bytes(qtype, k)
        h = ctypes.c_void_p()
        check(lib.b2_qmatrix_upload(qtype, ptr(gguf_bytes), n_rows, k, ctypes.byref(h)), "qmatrix_upload")
        self.h = h.value
        self.qtype, self.n_rows, self.k = qtype, n_rows, k

    def device_bytes(self) -> int:
        v = ctypes.c_int64()
        check(lib.b2_qmatrix_device_bytes(self.h, ctypes.byref(v)), "qmatrix_device_bytes")
        return v.value

    def dequantize(self) -> np.ndarray:
        buf = DeviceBuffer(self.n_rows * self.k * 4)
        check(lib.b2_qmatrix_dequantize(self.h, buf.ptr, None), "qmatrix_dequantize")
        return buf.download(np.float32).reshape(self.n_rows, self.k)

    def gemv_device(self, x: DeviceBuffer, n_tok: int, y: DeviceBuffer, stream: int | None = None) -> None:
        check(lib.b2_gemv(self.h, x.ptr, n_tok, y.ptr, stream), "gemv")

    def gemm_workspace_bytes(self, n_tok: int) -> int:
        v = ctypes.c_size_t()
        check(lib.b2_gemm_workspace_bytes(self.h, n_tok, ctypes.byref(v)), "gemm_workspace_bytes")
        return v.value

    def gemm_device(self, x: DeviceBuffer, n_tok: int, y: DeviceBuffer, status: DeviceBuffer | None = None,
                    stream: int | None = None, workspace: DeviceBuffer | None = None) -> None:
        """Tensor-core prefill GEMM (Q4_K or Q8_0 weights): x fp32 [n_tok, k] -> y fp32 [n_tok, n_rows] on the device."""
        check(lib.b2_gemm(self.h, x.ptr, n_tok, y.ptr, workspace.ptr if workspace else None,
                          workspace.nbytes if workspace else 0, status.ptr if status else None, stream), "gemm")

    def gemm(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Prefill GEMM from host arrays (the e2e path; pass pinned arrays for
        full copy bandwidth); raises if a pipeline wait expired."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        y = out if out is not None else np.empty((x.shape[0], self.n_rows), np.float32)
        assert y.shape == (x.shape[0], self.n_rows) and y.dtype == np.float32 and y.flags.c_contiguous
        check(lib.b2_gemm_host(self.h, ptr(x), x.shape[0], ptr(y)), "gemm_host")
        return y

    def gemv(self, x: np.ndarray) -> np.ndarray:
        """Device GEMV from host arrays (the e2e path): x [n_tok, k] -> y [n_tok, n_rows]."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        y = np.empty((x.shape[0], self.n_rows), np.float32)
        check(lib.b2_gemv_host(self.h, ptr(x), x.shape[0], ptr(y)), "gemv_host")
        return y

    def block_dots(self, row: int, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        nb = self.k // BLOCK[self.qtype]
        xd = DeviceBuffer.from_array(x)
        oi = DeviceBuffer(nb * 4)
        om = DeviceBuffer(nb * 4) if self.qtype == Q4_K else None
        check(lib.b2_block_dots(self.h, row, xd.ptr, oi.ptr, om.ptr if om else None, None), "block_dots")
        a = oi.download(np.int32)
        return (a, om.download(np.int32)) if om else a

    def __del__(self):
        if getattr(self, "h", None):
            lib.b2_qmatrix_free(self.h)
            self.h = None


def quantize_act(act_type: int, x: np.ndarray) -> np.ndarray:
    """Device activation quantization -> GGUF block bytes [n_tok, row_bytes]."""
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    n_tok, k = x.shape
    xd = DeviceBuffer.from_array(x)
    out = DeviceBuffer(n_tok * row_bytes(act_type, k))
    check(lib.b2_quantize_act(act_type, xd.ptr, n_tok, k, out.ptr, None), "quantize_act")
    return out.download(np.uint8).reshape(n_tok, -1)


# ---- GGUF models and the engine -------------------------------------------------------------
class LlamaHParams(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int32), ("n_embd", ctypes.c_int32), ("n_ff", ctypes.c_int32),
                ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32), ("n_vocab", ctypes.c_int32),
                ("n_ctx_train", ctypes.c_int32), ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("wtype", ctypes.c_int32), ("embd_type", ctypes.c_int32), ("out_type", ctypes.c_int32),
                ("seed", ctypes.c_uint64), ("w_std", ctypes.c_float)]


def write_synthetic_llama(path: str, n_layer: int, n_embd: int, n_ff: int, n_head: int, n_head_kv: int,
                          n_vocab: int, wtype: int, embd_type: int | None = None, out_type: int | None = None,
                          seed: int = 0, w_std: float = 0.02, rms_eps: float = 1e-5, rope_theta: float = 10000.0,
                          n_ctx_train: int = 4096, n_threads: int = 0) -> None:
    hp = LlamaHParams(n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab, n_ctx_train, rms_eps, rope_theta, wtype,
                      wtype if embd_type is None else embd_type, wtype if out_type is None else out_type, seed, w_std)
    nt = n_threads or (os.cpu_count() or 1)
    check(lib.b2_gguf_write_synthetic_llama(ctypes.byref(hp), path.encode(), nt), "write_synthetic_llama")


class ModelParams(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32),
                ("nccl_id", ctypes.c_void_p), ("keep_page_cache", ctypes.c_int32)]


class ContextParams(ctypes.Structure):
    _fields_ = [("n_ctx", ctypes.c_int32), ("n_seq_max", ctypes.c_int32), ("use_graph", ctypes.c_int32),
                ("prefill_gemm", ctypes.c_int32), ("type_k", ctypes.c_int32), ("type_v", ctypes.c_int32)]


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib.b2_nccl_unique_id(buf), "nccl_unique_id")
    return buf.raw


class Model:
    INFO = ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "n_vocab", "head_dim", "n_ctx_train", "wtype",
            "out_type", "tp_rank", "tp_size")

    def __init__(self, path: str, device: int = -1, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None,
                 keep_page_cache: bool = False):
        self._id = ctypes.create_string_buffer(nccl_id, 128) if nccl_id else None
        p = ModelParams(device, tp_rank, tp_size, ctypes.cast(self._id, ctypes.c_void_p) if self._id else None,
                        1 if keep_page_cache else 0)
        h = ctypes.c_void_p()
        check(lib.b2_model_load(path.encode(), ctypes.byref(p), ctypes.byref(h)), "model_load")
        self.h = h.value
        info = (ctypes.c_int32 * 12)()
        check(lib.b2_model_info(self.h, info, 12), "model_info")
        for k, v in zip(self.INFO, info):
            setattr(self, k, int(v))

    def device_bytes(self) -> int:
        v = ctypes.c_int64()
        check(lib.b2_model_device_bytes(self.h, ctypes.byref(v)), "model_device_bytes")
        return v.value

    def free(self) -> None:
        if getattr(self, "h", None):
            lib.b2_model_free(self.h)
            self.h = None

    def __del__(self):
        self.free()


class SamplerParams(ctypes.Structure):
    _fields_ = [("penalty_last_n", ctypes.c_int32), ("penalty_repeat", ctypes.c_float),
                ("penalty_freq", ctypes.c_float), ("penalty_present", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("top_p", ctypes.c_float), ("min_p", ctypes.c_float), ("temperature", ctypes.c_float),
                ("seed", ctypes.c_uint32)]


class Sampler:
    """A sampler chain on a context's GPU (Milda's rebuild_sampler chain);
    keyword arguments override Milda's defaults."""

    def __init__(self, ctx, **kw):
        p = SamplerParams()
        lib.b2_sampler_default_params(ctypes.byref(p))
        for k, v in kw.items():
            setattr(p, k, v)
        self.params = p
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(lib.b2_sampler_create(ctx.h, ctypes.byref(p), ctypes.byref(h)), "sampler_create")
        self.h = h.value

    def sample(self, idx: int = -1) -> int:
        t = ctypes.c_int32()
        check(lib.b2_sampler_sample(self.h, idx, ctypes.byref(t)), "sampler_sample")
        return t.value

    def sample_logits(self, logits_dev, n_vocab: int) -> int:
        t = ctypes.c_int32()
        check(lib.b2_sampler_sample_logits(self.h, logits_dev, n_vocab, ctypes.byref(t)), "sampler_sample_logits")
        return t.value

    def accept(self, tok: int) -> None:
        check(lib.b2_sampler_accept(self.h, tok), "sampler_accept")

    def reset(self) -> None:
        check(lib.b2_sampler_reset(self.h), "sampler_reset")

    def free(self) -> None:
        if getattr(self, "h", None):
            lib.b2_sampler_free(self.h)
            self.h = None

    def __del__(self):
        self.free()


class Context:
    def __init__(self, model: Model, n_ctx: int = 4096, n_seq: int = 1, use_graph: bool = True,
                 prefill_gemm: bool = True, type_k: int = F16, type_v: int = F16):
        self.model = model
        p = ContextParams(n_ctx, n_seq, 1 if use_graph else 0, 1 if prefill_gemm else 0, type_k, type_v)
        h = ctypes.c_void_p()
        check(lib.b2_context_create(model.h, ctypes.byref(p), ctypes.byref(h)), "context_create")
        self.h = h.value
        s = ctypes.c_void_p()
        check(lib.b2_context_stream(self.h, ctypes.byref(s)), "context_stream")
        self.stream = s.value
        self.last_n = 0

    def decode(self, tokens, pos=None, seq=None, want_logits: int = 2) -> int:
        t = np.ascontiguousarray(tokens, np.int32)
        pp = None if pos is None else np.ascontiguousarray(pos, np.int32)
        ss = None if seq is None else np.ascontiguousarray(seq, np.int32)
        rc = lib.b2_decode(self.h, ptr(t), ptr(pp) if pp is not None else None, ptr(ss) if ss is not None else None,
                           t.size, want_logits)
        check(rc, "decode")
        n = ctypes.c_int32()
        check(lib.b2_get_last_rows(self.h, ctypes.byref(n)), "get_last_rows")
        self.last_n = n.value if n.value else min(t.size, 8)
        return rc

    def logits(self, i: int = -1) -> np.ndarray:
        out = np.empty(self.model.n_vocab, np.float32)
        check(lib.b2_get_logits(self.h, i, ptr(out), out.size), "get_logits")
        return out

    def argmax(self, n: int | None = None):
        n = self.last_n if n is None else n
        ids = np.empty(max(n, 8), np.int32)
        top = np.empty(max(n, 8), np.float32)
        mar = np.empty(max(n, 8), np.float32)
        check(lib.b2_get_argmax(self.h, ptr(ids), ptr(top), ptr(mar), ids.size), "get_argmax")
        return ids[:n], top[:n], mar[:n]

    def generate(self, first, n_steps: int, seq=None) -> np.ndarray:
        """Greedy continuation on the device: returns ids [n_steps, n]."""
        f = np.ascontiguousarray(first, np.int32).ravel()
        ss = None if seq is None else np.ascontiguousarray(seq, np.int32)
        out = np.zeros((max(n_steps, 1), f.size), np.int32)
        rc = lib.b2_generate(self.h, ptr(f), ptr(ss) if ss is not None else None, f.size, n_steps, ptr(out))
        check(rc, "generate")
        self.last_n = f.size
        return out[:n_steps]

    def generate_sampled(self, samplers, first, n_steps: int, seq=None) -> np.ndarray:
        """Sampled continuation on the device (row i drawn by samplers[i]): ids [n_steps, n]."""
        f = np.ascontiguousarray(first, np.int32).ravel()
        ss = None if seq is None else np.ascontiguousarray(seq, np.int32)
        arr = (ctypes.c_void_p * len(samplers))(*[s.h for s in samplers])
        out = np.zeros((max(n_steps, 1), f.size), np.int32)
        rc = lib.b2_generate_sampled(self.h, arr, ptr(f), ptr(ss) if ss is not None else None, f.size, n_steps,
                                     ptr(out))
        check(rc, "generate_sampled")
        self.last_n = f.size
        return out[:n_steps]

    def exchange_wait_ns(self, reset: bool = False) -> int:
        v = ctypes.c_uint64()
        check(lib.b2_context_exchange_wait_ns(self.h, ctypes.byref(v), 1 if reset else 0), "context_exchange_wait_ns")
        return v.value

    def synchronize(self) -> None:
        check(lib.b2_synchronize_context(self.h), "synchronize_context")

    EVAL = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p)

    def set_eval_callback(self, fn) -> None:
        """fn(name, layer, np.ndarray) with each intermediate of eager steps (llama cb_eval)."""
        if fn is None:
            self._eval = None
            check(lib.b2_set_eval_callback(self.h, None, None), "set_eval_callback")
            return
        def cb(name, layer, dptr, n, user):
            out = np.empty(n, np.float32)
            lib.b2_memcpy_d2h(out.ctypes.data, dptr, out.nbytes, None)
            lib.b2_device_synchronize()
            fn(name.decode(), layer, out)
        self._eval = self.EVAL(cb)
        check(lib.b2_set_eval_callback(self.h, ctypes.cast(self._eval, ctypes.c_void_p), None), "set_eval_callback")

    def kv_clear(self) -> None:
        check(lib.b2_kv_clear(self.h), "kv_clear")

    def kv_seq_rm(self, seq: int, p0: int, p1: int) -> None:
        check(lib.b2_kv_seq_rm(self.h, seq, p0, p1), "kv_seq_rm")

    def kv_seq_add(self, seq: int, p0: int, p1: int, delta: int) -> None:
        check(lib.b2_kv_seq_add(self.h, seq, p0, p1, delta), "kv_seq_add")

    def kv_pos_max(self, seq: int) -> int:
        v = ctypes.c_int32()
        check(lib.b2_kv_seq_pos_max(self.h, seq, ctypes.byref(v)), "kv_seq_pos_max")
        return v.value

    def n_ctx(self) -> int:
        v = ctypes.c_int32()
        check(lib.b2_n_ctx(self.h, ctypes.byref(v)), "n_ctx")
        return v.value

    def can_shift(self) -> bool:
        v = ctypes.c_int32()
        check(lib.b2_memory_can_shift(self.h, ctypes.byref(v)), "memory_can_shift")
        return bool(v.value)

    def state_seq_get(self, seq: int) -> bytes:
        """Snapshot of one sequence's KV state (llama_state_seq_get_data)."""
        n = ctypes.c_size_t()
        check(lib.b2_state_seq_get_size(self.h, seq, ctypes.byref(n)), "state_seq_get_size")
        buf = ctypes.create_string_buffer(n.value)
        w = ctypes.c_size_t()
        check(lib.b2_state_seq_get_data(self.h, seq, buf, n.value, ctypes.byref(w)), "state_seq_get_data")
        return buf.raw[:w.value]

    def state_seq_set(self, seq: int, data: bytes) -> int:
        """Restores a snapshot into sequence seq (llama_state_seq_set_data); returns bytes read."""
        r = ctypes.c_size_t()
        check(lib.b2_state_seq_set_data(self.h, seq, data, len(data), ctypes.byref(r)), "state_seq_set_data")
        return r.value

    def set_abort_callback(self, fn) -> None:
        """fn() -> bool polled between decode steps; True stops the call with status 2 (llama abort callback)."""
        if fn is None:
            self._abort = None
            check(lib.b2_set_abort_callback(self.h, None, None), "set_abort_callback")
            return
        self._abort = self.ABORT(lambda user: 1 if fn() else 0)
        check(lib.b2_set_abort_callback(self.h, ctypes.cast(self._abort, ctypes.c_void_p), None),
              "set_abort_callback")

    ABORT = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)

    def free(self) -> None:
        if getattr(self, "h", None):
            lib.b2_context_free(self.h)
            self.h = None

    def __del__(self):
        self.free()
