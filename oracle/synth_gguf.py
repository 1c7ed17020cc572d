"""Test infrastructure: a numpy GGUF v3 writer for random-init
Llama-architecture files, used by the benchmark's CPU reference arm so that
its process loads the oracle alone (no product library).

The file has the metadata keys and tensor names the engines bind
(Singularity/src/core/cortex_a5_engine.cpp:579-654) and the block types of
the workload.  Quantized blocks hold valid random contents drawn from a
seeded generator — small positive fp16 scales, uniform codes — instead of
quantized normal weights: the CPU forward's time does not depend on the
weight values, and the parity tests use the library's own writer."""
import struct

import numpy as np

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), F32: (1, 4), F16: (1, 2)}
ALIGN = 32


def row_bytes(t: int, k: int) -> int:
    be, bb = BLOCK[t]
    return k // be * bb


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _str(key) + struct.pack("<I", vtype) + payload


def _blocks(rng: np.random.Generator, t: int, n_blocks: int) -> np.ndarray:
    """n_blocks valid random blocks of type t as uint8 [n_blocks][bytes]."""
    bb = BLOCK[t][1]
    out = rng.integers(0, 256, (n_blocks, bb), dtype=np.uint8)
    d = np.float16(0.0006)
    if t == Q4_0:
        out[:, 0:2] = np.frombuffer(d.tobytes(), np.uint8)
    elif t == Q8_0:
        out[:, 0:2] = np.frombuffer(np.float16(0.0002).tobytes(), np.uint8)
    elif t == Q4_K:
        out[:, 0:2] = np.frombuffer(np.float16(0.0004).tobytes(), np.uint8)
        out[:, 2:4] = np.frombuffer(np.float16(0.0003).tobytes(), np.uint8)
    elif t == Q6_K:
        out[:, 192:208] &= 0x3F                      # int8 scales in [0, 63]
        out[:, 208:210] = np.frombuffer(np.float16(0.0001).tobytes(), np.uint8)
    return out


def write_llama(path: str, n_layer: int, n_embd: int, n_ff: int, n_head: int, n_head_kv: int, n_vocab: int,
                wtype: int, embd_type: int, out_type: int, seed: int, rope_theta: float = 10000.0,
                n_ctx_train: int = 2048, rms_eps: float = 1e-5) -> None:
    hd = n_embd // n_head
    kvs = [
        _kv("general.architecture", 8, _str("llama")),
        _kv("general.name", 8, _str("b2-synthetic-llama-cpu-arm")),
        _kv("general.alignment", 4, struct.pack("<I", ALIGN)),
        _kv("llama.block_count", 4, struct.pack("<I", n_layer)),
        _kv("llama.context_length", 4, struct.pack("<I", n_ctx_train)),
        _kv("llama.embedding_length", 4, struct.pack("<I", n_embd)),
        _kv("llama.feed_forward_length", 4, struct.pack("<I", n_ff)),
        _kv("llama.attention.head_count", 4, struct.pack("<I", n_head)),
        _kv("llama.attention.head_count_kv", 4, struct.pack("<I", n_head_kv)),
        _kv("llama.rope.dimension_count", 4, struct.pack("<I", hd)),
        _kv("llama.vocab_size", 4, struct.pack("<I", n_vocab)),
        _kv("llama.attention.layer_norm_rms_epsilon", 6, struct.pack("<f", rms_eps)),
        _kv("llama.rope.freq_base", 6, struct.pack("<f", rope_theta)),
    ]
    tensors = [("token_embd.weight", embd_type, n_embd, n_vocab), ("output_norm.weight", F32, n_embd, 1),
               ("output.weight", out_type, n_embd, n_vocab)]
    for l in range(n_layer):
        b = f"blk.{l}."
        tensors += [(b + "attn_norm.weight", F32, n_embd, 1), (b + "attn_q.weight", wtype, n_embd, n_head * hd),
                    (b + "attn_k.weight", wtype, n_embd, n_head_kv * hd),
                    (b + "attn_v.weight", wtype, n_embd, n_head_kv * hd),
                    (b + "attn_output.weight", wtype, n_head * hd, n_embd), (b + "ffn_norm.weight", F32, n_embd, 1),
                    (b + "ffn_gate.weight", wtype, n_embd, n_ff), (b + "ffn_up.weight", wtype, n_embd, n_ff),
                    (b + "ffn_down.weight", wtype, n_ff, n_embd)]
    infos, offsets, off = [], [], 0
    for name, t, ne0, ne1 in tensors:
        nd = 1 if ne1 == 1 else 2
        dims = struct.pack("<Q", ne0) + (struct.pack("<Q", ne1) if nd == 2 else b"")
        offsets.append(off)
        infos.append(_str(name) + struct.pack("<I", nd) + dims + struct.pack("<I", t) + struct.pack("<Q", off))
        off += (row_bytes(t, ne0) * ne1 + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)) + b"".join(kvs) + b"".join(infos)
    data_off = (len(head) + ALIGN - 1) // ALIGN * ALIGN
    rng = np.random.default_rng(seed)
    with open(path, "wb") as f:
        f.write(head + b"\0" * (data_off - len(head)))
        for (name, t, ne0, ne1), o in zip(tensors, offsets):
            f.seek(data_off + o)
            if t == F32:
                f.write(np.ones(ne0 * ne1, np.float32).tobytes())
                continue
            nb = ne0 // BLOCK[t][0]
            rows = max(1, (64 << 20) // row_bytes(t, ne0))
            for r0 in range(0, ne1, rows):
                n = min(rows, ne1 - r0)
                f.write(_blocks(rng, t, n * nb).tobytes())
        f.truncate(data_off + off)
