"""Tensor parallelism on 2 GPUs through the C ABI, one process per rank.

The ranks exchange the attention-out / FFN-down partial outputs and the
head's logit shards through peer memory and sum the partials in rank order,
so the result is deterministic and the oracle reproduces it: its
reference-order forward with the same two column-slice partials per
row-split projection, each slice in block order (orc_model_set_tp).  Both ranks' logits must equal the oracle's
bit for bit, prefill and greedy steps, host loop and device loop alike."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

b2 = pytest.importorskip("b2gguf")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from tests import tp_worker as W  # noqa: E402

MODELS = {
    # name: (layers, d, ff, heads, kv heads, vocab, wtype, out type, theta)
    "q4_k_hd128": (2, 512, 1024, 4, 2, 768, 12, 14, 500000.0),
    "q4_0_hd64": (2, 256, 512, 4, 2, 512, 2, 2, 10000.0),
}


def _gpus() -> int:
    n = b2.ctypes.c_int()
    return n.value if b2.lib.b2_device_count(b2.ctypes.byref(n)) == 0 else 0


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name,kind", [(n, "short") for n in sorted(MODELS)] + [("q4_k_hd128", "long")])
def test_tp2_bit_exact_with_oracle(tmp_path, name, kind):
    """Two ranks against the oracle's two-rank emulation.  The long prompt
    runs all but its last 8 tokens through the tensor-core prefill, whose
    attention-out and FFN-down partials the ranks all-gather and sum in rank
    order."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    L, d, ff, nh, nkv, V, wt, ot, theta = MODELS[name]
    path = str(tmp_path / f"{name}.gguf")
    b2.write_synthetic_llama(path, L, d, ff, nh, nkv, V, wt, out_type=ot, seed=21, rope_theta=theta)
    id_file = tmp_path / "nccl.id"
    id_file.write_bytes(b2.nccl_unique_id())
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-m", "tests.tp_worker", str(r), "2", str(id_file), path,
                               str(tmp_path / f"r{r}.npz"), kind], cwd=ROOT, env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=300)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{outs[r][-3000:]}"
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(2)]
    for key in ("logits", "toks", "gen", "gen_last"):
        assert np.array_equal(_bits(res[0][key]) if res[0][key].dtype == np.float32 else res[0][key],
                              _bits(res[1][key]) if res[1][key].dtype == np.float32 else res[1][key]), key

    prompt = W.LONG_PROMPT if kind == "long" else W.PROMPT
    om = O.Model(path)
    om.set_tp(2)
    om.init_cache(2, 128)
    for p, t in enumerate(prompt):
        want = om.forward(0, t, p, logits=(p == len(prompt) - 1))
    got = res[0]["logits"]
    assert np.array_equal(_bits(got[0]), _bits(want)), "prefill logits"
    tok, pos = int(np.argmax(want)), len(prompt)
    assert res[0]["toks"][0] == tok
    for k in range(W.HOST_STEPS):
        want = om.forward(0, tok, pos + k)
        assert np.array_equal(_bits(got[k + 1]), _bits(want)), f"host-loop step {k}"
        tok = int(np.argmax(want))
        assert res[0]["toks"][k + 1] == tok
    for p, t in enumerate(prompt):
        want = om.forward(1, t, p, logits=(p == len(prompt) - 1))
    tok = int(np.argmax(want))
    assert int(res[0]["gen_first"]) == tok
    for k in range(W.GEN_STEPS):
        want = om.forward(1, tok, pos + k)
        tok = int(np.argmax(want))
        assert res[0]["gen"][k] == tok, f"device-loop step {k}"
    assert np.array_equal(_bits(res[0]["gen_last"]), _bits(want)), "device-loop last logits"


def test_tp2_lost_peer_times_out(tmp_path):
    """Failure detection without a GPU fault: rank 1 skips a decode step while
    staying alive with its exchange buffer mapped (NVLS off, plain peer
    stores and flag loads).  Rank 0's exchange waits, bounded to 2 s of wall
    time, expire; the step's synchronization returns B2_ERR_TIMEOUT and both
    processes end normally."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    L, d, ff, nh, nkv, V, wt, ot, theta = MODELS["q4_0_hd64"]
    path = str(tmp_path / "m.gguf")
    b2.write_synthetic_llama(path, L, d, ff, nh, nkv, V, wt, out_type=ot, seed=21, rope_theta=theta)
    id_file = tmp_path / "nccl.id"
    id_file.write_bytes(b2.nccl_unique_id())
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-m", "tests.tp_worker", str(r), "2", str(id_file), path,
                               str(tmp_path / f"r{r}.npz"), "skip"], cwd=ROOT, env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=300)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{outs[r][-3000:]}"
    r0 = np.load(tmp_path / "r0.npz")
    assert int(r0["rc"]) == b2.ERR_TIMEOUT, f"rank 0 returned {int(r0['rc'])}"
    print(f"lost peer: b2_decode returned B2_ERR_TIMEOUT after {float(r0['secs']):.1f} s")
