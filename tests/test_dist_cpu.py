"""The multi-rank plumbing of bench.py on CPU: two gloo ranks (no GPU) share
rank 0's NCCL id and model path and agree on max-over-ranks timings."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    d, r, w, local = bench.dist_init()
    assert (r, w, local) == (rank, world, rank)
    nccl_id, path = bench.tp_share(d, r, w, lambda: bytes(range(128)), f"/dev/shm/model_from_rank{r}.gguf")
    slowest = bench.dist_max(d, 1.5 + r)
    bench.barrier(d)
    q.put((r, nccl_id, path, slowest))
    d.destroy_process_group()


def test_two_gloo_ranks_share_tp_setup():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    got = sorted(q.get(timeout=10) for _ in range(2))
    for r, nccl_id, path, slowest in got:
        assert nccl_id == bytes(range(128))
        assert path == "/dev/shm/model_from_rank0.gguf"
        assert slowest == 2.5
