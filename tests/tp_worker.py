"""One tensor-parallel rank of the multi-GPU parity tests, run as a child
process: python -m tests.tp_worker RANK WORLD ID_FILE MODEL OUT_NPZ.

Loads MODEL as rank RANK of WORLD (device = rank, NCCL id from ID_FILE),
prefills a fixed prompt, then runs greedy steps both through the host loop
(b2_decode + logits) and through b2_generate, and saves logits and ids."""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "arkantos-ai-stack-suite_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import b2gguf as b2  # noqa: E402

PROMPT = [5, 17, 250, 3, 99, 42, 7, 11, 300, 1, 64]
# a prompt long enough for the tensor-core prefill (all but its last 8 tokens)
LONG_PROMPT = [(37 * i + 11) % 500 for i in range(90)]
HOST_STEPS = 5
GEN_STEPS = 6


def main() -> int:
    rank, world, id_file, model, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5]
    prompt = LONG_PROMPT if len(sys.argv) > 6 and sys.argv[6] == "long" else PROMPT
    with open(id_file, "rb") as f:
        nccl_id = f.read()
    m = b2.Model(model, device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    ctx = b2.Context(m, n_ctx=128, n_seq=2)
    if len(sys.argv) > 6 and sys.argv[6] == "skip":
        return skip_step(rank, ctx, out)
    ctx.decode(prompt, want_logits=2)
    logits = [ctx.logits(-1)]
    tok = int(ctx.argmax()[0][-1])
    toks = [tok]
    for k in range(HOST_STEPS):
        ctx.decode([tok], want_logits=1)
        logits.append(ctx.logits(0))
        tok = int(ctx.argmax()[0][0])
        toks.append(tok)
    # sequence 1: the same prompt, then the device-side greedy loop
    ctx.decode(prompt, pos=list(range(len(prompt))), seq=[1] * len(prompt), want_logits=2)
    first = int(ctx.argmax()[0][-1])
    gen = ctx.generate([first], GEN_STEPS, seq=[1])
    last = ctx.logits(0)
    ctx.synchronize()
    np.savez(out, logits=np.stack(logits), toks=np.array(toks, np.int32), gen=gen.ravel(), gen_first=first,
             gen_last=last)
    return 0


def skip_step(rank: int, ctx, out: str) -> int:
    """A lost peer, made on the host: both ranks run the prompt; then rank 0
    decodes one more token while rank 1 skips it, alive and with its
    exchange buffer mapped.  Rank 0's bounded exchange waits run out and the
    step's synchronization (b2_decode is asynchronous) returns
    B2_ERR_TIMEOUT; rank 1 then exits between steps, with nothing of its own
    in flight."""
    ctx.decode(PROMPT, want_logits=2)
    ctx.synchronize()
    done = out + ".done"
    rc, secs = 0, 0.0
    if rank == 0:
        toks = np.array([7], np.int32)
        pos = np.array([len(PROMPT)], np.int32)
        seq = np.array([0], np.int32)
        t0 = time.time()
        rc = b2.lib.b2_decode(ctx.h, b2.ptr(toks), b2.ptr(pos), b2.ptr(seq), 1, 1)
        if rc == 0:   # the step runs asynchronously; its status comes with the synchronization
            rc = b2.lib.b2_synchronize_context(ctx.h)
        secs = time.time() - t0
        with open(done, "w") as f:
            f.write("1")
    else:
        t0 = time.time()
        while not os.path.exists(done.replace("r1.npz", "r0.npz")) and time.time() - t0 < 120:
            time.sleep(0.05)
    np.savez(out, rc=rc, secs=secs)
    return 0


if __name__ == "__main__":
    sys.exit(main())
