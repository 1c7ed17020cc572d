"""One tensor-parallel rank of the multi-GPU parity tests, run as a child
process: python -m tests.tp_worker RANK WORLD ID_FILE MODEL OUT_NPZ.

Loads MODEL as rank RANK of WORLD (device = rank, NCCL id from ID_FILE),
prefills a fixed prompt, then runs greedy steps both through the host loop
(b2_decode + logits) and through b2_generate, and saves logits and ids."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "arkantos-ai-stack-suite_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import b2gguf as b2  # noqa: E402

PROMPT = [5, 17, 250, 3, 99, 42, 7, 11, 300, 1, 64]
HOST_STEPS = 5
GEN_STEPS = 6


def main() -> int:
    rank, world, id_file, model, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5]
    with open(id_file, "rb") as f:
        nccl_id = f.read()
    m = b2.Model(model, device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    ctx = b2.Context(m, n_ctx=64, n_seq=2)
    ctx.decode(PROMPT, want_logits=2)
    logits = [ctx.logits(-1)]
    tok = int(ctx.argmax()[0][-1])
    toks = [tok]
    for k in range(HOST_STEPS):
        ctx.decode([tok], want_logits=1)
        logits.append(ctx.logits(0))
        tok = int(ctx.argmax()[0][0])
        toks.append(tok)
    # sequence 1: the same prompt, then the device-side greedy loop
    ctx.decode(PROMPT, pos=list(range(len(PROMPT))), seq=[1] * len(PROMPT), want_logits=2)
    first = int(ctx.argmax()[0][-1])
    gen = ctx.generate([first], GEN_STEPS, seq=[1])
    last = ctx.logits(0)
    ctx.synchronize()
    np.savez(out, logits=np.stack(logits), toks=np.array(toks, np.int32), gen=gen.ravel(), gen_first=first,
             gen_last=last)
    return 0


if __name__ == "__main__":
    sys.exit(main())
