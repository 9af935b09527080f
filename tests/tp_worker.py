"""One rank of a tensor-parallel run, for tests/test_gpu_tp.py (not a test file).

    python tests/tp_worker.py RANK WORLD GGUF IDFILE OUT [VOCAB]

Runs on the GPU named by CUDA_VISIBLE_DEVICES. Rank 0 creates the NCCL group
id and writes it to IDFILE; the other ranks wait for it (bounded). Every rank
makes the same calls in the same order: prefill, teacher-forced decode steps,
a greedy loop, batched decode of sessions forked from the prompt. Rank 0
writes the logits and ids to OUT (.npz).
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from imurun_b200 import native  # noqa: E402

N_PROMPT, N_DEC, N_GREEDY = 40, 6, 8


def main() -> int:
    rank, world, path, idfile, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], sys.argv[5]
    vocab = int(sys.argv[6]) if len(sys.argv) > 6 else 128256
    lib = native.load_library()
    if rank == 0:
        gid = native.tp_unique_id(lib)
        tmp = idfile + ".tmp"
        with open(tmp, "wb") as f:
            f.write(gid)
        os.replace(tmp, idfile)
    else:
        t0 = time.time()
        while not os.path.exists(idfile):
            if time.time() - t0 > 120:
                print("no group id", file=sys.stderr)
                return 2
            time.sleep(0.05)
        gid = open(idfile, "rb").read()
    ids = np.random.default_rng(21).integers(3, vocab, N_PROMPT + N_DEC).astype(np.int32)
    with native.Model(path, 1024, lib=lib, tp=(rank, world, gid)) as m:
        steps = [m.prefill(ids[:N_PROMPT], 0)]
        am = []
        for s in range(N_PROMPT, N_PROMPT + N_DEC):
            lg, a = m.decode(ids[s:s + 1], s)
            steps.append(lg[0].copy())
            am.append(int(a[0]))
        # greedy from the last prompt token, and the same steps teacher-forced
        m.set_kv_len(N_PROMPT + N_DEC)
        first = int(am[-1])
        greedy = m.greedy(first, N_GREEDY)
        m.set_kv_len(N_PROMPT + N_DEC)
        tok, forced = first, []
        for s in range(N_GREEDY):
            _, a = m.decode(np.array([tok], np.int32), N_PROMPT + N_DEC + s)
            tok = int(a[0])
            forced.append(tok)
        # batched decode: three sessions forked from the prompt, fed the same
        # ids on every run (not their argmax, which may differ where the
        # margin is below the bar)
        sids = [m.session_fork(0, N_PROMPT) for _ in range(3)]
        for k in range(2):
            _, blg = m.decode_batch(sids, ids[N_PROMPT + 3 * k:N_PROMPT + 3 * k + 3], logits=True)
            steps.extend(blg.copy())
    if rank == 0:
        np.savez(out, logits=np.stack(steps), argmax=np.array(am, np.int32), greedy=np.asarray(greedy, np.int32),
                 forced=np.array(forced, np.int32), ids=ids)
    return 0


if __name__ == "__main__":
    sys.exit(main())
