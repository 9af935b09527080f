"""Host logic of the multi-GPU runs, on the CPU: two gloo ranks (as
torch.distributed.run starts them) through bench.py's own helpers — the
per-rank device choice, the NCCL group id handed from rank 0 to every rank,
the max-over-ranks timing and the barrier. No GPU and no NCCL are touched."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

RANK_CODE = r"""
import json, os, sys
sys.path.insert(0, {root!r})
import bench
dist = bench.dist_init()
gid = bench.share_group_id(dist, lambda: bytes(range(128)))
t = bench.max_over_ranks(dist, 1.5 + bench.RANK)
bench.barrier(dist)
with open({out!r} + str(bench.RANK), "w") as f:
    json.dump({{"rank": bench.RANK, "world": bench.WORLD, "vis": os.environ["CUDA_VISIBLE_DEVICES"],
               "gid": list(gid), "tmax": t}}, f)
dist.destroy_process_group()
"""


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_share_group_id_and_max_time(tmp_path):
    out = str(tmp_path / "rank")
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="4,5")
        procs.append(subprocess.Popen([sys.executable, "-c", RANK_CODE.format(root=str(ROOT), out=out)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    logs = [p.communicate(timeout=300)[0].decode(errors="replace") for p in procs]
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)
    res = [json.load(open(out + str(r))) for r in range(2)]
    for r, d in enumerate(res):
        assert d["rank"] == r and d["world"] == 2
        assert d["gid"] == list(range(128))          # rank 0's id reached every rank
        assert d["tmax"] == 2.5                        # the slower rank's time
    assert [d["vis"] for d in res] == ["4", "5"]     # one visible GPU per rank, in rank order


def test_rank_device_choice_without_visible_list():
    code = f"import sys; sys.path.insert(0, {str(ROOT)!r}); import bench, os; print(os.environ['CUDA_VISIBLE_DEVICES'])"
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    env.pop("CUDA_VISIBLE_DEVICES", None)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().splitlines()[-1] == "1", r.stdout + r.stderr
