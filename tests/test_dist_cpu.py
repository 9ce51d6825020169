"""bench.py's multi-rank logic on the host (no GPU): two gloo ranks (world size 2) as separate processes.

The data path has no collective (utterances are sharded by rank); the only cross-rank steps are the
start/stop barriers and the max-over-ranks of the timed region, and those are what is checked here. The
reference arm runs on rank 0 alone; another rank exits 0 at once without a process group."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

RANK_CODE = r"""
import json, os, sys, torch
sys.path.insert(0, os.getcwd())
import bench
world, rank, local = bench.setup_dist()
import torch.distributed as dist
assert dist.get_backend() == "gloo"
bench.barrier(world)
t = bench.max_over_ranks(1.5 + rank, world, torch.device("cpu"))
bench.barrier(world)
dist.destroy_process_group()
print(json.dumps({"rank": rank, "world": world, "max": t}))
"""


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> dict:
    env = dict(os.environ)
    env.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
               WORLD_SIZE=str(world), CUDA_VISIBLE_DEVICES="")  # fmt: skip
    return env


def test_two_gloo_ranks_take_the_max_time():
    port = _port()
    procs = [subprocess.Popen([sys.executable, "-c", RANK_CODE], cwd=ROOT, env=_env(r, 2, port),
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in range(2)]  # fmt: skip
    outs = []
    for p in procs:
        out, err = p.communicate(timeout=240)
        assert p.returncode == 0, err[-2000:]
        outs.append(json.loads(out.strip().splitlines()[-1]))
    assert sorted(o["rank"] for o in outs) == [0, 1]
    assert all(o["world"] == 2 and o["max"] == 2.5 for o in outs)


def test_reference_arm_other_ranks_exit_without_work():
    """Under torchrun the reference arm's rank 1 prints nothing and exits 0 (no process group is made)."""
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "1"], cwd=ROOT, env=_env(1, 2, _port()), capture_output=True, text=True,
                       timeout=240)  # fmt: skip
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""
