"""Host-side logic of the multi-GPU bench on CPU (gloo, world size 2): the max-over-ranks
time, the barrier, disjoint frame shares per rank, and the reference arm printing only on
rank 0. The GPU data path has no collective, so nothing else crosses ranks."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, str(ROOT))
    import bench
    import torch.distributed as dist
    w, r, _ = bench.dist_setup(backend="gloo")
    m = bench.dist_max(1.5 + r, w)
    bench.dist_barrier(w)
    seeds = bench.frame_seeds(r, 8)
    Path(out_dir, f"r{r}.json").write_text(json.dumps({"world": w, "max": m, "seeds": seeds,
                                                        "nccl_log": [os.environ.get("NCCL_DEBUG"),
                                                                     os.environ.get("NCCL_DEBUG_FILE")]}))
    dist.destroy_process_group()


def test_gloo_world2_max_and_disjoint_frame_shares(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    res = [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(2)]
    assert all(x["world"] == 2 for x in res)
    assert all(x["max"] == 2.5 for x in res)  # max over ranks, seen by every rank
    assert not set(res[0]["seeds"]) & set(res[1]["seeds"])
    # stdout carries only the JSON line: NCCL's log (its version banner included) goes to stderr
    assert all(x["nccl_log"] == ["WARN", "/dev/stderr"] for x in res)


def test_reference_arm_prints_only_on_rank0():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1"],
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0
    assert r.stdout.strip() == ""


def test_reference_arm_line_on_rank0():
    env = dict(os.environ, RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "frames/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
