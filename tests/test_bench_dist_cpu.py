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


def _fake_smi(tmp_path: Path, monkeypatch):
    """An `nvidia-smi` on PATH that prints one CSV row every 20 ms with a rising SM clock
    and sw_power_cap active, as `--query-gpu ... -lms` does."""
    smi = tmp_path / "nvidia-smi"
    smi.write_text(
        f"#!{sys.executable}\n"
        "import sys, time\n"
        "i = 0\n"
        "while True:\n"
        "    print(f'0, {1000 + i}, 1965, 700.5, 0x4, Not Active, Not Active, Not Active, Active', flush=True)\n"
        "    i += 1\n"
        "    time.sleep(0.02)\n")
    smi.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ.get('PATH', '')}")


def test_clock_sampler_keeps_only_the_timed_window(tmp_path, monkeypatch):
    import time
    sys.path.insert(0, str(ROOT))
    import bench
    _fake_smi(tmp_path, monkeypatch)
    clk = bench.ClockSampler(None).start()
    try:
        clk.wait_first(10.0)
        assert clk.rows, "the sampler saw no row before the window"
        time.sleep(0.2)
        with clk.window():
            time.sleep(0.3)
        time.sleep(0.2)
    finally:
        clk.stop()
    s = clk.summary()
    inside = [float(r[1]) for t, r in clk.rows if clk.t0 <= t <= clk.t1]
    assert s["samples"] == len(inside) >= 3
    assert len(clk.rows) > s["samples"]  # rows before and after the window are dropped
    assert min(inside) <= s["sm_mhz"] <= max(inside)
    assert s["sm_max_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 700.5


def test_clock_sampler_short_window_takes_the_next_row(tmp_path, monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    _fake_smi(tmp_path, monkeypatch)
    clk = bench.ClockSampler(None).start()
    try:
        clk.wait_first(10.0)
        with clk.window():
            pass
    finally:
        clk.stop()
    s = clk.summary()
    assert s["samples"] >= 1 and s["sm_mhz"] is not None and s["reasons"] == ["sw_power_cap"]


def test_clock_sampler_without_nvidia_smi_reports_unsampled(tmp_path, monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setenv("PATH", str(tmp_path))
    clk = bench.ClockSampler(None).start()
    clk.wait_first(0.5)
    with clk.window():
        pass
    clk.stop()
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
