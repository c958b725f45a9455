"""Per-layer 1-row halo exchange of a frame split into row strips (host bookkeeping), on
CPU: the plan, the moves, and a chain of 3x3 convs run strip by strip with the exchange
between layers, both as gloo ranks (world size 2 and 3, torch.distributed point-to-point
ops, as the GPUs use NCCL) and in one process. The convs stand in for the engine's layers:
each computes all of its local rows, halo rows included, with zero padding beyond them, as
the tensor-core kernel does; integer-valued data keeps the float64 sums exact, so the
stitched strips must equal the whole-frame chain bit for bit."""

from __future__ import annotations

import json
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

from arthip_b200.strips import HaloStrip, exchange_local, halo_moves, halo_window, plan_halo_strips

ROOT = Path(__file__).resolve().parents[1]


def _layers(seed: int, n: int, c: int):
    rng = np.random.default_rng(seed)
    return [rng.integers(-2, 3, size=(c, c, 3, 3)).astype(np.float64) for _ in range(n)]


def _conv(x, w):
    import torch
    import torch.nn.functional as F
    t = torch.from_numpy(x)[None]
    return F.conv2d(t, torch.from_numpy(w), padding=1)[0].numpy()


def _whole(frame, layers):
    x = frame
    for w in layers:
        x = _conv(x, w)
    return x


def _strip_chain(frame, st: HaloStrip, layers, exchange):
    """One rank: its window (C, rows + 2, W), each layer then the exchange (as a
    [rows + 2, W * C] view of an NHWC activation)."""
    x = halo_window(frame[None], st)[0]
    for k, w in enumerate(layers):
        x = _conv(x, w)
        if k + 1 < len(layers):
            nhwc = np.ascontiguousarray(x.transpose(1, 2, 0))
            view = nhwc.reshape(st.local_rows, -1)
            exchange(view)
            x = np.ascontiguousarray(view.reshape(nhwc.shape).transpose(2, 0, 1))
    return x[:, 1:st.rows + 1, :]


@pytest.mark.parametrize("height,n", [(4320, 8), (37, 2), (11, 5), (6, 3)])
def test_plan_owns_every_row_once(height, n):
    s = plan_halo_strips(height, n)
    assert s[0].lo == 0 and s[-1].hi == height
    assert all(a.hi == b.lo for a, b in zip(s, s[1:]))
    assert all(x.rows >= 2 and x.local_rows == x.rows + 2 for x in s)


def test_moves_pair_up_and_edges_are_zero_padding():
    s = plan_halo_strips(100, 4)
    for st in s:
        moves, zero = halo_moves(st)
        for m in moves:
            peer_moves = {pm.peer: pm for pm in halo_moves(s[m.peer])[0]}
            back = peer_moves[st.rank]
            # what I send lands in the peer's halo row next to my strip, and vice versa
            assert (m.recv_row == 0) == (back.recv_row == s[m.peer].rows + 1)
            assert m.send_row in (1, st.rows) and m.recv_row in (0, st.rows + 1)
        assert zero == ([0] if st.rank == 0 else []) + ([st.rows + 1] if st.rank == 3 else [])


def test_halo_window_zero_beyond_the_frame():
    f = np.arange(2 * 6 * 3, dtype=np.float64).reshape(1, 2, 6, 3) + 1
    s = plan_halo_strips(6, 2)
    w0, w1 = halo_window(f, s[0]), halo_window(f, s[1])
    assert (w0[:, :, 0] == 0).all() and (w1[:, :, -1] == 0).all()
    np.testing.assert_array_equal(w0[:, :, 1:], f[:, :, 0:4])
    np.testing.assert_array_equal(w1[:, :, :-1], f[:, :, 2:6])


@pytest.mark.parametrize("height,n", [(23, 2), (30, 3), (19, 4)])
def test_local_exchange_chain_equals_whole_frame(height, n):
    import torch
    c, w = 3, 9
    layers = _layers(7, 5, c)
    frame = np.random.default_rng(1).integers(0, 4, size=(c, height, w)).astype(np.float64)
    want = _whole(frame, layers)
    strips = plan_halo_strips(height, n)
    xs = [halo_window(frame[None], st)[0] for st in strips]
    for k, wk in enumerate(layers):
        xs = [_conv(x, wk) for x in xs]
        if k + 1 < len(layers):
            nhwc = [torch.from_numpy(np.ascontiguousarray(x.transpose(1, 2, 0))) for x in xs]
            views = [t.reshape(st.local_rows, -1) for t, st in zip(nhwc, strips)]
            exchange_local(views, strips)
            xs = [t.numpy().transpose(2, 0, 1).copy() for t in nhwc]
    got = np.concatenate([x[:, 1:st.rows + 1] for x, st in zip(xs, strips)], axis=1)
    np.testing.assert_array_equal(got, want)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, height: int, out_dir: str):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": str(port)})
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch
    import torch.distributed as dist

    from arthip_b200.strips import exchange_dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    c, w = 3, 9
    layers = _layers(11, 4, c)
    frame = np.random.default_rng(2).integers(0, 4, size=(c, height, w)).astype(np.float64)
    st = plan_halo_strips(height, world)[rank]

    def exchange(view):
        t = torch.from_numpy(view)
        exchange_dist(t, st)

    mine = _strip_chain(frame, st, layers, exchange)
    np.save(Path(out_dir) / f"r{rank}.npy", mine)
    if rank == 0:
        np.save(Path(out_dir) / "whole.npy", _whole(frame, layers))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,height", [(2, 21), (3, 26)])
def test_gloo_ranks_exchange_halos_and_stitch_exactly(tmp_path, world, height):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), height, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    parts = [np.load(tmp_path / f"r{r}.npy") for r in range(world)]
    np.testing.assert_array_equal(np.concatenate(parts, axis=1), np.load(tmp_path / "whole.npy"))
