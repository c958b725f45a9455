"""Row-strip split of one large frame across GPUs (overlap-recompute).

A conv chain of L 3x3 layers (stride 1) has a receptive field of L rows above and below
each output row, so a frame split into horizontal strips can be run strip by strip, one
strip per GPU, with each strip extended by `halo = L` input rows on each side: the output
rows of the strip's own range are then identical to the whole-frame result, and no row
needs to be exchanged between GPUs. The extra work is 2 * halo rows per interior strip
(6.7 % for 8 strips of a 4320-row frame with the 18 convs of R8F64), in place of one halo
exchange per layer.

``plan_strips`` gives each rank's input window and the output rows it owns;
``run_strip`` runs one rank's window through an :class:`~arthip_b200.engine.Engine` and
returns its own output rows (host NCHW), and ``stitch`` concatenates the ranks' rows.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Strip:
    rank: int
    out_lo: int   # first input-resolution row this rank owns
    out_hi: int   # one past the last owned row
    in_lo: int    # first input row of the window (owned rows - halo, clamped)
    in_hi: int    # one past the last input row of the window

    @property
    def rows(self) -> int:
        return self.in_hi - self.in_lo


def conv_depth(model_path) -> int:
    """Number of 3x3 convs on the model's path, i.e. the receptive-field radius in rows
    (from the host-side parse and fusion, no GPU needed)."""
    from .engine import inspect_model
    return sum(1 for line in inspect_model(model_path)["ops"] if line.startswith("Conv"))


def plan_strips(height: int, n: int, halo: int) -> list[Strip]:
    """Split `height` rows into `n` contiguous owned ranges (as even as possible) and the
    input windows that reproduce them."""
    if n < 1 or height < n:
        raise ValueError(f"cannot split {height} rows into {n} strips")
    out = []
    for r in range(n):
        lo = r * height // n
        hi = (r + 1) * height // n
        out.append(Strip(r, lo, hi, max(0, lo - halo), min(height, hi + halo)))
    return out


def run_strip(engine, frame: np.ndarray, strip: Strip, scale: int) -> np.ndarray:
    """Run one strip's input window (NCHW host frame) and return the output rows it owns.
    `scale` is the model's upscale factor (output rows per input row)."""
    window = np.ascontiguousarray(frame[:, :, strip.in_lo:strip.in_hi, :])
    out = engine.run(window)
    a = (strip.out_lo - strip.in_lo) * scale
    return out[:, :, a:a + (strip.out_hi - strip.out_lo) * scale, :]


def stitch(parts: list[np.ndarray]) -> np.ndarray:
    """Concatenate the ranks' owned output rows (in rank order) into the frame."""
    return np.concatenate(parts, axis=2)


# ---------------------------------------------------------------------------
# Row strips with a 1-row halo exchange per layer
# ---------------------------------------------------------------------------
#
# Each rank owns rows [lo, hi) of the frame and runs its engine on rows + 2 rows: local row
# 0 is global row lo - 1 (the row above), rows 1..rows are its own, local row rows + 1 is
# global row hi (the row below). Before every layer, each activation's halo rows must hold
# the neighbours' values of the previous layer's output: after each op, a rank sends its
# first own row (local 1) to the rank above, which stores it as its local row rows + 1, and
# its last own row (local rows) to the rank below, which stores it as its local row 0. At
# the frame's top and bottom the halo row is the conv's zero padding and is zeroed instead.
# A conv computes its two halo output rows too (from a missing outer row), and the exchange
# then overwrites them. Only the 3x3 convs' one-row reach needs this: elementwise ops read
# the same row.


@dataclass(frozen=True)
class HaloStrip:
    rank: int
    world: int
    lo: int   # first owned row
    hi: int   # one past the last owned row

    @property
    def rows(self) -> int:
        return self.hi - self.lo

    @property
    def local_rows(self) -> int:
        """Rows the engine runs: the owned ones plus one halo row on each side."""
        return self.rows + 2


@dataclass(frozen=True)
class HaloMove:
    peer: int
    send_row: int   # local row sent to the peer
    recv_row: int   # local row the peer's row is stored in


def plan_halo_strips(height: int, n: int) -> list[HaloStrip]:
    """Split `height` rows into `n` contiguous owned ranges, as even as possible."""
    if n < 1 or height < 2 * n:
        raise ValueError(f"cannot split {height} rows into {n} strips of at least 2 rows")
    return [HaloStrip(r, n, r * height // n, (r + 1) * height // n) for r in range(n)]


def halo_moves(st: HaloStrip) -> tuple[list[HaloMove], list[int]]:
    """One layer's exchange for `st`: the row moves with each neighbour (upper first), and
    the local halo rows that are zero padding (frame edges)."""
    moves, zero = [], []
    if st.rank > 0:
        moves.append(HaloMove(st.rank - 1, 1, 0))
    else:
        zero.append(0)
    if st.rank < st.world - 1:
        moves.append(HaloMove(st.rank + 1, st.rows, st.rows + 1))
    else:
        zero.append(st.rows + 1)
    return moves, zero


def halo_window(frame: np.ndarray, st: HaloStrip) -> np.ndarray:
    """The strip's engine input (NCHW): its own rows plus the frame rows above and below,
    zero rows beyond the frame edges."""
    n, c, h, w = frame.shape
    out = np.zeros((n, c, st.local_rows, w), dtype=frame.dtype)
    a, b = max(0, st.lo - 1), min(h, st.hi + 1)
    out[:, :, a - (st.lo - 1):b - (st.lo - 1), :] = frame[:, :, a:b, :]
    return out


def exchange_dist(rows_view, st: HaloStrip) -> None:
    """One layer's halo exchange through torch.distributed point-to-point ops (NCCL over
    NVLink on GPUs, gloo on CPU). `rows_view` is this rank's activation as a [local_rows,
    row_bytes] tensor; with NCCL the copies are ordered on the current CUDA stream."""
    import torch.distributed as dist
    moves, zero = halo_moves(st)
    ops = []
    for m in moves:
        ops.append(dist.P2POp(dist.isend, rows_view[m.send_row], m.peer))
        ops.append(dist.P2POp(dist.irecv, rows_view[m.recv_row], m.peer))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    for r in zero:
        rows_view[r].zero_()


def exchange_local(views: list, strips: list[HaloStrip]) -> None:
    """The same exchange for all strips held in one process (one device): direct row
    copies between the strips' activations."""
    for st, v in zip(strips, views):
        moves, zero = halo_moves(st)
        for m in moves:
            v[m.recv_row].copy_(views[m.peer][_peer_send_row(strips[m.peer], st.rank)])
        for r in zero:
            v[r].zero_()


def _peer_send_row(peer: HaloStrip, to_rank: int) -> int:
    for m in halo_moves(peer)[0]:
        if m.peer == to_rank:
            return m.send_row
    raise ValueError(f"strip {peer.rank} sends nothing to {to_rank}")


def device_rows_view(ptr: int, rows: int, row_bytes: int, device):
    """A [rows, row_bytes] uint8 torch view of device memory owned by the engine."""
    import torch

    class _Buf:
        __cuda_array_interface__ = {"shape": (rows, row_bytes), "typestr": "|u1", "data": (ptr, False),
                                    "version": 3}
    return torch.as_tensor(_Buf(), device=device)


class HaloStripRunner:
    """One rank's strip of a large frame on its engine, with the per-layer halo exchange.

    `exchange(view)` performs one layer's exchange on this rank's [local_rows, row_bytes]
    activation view (``exchange_dist`` under torch.distributed). Ops are launched one at a
    time (``Engine.enqueue_ops``), with the exchange after every op but the last, all on the
    engine stream."""

    def __init__(self, engine, st: HaloStrip, width: int, channels: int, device):
        self.engine, self.st, self.device, self.width = engine, st, device, width
        self.in_ptr, self.out_ptr, self.in_bytes, self.out_bytes = engine.prepare(channels, st.local_rows, width)
        self.n_ops = len(engine.ops())
        self.views = []
        for i in range(self.n_ops):
            ptr, rows, rb, boundary = engine.op_output(i)
            self.views.append(None if boundary else device_rows_view(ptr, rows, rb, device))

    def load_input(self, window: np.ndarray) -> None:
        import torch
        src = torch.from_numpy(np.ascontiguousarray(window).reshape(-1).view(np.uint8)).to(self.device)
        dst = device_rows_view(self.in_ptr, 1, self.in_bytes, self.device)[0]
        dst.copy_(src)
        torch.cuda.synchronize(self.device)

    def run(self, exchange) -> None:
        import torch
        stream = torch.cuda.ExternalStream(self.engine.stream, device=self.device)
        with torch.cuda.stream(stream):
            for i in range(self.n_ops):
                self.engine.enqueue_ops(i, i + 1)
                if i + 1 < self.n_ops and self.views[i] is not None:
                    exchange(self.views[i])

    def own_output(self, scale: int) -> np.ndarray:
        """Host copy of the owned output rows (NCHW): local output rows [scale, scale * (rows + 1))."""
        dt = np.float32 if self.engine.out_fp32 else np.float16
        _, c, full_rows, full_w = self.engine.output_shape(self.engine.in_channels, self.st.local_rows, self.width)
        buf = device_rows_view(self.out_ptr, 1, self.out_bytes, self.device)[0].cpu().numpy().view(dt)
        full = buf.reshape(1, c, full_rows, full_w)
        return full[:, :, scale:scale * (self.st.rows + 1), :].copy()
