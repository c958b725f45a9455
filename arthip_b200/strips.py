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
