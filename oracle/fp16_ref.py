"""Bit-level fp16 conversion references (numpy) — TEST INFRASTRUCTURE ONLY.

* ``to_half_rne``: IEEE round-to-nearest-even with subnormals, saturating to inf and
  keeping NaN — the semantics of the reference engine's ``FloatToHalfBitsRNE``
  (``src/vapoursynth/hip_engine.cc:1190-1232``); numpy's float32->float16 cast is
  exactly this rounding.
* ``to_half_ftz``: the load-time converter's ``float_to_half``
  (``src/vapoursynth/convert_float_to_float16.cpp:165-186``): the same rounding for
  normal results, but every input below the smallest normal half (|x| < 2^-14) becomes a
  signed zero and NaN becomes a signed infinity.
"""

from __future__ import annotations

import numpy as np


def to_half_rne(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_half_ftz(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    sign = ((bits >> 16) & 0x8000).astype(np.uint16)
    h = to_half_rne(x).copy()
    tiny = np.abs(x) < np.float32(2.0 ** -14)
    h[tiny] = sign[tiny]
    nan = np.isnan(x)
    h[nan] = sign[nan] | np.uint16(0x7C00)
    return h
