"""The native library loads on a CPU-only host and exports the whole C ABI; host-side
conversions are bit-exact against the numpy references. No GPU compute is called."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from arthip_b200 import native
from oracle import fp16_ref

HEADER = Path(__file__).resolve().parents[1] / "include" / "arthip_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)
    keywords = {"if", "sizeof", "return", "defined"}
    return sorted({n for n in names if n not in keywords and (n.startswith("ah_") or n.startswith("engine_"))})


def test_library_loads_and_exports_every_declared_symbol():
    lib = native.lib()
    decl = declared_functions()
    assert len(decl) >= 25
    missing = [n for n in decl if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # The binding table covers the same set.
    assert set(decl) == set(native.SIGNATURES), set(decl) ^ set(native.SIGNATURES)
    assert lib.ah_version().decode().startswith("arthip_b200")


def _all_special_floats():
    rng = np.random.default_rng(0)
    vals = [rng.standard_normal(200_000).astype(np.float32) * s for s in (1e-9, 1e-7, 6e-5, 1e-3, 1.0, 3e4, 7e4)]
    # every fp16 value, its neighbours and midpoints (exercises ties and boundaries)
    h = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    h = h[np.isfinite(h)]
    up = np.nextafter(h, np.float32(np.inf))
    dn = np.nextafter(h, np.float32(-np.inf))
    mids = ((h[:-1].astype(np.float64) + h[1:].astype(np.float64)) / 2).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 65504, 65519.99, 65520, 65536, 2 ** -14, 2 ** -24,
                        2 ** -25, 2 ** -25 * 1.0000001, 3e-8, 6.1e-5], dtype=np.float32)
    return np.concatenate(vals + [h, up, dn, mids, special, -special]).astype(np.float32)


def test_float_to_half_rne_bit_exact():
    lib = native.lib()
    x = np.ascontiguousarray(_all_special_floats())
    out = np.zeros(x.size, dtype=np.uint16)
    lib.ah_float_to_half_rne(x.ctypes.data, out.ctypes.data, x.size)
    ref = fp16_ref.to_half_rne(x)
    nan = np.isnan(x)
    assert np.array_equal(out[~nan], ref[~nan])
    assert np.all((out[nan] & 0x7C00) == 0x7C00) and np.all((out[nan] & 0x3FF) != 0)


def test_float_to_half_ftz_bit_exact():
    lib = native.lib()
    x = np.ascontiguousarray(_all_special_floats())
    out = np.zeros(x.size, dtype=np.uint16)
    lib.ah_float_to_half_ftz(x.ctypes.data, out.ctypes.data, x.size)
    assert np.array_equal(out, fp16_ref.to_half_ftz(x))


def test_half_to_float_exact_for_every_half():
    lib = native.lib()
    h = np.arange(65536, dtype=np.uint16)
    out = np.zeros(h.size, dtype=np.float32)
    lib.ah_half_to_float(h.ctypes.data, out.ctypes.data, h.size)
    ref = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(out[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.array_equal(np.isnan(out), np.isnan(ref))
