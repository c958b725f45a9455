"""Helpers shared by the GPU tests (tolerances and torch references)."""

from __future__ import annotations

import numpy as np

#: BASELINE parity bar, defined on the [0,1] output: max-abs and PSNR (peak 1.0).
MAX_ABS_TOL = 4e-3
PSNR_MIN_DB = 55.0


def ulp16(v: np.ndarray) -> np.ndarray:
    """Spacing of fp16 values at |v| (normal range; subnormal spacing below 2^-14)."""
    a = np.maximum(np.abs(v.astype(np.float64)), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(a)) - 10)


def assert_fp16_layer_close(got: np.ndarray, ref: np.ndarray, label: str, scale: np.ndarray | None = None,
                            min_exact: float = 0.99, ulps: float = 2.0) -> None:
    """One fused layer against an fp32 reference that applies the same fp16 roundings.

    Both compute the conv in fp32 with different summation orders (errors ~1e-6 of the
    sum of |terms|), so an element may land on the other side of an fp16 rounding
    boundary: allow one fp16 ulp of the largest intermediate magnitude (`scale`, default
    |ref|; with residual adds |ref| + sum |adds|), doubled for the cascade through the
    adds, plus 1e-4 absolute; nearly every element must match exactly."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert got.shape == ref.shape, f"{label}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{label}: non-finite output"
    s = np.abs(ref) if scale is None else np.maximum(np.abs(ref), scale)
    d = np.abs(got - ref)
    lim = ulps * ulp16(s) + 1e-4
    bad = d > lim
    assert not bad.any(), (f"{label}: {int(bad.sum())} elements beyond tolerance; max diff {d.max():.3g}"
                           f" at |ref|={np.abs(ref).flat[int(np.argmax(d))]:.3g}")
    exact = float((d == 0).mean())
    assert exact >= min_exact, f"{label}: only {exact:.4f} of elements exact"


def assert_frame_parity(got: np.ndarray, ref: np.ndarray, label: str, tol: float | None = None,
                        rel_tol: float | None = None) -> tuple[float, float]:
    """BASELINE's bar for a frame: max-abs <= 4e-3 and PSNR >= 55 dB on the [0,1] output.

    The synthetic ReLU configs end without a Clip and span about [-7, 7], where one fp16
    ulp is 3.9e-3; there the bar is applied to the [0,1]-clipped frame (what the metric
    is defined on), and the full range is checked relative to magnitude: every element
    within `rel_tol` (default max(tol, 2^-8)) * max(1, |ref|), PSNR >= 55 dB with the
    frame's own peak."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert got.shape == ref.shape, f"{label}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{label}: non-finite output"
    tol = MAX_ABS_TOL if tol is None else tol
    gc, rc = np.clip(got, 0, 1), np.clip(ref, 0, 1)
    d01 = float(np.abs(gc - rc).max())
    mse01 = float(np.mean((gc - rc) ** 2))
    psnr01 = float("inf") if mse01 == 0 else 10 * np.log10(1.0 / mse01)
    assert d01 <= tol, f"{label}: [0,1] max abs diff {d01:.4g} > {tol:.4g}"
    assert psnr01 >= PSNR_MIN_DB, f"{label}: [0,1] PSNR {psnr01:.2f} dB < {PSNR_MIN_DB}"
    rel = np.abs(got - ref) / np.maximum(1.0, np.abs(ref))
    rtol = max(tol, 2.0 ** -8) if rel_tol is None else rel_tol
    assert float(rel.max()) <= rtol, f"{label}: full-range relative diff {rel.max():.4g} > {rtol:.4g}"
    peak = float(np.abs(ref).max()) or 1.0
    mse = float(np.mean((got - ref) ** 2))
    psnr = float("inf") if mse == 0 else 10 * np.log10(peak * peak / mse)
    assert psnr >= PSNR_MIN_DB, f"{label}: full-range PSNR {psnr:.2f} dB"
    return d01, psnr01


ULP1 = 2.0 ** -10  # fp16 spacing just below 1.0


def report_parity(label: str, d16: float, p16: float, d32: float, p32: float, bar: float) -> None:
    """Prints the achieved parity of a frame test and, when ARTHIP_PARITY_LOG names a file,
    appends it there as one tab-separated line (label, max-abs and [0,1] PSNR against the
    typed fp16 graph, the same against fp32 between nodes, the max-abs bar applied)."""
    import os
    line = f"{label}\t{d16:.4g}\t{p16:.2f}\t{d32:.4g}\t{p32:.2f}\t{bar:.4g}"
    print("PARITY " + line)
    path = os.environ.get("ARTHIP_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")


def _gap01(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.abs(np.clip(a, 0, 1) - np.clip(b, 0, 1)).max())


def _relgap(a: np.ndarray, b: np.ndarray) -> float:
    return float((np.abs(a - b) / np.maximum(1.0, np.abs(b))).max())


def check_against_oracles(got: np.ndarray, ref16: np.ndarray, ref32: np.ndarray, variants16: list, label: str):
    """The engine against the oracle, with the bar derived from the oracle itself.

    `ref16` is the typed fp16 graph (every node rounded to fp16, fp32 sums): the engine
    must be within max-abs 4e-3 (PSNR >= 55 dB) of it on the [0,1] output, or, where
    other valid executions of the same fp16 graph (`variants16`: other summation orders,
    float64 sums) are already further apart than that, within their spread plus one fp16
    ulp at 1.0; the full-range relative check is widened the same way. `ref32` (fp32
    between nodes) brackets how a runtime may execute the graph instead: the engine must
    be within that bracket's width of it (the fp16 bar plus the two oracles' own gap),
    with PSNR >= 55 dB."""
    allv = [ref16] + list(variants16)
    spread = max((_gap01(a, b) for i, a in enumerate(allv) for b in allv[i + 1:]), default=0.0)
    rspread = max((_relgap(a, b) for i, a in enumerate(allv) for b in allv[i + 1:]), default=0.0)
    tol16 = MAX_ABS_TOL if spread <= MAX_ABS_TOL - ULP1 else spread + ULP1
    rel16 = max(tol16, 2.0 ** -8, rspread + ULP1)
    gap, rgap = _gap01(ref16, ref32), _relgap(ref32, ref16)
    print(f"{label}: engine vs fp16_nodes {_gap01(got, ref16):.4g} (oracle spread {spread:.4g}, bar {tol16:.4g}); "
          f"vs fp32_nodes {_gap01(got, ref32):.4g} (oracle gap {gap:.4g})")
    d16, p16 = assert_frame_parity(got, ref16, f"{label} vs oracle fp16_nodes", tol16, rel16)
    d32, p32 = assert_frame_parity(got, ref32, f"{label} vs oracle fp32_nodes", tol16 + gap, rel16 + rgap)
    report_parity(f"{label} (oracle spread {spread:.3g})", d16, p16, d32, p32, tol16)


def torch_conv_layer(x_nhwc, w_oihw, bias, act, adds):
    """fp32 cuDNN reference of one fused layer with the engine's fp16 node roundings."""
    import torch
    import torch.nn.functional as F
    torch.backends.cudnn.allow_tf32 = False
    x = x_nhwc.float().permute(0, 3, 1, 2)
    w = torch.as_tensor(w_oihw.astype(np.float16).astype(np.float32), device=x.device)
    b = None if bias is None else torch.as_tensor(bias.astype(np.float16).astype(np.float32), device=x.device)
    y = F.conv2d(x, w, b, padding=1).half().float()
    if act == 1:
        y = torch.clamp_min(y, 0)
    elif act == 2:
        s = torch.sigmoid(y).half().float()
        y = (y * s).half().float()
    for a in adds:
        y = (y + a.float().permute(0, 3, 1, 2)).half().float()
    return y.permute(0, 2, 3, 1).contiguous()
