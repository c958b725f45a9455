"""Helpers shared by the GPU tests (tolerances and torch references)."""

from __future__ import annotations

import numpy as np

#: BASELINE parity bar for fp16 frame outputs in [0,1]-scale: max-abs and PSNR (peak 1.0).
MAX_ABS_TOL = 4e-3
PSNR_MIN_DB = 55.0


def ulp16(v: np.ndarray) -> np.ndarray:
    """Spacing of fp16 values at |v| (normal range; subnormal spacing below 2^-14)."""
    a = np.maximum(np.abs(v.astype(np.float64)), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(a)) - 10)


def assert_fp16_layer_close(got: np.ndarray, ref: np.ndarray, label: str, max_ulps: float = 2.0,
                            min_exact: float = 0.98) -> None:
    """A single fused layer against its fp32 reference rounded the same way: differences
    come only from accumulation order flipping an fp16 rounding, so every element must be
    within `max_ulps` fp16 ulps and nearly all must match exactly."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert got.shape == ref.shape, f"{label}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{label}: non-finite output"
    d = np.abs(got - ref)
    lim = max_ulps * ulp16(ref) + 1e-7
    worst = float((d / lim).max())
    assert worst <= 1.0, f"{label}: max diff {d.max():.3g} ({worst * max_ulps:.2f} ulp)"
    exact = float((d == 0).mean())
    assert exact >= min_exact, f"{label}: only {exact:.4f} of elements exact"


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
