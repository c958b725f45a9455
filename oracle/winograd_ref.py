"""The reference's Winograd F(2x2,3x3) convolution numerics, restated in torch — TEST
INFRASTRUCTURE ONLY (the checker of the Winograd kernel; nothing in the product imports it).

Follows the reference's gfx1100 kernel and weight transform:
* weights ``U = G g G^T`` per (output, input channel), computed in fp32 in the order of
  ``src/vapoursynth/hip_engine.cc:972-998`` (``Gg = G g``, then ``Gg G^T``, sums over k in
  ascending order) and rounded to fp16 with round-to-nearest-even (``:999-1000``);
* input transform ``V = B^T d B`` on the 4x4 input tile in fp16 arithmetic: the column
  combinations of each row first, each rounded to fp16, then the row combinations, rounded
  again (``winograd_in4_v4``, ``src/common/hip_kernels.h:86-97``);
* the 16 per-point channel contractions ``M = sum_c U V`` accumulated in fp32 (the WMMA
  f32 accumulators, ``:242-276``), the output transform ``Y = A^T M A`` in fp32 (``FOLD4``,
  ``:133-141``).
The epilogue then follows the ONNX graph as the engine does: ``Y + bias`` rounded to fp16
once (the Conv node), the activation, and the residual adds each rounded to fp16.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

_G = np.array([[1.0, 0.0, 0.0], [0.5, 0.5, 0.5], [0.5, -0.5, 0.5], [0.0, 0.0, 1.0]], dtype=np.float32)


def weight_transform(w_oihw: np.ndarray) -> np.ndarray:
    """U[m, c, 4, 4] as fp16, from fp16-valued weights [M, C, 3, 3]."""
    g = w_oihw.astype(np.float32)
    gg = np.zeros(g.shape[:2] + (4, 3), dtype=np.float32)
    for r in range(4):
        for cc in range(3):
            acc = np.zeros(g.shape[:2], dtype=np.float32)
            for k in range(3):
                acc = acc + np.float32(_G[r, k]) * g[:, :, k, cc]
            gg[:, :, r, cc] = acc
    u = np.zeros(g.shape[:2] + (4, 4), dtype=np.float32)
    for r in range(4):
        for cc in range(4):
            acc = np.zeros(g.shape[:2], dtype=np.float32)
            for k in range(3):
                acc = acc + gg[:, :, r, k] * np.float32(_G[cc, k])
            u[:, :, r, cc] = acc
    return u.astype(np.float16)


def _input_transform(d: torch.Tensor) -> torch.Tensor:
    """d: [..., 4, 4] fp16 tiles -> V [..., 4, 4] fp16 (columns first, then rows)."""
    c0, c1, c2, c3 = d[..., 0], d[..., 1], d[..., 2], d[..., 3]
    t = torch.stack([c0 - c2, c1 + c2, c2 - c1, c1 - c3], dim=-1)  # fp16 ops round each result
    r0, r1, r2, r3 = t[..., 0, :], t[..., 1, :], t[..., 2, :], t[..., 3, :]
    return torch.stack([r0 - r2, r1 + r2, r2 - r1, r1 - r3], dim=-2)


def conv_layer(x_nhwc: torch.Tensor, w_oihw: np.ndarray, bias, act: int, adds) -> torch.Tensor:
    """One fused layer with the Winograd numerics above; x and adds are fp16 NHWC
    [1, H, W, C] tensors (any device). Returns fp32 NHWC holding fp16 values."""
    dev = x_nhwc.device
    _, H, W, C = x_nhwc.shape
    M = w_oihw.shape[0]
    th, tw = (H + 1) // 2, (W + 1) // 2
    x = x_nhwc.permute(0, 3, 1, 2).half()
    xp = F.pad(x, (1, 2 * tw + 2 - W - 1, 1, 2 * th + 2 - H - 1))
    d = xp.unfold(2, 4, 2).unfold(3, 4, 2)  # [1, C, th, tw, 4, 4]
    v = _input_transform(d)  # fp16 arithmetic: every add / sub rounded to fp16
    u = torch.from_numpy(weight_transform(w_oihw)).to(dev).float()  # [M, C, 4, 4]
    vf = v.float()[0]  # [C, th, tw, 4, 4]
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        m = torch.einsum("mcpq,ctupq->mtupq", u, vf)  # fp32 sums over C
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    # fold the columns q first (j), then the rows p (i), as FOLD4 does
    sq = [m[..., 0] + m[..., 1] + m[..., 2], m[..., 1] - m[..., 2] - m[..., 3]]  # j = 0, 1: [M, th, tw, 4(p)]
    y = torch.stack([torch.stack([s[..., 0] + s[..., 1] + s[..., 2], s[..., 1] - s[..., 2] - s[..., 3]], dim=-1)
                     for s in sq], dim=-1)  # [M, th, tw, 2(i), 2(j)]
    y = y.permute(0, 1, 3, 2, 4).reshape(M, 2 * th, 2 * tw)[:, :H, :W]
    if bias is not None:
        y = y + torch.as_tensor(np.asarray(bias, dtype=np.float16).astype(np.float32), device=dev).view(-1, 1, 1)
    y = y.half().float()
    if act == 1:
        y = torch.clamp_min(y, 0)
    elif act == 2:
        y = (y * torch.sigmoid(y).half().float()).half().float()
    y = y.permute(1, 2, 0)[None]
    for a in adds:
        y = (y + a.float()).half().float()
    return y.contiguous()


def conv2d_nchw(x: torch.Tensor, w: torch.Tensor, b) -> torch.Tensor:
    """Conv output before the node's fp16 rounding (Y + bias in fp32) with the Winograd
    numerics, for an NCHW fp32 tensor holding fp16 values: the form the ONNX oracle's
    executor takes for its Conv node (``onnx_cpu._Exec.conv``)."""
    _, C, H, W = x.shape
    M = w.shape[0]
    th, tw = (H + 1) // 2, (W + 1) // 2
    xp = F.pad(x.half(), (1, 2 * tw + 2 - W - 1, 1, 2 * th + 2 - H - 1))
    v = _input_transform(xp.unfold(2, 4, 2).unfold(3, 4, 2)).float()[0]
    u = torch.from_numpy(weight_transform(w.cpu().numpy().astype(np.float16))).to(x.device).float()
    m = torch.einsum("mcpq,ctupq->mtupq", u, v)
    sq = [m[..., 0] + m[..., 1] + m[..., 2], m[..., 1] - m[..., 2] - m[..., 3]]
    y = torch.stack([torch.stack([s[..., 0] + s[..., 1] + s[..., 2], s[..., 1] - s[..., 2] - s[..., 3]], dim=-1)
                     for s in sq], dim=-1)
    y = y.permute(0, 1, 3, 2, 4).reshape(M, 2 * th, 2 * tw)[:, :H, :W][None]
    if b is not None:
        y = y + b.float().view(1, -1, 1, 1)
    return y
