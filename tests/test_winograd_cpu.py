"""The Winograd F(2x2,3x3) restatement on CPU (oracle/winograd_ref.py): its weight
transform against float64, its conv against the exact-product conv, and what its fp16
transformed operands do over a whole chain. The chain test prints the figures and
asserts the finding the engine's default rests on: on BASELINE's random-weight R8F64 chain
the Winograd numerics drift further from the typed fp16 graph than two exact-product
executions of it do, while on the shipped trained luma model they stay inside 4e-3."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from arthip_b200 import modelgen, onnx_proto as op
from oracle import onnx_cpu, winograd_ref

G = np.array([[1, 0, 0], [.5, .5, .5], [.5, -.5, .5], [0, 0, 1]], dtype=np.float64)


def test_weight_transform_is_ggt_rounded_to_fp16():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((8, 8, 3, 3)) * 0.2).astype(np.float16)
    u = winograd_ref.weight_transform(w).astype(np.float64)
    exact = np.einsum("ij,mcjk,lk->mcil", G, w.astype(np.float64), G)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 2 ** -14))) - 10)
    assert np.all(np.abs(u - exact) <= ulp)  # within one fp16 ulp (fp32 sums, then RNE)


def test_winograd_conv_is_close_to_the_exact_conv():
    rng = np.random.default_rng(1)
    x = torch.from_numpy(rng.uniform(0, 1, (1, 16, 9, 13)).astype(np.float16)).float()
    w = torch.from_numpy((rng.standard_normal((16, 16, 3, 3)) * 0.1).astype(np.float16)).float()
    b = torch.from_numpy((rng.standard_normal(16) * 0.05).astype(np.float16)).float()
    got = winograd_ref.conv2d_nchw(x, w, b).double()
    exact = F.conv2d(x.double(), w.double(), b.double(), padding=1)
    d = float((got - exact).abs().max())
    assert 0 < d < 4e-3, d  # transformed-operand rounding only


def _chain(model, x, winograd):
    orig = onnx_cpu._Exec.conv

    def conv(self, xx, w, b, pads):
        if winograd and w.shape[0] == 64 and w.shape[1] == 64:
            return winograd_ref.conv2d_nchw(xx, w, b)
        return orig(self, xx, w, b, pads)
    onnx_cpu._Exec.conv = conv
    try:
        return onnx_cpu.run_model(model, x, mode="fp16_nodes", convert_fp32_weights_to_fp16=True)
    finally:
        onnx_cpu._Exec.conv = orig


def _gap(a, b):
    return float(np.abs(np.clip(a, 0, 1) - np.clip(b, 0, 1)).max())


def test_winograd_numerics_over_the_r8f64_chain_and_a_shipped_model():
    torch.set_num_threads(8)
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=2)
    x = modelgen.synthetic_frame(2, 1, 96, 192).astype(np.float64)
    ref = _chain(cm.model, x, False)
    alt = onnx_cpu.run_model(cm.model, x, mode="fp16_nodes", reverse_channels=True)
    wino = _chain(cm.model, x, True)
    spread, dw = _gap(alt, ref), _gap(wino, ref)
    path = Path(__file__).resolve().parent / "fixtures" / "models" / "ArtCNN_R8F64_fp16.onnx"
    model = op.load_model(path)
    from PIL import Image
    im = Image.open(path.parents[1] / "images" / "test_256.png").convert("L")
    xs = (np.asarray(im, dtype=np.float32)[:96, :128] / 255.0).astype(np.float16).astype(np.float64)[None, None]
    ds = _gap(_chain(model, xs, True), _chain(model, xs, False))
    print(f"R8F64 96x192: exact-product spread {spread:.4g}, winograd {dw:.4g}; shipped luma: winograd {ds:.4g}")
    assert dw > spread
    assert ds <= 4e-3
