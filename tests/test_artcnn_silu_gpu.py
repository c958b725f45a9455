"""The shipped ArtCNN model topology on the GPU against the oracle (random weights of the
same shapes, since the shipped .onnx files are not available where the GPU tests run).

Covers the SiLU epilogue (Sigmoid + Mul fused into the conv), three-conv residual blocks,
the body conv with the global skip, Clip fused into the tail (with and without a 2x
DepthToSpace), fp16 and fp32 boundary IO, and 1 / 2 / 3 output channels, so every
specialised tail store path runs: the luma model (1 -> 1, 2x), the chroma model
(3 -> 2, fp32 IO), the dehalo model (3 -> 3, fp32 IO) and 2x variants with 2 and 3 output
channels.
"""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import Engine
from gpu_util import check_against_oracles
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu

CASES = [
    # name, in_ch, out_ch, scale, fp32_io, h, w
    ("luma", 1, 1, 2, False, 40, 136),
    ("chroma", 3, 2, 1, True, 36, 150),
    ("dehalo", 3, 3, 1, True, 33, 140),
    ("uv2x_fp32", 3, 2, 2, True, 24, 130),
    ("rgb2x_fp16", 1, 3, 2, False, 20, 129),
]


@pytest.mark.parametrize("name,cin,cout,scale,fp32_io,h,w", CASES)
def test_artcnn_silu_vs_oracle(tmp_path, name, cin, cout, scale, fp32_io, h, w):
    cm = modelgen.artcnn_silu(in_ch=cin, out_ch=cout, scale=scale, fp32_io=fp32_io, seed=7)
    p = tmp_path / f"{name}.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(11, cin, h, w)
    if fp32_io:
        x = x.astype(np.float32)
    got = Engine(p).run(x).astype(np.float64)
    assert got.shape == (1, cout, h * scale, w * scale)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes")
    ref32 = onnx_cpu.run_model(cm.model, xd, mode="fp32_nodes")
    variants = [onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", reverse_channels=True),
                onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", use_torch=False)]
    check_against_oracles(got, ref16, ref32, variants, name)


def test_artcnn_silu_luma_full_hd_vs_fp32_reference(tmp_path):
    """The luma topology at 1920x1080 against the oracle's fp32 GPU path (cuDNN, TF32 off)."""
    cm = modelgen.artcnn_silu(seed=9)
    p = tmp_path / "luma.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(13, 1, 1080, 1920)
    got = Engine(p).run(x).astype(np.float64)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", device="cuda:0")
    ref32 = onnx_cpu.run_model(cm.model, xd, mode="fp32_nodes", device="cuda:0")
    alt = onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", device="cuda:0", reverse_channels=True)
    check_against_oracles(got, ref16, ref32, [alt], "SiLU luma 1080p (GPU fp32 reference)")
