"""The reference's shipped ArtCNN R8F64 models (luma fp16 2x, chroma 3->2 fp32 IO, dehalo
3->3 fp32 IO) on its photo fixtures, engine against the oracle, on BASELINE's fixed bar:
max-abs <= 4e-3 and PSNR >= 55 dB on the [0,1] output, against both the typed fp16 graph
and the fp32-between-nodes execution (the bar is not widened here).

The models and photos are copies of the reference project's test fixtures, committed under
`tests/fixtures/` (see the README there); ARTHIP_SHIPPED_DIR may name another directory
with the same layout. Inputs are photo crops: grayscale for the luma model, YCbCr for the
three-channel models (full-range, scaled to [0, 1]) as the reference's chroma tests feed
them (tests/correctness/test_plugin.py:204,241-251).
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from arthip_b200 import onnx_proto as op
from arthip_b200.engine import Engine
from gpu_util import MAX_ABS_TOL, assert_frame_parity, report_parity
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu

ROOT = Path(os.environ.get("ARTHIP_SHIPPED_DIR") or Path(__file__).resolve().parent / "fixtures")

MODELS = [
    # file, PIL mode of the input, channels kept, fp32 IO, output channels, scale
    ("ArtCNN_R8F64_fp16.onnx", "L", 1, False, 1, 2),
    ("ArtCNN_R8F64_Chroma.onnx", "YCbCr", 3, True, 2, 1),
    ("ArtCNN_R8F64_YCbCr_DEHALO.onnx", "YCbCr", 3, True, 3, 1),
]


def _photo(name: str, mode: str, y0: int, x0: int, h: int, w: int) -> np.ndarray:
    from PIL import Image
    im = Image.open(ROOT / "images" / name).convert("RGB").convert(mode)
    a = np.asarray(im, dtype=np.float32)
    if a.ndim == 2:
        a = a[:, :, None]
    a = a[y0:y0 + h, x0:x0 + w, :] / 255.0
    return np.ascontiguousarray(a.transpose(2, 0, 1)[None])


@pytest.mark.parametrize("fname,mode,cin,fp32_io,cout,scale", MODELS)
def test_shipped_model_on_photo_crop(fname, mode, cin, fp32_io, cout, scale):
    path = ROOT / "models" / fname
    model = op.load_model(path)
    x = _photo("test_256.png", mode, 70, 50, 80, 136)
    x = x.astype(np.float32 if fp32_io else np.float16)
    got = Engine(path).run(x).astype(np.float64)
    assert got.shape == (1, cout, 80 * scale, 136 * scale)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(model, xd, mode="fp16_nodes")
    ref32 = onnx_cpu.run_model(model, xd, mode="fp32_nodes")
    d16, p16 = assert_frame_parity(got, ref16, f"{fname} vs fp16_nodes", MAX_ABS_TOL)
    d32, p32 = assert_frame_parity(got, ref32, f"{fname} vs fp32_nodes", MAX_ABS_TOL)
    report_parity(f"shipped {fname}, 80x136 crop of test_256.png", d16, p16, d32, p32, MAX_ABS_TOL)


def test_shipped_luma_model_on_full_hd_photo():
    """The luma model on the whole 1920x1080 photo against the oracle's fp32 GPU path
    (cuDNN, TF32 off), as the reference upscales a 1080p frame."""
    path = ROOT / "models" / "ArtCNN_R8F64_fp16.onnx"
    model = op.load_model(path)
    x = _photo("test_1920_luma.png", "L", 0, 0, 1080, 1920).astype(np.float16)
    got = Engine(path).run(x).astype(np.float64)
    assert got.shape == (1, 1, 2160, 3840)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(model, xd, mode="fp16_nodes", device="cuda:0")
    ref32 = onnx_cpu.run_model(model, xd, mode="fp32_nodes", device="cuda:0")
    d16, p16 = assert_frame_parity(got, ref16, "luma 1080p vs fp16_nodes", MAX_ABS_TOL)
    d32, p32 = assert_frame_parity(got, ref32, "luma 1080p vs fp32_nodes", MAX_ABS_TOL)
    report_parity("shipped ArtCNN_R8F64_fp16.onnx, 1920x1080 test_1920 luma (GPU fp32 oracle)", d16, p16, d32, p32,
                  MAX_ABS_TOL)
