"""The reference's shipped ArtCNN R8F64 models (luma fp16 2x, chroma 3->2 fp32 IO, dehalo
3->3 fp32 IO) on its photo fixtures, engine against the oracle.

The model and photo files belong to the reference project and are not part of this
repository. The test runs when ARTHIP_SHIPPED_DIR names a directory laid out like the
reference's `tests/fixtures/` (`models/ArtCNN_R8F64_*.onnx`, `images/test_*.png`), and is
skipped otherwise. Inputs are photo crops: grayscale for the luma model, YCbCr for the
three-channel models (full-range, scaled to [0, 1]).
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from arthip_b200 import onnx_proto as op
from arthip_b200.engine import Engine
from gpu_util import check_against_oracles
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu

_DIR = os.environ.get("ARTHIP_SHIPPED_DIR")
if not _DIR or not (Path(_DIR) / "models").is_dir():
    pytest.skip("ARTHIP_SHIPPED_DIR does not name the shipped models and photos", allow_module_level=True)
ROOT = Path(_DIR)

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
    variants = [onnx_cpu.run_model(model, xd, mode="fp16_nodes", reverse_channels=True),
                onnx_cpu.run_model(model, xd, mode="fp16_nodes", use_torch=False)]
    check_against_oracles(got, ref16, ref32, variants, fname)


def test_shipped_luma_model_on_full_hd_photo():
    """The luma model on the whole 1920x1080 photo against the oracle's fp32 GPU path
    (cuDNN, TF32 off), as the reference upscales a 1080p frame."""
    path = ROOT / "models" / "ArtCNN_R8F64_fp16.onnx"
    model = op.load_model(path)
    x = _photo("test_1920.png", "L", 0, 0, 1080, 1920).astype(np.float16)
    got = Engine(path).run(x).astype(np.float64)
    assert got.shape == (1, 1, 2160, 3840)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(model, xd, mode="fp16_nodes", device="cuda:0")
    ref32 = onnx_cpu.run_model(model, xd, mode="fp32_nodes", device="cuda:0")
    alt = onnx_cpu.run_model(model, xd, mode="fp16_nodes", device="cuda:0", reverse_channels=True)
    check_against_oracles(got, ref16, ref32, [alt], "shipped luma model, 1080p photo (GPU fp32 reference)")
