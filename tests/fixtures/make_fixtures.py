"""Copy the reference project's shipped ArtCNN models and photo fixtures into this test
tree (test data: the ONNX models are weights, the photos are inputs).

    python tests/fixtures/make_fixtures.py <reference project root>

Writes ``models/ArtCNN_R8F64_{fp16,Chroma,YCbCr_DEHALO}.onnx`` (byte copies),
``images/test_256.png`` (byte copy) and ``images/test_1920_luma.png``: the luma plane
(PIL "L" conversion of the RGB photo) of the 1920x1080 ``test_1920.png``, stored as an
8-bit grayscale PNG, which is the input the luma test takes from that photo.
"""

from __future__ import annotations

import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
MODELS = ["ArtCNN_R8F64_fp16.onnx", "ArtCNN_R8F64_Chroma.onnx", "ArtCNN_R8F64_YCbCr_DEHALO.onnx"]


def main(argv: list[str]) -> int:
    if len(argv) != 1:
        print(__doc__)
        return 2
    src = Path(argv[0]) / "tests" / "fixtures"
    (HERE / "models").mkdir(exist_ok=True)
    (HERE / "images").mkdir(exist_ok=True)
    for m in MODELS:
        shutil.copyfile(src / "models" / m, HERE / "models" / m)
    shutil.copyfile(src / "images" / "test_256.png", HERE / "images" / "test_256.png")
    from PIL import Image
    Image.open(src / "images" / "test_1920.png").convert("RGB").convert("L").save(
        HERE / "images" / "test_1920_luma.png", optimize=True)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
