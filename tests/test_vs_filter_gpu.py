"""The VapourSynth filter core on the GPU, through its C ABI on numpy planes: the
reference plugin suite's cases (tests/correctness/test_plugin.py) with the oracle in place
of ONNX Runtime. Each shipped model runs after the load-time fp16 conversion, and the oracle
runs the same converted model, so the bar is BASELINE's 4e-3 on the [0,1] output."""

from __future__ import annotations

import threading
from pathlib import Path

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import EngineHarnessError
from arthip_b200.vsfilter import FLOAT, GRAY, INTEGER, RGB, YUV, ClipFormat, Model, convert_float_to_float16
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu

MODELS = Path(__file__).resolve().parent / "fixtures" / "models"
TOL = 4e-3


def _oracle(model_bytes: bytes, x: np.ndarray) -> np.ndarray:
    return onnx_cpu.run_model(op.decode_model(model_bytes), x.astype(np.float64), mode="fp16_nodes")


def _rand_planes(n, h, w, dtype, seed):
    rng = np.random.default_rng(seed)
    return [rng.uniform(0, 1, (h, w)).astype(dtype) for _ in range(n)]


def test_gray8_luma_defaults_to_fp16_output_at_2x():
    clip = ClipFormat(GRAY, INTEGER, 8, 1, 64, 48)
    m = Model(clip, MODELS / "ArtCNN_R8F64_fp16.onnx")
    assert (m.out_format.color_family, m.out_format.sample_type, m.out_format.bits_per_sample) == (GRAY, FLOAT, 16)
    assert (m.out_format.width, m.out_format.height) == (128, 96) and m.num_output_channels == 1
    src = np.random.default_rng(3).integers(0, 256, (48, 64)).astype(np.uint8)
    (got,) = m.get_frame([src])
    x = (src.astype(np.float32) / 255.0).astype(np.float16)[None, None]
    ref = _oracle((MODELS / "ArtCNN_R8F64_fp16.onnx").read_bytes(), x)
    assert float(np.abs(got.astype(np.float64) - ref[0, 0]).max()) <= TOL


def test_yuv444ps_chroma_flexible_two_fp32_planes():
    clip = ClipFormat(YUV, FLOAT, 32, 3, 64, 64)
    m = Model(clip, MODELS / "ArtCNN_R8F64_Chroma.onnx", fp16=1, flexible_output_prop="MlrtFlexible")
    assert m.num_output_channels == 2 and m.out_format.color_family == GRAY and m.out_format.bits_per_sample == 32
    planes = _rand_planes(3, 64, 64, np.float32, 1234)
    u, v = m.get_frame(planes)
    conv = convert_float_to_float16((MODELS / "ArtCNN_R8F64_Chroma.onnx").read_bytes(), cast_input=True,
                                    cast_output=True)
    ref = _oracle(conv, np.stack(planes)[None])
    for c, p in enumerate((u, v)):
        assert np.isfinite(p).all()
        assert float(np.abs(p.astype(np.float64) - ref[0, c]).max()) <= TOL, c
    assert abs(float(u.mean()) - float(v.mean())) > 1e-6  # two distinct planes


@pytest.mark.parametrize("fam", [YUV, RGB])
def test_fp16_three_plane_dehalo_comes_back_planar(fam):
    clip = ClipFormat(fam, FLOAT, 16, 3, 64, 64)
    m = Model(clip, MODELS / "ArtCNN_R8F64_YCbCr_DEHALO.onnx", fp16=1)
    assert m.out_format.color_family == RGB and m.num_output_channels == 3
    planes = _rand_planes(3, 64, 64, np.float16, 4242)
    outs = m.get_frame(planes)
    conv = convert_float_to_float16((MODELS / "ArtCNN_R8F64_YCbCr_DEHALO.onnx").read_bytes())
    ref = _oracle(conv, np.stack(planes)[None])
    for c in range(3):
        assert float(np.abs(outs[c].astype(np.float64) - ref[0, c]).max()) <= TOL, c


def test_integer_clip_into_an_fp32_model_without_conversion(tmp_path):
    """GRAY8 128 into an fp32-IO identity model with fp16=0 must arrive as ~0.502
    (test_plugin.py:395-414)."""
    fx = modelgen.FIXTURES["identity_fp32io"]()
    p = tmp_path / "identity_fp32io.onnx"
    op.save_model(fx.model, p)
    m = Model(ClipFormat(GRAY, INTEGER, 8, 1, 16, 16), p, fp16=0)
    assert m.out_format.bits_per_sample == 32
    (got,) = m.get_frame([np.full((16, 16), 128, dtype=np.uint8)])
    assert np.isfinite(got).all() and float(np.abs(got - 128 / 255).max()) < 1e-3


def test_fp16_off_gives_a_16_bit_integer_clip_for_an_fp16_model():
    clip = ClipFormat(GRAY, INTEGER, 8, 1, 32, 32)
    m = Model(clip, MODELS / "ArtCNN_R8F64_fp16.onnx", fp16=0)
    assert (m.out_format.sample_type, m.out_format.bits_per_sample) == (INTEGER, 16)
    src = np.random.default_rng(5).integers(0, 256, (32, 32)).astype(np.uint8)
    (got,) = m.get_frame([src])
    f16 = Model(clip, MODELS / "ArtCNN_R8F64_fp16.onnx").get_frame([src])[0].astype(np.float32)
    want = np.clip(f16 * np.float32(65535) + np.float32(0.5), 0, 65535).astype(np.int64)
    assert got.dtype == np.uint16
    assert int(np.abs(got.astype(np.int64) - want).max()) <= 1


@pytest.mark.parametrize("model,fmt,match", [
    ("ArtCNN_R8F64_YCbCr_DEHALO.onnx", ClipFormat(GRAY, INTEGER, 8, 1, 64, 64), "plane\\(s\\)"),
    ("ArtCNN_R8F64_Chroma.onnx", ClipFormat(GRAY, INTEGER, 8, 1, 64, 64), "plane\\(s\\)"),
    ("ArtCNN_R8F64_fp16.onnx", ClipFormat(YUV, FLOAT, 32, 3, 64, 64), "plane\\(s\\)"),
])
def test_plane_count_mismatch_is_refused(model, fmt, match):
    with pytest.raises(EngineHarnessError, match=match):
        Model(fmt, MODELS / model)


def test_more_model_channels_than_planes_is_refused(tmp_path):
    p = tmp_path / "c4m4.onnx"
    op.save_model(modelgen.FIXTURES["conv_c4m4"]().model, p)
    with pytest.raises(EngineHarnessError, match="input channels"):
        Model(ClipFormat(YUV, FLOAT, 32, 3, 64, 64), p)


def test_frame_size_tilesize_is_accepted_and_flexible_plane_count_follows_the_output():
    clip = ClipFormat(GRAY, INTEGER, 8, 1, 64, 64)
    m = Model(clip, MODELS / "ArtCNN_R8F64_fp16.onnx", tilesize=[64, 64], flexible_output_prop="MlrtFlexible")
    assert m.num_output_channels == 1  # the tail conv's 4 channels become 1 after DepthToSpace


def test_per_frame_subsampled_frame_is_refused():
    m = Model(ClipFormat(YUV, FLOAT, 32, 3, 32, 32), MODELS / "ArtCNN_R8F64_Chroma.onnx")
    bad = ClipFormat(YUV, FLOAT, 32, 3, 32, 32, 1, 1)
    with pytest.raises(EngineHarnessError, match="subsampled input frame"):
        m.get_frame(_rand_planes(3, 32, 32, np.float32, 1), bad)


def test_engine_pool_round_robin_from_threads_gives_identical_frames():
    clip = ClipFormat(GRAY, FLOAT, 16, 1, 96, 64)
    m = Model(clip, MODELS / "ArtCNN_R8F64_fp16.onnx", num_streams=2)
    src = _rand_planes(1, 64, 96, np.float16, 9)
    want = m.get_frame(src)[0]
    res, errs = [], []

    def work():
        try:
            for _ in range(4):
                res.append(m.get_frame(src)[0])
        except Exception as e:  # surfaced below
            errs.append(e)
    ts = [threading.Thread(target=work) for _ in range(3)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs and len(res) == 12
    assert all(np.array_equal(r, want) for r in res)
