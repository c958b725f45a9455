"""The VapourSynth loading path on CPU (no GPU, no VapourSynth): the fp32 -> fp16 model
conversion (src/vapoursynth/convert_float_to_float16.cpp:165-186,294-611), loadONNX's shape
fixing (src/vapoursynth/onnx_utils.cpp:29-128) and hip.Model's creation-time argument and
clip-format checks (src/vapoursynth/vs_hip.cpp:337-442; the cases of the reference's
tests/correctness/test_plugin.py:105-140,455-475)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import EngineHarnessError, inspect_model
from arthip_b200.ep import Capability
from arthip_b200.vsfilter import FLOAT, GRAY, INTEGER, RGB, YUV, ClipFormat, Model, convert_float_to_float16, load_onnx
from oracle import fp16_ref

MODELS = Path(__file__).resolve().parent / "fixtures" / "models"


def _chroma() -> bytes:
    return (MODELS / "ArtCNN_R8F64_Chroma.onnx").read_bytes()


def _inits(m: op.Model) -> dict:
    return {t.name: t for t in m.graph.initializers}


def test_conversion_rounds_every_weight_with_the_flush_to_zero_rule():
    src = op.decode_model(_chroma())
    conv = op.decode_model(convert_float_to_float16(_chroma()))
    a, b = _inits(src), _inits(conv)
    assert set(a) == set(b)
    n_tiny = 0
    for name, t in a.items():
        assert t.data_type == op.FLOAT
        assert b[name].data_type == op.FLOAT16
        x = t.to_numpy()
        want = fp16_ref.to_half_ftz(x)
        got = b[name].to_numpy().view(np.uint16)
        np.testing.assert_array_equal(got, want, err_msg=name)
        n_tiny += int(((np.abs(x) < 2.0 ** -14) & (x != 0)).sum())
    assert n_tiny > 0  # the model has weights below the fp16 normal range: the flush is exercised


def test_conversion_without_casts_makes_an_fp16_graph():
    conv = op.decode_model(convert_float_to_float16(_chroma()))
    assert conv.graph.inputs[0].elem_type == op.FLOAT16 and conv.graph.outputs[0].elem_type == op.FLOAT16
    assert not any(n.op_type == "Cast" for n in conv.graph.nodes)


def test_conversion_with_casts_keeps_fp32_io_and_folds_to_27_convs(tmp_path):
    b = convert_float_to_float16(_chroma(), cast_input=True, cast_output=True)
    m = op.decode_model(b)
    assert m.graph.inputs[0].elem_type == op.FLOAT and m.graph.outputs[0].elem_type == op.FLOAT
    first, last = m.graph.nodes[0], m.graph.nodes[-1]
    assert first.op_type == "Cast" and first.name == "graph_input_cast_0" and first.inputs == ["input"]
    assert last.op_type == "Cast" and last.name == "graph_output_cast_0" and last.outputs == ["output"]
    p = tmp_path / "chroma_fp16.onnx"
    p.write_bytes(b)
    info = inspect_model(p)
    ops = [l for l in info["ops"] if not l.startswith(("input", "output"))]
    assert len(ops) == 27 and all(l.startswith("Conv") for l in ops)
    assert info["in_fp32"] and info["out_fp32"] and info["in_channels"] == 3 and info["out_channels"] == 2
    # the converted model is what the execution provider claims whole (fp16 body, boundary Casts)
    cap = Capability(b)
    assert len(cap.regions) == 1 and len(cap.regions[0].nodes) == len(m.graph.nodes)


def test_block_list_keeps_ops_fp32_behind_casts():
    b = convert_float_to_float16(_chroma(), op_block_list=["Clip"])
    m = op.decode_model(b)
    clip = [n for n in m.graph.nodes if n.op_type == "Clip"][0]
    casts = {n.outputs[0]: n for n in m.graph.nodes if n.op_type == "Cast"}
    # Clip's fp16 bound initializers are cast to fp32 in front of it, and its fp16 graph
    # output is produced by a Cast behind it
    assert any(i in casts for i in clip.inputs[1:])
    assert any(n.op_type == "Cast" and n.inputs == clip.outputs for n in m.graph.nodes)


def test_load_onnx_fixes_the_input_shape_and_checks_rank():
    fixed = op.decode_model(load_onnx((MODELS / "ArtCNN_R8F64_fp16.onnx").read_bytes(), tile_w=320, tile_h=240))
    assert fixed.graph.inputs[0].shape[0] == 1 and list(fixed.graph.inputs[0].shape[2:]) == [240, 320]
    two = modelgen.FIXTURES["ep_two_inputs"]().model
    with pytest.raises(EngineHarnessError, match="single input"):
        load_onnx(op.encode_model(two))
    with pytest.raises(EngineHarnessError, match="parse"):
        load_onnx(path="/nonexistent/model.onnx")


def _fmt(fam, st, bits, planes, w=64, h=64, ssw=0, ssh=0):
    return ClipFormat(fam, st, bits, planes, w, h, ssw, ssh)


@pytest.mark.parametrize("fmt,match", [
    (_fmt(YUV, INTEGER, 8, 3, ssw=1, ssh=1), "subsampled"),   # YUV420P8
    (_fmt(YUV, INTEGER, 8, 3, ssw=1, ssh=0), "subsampled"),   # YUV422P8
    (_fmt(0, INTEGER, 8, 1), "gray, YUV or RGB"),             # variable format
    (_fmt(GRAY, INTEGER, 10, 1), "8/16-bit int"),             # 10-bit
    (_fmt(GRAY, FLOAT, 64, 1), "8/16-bit int"),
])
def test_clip_formats_are_refused_before_loading(fmt, match):
    with pytest.raises(EngineHarnessError, match=match) as e:
        Model(fmt, MODELS / "ArtCNN_R8F64_YCbCr_DEHALO.onnx")
    assert str(e.value).startswith("hip.Model: ")


@pytest.mark.parametrize("kw,match", [
    (dict(overlap=[1, 1]), "overlap"),
    (dict(overlap=[-1]), "non-negative"),
    (dict(tilesize=[32, 32]), "tilesize"),
    (dict(tilesize=[64, 32]), "tilesize"),
])
def test_tiling_arguments_other_than_the_default_are_refused(kw, match):
    with pytest.raises(EngineHarnessError, match=match):
        Model(_fmt(GRAY, INTEGER, 8, 1), MODELS / "ArtCNN_R8F64_fp16.onnx", **kw)


def test_model_file_errors_are_reported():
    with pytest.raises(EngineHarnessError, match="parse .* failed"):
        Model(_fmt(GRAY, INTEGER, 8, 1), "/nonexistent/model.onnx")
