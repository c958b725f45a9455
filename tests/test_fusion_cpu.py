"""Parse / fusion / rejection behaviour of the engine core, on the host only (no GPU).

Mirrors the rejection and fusion checks of the reference suite
(tests/correctness/test_engine.py: P1-2, P1-3, P1-8, P2-13, P2-14) through
``ah_model_inspect``, which runs the engine's Build() minus its CUDA set-up.
"""

from __future__ import annotations

from pathlib import Path

import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import EngineHarnessError, inspect_model

# The reference's shipped models, committed as test data (tests/fixtures/README.md).
FIXTURE_MODELS = Path(__file__).resolve().parent / "fixtures" / "models"

REF_MODELS = {
    "luma": "ArtCNN_R8F64_fp16.onnx",
    "chroma": "ArtCNN_R8F64_Chroma.onnx",
    "dehalo": "ArtCNN_R8F64_YCbCr_DEHALO.onnx",
}


@pytest.fixture(scope="module")
def fx_path(tmp_path_factory):
    d = tmp_path_factory.mktemp("fx")

    def get(name):
        _, p = modelgen.write_fixture(name, d)
        return p
    return get


@pytest.mark.parametrize("name,match", [
    ("conv_1x1", "3x3"),
    ("conv_short_bias", "bias"),
    ("conv_external", "external data"),
    ("conv_pads_asym", "pads"),
    ("clip_dynamic_bound", "dynamic Clip bounds"),
    ("add_const", "not an activation produced"),
    ("conv_m512", "256 output channels"),
    ("dts_crd", "DCR"),
])
def test_rejections(fx_path, name, match):
    with pytest.raises(EngineHarnessError, match=match):
        inspect_model(fx_path(name))


def test_unsupported_op_rejected(tmp_path):
    g = op.Graph(nodes=[op.make_node("Tanh", ["x"], ["y"])],
                 inputs=[op.value_info("x", op.FLOAT16, [1, 1, "h", "w"])],
                 outputs=[op.value_info("y", op.FLOAT16, [1, 1, "h", "w"])], initializers=[])
    p = tmp_path / "tanh.onnx"
    op.save_model(op.Model(graph=g), p)
    with pytest.raises(EngineHarnessError, match="unsupported op 'Tanh'"):
        inspect_model(p)


def test_malformed_file_rejected(tmp_path):
    p = tmp_path / "bad.onnx"
    p.write_bytes(b"\x0a\xff\xff\xff\xff\xff\xff")
    with pytest.raises(EngineHarnessError, match="parse"):
        inspect_model(p)


def test_shared_intermediates_decline_fusion(fx_path):
    silu = inspect_model(fx_path("silu_shared"))["ops"]
    assert any(l.startswith("Sigmoid") for l in silu) and any(l.startswith("Mul") for l in silu)
    assert not any("+silu" in l for l in silu)
    relu = inspect_model(fx_path("relu_shared"))["ops"]
    assert any(l.startswith("Relu") for l in relu) and not any("+relu" in l for l in relu)
    add = inspect_model(fx_path("add_shared_conv_out"))["ops"]
    assert any(l.startswith("Add") for l in add), add


@pytest.mark.parametrize("cfg", ["C4F32", "R8F64", "R16F96"])
def test_conv_chain_fuses_to_one_op_per_conv(tmp_path, cfg):
    spec = modelgen.CONFIGS[cfg]
    cm = modelgen.conv_chain(spec, seed=0)
    p = tmp_path / f"{cfg}.onnx"
    op.save_model(cm.model, p)
    info = inspect_model(p)
    ops = [l for l in info["ops"] if not l.startswith(("input", "output"))]
    assert len(ops) == 2 * spec.blocks + 2, ops
    assert all(l.startswith("Conv") for l in ops)
    assert sum("+relu" in l for l in ops) == spec.blocks
    # every second block conv carries the residual add; the last one also the global skip
    assert sum("+add(" in l for l in ops) == spec.blocks
    assert ops[-2].count("+add(") == 2
    assert "+dts2" in ops[-1]
    assert info["in_channels"] == 1 and info["out_channels"] == 4


def test_shipped_luma_model_fusion(tmp_path):
    import os
    ref = os.environ.get("ARTHIP_REF_MODELS", str(FIXTURE_MODELS))
    path = os.path.join(ref, REF_MODELS["luma"])
    if not os.path.exists(path):
        pytest.skip("shipped models not present")
    info = inspect_model(path)
    ops = [l for l in info["ops"] if not l.startswith(("input", "output"))]
    assert len(ops) == 27 and all(l.startswith("Conv") for l in ops)
    assert sum("+silu" in l for l in ops) == 16
    assert "+dts2" in ops[-1] and "clip[0,1]" in ops[-1]


def test_shipped_chroma_model_folds_fp32_casts(tmp_path):
    import os
    ref = os.environ.get("ARTHIP_REF_MODELS", str(FIXTURE_MODELS))
    path = os.path.join(ref, REF_MODELS["chroma"])
    if not os.path.exists(path):
        pytest.skip("shipped models not present")
    info = inspect_model(path)
    assert info["in_fp32"] and info["out_fp32"]
    assert info["in_channels"] == 3 and info["out_channels"] == 2
    ops = [l for l in info["ops"] if not l.startswith(("input", "output"))]
    assert len(ops) == 27 and all(l.startswith("Conv") for l in ops)
    assert "clip[0,1]" in ops[-1]  # Clip fused into the 2-channel tail conv


@pytest.mark.parametrize("kw", [dict(in_ch=1, out_ch=1, scale=2), dict(in_ch=3, out_ch=2, scale=1, fp32_io=True),
                                dict(in_ch=3, out_ch=3, scale=2, fp32_io=True)])
def test_artcnn_silu_topology_fuses_to_one_op_per_conv(tmp_path, kw):
    """The shipped ArtCNN topology (SiLU blocks, body conv + global skip, tail, optional
    DepthToSpace, Clip, optional fp32 boundary Casts) fuses to its 27 convs."""
    cm = modelgen.artcnn_silu(seed=5, **kw)
    p = tmp_path / "m.onnx"
    op.save_model(cm.model, p)
    info = inspect_model(p)
    ops = [l for l in info["ops"] if not l.startswith(("input", "output"))]
    assert len(ops) == 27 and all(l.startswith("Conv") for l in ops)
    assert sum("+silu" in l for l in ops) == 16
    assert sum("+add" in l for l in ops) == 9
    assert "clip[0,1]" in ops[-1] and (("+dts2" in ops[-1]) == (kw["scale"] == 2))
    assert info["in_fp32"] == info["out_fp32"] == kw.get("fp32_io", False)
