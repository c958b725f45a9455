"""ONNX Runtime execution-provider partition rules on CPU (no GPU, no ORT): the node
predicate, the claimed runs and their MetaDef values, and what a claimed run compiles to.

Cases follow the reference's EP suite (tests/correctness/test_ep.py): boundary-Cast fp32
IO claimed (:53-66), no claim without a usable device (:85-95), a two-activation-input
region refused (:141-159), a graph input shared by two convs deduplicated (:162-178); and
the predicate's rules (src/onnxruntime-hip/hip_execution_provider.cc:22-161)."""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.ep import Capability, device_usable, node_supported


def _bytes(model: op.Model) -> bytes:
    return op.encode_model(model)


def _fx(name: str) -> bytes:
    return _bytes(modelgen.FIXTURES[name]().model)


def _conv_model(*, pads=(1, 1, 1, 1), kernel=3, strides=None, dtype=op.FLOAT16, auto_pad=None, group=None):
    w = np.zeros((4, 4, kernel, kernel), dtype=np.float16 if dtype == op.FLOAT16 else np.float32)
    attrs = {"kernel_shape": [kernel, kernel]}
    if pads is not None:
        attrs["pads"] = list(pads)
    if strides is not None:
        attrs["strides"] = list(strides)
    if auto_pad is not None:
        attrs["auto_pad"] = auto_pad
    if group is not None:
        attrs["group"] = group
    nodes = [op.make_node("Conv", ["x", "w"], ["y"], **attrs)]
    g = op.Graph(nodes=nodes, inputs=[op.value_info("x", dtype, [1, 4, "h", "w"])],
                 outputs=[op.value_info("y", dtype, [1, 4, "h", "w"])],
                 initializers=[op.tensor_from_array("w", w)], name="t")
    return _bytes(op.Model(graph=g, opset=modelgen.OPSET))


def test_boundary_casts_fp32_io_region_is_claimed():
    cap = Capability(_fx("ep_conv_fp32io"))
    assert len(cap.regions) == 1
    r = cap.regions[0]
    assert r.nodes == [0, 1, 2] and r.activations == ["x"] and r.outputs == ["y"]
    assert sorted(r.constants) == ["b", "w"]
    assert r.name.startswith("HipKernel_graph_")
    ops = cap.inspect(0)
    # the boundary Casts fold into fp32 IO of the compiled engine
    assert ops[0].startswith("input") and ops[0].endswith("fp32") and ops[-1].endswith("fp32")
    assert sum(l.startswith("Conv") for l in ops) == 1 and not any(l.startswith("Cast") for l in ops)


def test_no_usable_device_claims_nothing():
    assert not device_usable(999)
    assert Capability(_fx("ep_conv_fp32io"), context_ok=False).regions == []


def test_two_activation_inputs_are_not_claimed():
    assert node_supported(_fx("ep_two_inputs"), 0)  # the Add itself is supported
    assert Capability(_fx("ep_two_inputs")).regions == []


def test_shared_graph_input_is_deduplicated():
    cap = Capability(_fx("ep_two_convs_one_input"))
    assert len(cap.regions) == 1
    r = cap.regions[0]
    assert r.activations == ["x"] and r.outputs == ["y"] and r.nodes == [0, 1, 2]


def test_metadef_names_are_unique():
    a = Capability(_fx("ep_conv_fp32io")).regions[0].name
    b = Capability(_fx("ep_conv_fp32io")).regions[0].name
    assert a != b


@pytest.mark.parametrize("kw,ok", [
    (dict(), True),
    (dict(pads=None, auto_pad="SAME_UPPER"), True),
    (dict(pads=None, auto_pad="SAME_LOWER"), True),
    (dict(pads=(1, 0, 1, 0)), False),          # asymmetric: a different convolution
    (dict(pads=(0, 0, 0, 0)), False),
    (dict(pads=None), False),                   # no padding at all
    (dict(pads=None, auto_pad="VALID"), False),
    (dict(kernel=1, pads=(0, 0, 0, 0)), False),  # 1x1
    (dict(strides=(2, 2)), False),
    (dict(group=2), False),
    (dict(dtype=op.FLOAT), False),              # fp32 tensors
])
def test_conv_predicate(kw, ok):
    assert node_supported(_conv_model(**kw), 0) is ok


def test_clip_bounds_must_be_initializers_and_depthtospace_must_be_dcr():
    assert not node_supported(_fx("clip_dynamic_bound"), 1)
    assert node_supported(_fx("clip_no_bounds"), 1)
    crd = modelgen.FIXTURES["dts_crd"]().model
    dts = [i for i, n in enumerate(crd.graph.nodes) if n.op_type == "DepthToSpace"][0]
    assert not node_supported(_bytes(crd), dts)


def test_interior_cast_is_not_claimed_and_splits_runs():
    """A Cast between two convs is neither a boundary input nor output Cast: it stays on
    another provider, and the convs on either side form runs of their own (each claimed only
    if it has one activation input and one output)."""
    w = np.zeros((4, 4, 3, 3), dtype=np.float16)
    conv = dict(kernel_shape=[3, 3], pads=[1, 1, 1, 1])
    nodes = [op.make_node("Conv", ["x", "w"], ["a"], **conv),
             op.make_node("Cast", ["a"], ["a32"], to=op.FLOAT),
             op.make_node("Cast", ["a32"], ["a16"], to=op.FLOAT16),
             op.make_node("Conv", ["a16", "w"], ["y"], **conv)]
    g = op.Graph(nodes=nodes, inputs=[op.value_info("x", op.FLOAT16, [1, 4, "h", "w"])],
                 outputs=[op.value_info("y", op.FLOAT16, [1, 4, "h", "w"])],
                 initializers=[op.tensor_from_array("w", w)], name="t")
    b = _bytes(op.Model(graph=g, opset=modelgen.OPSET))
    assert [node_supported(b, i) for i in range(4)] == [True, False, False, True]
    cap = Capability(b)
    assert [r.nodes for r in cap.regions] == [[0], [3]]
    assert cap.regions[0].activations == ["x"] and cap.regions[0].outputs == ["a"]
    assert cap.regions[1].activations == ["a16"] and cap.regions[1].outputs == ["y"]


def test_value_needed_outside_the_run_makes_a_second_output():
    """An intermediate that a node outside the run also reads must be exported: the run then
    has two outputs and is left unclaimed (the reference's multi-output rule)."""
    w = np.zeros((4, 4, 3, 3), dtype=np.float16)
    conv = dict(kernel_shape=[3, 3], pads=[1, 1, 1, 1])
    nodes = [op.make_node("Conv", ["x", "w"], ["a"], **conv),
             op.make_node("Conv", ["a", "w"], ["b"], **conv),
             op.make_node("Cast", ["a"], ["a32"], to=op.FLOAT)]
    g = op.Graph(nodes=nodes, inputs=[op.value_info("x", op.FLOAT16, [1, 4, "h", "w"])],
                 outputs=[op.value_info("b", op.FLOAT16, [1, 4, "h", "w"]),
                          op.value_info("a32", op.FLOAT, [1, 4, "h", "w"])],
                 initializers=[op.tensor_from_array("w", w)], name="t")
    cap = Capability(_bytes(op.Model(graph=g, opset=modelgen.OPSET)))
    assert cap.regions == []


def test_relu_chain_and_clip_defaults_compile_to_the_engine_core():
    """The R8F64 conv chain is claimed whole (Relu included) and fuses as the standalone
    path does; a Clip without bounds is a no-op (+-inf) through the provider path too."""
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=1)
    cap = Capability(_bytes(cm.model))
    assert len(cap.regions) == 1 and len(cap.regions[0].nodes) == len(cm.model.graph.nodes)
    ops = [l for l in cap.inspect(0) if not l.startswith(("input", "output"))]
    assert len(ops) == 18 and sum("+relu" in l for l in ops) == 8
    clip = Capability(_fx("clip_no_bounds"))
    assert len(clip.regions) == 1
    (line,) = [l for l in clip.inspect(0) if "clip[" in l]
    assert "clip[-inf,inf]" in line


def test_shipped_models_fp16_luma_claimed_whole_fp32_chroma_not():
    """The shipped fp16 luma model is one region (27 fused convs, Clip folded into the
    tail). The Chroma model is an fp32 graph (fp32 weights, no Casts): the provider claims
    only fp16 tensors, so it claims none of it, as the reference's provider does; it runs
    on the GPU after the fp16 conversion of the loading path."""
    from pathlib import Path
    d = Path(__file__).resolve().parent / "fixtures" / "models"
    luma = Capability((d / "ArtCNN_R8F64_fp16.onnx").read_bytes())
    assert len(luma.regions) == 1
    ops = luma.inspect(0)
    assert sum(l.startswith("Conv") for l in ops) == 27 and "clip[0,1]" in ops[-2]
    assert Capability((d / "ArtCNN_R8F64_Chroma.onnx").read_bytes()).regions == []
