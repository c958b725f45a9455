"""The wire-format ONNX writer/reader round-trips every generated model."""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op


@pytest.mark.parametrize("name", sorted(modelgen.FIXTURES))
def test_fixture_roundtrip(name):
    fx = modelgen.FIXTURES[name]()
    blob = op.encode_model(fx.model)
    m = op.decode_model(blob)
    assert [n.op_type for n in m.graph.nodes] == [n.op_type for n in fx.model.graph.nodes]
    assert [vi.name for vi in m.graph.inputs] == [vi.name for vi in fx.model.graph.inputs]
    for a, b in zip(m.graph.initializers, fx.model.graph.initializers):
        assert a.name == b.name and a.dims == b.dims and a.data_type == b.data_type
        if not b.external:
            np.testing.assert_array_equal(a.to_numpy(), b.to_numpy())
    for n1, n2 in zip(m.graph.nodes, fx.model.graph.nodes):
        for k in n2.attrs:
            assert n1.attr(k) == n2.attr(k)


def test_typed_half_initializer_is_bit_pattern():
    w = np.array([[1.0, -2.5], [0.333, 65504.0]], dtype=np.float16)
    t = op.tensor_from_array("w", w, typed_half=True)
    assert t.raw_data is None and len(t.int32_data) == 4
    back = op.decode_model(op.encode_model(op.Model(graph=op.Graph(nodes=[], inputs=[], outputs=[],
                                                                    initializers=[t]))))
    np.testing.assert_array_equal(back.graph.initializers[0].to_numpy(), w)


def test_conv_chain_structure():
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=2)
    counts = {}
    for n in cm.model.graph.nodes:
        counts[n.op_type] = counts.get(n.op_type, 0) + 1
    assert counts == {"Conv": 18, "Relu": 8, "Add": 9, "DepthToSpace": 1}
    flops, by = modelgen.conv_chain_flops(modelgen.CONFIGS["R8F64"], 1080, 1920)
    assert abs(flops / 1e9 - 2458.1) < 1.0
    assert abs(by / 1e9 - 11.43) < 0.05
