"""The CPU oracle against the golden vectors produced by the reference's own NumPy code.

This pins the oracle before it is trusted as the parity checker for the GPU path.
"""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen
from conftest import golden_cases, load_golden
from oracle import onnx_cpu

CASES = golden_cases()


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("mode", ["float64", "fp32_nodes"])
def test_oracle_matches_reference_golden(case, mode):
    fx = modelgen.FIXTURES[CASES[case]["fixture"]]()
    x, expected = load_golden(case)
    got = onnx_cpu.run_model(fx.model, x, mode=mode, use_torch=(mode != "float64"))
    assert got.shape == expected.shape
    # float64 mode is the same math as the reference's float64 references, up to
    # the float32 storage of the golden values; fp32_nodes adds fp32 accumulation
    # and the final fp16 rounding of an fp16 graph output.
    if mode == "float64":
        out_fp16 = fx.model.graph.outputs[0].elem_type == 10
        tol = 2e-3 if out_fp16 else 1e-5
        if not out_fp16:
            np.testing.assert_allclose(got, expected, rtol=1e-5, atol=1e-5)
        assert np.abs(got - expected).max() <= tol * max(1.0, np.abs(expected).max())
    else:
        assert np.abs(got - expected).max() <= 4e-3 * max(1.0, np.abs(expected).max())


def test_ramp_matches_reference_definition():
    r = onnx_cpu.ramp(300)
    assert r[0] == np.float32(11 / 251)
    assert r[1] == np.float32(48 / 251)
    assert float(r.max()) < 1.0 and float(r.min()) >= 0.0


def test_depth_to_space_dcr_vs_crd_channel_order():
    x = np.arange(2 * 4 * 3 * 3, dtype=np.float64).reshape(1, 8, 3, 3)
    dcr = onnx_cpu.depth_to_space(x, 2, "DCR")
    crd = onnx_cpu.depth_to_space(x, 2, "CRD")
    # DCR: output (c, 2h+r, 2w+q) = input channel (r*2+q)*Cout + c
    for c in range(2):
        for r in range(2):
            for q in range(2):
                assert dcr[0, c, r, q] == x[0, (r * 2 + q) * 2 + c, 0, 0]
                assert crd[0, c, r, q] == x[0, c * 4 + r * 2 + q, 0, 0]


def test_fp16_node_rounding_differs_from_fp32_only_by_rounding():
    spec = modelgen.CONFIGS["C4F32"]
    cm = modelgen.conv_chain(spec, seed=0)
    x = modelgen.synthetic_frame(0, 1, 32, 40).astype(np.float64)
    a = onnx_cpu.run_model(cm.model, x, mode="fp16_nodes")
    b = onnx_cpu.run_model(cm.model, x, mode="fp32_nodes")
    c = onnx_cpu.run_model(cm.model, x, mode="float64", use_torch=False)
    assert a.shape == (1, 1, 64, 80)
    assert np.abs(b - c).max() < 2e-3
    assert np.abs(a - c).max() < 1e-2
