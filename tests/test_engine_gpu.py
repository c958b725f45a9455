"""The engine through the reference-compatible driver ABI, on the GPU.

Ports the reference suite's engine checks (tests/correctness/test_engine.py) with the
expected values taken from the golden vectors the reference's own float64 NumPy code
produced (tests/golden/), at the stricter BASELINE tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import EngineHarness, EngineHarnessError, ramp_input
from conftest import golden_cases, load_golden
from gpu_util import MAX_ABS_TOL

pytestmark = pytest.mark.gpu

CASES = golden_cases()


@pytest.fixture(scope="module")
def engine():
    h = EngineHarness()
    if h.device_count() < 1:
        pytest.skip("no CUDA device")
    return h


@pytest.fixture(scope="module")
def fx(tmp_path_factory):
    d = tmp_path_factory.mktemp("gpu_fx")
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = modelgen.write_fixture(name, d)
        return cache[name]
    return get


def _tol(expected):
    # fp16 outputs: the BASELINE bar, widened to one fp16 ulp for values beyond [0, 2)
    return max(MAX_ABS_TOL, 2.0 ** (np.floor(np.log2(max(np.abs(expected).max(), 1e-3))) - 9))


@pytest.mark.parametrize("case", sorted(CASES))
def test_golden_case(engine, fx, device, case):
    name = CASES[case]["fixture"]
    f, path = fx(name)
    x, expected = load_golden(case)
    _, c, h, w = x.shape
    raw = x.astype(np.float32 if f.fp32_io and f.model.graph.inputs[0].elem_type == op.FLOAT else np.float16)
    res = engine.run(path, h=h, w=w, c=c, device=device, raw_input=raw.reshape(-1))
    assert res.shape == expected.shape
    assert np.isfinite(res.output).all()
    diff = float(np.abs(res.output - expected).max())
    assert diff <= _tol(expected), f"{case}: max abs diff {diff:.3g}"


def test_identity_is_bit_exact_raw_and_typed(engine, fx, device):
    """FLOAT16 values in int32_data are bit patterns (test_engine.py:109-119)."""
    h, w = 17, 8
    raw = engine.run(fx("identity_raw")[1], h=h, w=w, c=1, device=device)
    typed = engine.run(fx("identity_typed_half")[1], h=h, w=w, c=1, device=device)
    expected = ramp_input(1, h, w, False).astype(np.float64).reshape(1, 1, h, w)
    np.testing.assert_array_equal(raw.output, expected)
    np.testing.assert_array_equal(typed.output, raw.output)


def test_fp32_io_identity(engine, fx, device):
    res = engine.run(fx("identity_fp32io")[1], h=9, w=13, c=1, device=device)
    x = ramp_input(1, 9, 13, True).reshape(1, 1, 9, 13)
    np.testing.assert_allclose(res.output, x.astype(np.float16).astype(np.float64), atol=0, rtol=0)


@pytest.mark.parametrize("h,w", [(8, 8), (8, 17), (17, 17), (1082, 64), (54, 1920)])
def test_geometry_large_bands(engine, fx, device, h, w):
    """The reference's large geometry cases (a 1082-row band, a 1920-wide band) against
    the CPU oracle: every row and column must be produced."""
    from oracle import onnx_cpu
    for name in ("conv_c1m8", "conv_c4m4", "wide_c64m64_relu"):
        f, path = fx(name)
        res = engine.run(path, h=h, w=w, c=f.input_channels, device=device)
        xin = onnx_cpu.logical_ramp_input(f.input_channels, h, w)
        ref = onnx_cpu.run_model(f.model, xin, mode="fp16_nodes")
        assert float(np.abs(res.output - ref).max()) <= _tol(ref), (name, h, w)


def test_batch_greater_than_one_rejected(engine, fx, device):
    with pytest.raises(EngineHarnessError, match="shape propagation failed"):
        engine.probe(fx("conv_c4m4")[1], n=2, h=16, w=16, c=4, device=device)


def test_broadcast_operand_rejected(engine, fx, device):
    with pytest.raises(EngineHarnessError, match="shape propagation failed"):
        engine.probe(fx("add_broadcast")[1], h=16, w=16, c=4, device=device)


def test_wide_output_channels_supported(engine, fx, device):
    """M=128 exceeds the reference kernels' 64 but is within this engine's 256."""
    from oracle import onnx_cpu
    f, path = fx("conv_m128")
    res = engine.run(path, h=12, w=20, c=4, device=device)
    ref = onnx_cpu.run_model(f.model, onnx_cpu.logical_ramp_input(4, 12, 20), mode="fp16_nodes")
    assert float(np.abs(res.output - ref).max()) <= _tol(ref)


def test_selected_device_is_used(engine, fx, device):
    p = engine.probe(fx("conv_c4m4")[1], h=16, w=16, c=4, device=device)
    assert (p.in_channels, p.out_channels) == (4, 4)
    assert not p.in_fp32 and not p.out_fp32


def test_invalid_device_is_reported(engine, fx):
    with pytest.raises(EngineHarnessError, match="cudaSetDevice|invalid device"):
        engine.probe(fx("conv_c4m4")[1], h=16, w=16, c=4, device=999)


def test_allocation_failure_is_reported_then_recovers(engine, fx, device):
    """An impossible allocation surfaces the CUDA error and the same engine still runs a
    16x16 frame afterwards (test_engine.py:273-281)."""
    f, path = fx("conv_c4m4")
    message, result = engine.alloc_failure_then_run(path, c=4, device=device)
    assert "cudaMalloc" in message, message
    expected = load_golden("winograd_c4m4_17x16")  # same weights; recompute at 16x16 below
    from oracle import onnx_cpu
    ref = onnx_cpu.run_model(f.model, onnx_cpu.logical_ramp_input(4, 16, 16), mode="float64", use_torch=False)
    assert float(np.abs(result.output - ref).max()) <= MAX_ABS_TOL
    del expected


def test_fresh_engines_agree(engine, tmp_path, device):
    """The same frame through fresh engines is bit-identical (test_engine.py:292-326)."""
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=2)
    p = tmp_path / "r8f64.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(2, 1, 270, 480)
    first = None
    for _ in range(4):
        out = engine.run(p, h=270, w=480, c=1, device=device, raw_input=x.reshape(-1)).output
        if first is None:
            first = out
        else:
            np.testing.assert_array_equal(out, first)


def test_dead_residuals_are_added_in_place(tmp_path, device):
    """Buffer assignment: a conv whose last residual operand dies at that conv writes over
    it (the tensor-core kernel then adds it with reduce-add stores). In R8F64 that is block
    convs B of blocks 2-8 and the global skip of block 8. Block 1's residual is the head
    output, which the global skip still needs, so that conv writes a new buffer."""
    from arthip_b200.engine import Engine
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=2)
    p = tmp_path / "r8f64.onnx"
    op.save_model(cm.model, p)
    eng = Engine(p, device=device)
    eng.prepare(1, 64, 200)
    labels = [o["label"] for o in eng.ops()]
    adds = [lb for lb in labels if "+add" in lb]
    assert len(adds) == 8
    assert "in place" not in adds[0]
    assert all("in place" in lb for lb in adds[1:]), adds
    assert not any("in place" in lb for lb in labels if "+add" not in lb)
    eng.close()
