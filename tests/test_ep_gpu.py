"""Execution-provider regions compiled and run on the GPU (the provider's Compile +
compute function, src/onnxruntime-hip/hip_execution_provider.cc:337-406), against the
oracle: fp32 boundary IO, a re-plan for a second input shape, multi-channel NCHW input and
output layouts, and the deduplicated shared input (tests/correctness/test_ep.py cases)."""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.ep import Capability
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu

TOL = 2e-3  # fp16 conv tolerance on these small fixtures (the reference suite uses 2e-2)


def _case(name, c, h, w, fp32=False):
    fx = modelgen.FIXTURES[name]()
    cap = Capability(op.encode_model(fx.model))
    assert len(cap.regions) == 1
    eng = cap.compile(0, device=0)
    x = onnx_cpu.logical_ramp_input(c, h, w, in_fp32=fp32)
    got = eng.run(x.astype(np.float32 if fp32 else np.float16)).astype(np.float64)
    ref = onnx_cpu.run_model(fx.model, x, mode="fp16_nodes")
    return got, ref, eng


@pytest.mark.parametrize("name,c,h,w,fp32", [
    ("ep_conv_fp32io", 1, 16, 16, True),
    ("conv_c1m8", 1, 16, 16, False),
    ("conv_c4m4", 4, 16, 16, False),
    ("ep_two_convs_one_input", 4, 8, 8, False),
])
def test_compiled_region_matches_the_oracle(name, c, h, w, fp32):
    got, ref, _ = _case(name, c, h, w, fp32)
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, atol=TOL, rtol=0)


def test_compiled_region_replans_for_a_new_shape():
    got, ref, eng = _case("ep_conv_fp32io", 1, 16, 16, True)
    np.testing.assert_allclose(got, ref, atol=TOL, rtol=0)
    fx = modelgen.FIXTURES["ep_conv_fp32io"]()
    x = onnx_cpu.logical_ramp_input(1, 4, 4, in_fp32=True)
    small = eng.run(x.astype(np.float32)).astype(np.float64)
    assert small.shape == (1, 1, 4, 4)
    np.testing.assert_allclose(small, onnx_cpu.run_model(fx.model, x, mode="fp16_nodes"), atol=TOL, rtol=0)


def test_compile_on_a_bad_device_fails_with_the_provider_message():
    cap = Capability(op.encode_model(modelgen.FIXTURES["ep_conv_fp32io"]().model))
    with pytest.raises(Exception, match="HIP EP: device context is not initialized"):
        cap.compile(0, device=999)
