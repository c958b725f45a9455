"""A frame split into row strips, each run with the model's receptive-field halo, stitches
back to exactly the whole-frame result (the single-large-frame path across GPUs, run here
strip after strip on one GPU)."""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import Engine
from arthip_b200.strips import conv_depth, plan_strips, run_strip, stitch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [2, 3, 5])
def test_strips_stitch_to_the_whole_frame(tmp_path, n):
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=4)
    p = tmp_path / "r8f64.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(4, 1, 270, 480)
    eng = Engine(p)
    full = eng.run(x)
    halo = conv_depth(p)
    assert halo == 18
    parts = [run_strip(eng, x, s, 2) for s in plan_strips(270, n, halo)]
    np.testing.assert_array_equal(stitch(parts), full)
