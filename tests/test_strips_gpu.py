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


@pytest.mark.parametrize("n,height", [(2, 270), (3, 200), (4, 131)])
def test_halo_exchange_strips_stitch_to_the_whole_frame(tmp_path, n, height):
    """The per-layer 1-row halo exchange variant, its ranks emulated on one GPU: one engine
    per strip (rows + 2 local rows), ops launched one at a time, and after each op the
    strips' halo rows copied from their neighbours (the row moves the multi-GPU run makes
    with NCCL send/recv). The owned output rows must equal the whole-frame result."""
    import torch

    from arthip_b200.strips import HaloStripRunner, exchange_local, halo_window, plan_halo_strips
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=4)
    p = tmp_path / "r8f64.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(4, 1, height, 480)
    full = Engine(p).run(x)
    dev = torch.device("cuda:0")
    strips = plan_halo_strips(height, n)
    runners = [HaloStripRunner(Engine(p), st, 480, 1, dev) for st in strips]
    for r, st in zip(runners, strips):
        r.load_input(halo_window(x, st))
    n_ops = runners[0].n_ops
    for i in range(n_ops):
        for r in runners:
            r.engine.enqueue_ops(i, i + 1)
        for r in runners:
            r.engine.synchronize()
        if i + 1 < n_ops:
            exchange_local([r.views[i] for r in runners], strips)
            torch.cuda.synchronize()
    got = np.concatenate([r.own_output(2) for r in runners], axis=2)
    np.testing.assert_array_equal(got, full)
