"""Row-strip plans for splitting one frame across GPUs (host logic only)."""

from __future__ import annotations

import pytest

from arthip_b200.strips import plan_strips


@pytest.mark.parametrize("height,n,halo", [(4320, 8, 18), (4320, 2, 18), (1080, 4, 18), (100, 7, 5), (9, 9, 3)])
def test_plan_covers_every_row_once_with_clamped_halos(height, n, halo):
    s = plan_strips(height, n, halo)
    assert [x.rank for x in s] == list(range(n))
    assert s[0].out_lo == 0 and s[-1].out_hi == height
    for a, b in zip(s, s[1:]):
        assert a.out_hi == b.out_lo
    for x in s:
        assert x.out_hi > x.out_lo
        assert x.in_lo == max(0, x.out_lo - halo) and x.in_hi == min(height, x.out_hi + halo)


def test_plan_rejects_more_strips_than_rows():
    with pytest.raises(ValueError):
        plan_strips(3, 4, 1)


def test_conv_depth_of_r8f64_is_18(tmp_path):
    from arthip_b200 import modelgen, onnx_proto as op
    from arthip_b200.strips import conv_depth
    cm = modelgen.conv_chain(modelgen.CONFIGS["R8F64"], seed=1)
    p = tmp_path / "m.onnx"
    op.save_model(cm.model, p)
    assert conv_depth(p) == 18
