"""The two-SM (cta_group::2) vertical-window conv against the single-SM kernel: the same
MMAs per output element in the same order, only the MMA shape differs (256 pixel rows over
an SM pair, each SM holding half of every weight block), so the outputs must be equal bit for
bit; and against the fp32 cuDNN reference of the fused layer."""

from __future__ import annotations

import numpy as np
import pytest

from gpu_util import assert_fp16_layer_close, torch_conv_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _layer(H, W, nadds, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, 64, generator=g).half().to(dev)
    w = (torch.randn(64, 64, 3, 3, generator=g) * (2.0 / 576) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(64, generator=g) * 0.05).numpy().astype(np.float16)
    adds = [torch.randn(1, H, W, 64, generator=g).half().to(dev) for _ in range(nadds)]
    return x, w, b, adds


def _run(algo, x, w, b, act, adds, out=None):
    from arthip_b200.engine import Conv3x3
    _, H, W, _ = x.shape
    if out is None:
        out = torch.full((1, H, W, 64), float("nan"), dtype=torch.float16, device=x.device)
    conv = Conv3x3(w, b.astype(np.float32), act=act, algo=algo)
    try:
        conv.run(x.data_ptr(), H, W, out.data_ptr(), *(a.data_ptr() for a in adds),
                 stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert conv.status() == 0
    finally:
        conv.close()
    return out


@pytest.mark.parametrize("H,W,act,nadds", [
    (5, 256, 1, 0),      # one cluster strip
    (37, 300, 1, 0),     # a partial second strip: the odd CTA of that pair has no pixels
    (19, 131, 0, 2),     # residual + skip, narrower than one pair strip
    (13, 520, 2, 1),     # SiLU
    (3, 1000, 0, 1),     # short segments
    (270, 480, 1, 0),    # many rows per cluster
])
def test_pair_kernel_equals_the_single_sm_kernel(H, W, act, nadds):
    x, w, b, adds = _layer(H, W, nadds, seed=H * 7 + W)
    want = _run("direct", x, w, b, act, adds)
    got = _run("pair", x, w, b, act, adds)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    ref = torch_conv_layer(x, w, b, act, adds)
    scale = ref.abs() + sum((a.float().abs() for a in adds), torch.zeros_like(ref))
    assert_fp16_layer_close(got.float().cpu().numpy(), ref.cpu().numpy(), f"pair {H}x{W}", scale.cpu().numpy(),
                            ulps=3.0 if act == 2 else 2.0)


def test_pair_kernel_in_place_residual():
    x, w, b, adds = _layer(37, 300, 2, seed=3)
    want = _run("pair", x, w, b, 0, adds)
    inplace = adds[1].clone()
    got = _run("pair", x, w, b, 0, [adds[0], inplace], out=inplace)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_pair_kernel_config1_full_size():
    x, w, b, _ = _layer(1080, 1920, 0, seed=1)
    want = _run("direct", x, w, b, 1, [])
    got = _run("pair", x, w, b, 1, [])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
