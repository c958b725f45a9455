"""Single fused conv layers on the GPU against an fp32 cuDNN reference of the same layer.

Covers the tcgen05 tensor-core kernel (every supported channel-chunk combination,
partial column strips, 1-row frames, channel-sliced launches, fused ReLU/SiLU and one or
two residual adds) and the CUDA-core kernel (C==1 heads, narrow tails, odd widths).
"""

from __future__ import annotations

import numpy as np
import pytest

from gpu_util import assert_fp16_layer_close, torch_conv_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(C, M, H, W, act, nadds, seed):
    from arthip_b200.engine import Conv3x3
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, C, generator=g).half().to(dev)
    w = (torch.randn(M, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(M, generator=g) * 0.05).numpy().astype(np.float16)
    adds = [torch.randn(1, H, W, M, generator=g).half().to(dev) for _ in range(nadds)]
    out = torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=dev)
    conv = Conv3x3(w, b.astype(np.float32), act=act)
    conv.run(x.data_ptr(), H, W, out.data_ptr(), *(a.data_ptr() for a in adds),
             stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert conv.status() == 0, "kernel reported a pipeline timeout"
    ref = torch_conv_layer(x, w, b, act, adds)
    scale = ref.abs() + sum((a.float().abs() for a in adds), torch.zeros_like(ref))
    return conv.kind, out.float().cpu().numpy(), ref.cpu().numpy(), scale.cpu().numpy()


TC_CASES = [
    # C, M, H, W, act, nadds
    (64, 64, 37, 300, 1, 0),     # 3 strips, last partial
    (64, 64, 9, 128, 0, 1),      # exactly one strip, residual add
    (64, 64, 5, 131, 1, 2),      # block conv with residual + global skip
    (64, 64, 1, 5, 1, 0),        # a single short row
    (64, 64, 64, 64, 2, 0),      # SiLU epilogue
    (32, 32, 33, 129, 1, 1),     # 64B-swizzle chunk
    (16, 16, 17, 200, 0, 0),     # 32B-swizzle chunk
    (48, 80, 11, 140, 1, 0),     # chunks 32+16, N=80
    (96, 96, 13, 150, 1, 1),     # chunks 64+32 (R16F96 layers)
    (128, 128, 8, 140, 1, 0),    # two 64-chunks; channel-sliced launch
    (64, 256, 6, 130, 0, 0),     # N split across CTAs
    (128, 16, 4, 129, 0, 0),     # two chunks, narrow N
    (64, 4, 21, 70, 0, 0),       # narrow tail (N padded to 16, per-element stores)
    (64, 2, 9, 9, 0, 0),
    (32, 12, 7, 140, 1, 1),
    (48, 16, 33, 150, 2, 1),     # vertical window with N = 48 (chunks 32+16), SiLU, NHWC stores
    (64, 8, 40, 260, 0, 2),      # vertical window, padded N, per-element stores with two adds
    (48, 48, 19, 200, 1, 0),     # vertical window, one 48-channel slice (N = 144)
    (96, 96, 11, 140, 0, 1),     # two 48-channel slices; residual TMA-loaded into the staging
    (96, 96, 7, 300, 0, 2),      # two slices, residual + global skip (first TMA-staged, second per lane)
    (32, 96, 9, 131, 2, 0),      # two slices from a 32-channel input, SiLU
    (64, 128, 10, 260, 0, 1),    # two 64-channel slices, staged residual
    (64, 64, 19, 300, 2, 2),     # SiLU, 64 channels: eight epilogue warps per pipe, two residuals
    (64, 4, 13, 300, 1, 0),      # narrow tail over three strips, partial last strip
    (32, 3, 9, 253, 2, 1),       # narrow output with SiLU and a residual (per-element stores)
    (16, 1, 5, 127, 0, 0),       # one output channel, one pixel short of a strip
    (48, 5, 7, 130, 1, 0),       # five output channels, two pixels past a strip
]


@pytest.mark.parametrize("C,M,H,W,act,nadds", TC_CASES)
def test_tensor_core_conv_matches_fp32_reference(C, M, H, W, act, nadds):
    kind, got, ref, scale = _case(C, M, H, W, act, nadds, seed=C * 1000 + M + H)
    assert kind == "conv_tc"
    # SiLU rounds the sigmoid to fp16 before the product: a one-ulp sigmoid difference
    # (fp32 exp error near a rounding boundary) moves the product by up to one more ulp.
    assert_fp16_layer_close(got, ref, f"tc C{C} M{M} {H}x{W} act{act} adds{nadds}", scale,
                            ulps=3.0 if act == 2 else 2.0)


SIMT_CASES = [
    (1, 64, 40, 77, 0, 0),    # head conv (register-weight sliding-window kernel)
    (1, 32, 19, 45, 2, 2),    # head kernel with SiLU and two residual adds
    (1, 64, 3, 2000, 1, 0),   # head kernel, rows longer than one block
    (1, 8, 17, 25, 1, 0),
    (3, 64, 16, 33, 2, 0),    # chroma head (tensor-core head kernel, K = 27 -> 2 k-steps)
    (2, 32, 9, 300, 1, 0),    # tensor-core head, partial last segment
    (4, 128, 5, 70, 0, 0),    # tensor-core head, 3 k-steps, 16 channel octets
    (3, 96, 7, 257, 2, 0),    # tensor-core head, 12 channel octets, one pixel past a segment
    (4, 4, 33, 17, 0, 1),
    (24, 8, 9, 30, 0, 0),     # C not a multiple of 16
    (160, 16, 6, 40, 1, 0),   # wider than the tensor-core tiling: CUDA-core path
]


@pytest.mark.parametrize("C,M,H,W,act,nadds", SIMT_CASES)
def test_cuda_core_conv_matches_fp32_reference(C, M, H, W, act, nadds):
    kind, got, ref, scale = _case(C, M, H, W, act, nadds, seed=C * 1000 + M + H + 7)
    assert kind == "conv_simt"
    assert_fp16_layer_close(got, ref, f"simt C{C} M{M} {H}x{W}", scale)


def test_microbench_layer_full_size():
    """conv 64->64 + bias + ReLU on a 1080x1920 NHWC frame."""
    kind, got, ref, scale = _case(64, 64, 1080, 1920, 1, 0, seed=1)
    assert kind == "conv_tc"
    assert_fp16_layer_close(got, ref, "C1 1080p", scale)


def test_repeated_launches_are_bit_identical():
    from arthip_b200.engine import Conv3x3
    dev = torch.device("cuda:0")
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.rand(1, 270, 480, 64, generator=g).half().to(dev)
    w = (torch.randn(64, 64, 3, 3, generator=g) * 0.06).numpy().astype(np.float16)
    conv = Conv3x3(w, None, act=1)
    outs = []
    for _ in range(4):
        o = torch.empty(1, 270, 480, 64, dtype=torch.float16, device=dev)
        conv.run(x.data_ptr(), 270, 480, o.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
        outs.append(o)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_timed_out_pipeline_wait_is_reported_and_recovers():
    """Failure detection without a GPU fault: every CTA arms one input row's slot without
    loading it, so the MMA issuer's bounded wait (shortened to 50 ms) runs out; the kernel
    must drain, free its tensor memory and report the timeout in the status word, and the
    same layer must then run correctly."""
    from arthip_b200.engine import Conv3x3
    from arthip_b200.native import lib
    H, W, C, M = 37, 300, 64, 64
    g = torch.Generator(device="cpu").manual_seed(5)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, C, generator=g).half().to(dev)
    w = (torch.randn(M, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(M, generator=g) * 0.05).numpy().astype(np.float16)
    out = torch.zeros(1, H, W, M, dtype=torch.float16, device=dev)
    conv = Conv3x3(w, b.astype(np.float32), act=1)
    s = torch.cuda.current_stream().cuda_stream
    lib().ah_test_set_conv_fault_hook(50, 1)  # every CTA reads >= 3 input rows
    try:
        conv.run(x.data_ptr(), H, W, out.data_ptr(), stream=s)
        assert conv.status() != 0, "a wait that cannot complete must be reported"
    finally:
        lib().ah_test_set_conv_fault_hook(0, -1)
    conv.run(x.data_ptr(), H, W, out.data_ptr(), stream=s)
    torch.cuda.synchronize()
    assert conv.status() == 0
    ref = torch_conv_layer(x, w, b, 1, [])
    assert_fp16_layer_close(out.float().cpu().numpy(), ref.cpu().numpy(), "after recovery", ref.abs().cpu().numpy())


@pytest.mark.parametrize("C,M,H,W,act,nadds", [
    (64, 64, 37, 300, 1, 1),    # vertical window, block conv B
    (64, 64, 19, 131, 1, 2),    # block residual + global skip (only the last operand in place)
    (64, 64, 13, 200, 2, 1),    # SiLU (eight epilogue warps per pipe), in place
    (32, 32, 9, 140, 1, 1),     # vertical window, 64B-swizzle chunk
    (96, 96, 13, 150, 1, 1),    # vertical window in two 48-channel slices
    (64, 128, 9, 140, 0, 2),    # two 64-channel slices, staged first operand, second in place
    (128, 128, 8, 140, 1, 1),   # standard formulation, channel-sliced launch
    (64, 8, 11, 150, 0, 1),     # narrow N: per-element output form, in place but no reduce
])
def test_in_place_residual_is_bit_identical(C, M, H, W, act, nadds):
    """Output buffer = the last residual operand (as the engine assigns it once that operand
    is dead): the tensor-core conv then leaves the operand to reduce-add tile stores in L2.
    The result must equal the out-of-place result bit for bit, including residuals in the
    fp16 subnormal range behind ReLU zeros (no flush to zero in the L2 addition)."""
    from arthip_b200.engine import Conv3x3
    g = torch.Generator(device="cpu").manual_seed(C + M + H + nadds)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, C, generator=g).half().to(dev)
    w = (torch.randn(M, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(M, generator=g) * 0.05).numpy().astype(np.float16)
    adds = []
    for _ in range(nadds):
        r = torch.randn(1, H, W, M, generator=g)
        tiny = torch.rand(1, H, W, M, generator=g) < 0.3
        adds.append(torch.where(tiny, r * 3e-6, r).half().to(dev))
    conv = Conv3x3(w, b.astype(np.float32), act=act)
    s = torch.cuda.current_stream().cuda_stream
    ref = torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=dev)
    conv.run(x.data_ptr(), H, W, ref.data_ptr(), *(a.data_ptr() for a in adds), stream=s)
    inplace = adds[-1].clone()
    ops = [a.data_ptr() for a in adds[:-1]] + [inplace.data_ptr()]
    conv.run(x.data_ptr(), H, W, inplace.data_ptr(), *ops, stream=s)
    torch.cuda.synchronize()
    assert conv.status() == 0
    assert int((adds[-1].abs() < 6.1e-5).sum()) > 0
    if act == 1:  # ReLU zeros leave subnormal residuals as results
        assert int((ref.abs() < 6.1e-5).sum()) > 0
    diff = (inplace.view(torch.int16) != ref.view(torch.int16))
    assert int(diff.sum()) == 0, f"{int(diff.sum())} elements differ in place"
