"""The luma head kernel (C = 1) and the kx-in-N 2x DepthToSpace tail on the GPU.

* Luma head (`conv3x3_head1_kernel`): every output width it is built for (M = 32, 64, 96,
  128: one 64B-swizzled box, 128B-swizzled boxes, both), every activation, frames that
  end inside a 16-pixel tile, a 128-pixel block and an 8-row (4-row) block, against an
  fp32 cuDNN reference of the same layer.
* kx-in-N tail: through the engine (the tail is planned with its DepthToSpace output),
  for every input channel count it takes (16 .. 96: 32B, 64B and 128B swizzled chunks and
  their mixes) and C = 128 (which keeps the three-kx form), on frames narrower than one
  sub-tile, ending one pixel before / after a 120-pixel strip, and one row high, against
  the CPU oracle in both precision modes. And the kx-in-N form against the three-kx form
  (`ARTHIP_TAIL_KXN=0`, read when a plan is built) on the same model and frame.
"""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import Engine
from gpu_util import assert_fp16_layer_close, check_against_oracles, torch_conv_layer
from oracle import onnx_cpu

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


HEAD_CASES = [
    # M, H, W, act
    (32, 21, 129, 0),     # one 32-channel (64B) box per tile; one pixel past a block
    (64, 1, 1, 1),        # a single pixel
    (64, 9, 16, 2),       # SiLU, one 16-pixel tile, one row past an 8-row block
    (64, 17, 250, 1),     # ReLU, partial last tile and block
    (96, 13, 300, 1),     # 64 + 32 channel boxes, 4-row blocks
    (96, 5, 130, 2),      # SiLU with both box kinds
    (128, 9, 140, 0),     # two 64-channel boxes
    (128, 4, 1000, 2),    # SiLU, exactly one 4-row block, eight 128-pixel blocks
]


@pytest.mark.parametrize("M,H,W,act", HEAD_CASES)
def test_luma_head_matches_fp32_reference(M, H, W, act):
    from arthip_b200.engine import Conv3x3
    g = torch.Generator(device="cpu").manual_seed(M * 100 + H)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, 1, generator=g).half().to(dev)
    w = (torch.randn(M, 1, 3, 3, generator=g) * (2.0 / 9) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(M, generator=g) * 0.05).numpy().astype(np.float16)
    out = torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=dev)
    conv = Conv3x3(w, b.astype(np.float32), act=act)
    assert conv.kind == "conv_simt"
    conv.run(x.data_ptr(), H, W, out.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = torch_conv_layer(x, w, b, act, [])
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all(), "pixels left unwritten"
    assert_fp16_layer_close(got, ref.cpu().numpy(), f"luma head M{M} {H}x{W} act{act}", ref.abs().cpu().numpy(),
                            ulps=3.0 if act == 2 else 2.0)


def _tail_model(tmp_path, C, seed):
    spec = modelgen.ChainSpec(f"tail{C}", 1, C)
    cm = modelgen.conv_chain(spec, seed=seed)
    p = tmp_path / f"tail{C}_{seed}.onnx"
    op.save_model(cm.model, p)
    return cm, p


TAIL_CASES = [
    # C, H, W
    (16, 7, 119),     # 32B-swizzled chunk; one pixel short of a strip
    (32, 9, 121),     # 64B chunk; one pixel past a strip
    (48, 1, 250),     # 32 + 16 chunks; one row
    (64, 5, 241),     # three strips, one pixel into the third
    (64, 3, 20),      # narrower than one sub-tile's 30 outputs
    (80, 6, 360),     # 64 + 16 chunks; exactly three strips
    (96, 4, 130),     # 64 + 32 chunks (the R16F96 tail)
    (128, 5, 200),    # too wide for two CTAs per SM: the three-kx form
]


@pytest.mark.parametrize("C,H,W", TAIL_CASES)
def test_tail_vs_cpu_oracle(tmp_path, C, H, W):
    cm, p = _tail_model(tmp_path, C, seed=C + H)
    x = modelgen.synthetic_frame(C + W, 1, H, W)
    eng = Engine(p)
    got = eng.run(x).astype(np.float64)
    assert got.shape == (1, 1, 2 * H, 2 * W)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes")
    ref32 = onnx_cpu.run_model(cm.model, xd, mode="fp32_nodes")
    variants = [onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", reverse_channels=True),
                onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", use_torch=False)]
    check_against_oracles(got, ref16, ref32, variants, f"tail C{C} {H}x{W}")


@pytest.mark.parametrize("cfg,H,W", [("R8F64", 37, 250), ("R16F96", 11, 241)])
def test_tail_kxn_matches_three_kx_form(tmp_path, monkeypatch, cfg, H, W):
    cm = modelgen.conv_chain(modelgen.CONFIGS[cfg], seed=5)
    p = tmp_path / f"{cfg}.onnx"
    op.save_model(cm.model, p)
    x = modelgen.synthetic_frame(5, 1, H, W)
    monkeypatch.delenv("ARTHIP_TAIL_KXN", raising=False)
    new = Engine(p).run(x).astype(np.float32)
    monkeypatch.setenv("ARTHIP_TAIL_KXN", "0")
    old = Engine(p).run(x).astype(np.float32)
    # Same fp16 inputs to the tail; only its fp32 summation order differs, so the fp16
    # outputs agree up to one rounding step (one ulp of the larger of the two), plus the
    # fp32 cancellation error of the 576-term sums where an output is near zero. Measured
    # on B200 (R8F64 37x250): 112 of 37,000 outputs differ, each time one of the two forms
    # equals the float64 oracle.
    d = np.abs(new - old)
    mag = np.maximum(np.maximum(np.abs(old), np.abs(new)), 2.0 ** -14)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 10)
    assert (d <= ulp + 2.0 ** -16).all(), f"{cfg}: max diff {d.max():.3g}"
    assert (d == 0).mean() > 0.99, f"{cfg}: only {(d == 0).mean():.4f} identical"


def test_tail_timed_out_wait_is_reported_and_recovers(tmp_path, monkeypatch):
    """Failure detection without a GPU fault, through the kx-in-N tail: a model whose only
    tensor-core launch is the 64 -> 4 DepthToSpace tail; every pipeline arms its second
    input row's slot without loading it, so the MMA issuer's bounded wait (shortened to
    50 ms) runs out. The engine must report the timed-out wait, and the same engine must
    then produce the oracle's frame, as must a new engine on the same context. The first
    engine launches its ops one by one (`ARTHIP_NO_GRAPH=1`): a captured CUDA graph would
    keep the launch arguments of the faulted frame."""
    from arthip_b200.engine import EngineHarnessError
    from arthip_b200.modelgen import _conv_node, _half, _model, kern, linspace
    from arthip_b200.native import lib
    C, H, W = 64, 29, 250
    w = kern(7, 4, C) * 0.25
    b = linspace(4, -0.05, 0.05)
    nodes = [_conv_node("x", "w", "b", "raw"),
             op.make_node("DepthToSpace", ["raw"], ["y"], blocksize=2, mode="DCR")]
    model = _model(nodes, "x", [1, C, "h", "w"], op.FLOAT16, "y", [1, 1, "2*h", "2*w"], op.FLOAT16,
                   [_half("w", w), _half("b", b)])
    p = tmp_path / "tail_only.onnx"
    op.save_model(model, p)
    x = modelgen.synthetic_frame(3, C, H, W)
    monkeypatch.setenv("ARTHIP_NO_GRAPH", "1")
    eng = Engine(p)
    monkeypatch.delenv("ARTHIP_NO_GRAPH")
    lib().ah_test_set_conv_fault_hook(50, 1)
    try:
        with pytest.raises(EngineHarnessError, match="timed-out"):
            eng.run(x)
    finally:
        lib().ah_test_set_conv_fault_hook(0, -1)
    got = eng.run(x).astype(np.float64)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(model, xd, mode="fp16_nodes")
    ref32 = onnx_cpu.run_model(model, xd, mode="fp32_nodes")
    variants = [onnx_cpu.run_model(model, xd, mode="fp16_nodes", use_torch=False)]
    check_against_oracles(got, ref16, ref32, variants, "tail only, after recovery")
    again = Engine(p).run(x).astype(np.float64)
    assert np.array_equal(again, got), "a new engine (CUDA graph) differs from the recovered one"
