"""BASELINE configs end to end on the GPU, against the oracle.

* C0 (C4F32 @256x256) and reduced-size C2/C3: the CPU oracle in both precision modes
  (fp16 rounding at every node, and fp32 between nodes) — max-abs <= 4e-3, PSNR >= 55 dB.
* Full-size C2 (R8F64 @1920x1080), C3 (R16F96 @1080p), C4 (R8F64 @3840x2160): the same
  graph through the oracle's torch path on the GPU in fp32 (cuDNN, TF32 off).
* Size-independent properties: a crop of a full frame equals the same crop computed from
  a frame-sized margin (receptive-field locality), determinism across engines.
"""

from __future__ import annotations

import numpy as np
import pytest

from arthip_b200 import modelgen, onnx_proto as op
from arthip_b200.engine import Engine
from gpu_util import assert_frame_parity, check_against_oracles
from oracle import onnx_cpu

pytestmark = pytest.mark.gpu


def _model(tmp_path, cfg, seed):
    cm = modelgen.conv_chain(modelgen.CONFIGS[cfg], seed=seed)
    p = tmp_path / f"{cfg}_{seed}.onnx"
    op.save_model(cm.model, p)
    return cm, p


def _oracle_gap(a, b):
    """[0,1]-output distance between two oracle runs."""
    return float(np.abs(np.clip(a, 0, 1) - np.clip(b, 0, 1)).max())


@pytest.mark.parametrize("cfg,seed,h,w", [("C4F32", 0, 256, 256), ("R8F64", 2, 96, 160), ("R16F96", 3, 64, 136)])
def test_config_vs_cpu_oracle(tmp_path, cfg, seed, h, w):
    cm, p = _model(tmp_path, cfg, seed)
    x = modelgen.synthetic_frame(seed, 1, h, w)
    eng = Engine(p)
    got = eng.run(x).astype(np.float64)
    xd = x.astype(np.float64)
    ref16 = onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes")
    ref32 = onnx_cpu.run_model(cm.model, xd, mode="fp32_nodes")
    variants = [onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", reverse_channels=True),
                onnx_cpu.run_model(cm.model, xd, mode="fp16_nodes", use_torch=False)]
    check_against_oracles(got, ref16, ref32, variants, f"{cfg} {h}x{w}")


@pytest.mark.parametrize("cfg,seed,h,w", [("R8F64", 2, 1080, 1920), ("R16F96", 3, 1080, 1920),
                                          ("R8F64", 4, 2160, 3840)])
def test_config_full_size_vs_fp32_reference(tmp_path, cfg, seed, h, w):
    cm, p = _model(tmp_path, cfg, seed)
    x = modelgen.synthetic_frame(seed, 1, h, w)
    eng = Engine(p)
    got = eng.run(x).astype(np.float64)
    assert got.shape == (1, 1, 2 * h, 2 * w)
    refs = [onnx_cpu.run_model(cm.model, x.astype(np.float64), mode=m, device="cuda:0")
            for m in ("fp16_nodes", "fp32_nodes")]
    alt = onnx_cpu.run_model(cm.model, x.astype(np.float64), mode="fp16_nodes", device="cuda:0",
                             reverse_channels=True)
    check_against_oracles(got, refs[0], refs[1], [alt], f"{cfg} {h}x{w} (GPU fp32 reference)")


def test_crop_locality(tmp_path):
    """18 conv layers see 18 pixels each way: an interior crop computed from a frame
    with a >= 18-pixel margin equals the same region of the full-frame result."""
    cm, p = _model(tmp_path, "R8F64", 7)
    x = modelgen.synthetic_frame(7, 1, 300, 520)
    eng = Engine(p)
    full = eng.run(x)
    y0, x0, hh, ww = 100, 200, 64, 96
    m = 20
    crop_in = np.ascontiguousarray(x[:, :, y0 - m:y0 + hh + m, x0 - m:x0 + ww + m])
    part = eng.run(crop_in)
    a = full[:, :, 2 * y0:2 * (y0 + hh), 2 * x0:2 * (x0 + ww)]
    b = part[:, :, 2 * m:2 * (m + hh), 2 * m:2 * (m + ww)]
    np.testing.assert_array_equal(a, b)


def _dev_bytes(ptr, nbytes):
    """A torch uint8 view of raw device memory (CUDA array interface)."""
    import torch

    class _Buf:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3}
    return torch.as_tensor(_Buf(), device="cuda")


def test_device_resident_path_matches_host_path(tmp_path):
    import torch
    cm, p = _model(tmp_path, "R8F64", 2)
    x = modelgen.synthetic_frame(2, 1, 135, 240)
    eng = Engine(p)
    host = eng.run(x)
    in_ptr, out_ptr, ib, ob = eng.prepare(1, 135, 240)
    _dev_bytes(in_ptr, ib).copy_(torch.from_numpy(x.reshape(-1).view(np.uint8)).cuda())
    torch.cuda.synchronize()
    for _ in range(3):
        eng.enqueue()
    eng.synchronize()
    dev = _dev_bytes(out_ptr, ob).cpu().numpy().view(np.float16).reshape(host.shape)
    np.testing.assert_array_equal(dev, host)
