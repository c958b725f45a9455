"""The allocation-free conv entry point (ah_conv3x3_run_noalloc) through the C ABI.

Some callers cannot call cudaMalloc while they run a layer: plugin hosts that hand their
plugins device buffers from the host's own memory pool and forbid allocation inside the
plugin. ah_conv3x3_run_noalloc serves them from a fixed __device__ array instead of
allocated weight / bias / error-word buffers. This checks it against the regular entry
point (ah_conv3x3_create + ah_conv3x3_run) on two calls in a row with different layers,
so the second call also shows that what the first left in the shared array does not leak
into its result. The file name sorts last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import assert_fp16_layer_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

_ERR_LEN = 512


def _layer(C, M, H, W, act, nadds, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.device("cuda:0")
    x = torch.rand(1, H, W, C, generator=g).half().to(dev)
    w = (torch.randn(M, C, 3, 3, generator=g) * (2.0 / (9 * C)) ** 0.5).numpy().astype(np.float16)
    b = (torch.randn(M, generator=g) * 0.05).numpy().astype(np.float16).astype(np.float32)
    adds = [torch.randn(1, H, W, M, generator=g).half().to(dev) for _ in range(nadds)]
    return x, w, b, adds


def _run_regular(x, w, b, act, adds):
    from arthip_b200.engine import Conv3x3
    _, H, W, _ = x.shape
    M = w.shape[0]
    out = torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=x.device)
    conv = Conv3x3(w, b, act=act)
    try:
        assert conv.kind == "conv_tc"
        conv.run(x.data_ptr(), H, W, out.data_ptr(), *(a.data_ptr() for a in adds),
                 stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert conv.status() == 0
    finally:
        conv.close()
    return out


def _run_noalloc(x, w, b, act, adds):
    from arthip_b200.native import lib
    _, H, W, C = x.shape
    M = w.shape[0]
    out = torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=x.device)
    w16 = np.ascontiguousarray(w).view(np.uint16)
    b32 = np.ascontiguousarray(b, dtype=np.float32)
    a = [t.data_ptr() for t in adds] + [None, None]
    err = ctypes.create_string_buffer(_ERR_LEN)
    rc = lib().ah_conv3x3_run_noalloc(0, C, M, w16.ctypes.data, b32.ctypes.data, act, x.data_ptr(), H, W,
                                      a[0], a[1], out.data_ptr(), torch.cuda.current_stream().cuda_stream,
                                      err, _ERR_LEN)
    assert rc == 0, err.value.decode(errors="replace")
    return out


def test_no_alloc_matches_regular_entry_point_on_consecutive_calls():
    cases = [
        # C, M, H, W, act, nadds: a vertical-window 64->64 block conv with both residual
        # adds, then a smaller channel-chunked layer whose weights cover less of the array.
        (64, 64, 37, 300, 1, 2),
        (48, 80, 11, 140, 2, 1),
    ]
    for i, (C, M, H, W, act, nadds) in enumerate(cases):
        x, w, b, adds = _layer(C, M, H, W, act, nadds, seed=4242 + i)
        want = _run_regular(x, w, b, act, adds).float()
        got = _run_noalloc(x, w, b, act, adds).float()
        scale = want.abs() + sum((t.float().abs() for t in adds), torch.zeros_like(want))
        assert_fp16_layer_close(got.cpu().numpy(), want.cpu().numpy(), f"no-alloc call {i + 1} C{C} M{M}",
                                scale.cpu().numpy(), ulps=3.0 if act == 2 else 2.0)


def test_no_alloc_rejects_unsupported_sizes():
    from arthip_b200.native import lib
    dev = torch.device("cuda:0")
    x = torch.zeros(1, 4, 4, 256, dtype=torch.float16, device=dev)
    out = torch.zeros(1, 4, 4, 8, dtype=torch.float16, device=dev)
    w16 = np.zeros((8, 256, 3, 3), dtype=np.uint16)
    err = ctypes.create_string_buffer(_ERR_LEN)
    rc = lib().ah_conv3x3_run_noalloc(0, 256, 8, w16.ctypes.data, None, 0, x.data_ptr(), 4, 4, None, None,
                                      out.data_ptr(), None, err, _ERR_LEN)
    assert rc == 1
    assert b"C <= 128" in err.value
