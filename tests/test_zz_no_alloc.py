"""The allocation-free conv entry point (ah_conv3x3_run_noalloc) through the C ABI.

Some callers cannot call cudaMalloc while they run a layer: plugin hosts that hand their
plugins device buffers from the host's own memory pool and forbid allocation inside the
plugin. ah_conv3x3_run_noalloc serves them from a fixed __device__ array instead of
allocated weight / bias / error-word buffers. Both entry points run the same kernel on the
same packed weights, so the no-alloc output must equal the regular entry point's
(ah_conv3x3_create + ah_conv3x3_run) bit for bit; it is also checked against the fp32
cuDNN reference of the layer. The cases run as consecutive calls with different layers,
so each call also shows that what the previous call left in the shared array does not leak
into its result. The file name sorts last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import assert_fp16_layer_close, torch_conv_layer

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


def _out_like(x, M, out):
    if out is not None:
        return out
    _, H, W, _ = x.shape
    return torch.full((1, H, W, M), float("nan"), dtype=torch.float16, device=x.device)


def _run_regular(x, w, b, act, adds, out=None):
    from arthip_b200.engine import Conv3x3
    _, H, W, _ = x.shape
    out = _out_like(x, w.shape[0], out)
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


def _call_noalloc(x, w, b, act, adds, out):
    from arthip_b200.native import lib
    _, H, W, C = x.shape
    M = w.shape[0]
    w16 = np.ascontiguousarray(w).view(np.uint16)
    b32 = np.ascontiguousarray(b, dtype=np.float32)
    a = [t.data_ptr() for t in adds] + [None, None]
    err = ctypes.create_string_buffer(_ERR_LEN)
    rc = lib().ah_conv3x3_run_noalloc(0, C, M, w16.ctypes.data, b32.ctypes.data, act, x.data_ptr(), H, W,
                                      a[0], a[1], out.data_ptr(), torch.cuda.current_stream().cuda_stream,
                                      err, _ERR_LEN)
    return rc, err.value.decode(errors="replace")


def _run_noalloc(x, w, b, act, adds, out=None):
    out = _out_like(x, w.shape[0], out)
    rc, msg = _call_noalloc(x, w, b, act, adds, out)
    assert rc == 0, msg
    return out


def _check_against_fp32(got, x, w, b, act, adds, label):
    ref = torch_conv_layer(x, w, b, act, adds)
    scale = ref.abs() + sum((t.float().abs() for t in adds), torch.zeros_like(ref))
    assert_fp16_layer_close(got.float().cpu().numpy(), ref.cpu().numpy(), label, scale.cpu().numpy(),
                            ulps=3.0 if act == 2 else 2.0)


CASES = [
    # C, M, H, W, act, nadds: a vertical-window 64->64 block conv with both residual adds;
    # a channel-chunked layer whose weights cover less of the array; M % 16 != 0 (the
    # per-element output form).
    (64, 64, 37, 300, 1, 2),
    (48, 80, 11, 140, 2, 1),
    (64, 40, 9, 133, 0, 1),
]


def test_no_alloc_matches_regular_entry_point_on_consecutive_calls():
    for i, (C, M, H, W, act, nadds) in enumerate(CASES):
        x, w, b, adds = _layer(C, M, H, W, act, nadds, seed=4242 + i)
        want = _run_regular(x, w, b, act, adds)
        got = _run_noalloc(x, w, b, act, adds)
        label = f"no-alloc call {i + 1} C{C} M{M}"
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"{label}: differs from the regular entry"
        _check_against_fp32(got, x, w, b, act, adds, label)


def test_no_alloc_in_place_residual():
    """Output buffer = the last residual operand (the in-place form the engine uses)."""
    C, M, H, W, act = 64, 64, 19, 131, 1
    x, w, b, adds = _layer(C, M, H, W, act, 2, seed=77)
    want = _run_regular(x, w, b, act, adds)
    inplace = adds[1].clone()
    got = _run_noalloc(x, w, b, act, [adds[0], inplace], out=inplace)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_no_alloc_reports_a_timed_out_wait_then_recovers():
    """A wait that cannot complete (test hook: one input row is never loaded, 50 ms bound)
    is reported as return 2 without a fault; the next call clears the error word and runs
    correctly."""
    from arthip_b200.native import lib
    C, M, H, W, act = 64, 64, 37, 300, 1
    x, w, b, adds = _layer(C, M, H, W, act, 0, seed=91)
    out = _out_like(x, M, None)
    lib().ah_test_set_conv_fault_hook(50, 1)
    try:
        rc, msg = _call_noalloc(x, w, b, act, adds, out)
    finally:
        lib().ah_test_set_conv_fault_hook(0, -1)
    assert rc == 2 and "timed-out" in msg, (rc, msg)
    got = _run_noalloc(x, w, b, act, adds)
    want = _run_regular(x, w, b, act, adds)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_no_alloc_call_allocates_no_device_memory():
    C, M, H, W, act = 64, 64, 64, 256, 1
    x, w, b, adds = _layer(C, M, H, W, act, 1, seed=5)
    out = _out_like(x, M, None)
    _run_noalloc(x, w, b, act, adds, out)  # warm-up: loads the kernel module
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    _run_noalloc(x, w, b, act, adds, out)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes across a call"


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
