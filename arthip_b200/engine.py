"""Python front end of the native engine.

* :class:`EngineHarness` mirrors the reference suite's ctypes wrapper
  (``tests/correctness/harness/engine.py:47-200``): ``probe`` / ``run`` /
  ``alloc_failure_then_run`` over the ``engine_*`` driver ABI, raising
  :class:`EngineHarnessError` with the engine's own message, so tests read like the
  reference's.
* :class:`Engine` holds one persistent engine (``ah_engine_*``): host frames, the
  device-resident path (``prepare`` / ``enqueue``) and per-op timing.
* :class:`Conv3x3` is one fused conv layer on device NHWC tensors (``ah_conv3x3_*``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .native import lib

_ERR_LEN = 2048
_MAX_RANK = 8


class EngineHarnessError(RuntimeError):
    """The engine rejected the model, the shape, or the run."""


@dataclass(frozen=True)
class Probe:
    in_fp32: bool
    out_fp32: bool
    in_channels: int
    out_channels: int
    shape: tuple[int, ...]  # NCHW


@dataclass(frozen=True)
class RunResult:
    output: np.ndarray  # logical NCHW float64
    shape: tuple[int, ...]


def _err() -> ctypes.Array:
    return ctypes.create_string_buffer(_ERR_LEN)


def _msg(buf, fallback: str) -> str:
    t = bytes(buf.value).decode(errors="replace").strip()
    return t or fallback


def decode_output(buf: bytes, shape, out_fp32: bool) -> np.ndarray:
    n, c, h, w = (int(v) for v in shape)
    return np.frombuffer(buf, dtype=np.float32 if out_fp32 else np.float16).reshape(n, c, h, w).astype(np.float64)


def ramp_input(c: int, h: int, w: int, in_fp32: bool) -> np.ndarray:
    """The deterministic ``((i*37+11) mod 251)/251`` ramp in the NCHW host layout."""
    i = np.arange(c * h * w, dtype=np.int64)
    flat = (((i * 37) + 11) % 251).astype(np.float32) / np.float32(251)
    return flat if in_fp32 else flat.astype(np.float16)


class EngineHarness:
    """Binding to the reference-compatible driver ABI (one fresh engine per call)."""

    def __init__(self):
        self._lib = lib()

    def device_count(self) -> int:
        n = ctypes.c_int(-1)
        if self._lib.engine_device_count(ctypes.byref(n)) != 0:
            return -1
        return n.value

    def probe(self, model, *, n=1, h=16, w=16, c=1, device=0) -> Probe:
        err = _err()
        i32 = ctypes.c_int
        in32, out32, cin, cout = i32(0), i32(0), i32(0), i32(0)
        shape, rank = (ctypes.c_int64 * _MAX_RANK)(), i32(0)
        rc = self._lib.engine_probe(str(model).encode(), n, h, w, c, device, err, _ERR_LEN, ctypes.byref(in32),
                                    ctypes.byref(out32), ctypes.byref(cin), ctypes.byref(cout), shape,
                                    ctypes.byref(rank))
        if rc != 0:
            raise EngineHarnessError(_msg(err, f"engine_probe failed (rc={rc})"))
        return Probe(bool(in32.value), bool(out32.value), cin.value, cout.value,
                     tuple(int(shape[i]) for i in range(rank.value)))

    def run(self, model, *, n=1, h=16, w=16, c=1, device=0, raw_input: np.ndarray | None = None) -> RunResult:
        probe = self.probe(model, n=n, h=h, w=w, c=c, device=device)
        if raw_input is None:
            raw_input = ramp_input(c, h, w, probe.in_fp32)
        raw_input = np.ascontiguousarray(raw_input)
        numel = int(np.prod(probe.shape))
        cap = numel * (4 if probe.out_fp32 else 2)
        out = ctypes.create_string_buffer(cap)
        out_bytes, out32 = ctypes.c_size_t(0), ctypes.c_int(0)
        shape, rank = (ctypes.c_int64 * _MAX_RANK)(), ctypes.c_int(0)
        err = _err()
        rc = self._lib.engine_run(str(model).encode(), n, h, w, c, device, raw_input.ctypes.data, raw_input.nbytes,
                                  ctypes.cast(out, ctypes.c_void_p), cap, ctypes.byref(out_bytes),
                                  ctypes.byref(out32), shape, ctypes.byref(rank), err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, f"engine_run failed (rc={rc})"))
        rs = tuple(int(shape[i]) for i in range(rank.value))
        return RunResult(decode_output(out.raw[: out_bytes.value], rs, bool(out32.value)), rs)

    def alloc_failure_then_run(self, model, *, big_h=200_000, big_w=200_000, n=1, c=1, h=16, w=16, device=0):
        probe = self.probe(model, n=n, h=h, w=w, c=c, device=device)
        raw = np.ascontiguousarray(ramp_input(c, h, w, probe.in_fp32))
        numel = int(np.prod(probe.shape))
        cap = numel * (4 if probe.out_fp32 else 2)
        out = ctypes.create_string_buffer(cap)
        out_bytes, out32 = ctypes.c_size_t(0), ctypes.c_int(0)
        shape, rank = (ctypes.c_int64 * _MAX_RANK)(), ctypes.c_int(0)
        ferr, rerr = _err(), _err()
        rc = self._lib.engine_alloc_failure_then_run(str(model).encode(), n, big_h, big_w, c, device, raw.ctypes.data,
                                                     raw.nbytes, ctypes.cast(out, ctypes.c_void_p), cap,
                                                     ctypes.byref(out_bytes), ctypes.byref(out32), shape,
                                                     ctypes.byref(rank), ferr, _ERR_LEN, rerr, _ERR_LEN)
        fail = _msg(ferr, "")
        if rc != 0:
            raise EngineHarnessError(f"driver rc={rc}; reported failure={fail!r}; recovery={_msg(rerr, '')!r}")
        rs = tuple(int(shape[i]) for i in range(rank.value))
        return fail, RunResult(decode_output(out.raw[: out_bytes.value], rs, bool(out32.value)), rs)


def inspect_model(path) -> dict:
    """Parse and fuse a model on the host only (no GPU); returns the fused op list."""
    l = lib()
    buf = ctypes.create_string_buffer(1 << 16)
    err = _err()
    i32 = ctypes.c_int
    in32, out32, cin, cout = i32(0), i32(0), i32(0), i32(0)
    rc = l.ah_model_inspect(str(path).encode(), buf, len(buf), ctypes.byref(in32), ctypes.byref(out32),
                            ctypes.byref(cin), ctypes.byref(cout), err, _ERR_LEN)
    if rc != 0:
        raise EngineHarnessError(_msg(err, "inspect failed"))
    return {"ops": buf.value.decode().strip().splitlines(), "in_fp32": bool(in32.value),
            "out_fp32": bool(out32.value), "in_channels": cin.value, "out_channels": cout.value}


class Engine:
    """One persistent native engine (the object a plugin keeps per stream)."""

    def __init__(self, model, device: int = 0, _handle=None):
        self._lib = lib()
        self._h = ctypes.c_void_p()
        err = _err()
        if _handle is not None:
            self._h = _handle  # an engine the native side created (e.g. an EP region compile)
        else:
            if isinstance(model, (bytes, bytearray)):
                buf = ctypes.create_string_buffer(bytes(model), len(model))
                rc = self._lib.ah_engine_create_from_bytes(buf, len(model), device, ctypes.byref(self._h), err,
                                                           _ERR_LEN)
            else:
                rc = self._lib.ah_engine_create_from_file(str(model).encode(), device, ctypes.byref(self._h), err,
                                                          _ERR_LEN)
            if rc != 0:
                raise EngineHarnessError(_msg(err, "engine creation failed"))
        i32 = ctypes.c_int
        a, b, c, d = i32(0), i32(0), i32(0), i32(0)
        self._lib.ah_engine_info(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), ctypes.byref(d))
        self.in_fp32, self.out_fp32, self.in_channels, self.out_channels = bool(a.value), bool(b.value), c.value, d.value

    @classmethod
    def from_handle(cls, handle) -> "Engine":
        return cls(None, _handle=handle)

    def close(self):
        if self._h:
            self._lib.ah_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def output_shape(self, c: int, h: int, w: int) -> tuple[int, int, int, int]:
        s = (ctypes.c_int64 * 4)()
        if self._lib.ah_engine_output_shape(self._h, 1, c, h, w, s) != 0:
            raise EngineHarnessError("shape propagation failed")
        return tuple(int(v) for v in s)

    def run(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """One frame from a host NCHW array (fp16, or fp32 for fp32-IO models)."""
        x = np.ascontiguousarray(x)
        _, c, h, w = x.shape
        oshape = self.output_shape(c, h, w)
        if out is None:
            out = np.empty(oshape, dtype=np.float32 if self.out_fp32 else np.float16)
        err = _err()
        rc = self._lib.ah_engine_run(self._h, 1, c, h, w, x.ctypes.data, x.nbytes, out.ctypes.data, out.nbytes, err,
                                     _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, f"run failed (rc={rc})"))
        return out

    def run_ptr(self, c, h, w, in_ptr: int, in_bytes: int, out_ptr: int, out_bytes: int):
        """One frame between raw host pointers (e.g. pinned torch tensors)."""
        err = _err()
        rc = self._lib.ah_engine_run(self._h, 1, c, h, w, in_ptr, in_bytes, out_ptr, out_bytes, err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, f"run failed (rc={rc})"))

    def prepare(self, c: int, h: int, w: int):
        """Build the plan; returns (in_dev_ptr, out_dev_ptr, in_bytes, out_bytes)."""
        ip, op_ = ctypes.c_void_p(), ctypes.c_void_p()
        ib, ob = ctypes.c_size_t(0), ctypes.c_size_t(0)
        err = _err()
        rc = self._lib.ah_engine_prepare(self._h, 1, c, h, w, ctypes.byref(ip), ctypes.byref(op_), ctypes.byref(ib),
                                         ctypes.byref(ob), err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, "prepare failed"))
        return ip.value, op_.value, ib.value, ob.value

    def enqueue(self):
        err = _err()
        if self._lib.ah_engine_enqueue(self._h, err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "enqueue failed"))

    def synchronize(self):
        err = _err()
        if self._lib.ah_engine_synchronize(self._h, err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "synchronize failed"))

    def set_conv_algo(self, algo: str):
        """"direct" (default) or "winograd" for the 64 -> 64 convs; drops the current plan."""
        err = _err()
        if self._lib.ah_engine_set_conv_algo(self._h, {"direct": 0, "winograd": 1}[algo], err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "set_conv_algo failed"))

    def enqueue_ops(self, begin: int, end: int):
        """Launch ops [begin, end) of the prepared plan on the engine stream (no graph)."""
        err = _err()
        if self._lib.ah_engine_enqueue_ops(self._h, begin, end, err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "enqueue_ops failed"))

    def op_output(self, i: int) -> tuple[int, int, int, bool]:
        """Op i's output buffer: (device pointer, rows, bytes per row, is the boundary output)."""
        ptr, rows, rb, bnd = ctypes.c_void_p(), ctypes.c_int(0), ctypes.c_size_t(0), ctypes.c_int(0)
        if self._lib.ah_engine_op_output(self._h, i, ctypes.byref(ptr), ctypes.byref(rows), ctypes.byref(rb),
                                         ctypes.byref(bnd)) != 0:
            raise EngineHarnessError(f"no output for op {i}")
        return ptr.value, rows.value, rb.value, bool(bnd.value)

    @property
    def stream(self) -> int:
        return self._lib.ah_engine_stream(self._h) or 0

    def timing_start(self, max_frames: int):
        err = _err()
        if self._lib.ah_engine_timing_start(self._h, max_frames, err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "timing_start failed"))

    def timing_read(self):
        n = self._lib.ah_engine_num_ops(self._h)
        arr = (ctypes.c_double * max(n, 1))()
        span, frames = ctypes.c_double(0), ctypes.c_int(0)
        err = _err()
        rc = self._lib.ah_engine_timing_read(self._h, arr, n, ctypes.byref(span), ctypes.byref(frames), err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, "timing_read failed"))
        return [arr[i] for i in range(n)], span.value, frames.value

    def ops(self) -> list[dict]:
        n = self._lib.ah_engine_num_ops(self._h)
        res = []
        for i in range(n):
            kind, label = ctypes.create_string_buffer(64), ctypes.create_string_buffer(256)
            fl, by = ctypes.c_double(0), ctypes.c_double(0)
            self._lib.ah_engine_op_info(self._h, i, kind, 64, label, 256, ctypes.byref(fl), ctypes.byref(by))
            res.append({"kind": kind.value.decode(), "label": label.value.decode(), "flops": fl.value,
                        "bytes": by.value})
        return res

    def describe(self) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        self._lib.ah_engine_describe(self._h, buf, len(buf))
        return buf.value.decode()


class Conv3x3:
    """One fused 3x3 conv layer on device NHWC fp16 tensors (pointers as ints).
    ``algo``: "direct" (the default selection), "winograd" (Winograd F(2x2,3x3), 64 -> 64
    channels) or "pair" (the direct conv on two SMs per MMA, 64 -> 64 channels)."""

    def __init__(self, weight_oihw: np.ndarray, bias: np.ndarray | None, act: int = 0, device: int = 0,
                 algo: str = "direct"):
        self._lib = lib()
        w16 = np.ascontiguousarray(weight_oihw.astype(np.float16)).view(np.uint16)
        m, c = int(weight_oihw.shape[0]), int(weight_oihw.shape[1])
        b = None if bias is None else np.ascontiguousarray(bias.astype(np.float16).astype(np.float32))
        self._h = ctypes.c_void_p()
        err = _err()
        code = {"direct": 0, "winograd": 1, "pair": 2}[algo]
        rc = self._lib.ah_conv3x3_create_algo(device, c, m, w16.ctypes.data, None if b is None else b.ctypes.data,
                                              act, code, ctypes.byref(self._h), err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, "conv create failed"))
        self.C, self.M = c, m

    @property
    def kind(self) -> str:
        return {0: "conv_tc", 1: "conv_simt", 2: "conv_wino", 3: "conv_pair"}[self._lib.ah_conv3x3_kind(self._h)]

    def run(self, in_ptr: int, h: int, w: int, out_ptr: int, add1: int = 0, add2: int = 0, stream: int = 0):
        err = _err()
        rc = self._lib.ah_conv3x3_run(self._h, in_ptr, h, w, add1 or None, add2 or None, out_ptr, stream or None,
                                      err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, "conv run failed"))

    def status(self) -> int:
        st = ctypes.c_uint32(0)
        if self._lib.ah_conv3x3_status(self._h, ctypes.byref(st)) != 0:
            raise EngineHarnessError("conv status read failed")
        return st.value

    def close(self):
        if self._h:
            self._lib.ah_conv3x3_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
