"""Python view of the VapourSynth filter core (``ah_vs_*``, ``ah_convert_float_to_float16``,
``ah_load_onnx`` in include/arthip_b200.h): what the plugin shim calls, usable without
VapourSynth. ``Model`` mirrors ``core.hip.Model(clip, network_path, overlap, tilesize,
device_id, num_streams, fp16, flexible_output_prop)`` (src/vapoursynth/vs_hip.cpp:616-641)
on numpy planes."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from .engine import EngineHarnessError, _ERR_LEN, _err, _msg
from .native import lib

GRAY, RGB, YUV = 1, 2, 3
INTEGER, FLOAT = 0, 1


class _Format(ctypes.Structure):
    _fields_ = [("color_family", ctypes.c_int), ("sample_type", ctypes.c_int), ("bits_per_sample", ctypes.c_int),
                ("subsampling_w", ctypes.c_int), ("subsampling_h", ctypes.c_int), ("num_planes", ctypes.c_int),
                ("width", ctypes.c_int), ("height", ctypes.c_int)]


class _Args(ctypes.Structure):
    _fields_ = [("device_id", ctypes.c_int), ("num_streams", ctypes.c_int), ("fp16_set", ctypes.c_int),
                ("fp16", ctypes.c_int64), ("overlap_n", ctypes.c_int), ("overlap", ctypes.c_int64 * 2),
                ("tilesize_n", ctypes.c_int), ("tilesize", ctypes.c_int64 * 2),
                ("flexible_output_prop", ctypes.c_char_p)]


@dataclass
class ClipFormat:
    color_family: int
    sample_type: int
    bits_per_sample: int
    num_planes: int
    width: int
    height: int
    subsampling_w: int = 0
    subsampling_h: int = 0

    def _c(self) -> _Format:
        return _Format(self.color_family, self.sample_type, self.bits_per_sample, self.subsampling_w,
                       self.subsampling_h, self.num_planes, self.width, self.height)

    @property
    def dtype(self):
        if self.sample_type == INTEGER:
            return np.uint8 if self.bits_per_sample == 8 else np.uint16
        return np.float16 if self.bits_per_sample == 16 else np.float32


def _bytes_out(call, *args) -> bytes:
    n = ctypes.c_size_t(0)
    err = _err()
    if call(*args, None, 0, ctypes.byref(n), err, _ERR_LEN) != 0:
        raise EngineHarnessError(_msg(err, "conversion failed"))
    buf = ctypes.create_string_buffer(n.value)
    if call(*args, buf, n.value, ctypes.byref(n), err, _ERR_LEN) != 0:
        raise EngineHarnessError(_msg(err, "conversion failed"))
    return buf.raw[:n.value]


def convert_float_to_float16(model: bytes, *, force_fp16_initializers: bool = True, op_block_list=(),
                             cast_input: bool = False, cast_output: bool = False) -> bytes:
    block = ",".join(op_block_list).encode() if op_block_list else None
    return _bytes_out(lib().ah_convert_float_to_float16, model, len(model), int(force_fp16_initializers), block,
                      int(cast_input), int(cast_output))


def load_onnx(model: bytes | None = None, path: str | None = None, tile_w: int = 0, tile_h: int = 0) -> bytes:
    return _bytes_out(lib().ah_load_onnx, model, len(model) if model else 0, path.encode() if path else None,
                      tile_w, tile_h)


class Model:
    """One hip.Model filter instance: frames in as per-plane 2-D numpy arrays, out as a list
    of per-channel planes in the output clip's sample type."""

    def __init__(self, clip: ClipFormat, network_path=None, *, model_bytes: bytes | None = None, overlap=None,
                 tilesize=None, device_id: int = 0, num_streams: int = 1, fp16=None,
                 flexible_output_prop: str | None = None):
        self._lib = lib()
        a = _Args()
        a.device_id, a.num_streams = device_id, num_streams
        a.fp16_set, a.fp16 = (0, 0) if fp16 is None else (1, int(fp16))
        for name, vals in (("overlap", overlap), ("tilesize", tilesize)):
            vals = list(vals or [])
            setattr(a, f"{name}_n", len(vals))
            arr = getattr(a, name)
            for i, v in enumerate(vals[:2]):
                arr[i] = v
        a.flexible_output_prop = flexible_output_prop.encode() if flexible_output_prop else None
        self.clip = clip
        self._h = ctypes.c_void_p()
        err = _err()
        path = str(network_path).encode() if network_path is not None else None
        rc = self._lib.ah_vs_model_create(ctypes.byref(clip._c()), model_bytes,
                                          len(model_bytes) if model_bytes else 0, path, ctypes.byref(a),
                                          ctypes.byref(self._h), err, _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, "hip.Model failed"))
        f, n = _Format(), ctypes.c_int(0)
        self._lib.ah_vs_model_output(self._h, ctypes.byref(f), ctypes.byref(n))
        self.out_format = ClipFormat(f.color_family, f.sample_type, f.bits_per_sample, f.num_planes, f.width,
                                     f.height)
        self.num_output_channels = n.value

    def get_frame(self, planes: list[np.ndarray], frame_format: ClipFormat | None = None) -> list[np.ndarray]:
        fmt = frame_format or self.clip
        planes = [np.ascontiguousarray(p) for p in planes]
        src = (ctypes.c_void_p * len(planes))(*[p.ctypes.data for p in planes])
        sstr = (ctypes.c_ssize_t * len(planes))(*[p.strides[0] for p in planes])
        of = self.out_format
        h, w = fmt.height * (of.height // max(1, self.clip.height)), fmt.width * (of.width // max(1, self.clip.width))
        outs = [np.zeros((h, w), dtype=of.dtype) for _ in range(self.num_output_channels)]
        dst = (ctypes.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        dstr = (ctypes.c_ssize_t * len(outs))(*[o.strides[0] for o in outs])
        err = _err()
        rc = self._lib.ah_vs_model_get_frame(self._h, ctypes.byref(fmt._c()), src, sstr, dst, dstr, len(outs), err,
                                             _ERR_LEN)
        if rc != 0:
            raise EngineHarnessError(_msg(err, f"get_frame failed (rc={rc})"))
        return outs

    def close(self):
        if self._h:
            self._lib.ah_vs_model_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
