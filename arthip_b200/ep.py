"""Python view of the execution-provider partition rules in the native core
(``ah_ep_*`` in include/arthip_b200.h): what an ONNX Runtime provider shim asks of the
engine. Mirrors HIPExecutionProvider::GetCapability / Compile
(src/onnxruntime-hip/hip_execution_provider.cc:180-406) on serialized model bytes."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from .engine import Engine, EngineHarnessError, _err, _msg, _ERR_LEN
from .native import lib

PROVIDER = "HIPExecutionProvider"


@dataclass
class Region:
    index: int
    name: str
    nodes: list[int]
    activations: list[str]
    constants: list[str]
    outputs: list[str]


def device_usable(device: int) -> bool:
    return lib().ah_ep_device_usable(device) == 1


def node_supported(model_bytes: bytes, node_index: int) -> bool:
    r = lib().ah_ep_node_supported(model_bytes, len(model_bytes), node_index)
    if r < 0:
        raise EngineHarnessError("malformed model")
    return r == 1


class Capability:
    """The claimed regions of one model (GetCapability), and their compilation."""

    def __init__(self, model_bytes: bytes, context_ok: bool = True):
        self._lib = lib()
        self._bytes = bytes(model_bytes)
        self._h = ctypes.c_void_p()
        err = _err()
        if self._lib.ah_ep_get_capability(self._bytes, len(self._bytes), 1 if context_ok else 0,
                                          ctypes.byref(self._h), err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "capability failed"))
        self.regions = [self._region(i) for i in range(self._lib.ah_ep_region_count(self._h))]

    def _region(self, i: int) -> Region:
        n = self._lib.ah_ep_region_nodes(self._h, i, None, 0)
        arr = (ctypes.c_int * max(n, 1))()
        self._lib.ah_ep_region_nodes(self._h, i, arr, n)

        def values(kind):
            out = []
            for j in range(self._lib.ah_ep_region_value_count(self._h, i, kind)):
                buf = ctypes.create_string_buffer(1024)
                self._lib.ah_ep_region_value(self._h, i, kind, j, buf, len(buf))
                out.append(buf.value.decode())
            return out
        name = ctypes.create_string_buffer(128)
        self._lib.ah_ep_region_name(self._h, i, name, len(name))
        return Region(i, name.value.decode(), list(arr[:n]), values(0), values(1), values(2))

    def inspect(self, i: int) -> list[str]:
        """The fused op list region i compiles to (no GPU needed)."""
        buf = ctypes.create_string_buffer(1 << 16)
        err = _err()
        if self._lib.ah_ep_region_inspect(self._h, i, buf, len(buf), err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "inspect failed"))
        return buf.value.decode().strip().splitlines()

    def compile(self, i: int, device: int = 0) -> Engine:
        h = ctypes.c_void_p()
        err = _err()
        if self._lib.ah_ep_compile_region(self._h, i, device, ctypes.byref(h), err, _ERR_LEN) != 0:
            raise EngineHarnessError(_msg(err, "compile failed"))
        return Engine.from_handle(h)

    def close(self):
        if self._h:
            self._lib.ah_ep_capability_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
