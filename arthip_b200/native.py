"""ctypes binding of the native library (``lib/libarthip_b200.so``, C ABI in
``include/arthip_b200.h``).

Loading fails loudly: there is no Python or CPU fallback for any compute entry point.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libarthip_b200.so"

# Every function the header declares, with (restype, argtypes).
_i32, _i64, _sz, _vp, _cp = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p
_i32p, _i64p, _szp = ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(_sz)
_dp = ctypes.POINTER(ctypes.c_double)
_u32p = ctypes.POINTER(ctypes.c_uint32)

SIGNATURES: dict[str, tuple] = {
    "engine_device_count": (_i32, [_i32p]),
    "engine_probe": (_i32, [_cp, _i32, _i32, _i32, _i32, _i32, _cp, _i32, _i32p, _i32p, _i32p, _i32p, _i64p, _i32p]),
    "engine_run": (_i32, [_cp, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _sz, _szp, _i32p, _i64p, _i32p, _cp,
                          _i32]),
    "engine_alloc_failure_then_run": (_i32, [_cp, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _sz, _szp, _i32p,
                                             _i64p, _i32p, _cp, _i32, _cp, _i32]),
    "ah_engine_create_from_file": (_i32, [_cp, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_engine_create_from_bytes": (_i32, [_vp, _sz, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_engine_destroy": (None, [_vp]),
    "ah_engine_info": (_i32, [_vp, _i32p, _i32p, _i32p, _i32p]),
    "ah_engine_output_shape": (_i32, [_vp, _i32, _i32, _i32, _i32, _i64p]),
    "ah_engine_run": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _sz, _cp, _i32]),
    "ah_engine_prepare": (_i32, [_vp, _i32, _i32, _i32, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _szp, _szp,
                                 _cp, _i32]),
    "ah_engine_enqueue": (_i32, [_vp, _cp, _i32]),
    "ah_engine_synchronize": (_i32, [_vp, _cp, _i32]),
    "ah_engine_set_conv_algo": (_i32, [_vp, _i32, _cp, _i32]),
    "ah_engine_enqueue_ops": (_i32, [_vp, _i32, _i32, _cp, _i32]),
    "ah_engine_op_output": (_i32, [_vp, _i32, ctypes.POINTER(_vp), _i32p, _szp, _i32p]),
    "ah_engine_stream": (_vp, [_vp]),
    "ah_engine_timing_start": (_i32, [_vp, _i32, _cp, _i32]),
    "ah_engine_timing_read": (_i32, [_vp, _dp, _i32, _dp, _i32p, _cp, _i32]),
    "ah_engine_num_ops": (_i32, [_vp]),
    "ah_engine_op_info": (_i32, [_vp, _i32, _cp, _i32, _cp, _i32, _dp, _dp]),
    "ah_engine_describe": (_i32, [_vp, _cp, _i32]),
    "ah_model_inspect": (_i32, [_cp, _cp, _i32, _i32p, _i32p, _i32p, _i32p, _cp, _i32]),
    "ah_ep_device_usable": (_i32, [_i32]),
    "ah_ep_node_supported": (_i32, [_vp, _sz, _i32]),
    "ah_ep_get_capability": (_i32, [_vp, _sz, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_ep_region_count": (_i32, [_vp]),
    "ah_ep_region_nodes": (_i32, [_vp, _i32, _i32p, _i32]),
    "ah_ep_region_value_count": (_i32, [_vp, _i32, _i32]),
    "ah_ep_region_value": (_i32, [_vp, _i32, _i32, _i32, _cp, _i32]),
    "ah_ep_region_name": (_i32, [_vp, _i32, _cp, _i32]),
    "ah_ep_region_inspect": (_i32, [_vp, _i32, _cp, _i32, _cp, _i32]),
    "ah_ep_compile_region": (_i32, [_vp, _i32, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_ep_capability_destroy": (None, [_vp]),
    "ah_conv3x3_create": (_i32, [_i32, _i32, _i32, _vp, _vp, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_conv3x3_create_algo": (_i32, [_i32, _i32, _i32, _vp, _vp, _i32, _i32, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_conv3x3_run": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _cp, _i32]),
    "ah_conv3x3_kind": (_i32, [_vp]),
    "ah_conv3x3_status": (_i32, [_vp, _u32p]),
    "ah_conv3x3_destroy": (None, [_vp]),
    "ah_conv3x3_run_noalloc": (_i32, [_i32, _i32, _i32, _vp, _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp,
                                      _cp, _i32]),
    "ah_test_set_conv_fault_hook": (None, [_i32, _i32]),
    "ah_convert_float_to_float16": (_i32, [_vp, _sz, _i32, _cp, _i32, _i32, _vp, _sz, _szp, _cp, _i32]),
    "ah_load_onnx": (_i32, [_vp, _sz, _cp, _i64, _i64, _vp, _sz, _szp, _cp, _i32]),
    "ah_vs_model_create": (_i32, [_vp, _vp, _sz, _cp, _vp, ctypes.POINTER(_vp), _cp, _i32]),
    "ah_vs_model_output": (_i32, [_vp, _vp, _i32p]),
    "ah_vs_model_get_frame": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _cp, _i32]),
    "ah_vs_model_destroy": (None, [_vp]),
    "ah_device_properties": (_i32, [_i32, _cp, _i32, _i64p, _i64p, _i64p]),
    "ah_float_to_half_rne": (None, [_vp, _vp, _sz]),
    "ah_float_to_half_ftz": (None, [_vp, _vp, _sz]),
    "ah_half_to_float": (None, [_vp, _vp, _sz]),
    "ah_version": (_cp, []),
}

_lib = None


class NativeLibraryMissing(RuntimeError):
    """The native library is not built (run ``python -m arthip_b200.build``)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("ARTHIP_LIB", LIB_PATH))
    if not path.exists():
        raise NativeLibraryMissing(
            f"native library not found at {path}; build it with `python -m arthip_b200.build` "
            "(there is no fallback implementation)")
    l = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args
    _lib = l
    return l
