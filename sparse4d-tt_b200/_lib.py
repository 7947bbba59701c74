"""ctypes binding of ``lib/libs4d_dfa.so`` (the C ABI declared in ``include/s4d_dfa.h``).

The library is loaded on first use.  If it is missing, every operator raises instead of
falling back to another implementation.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
# The in-tree build; S4D_LIB may point at another build of the same ABI.
LIB_PATH = os.environ.get("S4D_LIB") or os.path.join(_PKG, "lib", "libs4d_dfa.so")

S4D_OK = 0
S4D_ERR_INVALID_ARG = 1
S4D_ERR_UNSUPPORTED_SHAPE = 2
S4D_ERR_CUDA = 3
S4D_ERR_DEVICE_FAULT = 4

S4D_DTYPE_F32 = 0
S4D_DTYPE_BF16 = 1

S4D_LAYOUT_CAM_MAJOR = 0
S4D_LAYOUT_PT_MAJOR = 1
S4D_LAYOUT_GRID = 2

S4D_FLAG_BAD_LEVEL = 1
S4D_FLAG_WAIT_TIMEOUT = 2
S4D_FLAG_PEER_TIMEOUT = 4

S4D_MAPS_NCHW = 0
S4D_MAPS_NHWC = 1

S4D_RESIDUAL_NONE = 0
S4D_RESIDUAL_ADD = 1
S4D_RESIDUAL_CAT = 2

_i64, _int, _p, _sz = C.c_int64, C.c_int, C.c_void_p, C.c_size_t

# name -> (restype, argtypes); one entry per function of include/s4d_dfa.h
SIGNATURES = {
    "s4d_status_string": (C.c_char_p, [_int]),
    "s4d_last_error": (C.c_char_p, []),
    "s4d_abi_version": (_int, []),
    "s4d_kps_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "s4d_kps_project": (_int, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _int,
                               _p, _p, _p, _p, _p, _p, _sz, _p]),
    "s4d_kps_project_linear": (_int, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _p, _p, _i64, _i64, _i64,
                                      _int, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "s4d_set_tc_wait_limit_ns": (C.c_uint64, [C.c_uint64]),
    "s4d_kps_project_noalloc": (_int, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _int,
                                       _p, _p, _p, _p, _p, _p]),
    "s4d_kps_project_fused": (_int, [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _p, _p]),
    "s4d_deformable_aggregation": (_int, [_p, _int, _i64, _p, _p, _p, _p, _p, _int, _int,
                                          _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                          _p, _p, _p, _sz, _p]),
    "s4d_deformable_aggregation_anchors": (_int, [_p, _int, _i64, _p, _p, _p, _i64, _p, _i64, _p, _p, _p, _p, _p,
                                                  _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                                  _p, _p, _p, _sz, _p]),
    "s4d_deformable_aggregation_anchors_peer": (_int, [_p, _int, _i64, _p, _p, _p, _i64, _p, _i64, _p, _p, _p, _p,
                                                       _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                                       _p, _p, _i64, _i64, _p, _p, _sz, _p]),
    "s4d_dfa_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _int]),
    "s4d_dfa_camera_factors": (_int, [_p, _i64, _i64, _i64, _i64, _i64, _p, _sz, _p]),
    "s4d_dfa_weights_fc": (_int, [_p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "s4d_dfa_camera_logits": (_int, [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                     _p, _sz, _p]),
    "s4d_dfa_camera_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "s4d_dfa_camera_terms": (_int, [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                    _p, _sz, _p]),
    "s4d_pack_feature_maps": (_int, [_p, _int, _int, _i64, _i64, _i64, _p, _i64, _int, _p, _p]),
    "s4d_instance_bank_project": (_int, [_p, _p, _p, _i64, _i64, _p, _p]),
    "s4d_instance_bank_cache": (_int, [_p, _p, _p, _p, C.c_float, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "s4d_instance_bank_update": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "s4d_dfa_output_proj": (_int, [_p, _i64, _p, _p, _p, _i64, _int, _p, _i64, _i64, _p, _p]),
    "s4d_dfa_output_proj_sum": (_int, [_p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _int, _p, _i64, _i64, _p, _p]),
    "s4d_ipc_handle_bytes": (_sz, []),
    "s4d_ipc_export": (_int, [_p, _p, C.POINTER(C.c_uint64)]),
    "s4d_ipc_open": (_int, [_p, C.POINTER(C.c_void_p)]),
    "s4d_ipc_close": (_int, [_p]),
    "s4d_peer_signal_wait": (_int, [_p, _p, _int, _int, C.c_uint32, C.c_uint64, _p, _p]),
    "s4d_peer_signal_wait_counter": (_int, [_p, _p, _int, _int, _p, _int, C.c_uint64, _p, _p]),
    "s4d_layer_norm": (_int, [_p, _p, _p, _p, _i64, _i64, C.c_float, _p]),
}

_lib = None
_lock = threading.Lock()


class S4DError(RuntimeError):
    """A non-OK status from the C ABI."""

    def __init__(self, fn: str, status: int, msg: str):
        self.status = status
        super().__init__(f"{fn}: {status_string(status)}: {msg}")


# Version of include/s4d_dfa.h these bindings are written for (s4d_abi_version()).
ABI_VERSION = 109


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"CUDA library {LIB_PATH} is not built; run `python __graft_entry__.py build` "
                        "(or python sparse4d-tt_b200/build.py).  There is no CPU fallback.")
                handle = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                version = handle.s4d_abi_version()
                if version != ABI_VERSION:
                    raise RuntimeError(f"{LIB_PATH} has C ABI version {version}, these bindings expect "
                                       f"{ABI_VERSION}; rebuild it (python sparse4d-tt_b200/build.py)")
                _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().s4d_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status != S4D_OK:
        msg = lib().s4d_last_error().decode()
        if status in (S4D_ERR_INVALID_ARG, S4D_ERR_UNSUPPORTED_SHAPE):
            raise ValueError(f"{fn}: {status_string(status)}: {msg}")
        raise S4DError(fn, status, msg)
