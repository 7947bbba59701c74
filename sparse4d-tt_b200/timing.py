"""Device-side timing of kernels that run inside CUDA graphs.

``TimingEvent`` is a CUDA event (driver handle, timing enabled) whose ``record`` becomes an
event-record node of the graph when the stream is being captured, so that every replay of the
graph records it again (the events then hold the timestamps of the latest replay); outside
capture it records like ``torch.cuda.Event``.

Only the CUDA driver (``libcuda.so.1``) is used, through ctypes: the runtime handles torch hands
out (``cudaEvent_t``, ``cudaStream_t``) are the driver's.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

_CU_EVENT_DEFAULT = 0
_CU_EVENT_RECORD_EXTERNAL = 0x1

_lib: Optional[ctypes.CDLL] = None


def _cu() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL("libcuda.so.1")
        vp, u32 = ctypes.c_void_p, ctypes.c_uint
        sigs = {
            "cuEventCreate": [ctypes.POINTER(vp), u32],
            "cuEventDestroy_v2": [vp],
            "cuEventRecord": [vp, vp],
            "cuEventRecordWithFlags": [vp, vp, u32],
            "cuEventElapsedTime": [ctypes.POINTER(ctypes.c_float), vp, vp],
            "cuEventSynchronize": [vp],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = lib
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: CUresult {rc}")


class TimingEvent:
    """A timing CUDA event; ``record`` during stream capture adds an event-record node."""

    def __init__(self):
        torch.cuda.init()  # the driver context torch uses must exist and be current
        h = ctypes.c_void_p()
        _check(_cu().cuEventCreate(ctypes.byref(h), _CU_EVENT_DEFAULT), "cuEventCreate")
        self.handle = h.value

    def record(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream()).cuda_stream
        if torch.cuda.is_current_stream_capturing():
            _check(_cu().cuEventRecordWithFlags(self.handle, s, _CU_EVENT_RECORD_EXTERNAL), "cuEventRecordWithFlags")
        else:
            _check(_cu().cuEventRecord(self.handle, s), "cuEventRecord")

    def synchronize(self) -> None:
        _check(_cu().cuEventSynchronize(self.handle), "cuEventSynchronize")

    def elapsed_time(self, end: "TimingEvent") -> float:
        """Milliseconds from this event to ``end`` (both recorded and complete)."""
        ms = ctypes.c_float()
        _check(_cu().cuEventElapsedTime(ctypes.byref(ms), self.handle, end.handle), "cuEventElapsedTime")
        return float(ms.value)

    def __del__(self):
        h, self.handle = getattr(self, "handle", None), None
        if h and _lib is not None:
            _lib.cuEventDestroy_v2(h)
