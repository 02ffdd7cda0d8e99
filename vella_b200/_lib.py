"""ctypes binding of ``libvella_cuda.so`` (the C ABI declared in ``include/vella_cuda.h``).

There is no fallback: if the library is missing or fails to load, importing anything that
needs it raises, so a CPU or library path can never silently stand in for the kernels.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("VELLA_LIB", _PKG / "_lib" / "libvella_cuda.so"))

OK, E_UNSUPPORTED, E_INVALID, E_CUDA, E_NONFINITE, E_OOM = range(6)
BF16, F16 = 0, 1
EPI = {"none": 0, "bias": 1, "residual": 2, "biasResidual": 3, "siluGate": 4, "biasGelu": 5,
       "biasGeluResidual": 6}
STATUS_NAMES = {0: "VELLA_OK", 1: "VELLA_E_UNSUPPORTED", 2: "VELLA_E_INVALID", 3: "VELLA_E_CUDA",
                4: "VELLA_E_NONFINITE", 5: "VELLA_E_OOM"}


class VellaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code


class QgemmDesc(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("bits", ctypes.c_int32), ("group_size", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("epilogue", ctypes.c_int32)]


_vp = ctypes.c_void_p
_PROTOS = {
    "vella_version": (ctypes.c_char_p, []),
    "vella_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "vella_qgemm_supports": (ctypes.c_int, [ctypes.POINTER(QgemmDesc)]),
    "vella_qgemm_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(QgemmDesc)]),
    "vella_qgemm": (ctypes.c_int, [ctypes.POINTER(QgemmDesc)] + [_vp] * 10 + [_vp, ctypes.c_size_t, _vp]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises when it is absent: build it with ``python -m vella_b200.build``)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m vella_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _PROTOS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def declare(name: str, restype, argtypes) -> None:
    """Register the prototype of a further C-ABI function (used by the other modules)."""
    _PROTOS[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().vella_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int) -> int:
    if code != OK:
        raise VellaError(code, last_error())
    return code


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()
