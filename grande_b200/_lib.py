"""Loads ``libomg_b200.so`` (built in-tree by ``grande_b200.build``) and
declares the C ABI of ``include/omg_b200.h`` for ctypes.

There is no fallback: if the library is missing or fails to load, every entry
point raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libomg_b200.so"

_lib: C.CDLL | None = None

u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
u32p = C.POINTER(C.c_uint32)
i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)
f32p = C.POINTER(C.c_float)
szp = C.POINTER(C.c_size_t)


class OmgError(RuntimeError):
    """An error reported by the native engine (omg_last_error)."""


class Branch(C.Structure):
    _fields_ = [
        ("tokens", i32p),
        ("n_tokens", C.c_size_t),
        ("want", szp),
        ("n_want", C.c_size_t),
    ]


class GroupC(C.Structure):
    _fields_ = [
        ("prefix", u32p),
        ("n_prefix", C.c_size_t),
        ("branches", C.POINTER(Branch)),
        ("n_branches", C.c_size_t),
    ]


# name -> (restype, argtypes)
PROTOTYPES: dict[str, tuple] = {
    "omg_last_error": (C.c_char_p, []),
    "omg_version": (C.c_char_p, []),
    "omg_debug_gemm": (
        C.c_int,
        [C.c_int, u16p, C.c_int, C.c_int, C.c_int, u16p, C.c_int, C.c_int, C.c_int, C.c_int,
         C.c_int, C.c_void_p, C.c_int],
    ),
}


def lib() -> C.CDLL:
    """The loaded native library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OmgError(
                f"{LIB_PATH.name} is not built; run `python -m grande_b200.build` "
                "(there is no CPU fallback)"
            )
        _lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def check(rc: int) -> int:
    """Raise OmgError with the native message when a call returned -1."""
    if rc < 0:
        raise OmgError(lib().omg_last_error().decode("utf-8", "replace"))
    return rc


def ptr(arr, ctype):
    """ctypes pointer to a contiguous numpy array's data."""
    return arr.ctypes.data_as(C.POINTER(ctype))
