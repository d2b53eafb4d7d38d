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
    # omg_branch: the pointers as plain addresses (set from numpy buffers).
    _fields_ = [
        ("tokens", C.c_void_p),
        ("n_tokens", C.c_size_t),
        ("want", C.c_void_p),
        ("n_want", C.c_size_t),
    ]


class GroupC(C.Structure):
    _fields_ = [
        ("prefix", u32p),
        ("n_prefix", C.c_size_t),
        ("branches", C.POINTER(Branch)),
        ("n_branches", C.c_size_t),
    ]


class EngineInfo(C.Structure):
    _fields_ = [
        ("d", C.c_int), ("vocab", C.c_int), ("layers", C.c_int), ("embed_dtype", C.c_int),
        ("per_layer_dim", C.c_int), ("device", C.c_int), ("capacity", C.c_size_t),
        ("max_rows", C.c_size_t), ("bos", C.c_uint32),
    ]


class LayaSeqC(C.Structure):
    # omg_laya_sequence: the pointers as plain addresses (set from numpy buffers).
    _fields_ = [
        ("ids", C.c_void_p),
        ("n_ids", C.c_size_t),
        ("markers", C.c_void_p),
        ("n_markers", C.c_size_t),
        ("qtype", C.c_int),
    ]


vp = C.c_void_p
pp = C.POINTER(C.c_void_p)
cs = C.c_char_p
sz = C.c_size_t
GroupP = C.POINTER(GroupC)
BranchP = C.POINTER(Branch)

# name -> (restype, argtypes); every function of include/omg_b200.h.
PROTOTYPES: dict[str, tuple] = {
    "omg_last_error": (C.c_char_p, []),
    "omg_version": (C.c_char_p, []),
    "omg_device_count": (C.c_int, []),
    "omg_host_alloc": (C.c_int, [C.c_int, sz, pp]),
    "omg_host_free": (None, [vp]),
    "omg_config_check": (C.c_int, [cs, C.c_char_p, sz]),
    "omg_config_tensors": (C.c_int, [cs, C.c_char_p, sz, szp]),
    "omg_builder_new": (C.c_int, [cs, C.c_int, pp]),
    "omg_builder_push": (C.c_int, [vp, cs, C.c_int, i64p, C.c_int, vp, sz, vp, sz]),
    "omg_builder_set_per_layer_table": (C.c_int, [vp, C.c_int, i64p, C.c_int, vp, sz, vp, sz]),
    "omg_builder_missing": (C.c_int, [vp, C.c_char_p, sz, szp]),
    "omg_builder_finish": (C.c_int, [vp, sz, sz, pp]),
    "omg_builder_free": (None, [vp]),
    "omg_engine_evaluate_groups": (C.c_int, [vp, GroupP, sz, C.c_int, f32p, sz, i32p]),
    "omg_engine_evaluate": (C.c_int, [vp, u32p, sz, BranchP, sz, C.c_int, f32p, sz]),
    "omg_engine_evaluate_rows": (C.c_int, [vp, u32p, sz, BranchP, sz, C.c_int, vp, sz, f32p, sz]),
    "omg_engine_warmup": (C.c_int, [vp]),
    "omg_engine_prefix_source": (C.c_int, [vp]),
    "omg_engine_is_resident": (C.c_int, [vp, u32p, sz]),
    "omg_engine_evict_resident": (None, [vp]),
    "omg_engine_set_state_cache": (C.c_int, [vp, sz, cs, cs]),
    "omg_engine_save_state": (C.c_int, [vp, u32p, sz, pp]),
    "omg_engine_restore_state": (C.c_int, [vp, vp]),
    "omg_engine_state_image_bytes": (sz, [vp, sz]),
    "omg_engine_export_state_device": (C.c_int, [vp, u32p, sz, vp, sz]),
    "omg_engine_import_state_device": (C.c_int, [vp, u32p, sz, vp, sz]),
    "omg_engine_gather_per_layer": (C.c_int, [vp, u32p, sz, u8p, sz]),
    "omg_engine_get_info": (C.c_int, [vp, C.POINTER(EngineInfo)]),
    "omg_engine_time_forward": (C.c_int, [vp, GroupP, sz, C.c_int, C.c_int, C.c_int, f32p,
                                          C.POINTER(C.c_int)]),
    "omg_engine_profile_forward": (C.c_int, [vp, GroupP, sz, C.c_int, C.c_int, C.c_int,
                                             C.c_char_p, sz, szp]),
    "omg_debug_attention": (C.c_int, [C.c_int, u16p, u16p, i32p, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int, C.c_int, u16p]),
    "omg_debug_attention_time": (C.c_int, [C.c_int, u16p, u16p, i32p, C.c_int, C.c_int, C.c_int,
                                           C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.POINTER(C.c_float)]),
    "omg_gemm_splitk_noalloc": (C.c_int, [C.c_int, vp, C.c_int, C.c_int, C.c_int, vp, C.c_int,
                                          C.c_int, vp, C.c_int, vp]),
    "omg_engine_record_event": (C.c_int, [vp, C.c_int]),
    "omg_engine_elapsed_ms": (C.c_int, [vp, C.c_int, C.c_int, f32p]),
    "omg_engine_destroy": (None, [vp]),
    "omg_state_byte_len": (sz, [vp]),
    "omg_state_to_bytes": (C.c_int, [vp, cs, u8p, sz, szp]),
    "omg_state_from_bytes": (C.c_int, [u8p, sz, cs, pp]),
    "omg_state_prefix": (C.c_int, [vp, u32p, sz, szp]),
    "omg_state_free": (None, [vp]),
    "omg_state_key": (C.c_uint64, [cs, u32p, sz]),
    "omg_quantize": (C.c_int, [C.c_int, f32p, sz, u8p, u8p]),
    "omg_dequantize": (C.c_int, [C.c_int, u8p, u8p, sz, f32p]),
    "omg_synth_normal": (C.c_int, [C.c_uint64, cs, C.c_float, C.c_float, f32p, sz]),
    "omg_debug_gemm_q": (C.c_int, [C.c_int, u16p, C.c_int, C.c_int, C.c_int, C.c_int, u8p, u8p,
                                    C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, C.c_int]),
    "omg_debug_mlp_q": (C.c_int, [C.c_int, u16p, C.c_int, C.c_int, C.c_int, u8p, u8p, C.c_int,
                                   u8p, u8p, C.c_int, u16p, f32p]),
    "omg_debug_gemm_time_q": (C.c_int, [C.c_int] * 9 + [f32p]),
    "omg_debug_mlp_time": (C.c_int, [C.c_int] * 7 + [f32p]),
    "omg_debug_dequant": (C.c_int, [C.c_int, C.c_int, u8p, u8p, C.c_int, C.c_int, C.c_int, u16p,
                                     u16p]),
    "omg_engine_weight_f16": (C.c_int, [vp, C.c_char_p, u16p, sz]),
    "omg_engine_arm_wait_timeout": (C.c_int, [vp, C.c_longlong]),
    "omg_builder_set_weight_layout": (C.c_int, [vp, C.c_int]),
    "omg_debug_gemm": (
        C.c_int,
        [C.c_int, u16p, C.c_int, C.c_int, C.c_int, u16p, C.c_int, C.c_int, C.c_int, C.c_int,
         C.c_int, C.c_void_p, C.c_int],
    ),
    "omg_debug_gemm_time": (C.c_int, [C.c_int] * 8 + [f32p]),
    "omg_debug_mlp": (C.c_int, [C.c_int, u16p, C.c_int, C.c_int, u16p, C.c_int, u16p, C.c_int,
                                u16p, f32p]),
    "omg_laya_config_check": (C.c_int, [cs, C.c_char_p, sz]),
    "omg_laya_config_tensors": (C.c_int, [cs, C.c_char_p, sz, szp]),
    "omg_laya_builder_new": (C.c_int, [cs, C.c_int, pp]),
    "omg_laya_builder_push": (C.c_int, [vp, cs, C.c_int, i64p, C.c_int, vp, sz, vp, sz]),
    "omg_laya_builder_missing": (C.c_int, [vp, C.c_char_p, sz, szp]),
    "omg_laya_builder_finish": (C.c_int, [vp, sz, sz, pp]),
    "omg_laya_builder_free": (None, [vp]),
    "omg_laya_warmup": (C.c_int, [vp]),
    "omg_laya_hidden": (C.c_int, [vp, C.POINTER(LayaSeqC), sz, f32p, sz]),
    "omg_laya_evaluate": (C.c_int, [vp, C.POINTER(LayaSeqC), sz, f32p, sz, f32p]),
    "omg_laya_probabilities": (C.c_int, [vp, C.c_int, f32p, sz, C.POINTER(C.c_double)]),
    "omg_laya_time_forward": (C.c_int, [vp, C.POINTER(LayaSeqC), sz, C.c_int, f32p,
                                        C.POINTER(C.c_int)]),
    "omg_laya_profile_forward": (C.c_int, [vp, C.POINTER(LayaSeqC), sz, C.c_int, C.c_char_p, sz,
                                           szp]),
    "omg_laya_record_event": (C.c_int, [vp, C.c_int]),
    "omg_laya_elapsed_ms": (C.c_int, [vp, C.c_int, C.c_int, f32p]),
    "omg_laya_destroy": (None, [vp]),
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
