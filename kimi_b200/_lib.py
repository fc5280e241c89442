"""ctypes binding of ``libkimi_mla.so`` (the C ABI declared in include/kimi_mla.h).

The library is built in-tree by :mod:`kimi_b200.build`.  There is no other
implementation behind these calls: if the library is missing, every call
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libkimi_mla.so")

KIMI_OK = 0
KIMI_ERR_CUDA_BASE = 0x10000

# Symbols the header declares; tests check the library exports each one.
EXPORTED_SYMBOLS = (
    "kimi_abi_version",
    "kimi_status_string",
    "kimi_mla_decode_workspace_size",
    "kimi_mla_decode_num_splits",
    "kimi_mla_decode",
    "kimi_mla_reduce",
    "kimi_mxfp4_kv_append",
    "kimi_mxfp4_quantize",
    "kimi_mla_decode_static_workspace",
    "kimi_mla_decode_partial",
    "kimi_mla_decode_merge",
    "kimi_mla_q_absorb_rope_append",
    "kimi_ar_rmsnorm_mxfp4",
    "kimi_ar_rmsnorm_mxfp4_two_shot",
    "kimi_mla_v_up_o_proj",
    "kimi_device_status",
)

ABI_VERSION = 201

# Bits of the decode's device status word (KIMI_DEVICE_* in include/kimi_mla.h).
DEVICE_WAIT_BITS = 0x1FF
DEVICE_BAD_PAGE = 0x200
DEVICE_PEER_WAIT = 0x400
DEVICE_QABSORB_WAIT = 0x800
DEVICE_VUP_WAIT = 0x1000

AR_MAX_INPUTS = 8


class KimiMlaDecodeParams(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_b", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("kv_buffer", ctypes.c_void_p),
        ("kv_scales", ctypes.c_void_p),
        ("num_pages", ctypes.c_int64),
        ("kv_indptr", ctypes.c_void_p),
        ("kv_indices", ctypes.c_void_p),
        ("kv_last_page_len", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("o_stride_b", ctypes.c_int64),
        ("o_stride_h", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_splits", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("logit_cap", ctypes.c_float),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
    ]


class KimiMlaReduceParams(ctypes.Structure):
    _fields_ = [
        ("partial_o", ctypes.c_void_p),
        ("partial_lse", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("o_stride_b", ctypes.c_int64),
        ("o_stride_h", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
    ]


class KimiKvAppendParams(ctypes.Structure):
    _fields_ = [
        ("kv_c", ctypes.c_void_p),
        ("kv_c_stride", ctypes.c_int64),
        ("k_pe", ctypes.c_void_p),
        ("k_pe_stride", ctypes.c_int64),
        ("slot_mapping", ctypes.c_void_p),
        ("kv_buffer", ctypes.c_void_p),
        ("kv_scales", ctypes.c_void_p),
        ("num_pages", ctypes.c_int64),
        ("num_tokens", ctypes.c_int32),
        ("legacy_rule", ctypes.c_int32),
    ]


class KimiQAbsorbParams(ctypes.Structure):
    _fields_ = [
        ("q_nope", ctypes.c_void_p),
        ("q_nope_stride_t", ctypes.c_int64),
        ("q_nope_stride_h", ctypes.c_int64),
        ("q_pe", ctypes.c_void_p),
        ("q_pe_stride_t", ctypes.c_int64),
        ("q_pe_stride_h", ctypes.c_int64),
        ("w_uk", ctypes.c_void_p),
        ("kv_c", ctypes.c_void_p),
        ("kv_c_stride", ctypes.c_int64),
        ("k_pe", ctypes.c_void_p),
        ("k_pe_stride", ctypes.c_int64),
        ("positions", ctypes.c_void_p),
        ("cos_cache", ctypes.c_void_p),
        ("sin_cache", ctypes.c_void_p),
        ("max_position", ctypes.c_int64),
        ("slot_mapping", ctypes.c_void_p),
        ("kv_buffer", ctypes.c_void_p),
        ("kv_scales", ctypes.c_void_p),
        ("num_pages", ctypes.c_int64),
        ("q_out", ctypes.c_void_p),
        ("q_out_stride_t", ctypes.c_int64),
        ("q_out_stride_h", ctypes.c_int64),
        ("num_tokens", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("is_neox", ctypes.c_int32),
        ("legacy_rule", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


class KimiArRmsNormParams(ctypes.Structure):
    _fields_ = [
        ("inputs", ctypes.c_void_p * 8),
        ("num_inputs", ctypes.c_int32),
        ("residual", ctypes.c_void_p),
        ("residual_out", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("nibbles", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("rows", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("legacy_rule", ctypes.c_int32),
    ]


class KimiArTwoShotParams(ctypes.Structure):
    _fields_ = [
        ("inputs", ctypes.c_void_p * 8),
        ("residual_out", ctypes.c_void_p * 8),
        ("nibbles", ctypes.c_void_p * 8),
        ("scales", ctypes.c_void_p * 8),
        ("flags", ctypes.c_void_p * 8),
        ("counter", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("rows", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("legacy_rule", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
    ]


class KimiVUpOProjParams(ctypes.Structure):
    _fields_ = [
        ("o", ctypes.c_void_p),
        ("o_stride_h", ctypes.c_int64),
        ("o_stride_t", ctypes.c_int64),
        ("w_uv", ctypes.c_void_p),
        ("w_o", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_stride", ctypes.c_int64),
        ("num_tokens", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the library (once) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m kimi_b200.build` "
                "(this package has no CPU or Python fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        lib.kimi_abi_version.restype = ctypes.c_int
        lib.kimi_abi_version.argtypes = []
        lib.kimi_status_string.restype = ctypes.c_char_p
        lib.kimi_status_string.argtypes = [ctypes.c_int]
        lib.kimi_mla_decode_workspace_size.restype = sz
        lib.kimi_mla_decode_workspace_size.argtypes = [i32, i32, i32]
        lib.kimi_mla_decode_num_splits.restype = i32
        lib.kimi_mla_decode_num_splits.argtypes = [i32, i32, i32]
        lib.kimi_mla_decode.restype = ctypes.c_int
        lib.kimi_mla_decode.argtypes = [ctypes.POINTER(KimiMlaDecodeParams), vp, sz, vp]
        lib.kimi_mla_reduce.restype = ctypes.c_int
        lib.kimi_mla_reduce.argtypes = [ctypes.POINTER(KimiMlaReduceParams), vp]
        lib.kimi_mxfp4_kv_append.restype = ctypes.c_int
        lib.kimi_mxfp4_kv_append.argtypes = [ctypes.POINTER(KimiKvAppendParams), vp]
        for name in ("kimi_mla_decode_partial", "kimi_mla_decode_merge"):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(KimiMlaDecodeParams), vp, sz, vp]
        lib.kimi_mla_decode_static_workspace.restype = ctypes.c_int
        lib.kimi_mla_decode_static_workspace.argtypes = [ctypes.POINTER(KimiMlaDecodeParams), vp]
        lib.kimi_mla_q_absorb_rope_append.restype = ctypes.c_int
        lib.kimi_mla_q_absorb_rope_append.argtypes = [ctypes.POINTER(KimiQAbsorbParams), vp]
        lib.kimi_ar_rmsnorm_mxfp4.restype = ctypes.c_int
        lib.kimi_ar_rmsnorm_mxfp4.argtypes = [ctypes.POINTER(KimiArRmsNormParams), vp]
        lib.kimi_ar_rmsnorm_mxfp4_two_shot.restype = ctypes.c_int
        lib.kimi_ar_rmsnorm_mxfp4_two_shot.argtypes = [ctypes.POINTER(KimiArTwoShotParams), vp]
        lib.kimi_mla_v_up_o_proj.restype = ctypes.c_int
        lib.kimi_mla_v_up_o_proj.argtypes = [ctypes.POINTER(KimiVUpOProjParams), vp]
        lib.kimi_device_status.restype = ctypes.c_int
        lib.kimi_device_status.argtypes = [vp, i32, vp]
        lib.kimi_mxfp4_quantize.restype = ctypes.c_int
        lib.kimi_mxfp4_quantize.argtypes = [vp, i64, i64, i64, vp, vp, i32, vp]
        _lib = lib
        return _lib


def status_text(status: int) -> str:
    return load().kimi_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != KIMI_OK:
        kind = RuntimeError if status > 0 else ValueError
        raise kind(f"{what} failed: {status_text(status)} (status {status})")
