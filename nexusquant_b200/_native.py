"""ctypes binding of libnexusquant_b200.so (the C ABI in include/nexusquant_b200.h).

The shared library is built in-tree (``make -C nexusquant_b200/csrc``, or
``__graft_entry__.build()``) into ``nexusquant_b200/_lib/``.  There is no
fallback: if the library is missing, or the tensors handed to an entry point
are not CUDA tensors, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libnexusquant_b200.so")

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_f32 = ctypes.c_float
c_size = ctypes.c_size_t

NQ_OK = 0
_STATUS = {
    0: "ok", -1: "invalid argument", -2: "unsupported shape or dtype", -3: "CUDA error",
    -4: "device-side wait timed out", -5: "workspace missing or too small",
    -6: "pointer or stride not 16-byte aligned", -7: "problem exceeds the library's built-in scratch size",
}


class NexusQuantError(RuntimeError):
    """Raised when a native entry point returns a non-zero nq_status_t."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {_STATUS.get(status, 'unknown')} (status {status})")


class LayerIO(ctypes.Structure):
    _fields_ = [("k", c_vp), ("v", c_vp), ("k_codes", c_vp), ("v_codes", c_vp),
                ("k_scales", c_vp), ("v_scales", c_vp), ("k_scales_f32", c_vp), ("v_scales_f32", c_vp),
                ("k_out", c_vp), ("v_out", c_vp), ("key_levels", c_i32), ("value_levels", c_i32)]


class CompressParams(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("heads", c_i32), ("seq", c_i32), ("head_dim", c_i32),
                ("head_dim_padded", c_i32), ("n_kept", c_i32), ("kept_idx", c_vp), ("kept_count", c_vp),
                ("positions", c_vp), ("rope_cos", c_vp), ("rope_sin", c_vp), ("rope_rows", c_i32),
                ("in_dtype", c_i32), ("in_stride_b", c_i64), ("in_stride_h", c_i64), ("in_stride_t", c_i64),
                ("out_stride_b", c_i64), ("out_stride_h", c_i64), ("out_stride_t", c_i64),
                ("out_row_mode", c_i32), ("out_positions", c_vp), ("key_sharpen", c_f32),
                ("rotate", c_i32), ("inputs_host", c_i32), ("error_flag", c_vp), ("layers", ctypes.POINTER(LayerIO)), ("n_layers", c_i32)]


class DLayerIO(ctypes.Structure):
    _fields_ = [("k_codes", c_vp), ("v_codes", c_vp), ("k_scales", c_vp), ("v_scales", c_vp),
                ("k_out", c_vp), ("v_out", c_vp), ("key_levels", c_i32), ("value_levels", c_i32)]


class DecompressParams(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("heads", c_i32), ("n_tokens", c_i32), ("head_dim", c_i32),
                ("head_dim_padded", c_i32), ("count", c_vp), ("positions", c_vp), ("rope_cos", c_vp),
                ("rope_sin", c_vp), ("rope_rows", c_i32), ("out_stride_b", c_i64), ("out_stride_h", c_i64),
                ("out_stride_t", c_i64), ("key_sharpen", c_f32), ("layers", ctypes.POINTER(DLayerIO)),
                ("n_layers", c_i32)]


class AttendParams(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("q_heads", c_i32), ("heads", c_i32), ("head_dim", c_i32),
                ("head_dim_padded", c_i32), ("n_tokens", c_i32), ("count", c_vp), ("q", c_vp),
                ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("k_codes", c_vp), ("v_codes", c_vp),
                ("k_scales", c_vp), ("v_scales", c_vp), ("key_levels", c_i32), ("value_levels", c_i32),
                ("positions", c_vp), ("rope_cos", c_vp), ("rope_sin", c_vp), ("rope_rows", c_i32),
                ("key_sharpen", c_f32), ("scale", c_f32), ("out", c_vp), ("out_stride_b", c_i64),
                ("out_stride_h", c_i64)]


# name -> (restype, argtypes)
_PROTOS = {
    "nq_status_string": (ctypes.c_char_p, [c_i32]),
    "nq_abi_version": (c_i32, []),
    "nq_packed_bytes": (c_i32, [c_i32, c_i32]),
    "nq_compress_layers": (c_i32, [ctypes.POINTER(CompressParams), c_vp]),
    "nq_decompress_layers": (c_i32, [ctypes.POINTER(DecompressParams), c_vp]),
    "nq_score_keykey": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_i64, c_i32, c_i32,
                                c_i32, c_i32, c_vp, c_vp, c_size, c_vp]),
    "nq_score_keykey_workspace_size": (c_size, [c_i32, c_i32, c_i32, c_i32]),
    "nq_score_keykey_noalloc": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_i64, c_i32, c_i32,
                                        c_i32, c_i32, c_vp, c_vp]),
    "nq_score_attention": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64,
                                   c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp, c_vp, c_size, c_vp]),
    "nq_score_attention_workspace_size": (c_size, [c_i32, c_i32, c_i32, c_i32]),
    "nq_reduce_heads": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_f32, c_i32, c_vp, c_vp]),
    "nq_select_keep": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp, c_vp, c_size, c_vp]),
    "nq_select_keep_workspace_size": (c_size, [c_i32, c_i32]),
    "nq_gather_rows": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp, c_i32, c_vp,
                               c_i64, c_i64, c_i64, c_vp]),
    "nq_delta_codes": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "nq_code_histogram": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp]),
    "nq_code_symbols": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "nq_rans_encode": (c_i32, [c_vp, c_i64, c_vp, c_i32, c_vp, c_i64, ctypes.POINTER(c_i64)]),
    "nq_rans_decode": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_i32, c_vp]),
    "nq_attend_compressed_workspace_size": (c_size, [c_i32, c_i32, c_i32, c_i32]),
    "nq_attend_compressed": (c_i32, [ctypes.POINTER(AttendParams), c_vp, c_size, c_vp]),
    "nq_merge_centroid_accumulate": (c_i32, [ctypes.POINTER(c_vp), c_i32, c_i32, c_i32, c_i32, c_i32, c_i64,
                                             c_i64, c_i32, c_vp, c_vp]),
    "nq_merge_centroid_normalize": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "nq_merge_nearest": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_vp, c_i32, c_vp, c_vp]),
    "nq_merge_nearest_unit": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_vp, c_i32, c_vp, c_vp]),
    "nq_unpack_codes": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp]),
    "nq_pack_nibbles": (c_i32, [c_vp, c_i64, c_i32, c_vp, c_vp]),
    "nq_unpack_nibbles": (c_i32, [c_vp, c_i64, c_i32, c_vp, c_vp]),
    "nq_merge_apply": (c_i32, [ctypes.POINTER(c_vp), c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_vp, c_vp,
                               c_i32, c_vp, c_vp, c_vp]),
    "nq_device_error": (c_i32, [ctypes.POINTER(c_i32), c_vp]),
    "nq_wait_selftest": (c_i32, [ctypes.c_uint32, c_vp]),
}

EXPORTED = tuple(_PROTOS)

_lib = None
_lock = threading.Lock()


def library_path() -> str:
    return LIB_PATH


def load(path: str = LIB_PATH):
    """Load (once) and return the native library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise ImportError(
                    f"nexusquant_b200 native library not found at {path}; build it with "
                    f"`make -C {os.path.join(_HERE, 'csrc')}` (nvcc, sm_100a)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _PROTOS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.nq_abi_version() != 2:
                raise ImportError("nexusquant_b200 native library ABI mismatch")
            _lib = lib
    return _lib


def check(fn: str, status: int) -> None:
    if status != NQ_OK:
        raise NexusQuantError(fn, status)


def call(fn: str, *args) -> None:
    check(fn, getattr(load(), fn)(*args))
