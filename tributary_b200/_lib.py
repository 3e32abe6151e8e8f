"""ctypes binding of libtributary_b200.so (the C ABI in include/rt_attention.h).

This is the same binding a reference-side integration writes; the Python
host layer in ``tributary_b200.attention`` and the
tests call the library through it. There is no fallback: if the shared
library is missing or fails to load, ``load()`` raises.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

RT_OK = 0
RT_ERR_INVALID_ARGUMENT = 1
RT_ERR_UNSUPPORTED = 2
RT_ERR_CUDA = 3
RT_ERR_TIMEOUT = 4
RT_ERR_WORKSPACE = 5
RT_ERR_DEVICE = 6

RT_MASK_COLUMN = 0
RT_MASK_FEATURE = 1
RT_MASK_NEIGHBOR = 2
RT_MASK_FULL = 3

TILE = 128

EXPORTED = (
    "rt_tile_plan_bytes", "rt_tile_plan_bind", "rt_build_tile_plan",
    "rt_attention_fwd", "rt_attention_bwd_workspace_bytes", "rt_attention_bwd",
    "rt_attention_bwd_noalloc", "rt_attention_bwd_qkv", "rt_column_order", "rt_rcm_order",
    "rt_qk_prepare", "rt_qk_prepare_bwd", "rt_heads_unpermute", "rt_heads_permute",
    "rt_device_status", "rt_status_string", "rt_last_error", "rt_version",
    "rt_selftest_bounded_wait", "rt_column_order_device",
    "rt_rms_norm", "rt_rms_norm_bwd_workspace_bytes", "rt_rms_norm_bwd", "rt_gate_residual",
    "rt_gate_residual_bwd", "rt_swiglu", "rt_swiglu_bwd", "rt_residual_add", "rt_residual_add_bwd",
)


class RtTilePlan(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
        ("tiles", ctypes.c_int32),
        ("words", ctypes.c_int32),
        ("live_bits", ctypes.c_void_p),
        ("full_bits", ctypes.c_void_p),
        ("q2k_ptr", ctypes.c_void_p),
        ("q2k_idx", ctypes.c_void_p),
        ("k2q_ptr", ctypes.c_void_p),
        ("k2q_idx", ctypes.c_void_p),
        ("tile_masks", ctypes.c_void_p),
        ("tile_masks_t", ctypes.c_void_p),
        ("fk_bits", ctypes.c_void_p),
        ("nnz", ctypes.c_void_p),
    ]


class RtError(RuntimeError):
    def __init__(self, status: int, what: str, message: str):
        super().__init__(f"{what}: {message} (status {status})")
        self.status = status


_LIB = None


def _declare(lib):
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t
    plan_p = ctypes.POINTER(RtTilePlan)
    lib.rt_tile_plan_bytes.argtypes = [i32, i32, i32]
    lib.rt_tile_plan_bytes.restype = sz
    lib.rt_tile_plan_bind.argtypes = [vp, sz, i32, i32, i32, plan_p]
    lib.rt_tile_plan_bind.restype = ctypes.c_int
    lib.rt_build_tile_plan.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, plan_p, vp]
    lib.rt_build_tile_plan.restype = ctypes.c_int
    lib.rt_qk_prepare.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp]
    lib.rt_qk_prepare.restype = ctypes.c_int
    lib.rt_qk_prepare_bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, vp]
    lib.rt_qk_prepare_bwd.restype = ctypes.c_int
    lib.rt_heads_unpermute.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp]
    lib.rt_heads_unpermute.restype = ctypes.c_int
    lib.rt_heads_permute.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp]
    lib.rt_heads_permute.restype = ctypes.c_int
    lib.rt_column_order.argtypes = [vp, vp, i32, i32, vp]
    lib.rt_column_order.restype = ctypes.c_int
    lib.rt_rcm_order.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp]
    lib.rt_rcm_order.restype = ctypes.c_int
    lib.rt_attention_fwd.argtypes = [vp, vp, vp, i32, i32, i32, i32, f32, plan_p, vp, vp, vp]
    lib.rt_attention_fwd.restype = ctypes.c_int
    lib.rt_attention_bwd_workspace_bytes.argtypes = [i32, i32, i32]
    lib.rt_attention_bwd_workspace_bytes.restype = sz
    lib.rt_attention_bwd.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, plan_p,
                                     vp, vp, vp, vp, sz, vp]
    lib.rt_attention_bwd.restype = ctypes.c_int
    lib.rt_attention_bwd_qkv.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, plan_p,
                                         vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.rt_attention_bwd_qkv.restype = ctypes.c_int
    lib.rt_attention_bwd_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32,
                                             plan_p, vp, vp, vp, vp]
    lib.rt_attention_bwd_noalloc.restype = ctypes.c_int
    lib.rt_device_status.argtypes = [i32]
    lib.rt_device_status.restype = ctypes.c_int
    lib.rt_status_string.argtypes = [i32]
    lib.rt_status_string.restype = ctypes.c_char_p
    lib.rt_last_error.argtypes = []
    lib.rt_last_error.restype = ctypes.c_char_p
    lib.rt_version.argtypes = []
    lib.rt_version.restype = i32
    i64 = ctypes.c_int64
    lib.rt_rms_norm.argtypes = [vp, vp, i64, i32, f32, vp, vp, vp]
    lib.rt_rms_norm.restype = ctypes.c_int
    lib.rt_rms_norm_bwd_workspace_bytes.argtypes = [i64, i32]
    lib.rt_rms_norm_bwd_workspace_bytes.restype = sz
    lib.rt_rms_norm_bwd.argtypes = [vp, vp, vp, vp, i64, i32, vp, vp, vp, sz, vp]
    lib.rt_rms_norm_bwd.restype = ctypes.c_int
    lib.rt_gate_residual.argtypes = [vp, vp, vp, i64, f32, vp, vp]
    lib.rt_gate_residual.restype = ctypes.c_int
    lib.rt_gate_residual_bwd.argtypes = [vp, vp, vp, i64, f32, vp, vp, vp]
    lib.rt_gate_residual_bwd.restype = ctypes.c_int
    lib.rt_residual_add.argtypes = [vp, vp, i64, f32, vp, vp]
    lib.rt_residual_add.restype = ctypes.c_int
    lib.rt_residual_add_bwd.argtypes = [vp, i64, f32, vp, vp]
    lib.rt_residual_add_bwd.restype = ctypes.c_int
    lib.rt_swiglu.argtypes = [vp, i64, i32, vp, vp]
    lib.rt_swiglu.restype = ctypes.c_int
    lib.rt_swiglu_bwd.argtypes = [vp, vp, i64, i32, vp, vp]
    lib.rt_swiglu_bwd.restype = ctypes.c_int
    lib.rt_column_order_device.argtypes = [vp, vp, i32, i32, vp, vp]
    lib.rt_column_order_device.restype = ctypes.c_int
    lib.rt_selftest_bounded_wait.argtypes = [ctypes.c_int64, vp, vp]
    lib.rt_selftest_bounded_wait.restype = ctypes.c_int


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of the CUDA library."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"CUDA library not built: {p} (run python -m tributary_b200.build)")
    lib = ctypes.CDLL(p)
    _declare(lib)
    if path is None:
        _LIB = lib
    return lib


def check(status: int, what: str):
    if status != RT_OK:
        lib = load()
        msg = lib.rt_status_string(status).decode()
        if status == RT_ERR_CUDA:
            msg += " -- " + lib.rt_last_error().decode()
        raise RtError(status, what, msg)
