"""ctypes binding of ``libgraphkv_b200.so`` (C ABI in ``include/graphkv_b200.h``).

The library is built in-tree by ``graphkv_b200.build`` into
``graphkv_b200/lib/``.  There is no fallback: when the library is missing or a
CUDA device is not available, every compute call raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgraphkv_b200.so")

GKV_OK = 0
GKV_ERR_INVALID = -1
GKV_ERR_UNSUPPORTED = -2
GKV_ERR_CUDA = -3
GKV_ERR_WORKSPACE = -4
GKV_ERR_TOO_LARGE = -5

GKV_F32, GKV_F16, GKV_BF16 = 0, 1, 2
GKV_SYMMETRIC, GKV_AFFINE = 0, 1
GKV_AXIS_TOKEN, GKV_AXIS_CHANNEL = 0, 1
GKV_ROT_NONE, GKV_ROT_HADAMARD = 0, 1
STD_K, STD_V, COLD_K, COLD_V = 0, 1, 2, 3

DTYPE_CODE = {torch.float32: GKV_F32, torch.float16: GKV_F16, torch.bfloat16: GKV_BF16}

c_i32, c_i64, c_ptr = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class TensorSpec(ctypes.Structure):
    _fields_ = [("bits", c_i32), ("quantizer", c_i32), ("axis", c_i32), ("group_size", c_i32),
                ("rotation", c_i32), ("packed", c_i32), ("scale_dtype", c_i32), ("reserved", c_i32)]


class Plan(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("head_dim", c_i32), ("seq_len", c_i32), ("dtype", c_i32),
                ("n_retained", c_i32), ("n_standard", c_i32), ("n_cold", c_i32), ("out_seq_stride", c_i32),
                ("idx_retained", c_ptr), ("idx_standard", c_ptr), ("idx_cold", c_ptr),
                ("spec", TensorSpec * 4), ("hadamard_divisor", ctypes.c_float), ("reserved1", c_i32),
                ("retained_k", c_ptr), ("retained_v", c_ptr),
                ("codes", c_ptr * 4), ("scales", c_ptr * 4), ("zero_points", c_ptr * 4)]


class LayerIn(ctypes.Structure):
    _fields_ = [("k", c_ptr), ("v", c_ptr), ("k_stride", c_i64 * 3), ("v_stride", c_i64 * 3),
                ("heads", c_i32), ("reserved", c_i32)]


class SelectPolicy(ctypes.Structure):
    _fields_ = [("seq_len", c_i32), ("sink", c_i32), ("tail", c_i32), ("keep_protect", c_i32),
                ("keep_outlier", c_i32), ("keep_cold", c_i32), ("n_retained", c_i32), ("n_standard", c_i32),
                ("n_cold", c_i32), ("reserved", c_i32)]


_PROTOTYPES = {
    "gkv_abi_version": (c_i32, []),
    "gkv_last_error": (ctypes.c_char_p, []),
    "gkv_device_error": (c_i32, [ctypes.POINTER(c_i32)]),
    "gkv_select_workspace_bytes": (ctypes.c_size_t, [c_i32]),
    "gkv_select_tiers": (c_i32, [c_ptr, c_ptr, ctypes.POINTER(SelectPolicy), c_ptr, c_ptr, c_ptr, c_ptr,
                                 ctypes.c_size_t, c_ptr]),
    "gkv_select_tiers_static": (c_i32, [c_ptr, c_ptr, ctypes.POINTER(SelectPolicy), c_ptr, c_ptr, c_ptr, c_ptr]),
    "gkv_mean_scores": (c_i32, [c_ptr, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "gkv_outlier_scores": (c_i32, [ctypes.POINTER(LayerIn), c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "gkv_quantize_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Plan), ctypes.POINTER(LayerIn), c_i32]),
    "gkv_quantize": (c_i32, [ctypes.POINTER(Plan), ctypes.POINTER(LayerIn), c_i32, c_ptr, ctypes.c_size_t, c_ptr]),
    "gkv_dequantize_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Plan), c_i32]),
    "gkv_dequantize": (c_i32, [ctypes.POINTER(Plan), c_i32, c_ptr, c_ptr, c_ptr, ctypes.c_size_t, c_ptr]),
    "gkv_attention_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(Plan), c_i32, c_i32]),
    "gkv_attention": (c_i32, [ctypes.POINTER(Plan), c_i32, c_ptr, c_i32, c_ptr, c_ptr, ctypes.c_size_t, c_ptr]),
}

_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once) and declare the prototypes."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"graphkv_b200 CUDA library not found at {path}; build it with "
                    "`python -c 'import graphkv_b200.build as b; b.build()'`")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def lib() -> ctypes.CDLL:
    """The loaded library, checked to be usable for compute (CUDA present)."""
    if not torch.cuda.is_available():
        raise RuntimeError("graphkv_b200 needs a CUDA device; there is no CPU fallback.")
    return load()


def check(status: int) -> None:
    """Map a gkv_status to the reference's exception types."""
    if status == GKV_OK:
        return
    msg = (_lib.gkv_last_error() or b"").decode(errors="replace")
    if status in (GKV_ERR_INVALID, GKV_ERR_TOO_LARGE):
        raise ValueError(msg)
    raise RuntimeError(f"graphkv_b200 error {status}: {msg}")


def device_error() -> int:
    """Read and clear the device error word (synchronises the device)."""
    code = c_i32(0)
    check(lib().gkv_device_error(ctypes.byref(code)))
    return int(code.value)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()
