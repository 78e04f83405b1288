"""ctypes binding of the C ABI in ``include/fds_b200.h`` (``_lib/libfds_b200.so``).

The structures below mirror ``FdsFlexRelArgs`` / ``FdsRopeArgs`` field for
field. Loading fails loudly: there is no CPU or library fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

FDS_OK = 0
FDS_ERR_INVALID_ARGUMENT = 1
FDS_ERR_UNSUPPORTED_DEVICE = 2
FDS_ERR_CUDA = 3
FDS_ERR_TENSOR_MAP = 4

FDS_DTYPE_FP16 = 0
FDS_DTYPE_BF16 = 1

FDS_STATUS_TIMEOUT_LOAD = 0x1
FDS_STATUS_TIMEOUT_MMA = 0x2
FDS_STATUS_TIMEOUT_SOFTMAX = 0x4
FDS_STATUS_TIMEOUT_DRAIN = 0x8

FDS_DEBUG_FORCE_TIMEOUT = 0x1

FDS_ROPE_STATIC_SCRATCH_BYTES = 20 * 1024 * 1024

FDS_EPILOGUE_STORE = 0
FDS_EPILOGUE_ROPE = 1
FDS_EPILOGUE_ACCUMULATE_F32 = 2
FDS_GEMM_AUTO = 0
FDS_GEMM_SINGLE = 1
FDS_GEMM_PAIR = 2

ABI_VERSION = 4

# every symbol include/fds_b200.h declares (checked by the CPU test suite)
EXPORTED_SYMBOLS = (
    "fds_flexrel_attn_fwd",
    "fds_rope_attn_fwd",
    "fds_rope_attn_fwd_static",
    "fds_rope_split",
    "fds_abi_version",
    "fds_last_error",
    "fds_attn_smem_bytes",
    "fds_attn_workspace_bytes",
    "fds_attn_schedule",
    "fds_linear_fwd",
    "fds_flexrel_qr_attn_fwd",
)


class FdsFlexRelArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", ctypes.c_void_p),
        ("qkv_row_stride", ctypes.c_int64),
        ("rel", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_row_stride", ctypes.c_int64),
        ("kv_len", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("timeout_ns", ctypes.c_int64),
        ("debug_flags", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("grid_ctas", ctypes.c_int32),
        ("status_host", ctypes.c_void_p),
    ]


class FdsRopeArgs(ctypes.Structure):
    _fields_ = [
        ("qkv", ctypes.c_void_p),
        ("qkv_row_stride", ctypes.c_int64),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("qk_scratch", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_row_stride", ctypes.c_int64),
        ("status", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("timeout_ns", ctypes.c_int64),
        ("debug_flags", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("grid_ctas", ctypes.c_int32),
        ("status_host", ctypes.c_void_p),
        ("qk_rotated", ctypes.c_int32),
    ]


class FdsFlexRelQrArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("qr", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("kv_len", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("status_host", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("heads_last", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("timeout_ns", ctypes.c_int64),
        ("debug_flags", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("grid_ctas", ctypes.c_int32),
    ]


class FdsLinearArgs(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p),
        ("a_row_stride", ctypes.c_int64),
        ("w", ctypes.c_void_p),
        ("w_row_stride", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_row_stride", ctypes.c_int64),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("status_host", ctypes.c_void_p),
        ("m", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("epilogue", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("rope_cols", ctypes.c_int32),
        ("timeout_ns", ctypes.c_int64),
        ("grid_ctas", ctypes.c_int32),
        ("cta_pair", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()


def lib_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if the .so is missing) the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not path.exists():
            if not build_if_missing:
                raise RuntimeError(f"native library {path} is missing; run fastdialoguesidon_b200.build.build()")
            _build.build()
        lib = ctypes.CDLL(str(path))
        lib.fds_flexrel_attn_fwd.argtypes = [ctypes.POINTER(FdsFlexRelArgs), ctypes.c_void_p]
        lib.fds_flexrel_attn_fwd.restype = ctypes.c_int
        lib.fds_rope_attn_fwd.argtypes = [ctypes.POINTER(FdsRopeArgs), ctypes.c_void_p]
        lib.fds_rope_attn_fwd.restype = ctypes.c_int
        lib.fds_rope_attn_fwd_static.argtypes = [ctypes.POINTER(FdsRopeArgs), ctypes.c_void_p]
        lib.fds_rope_attn_fwd_static.restype = ctypes.c_int
        lib.fds_flexrel_qr_attn_fwd.argtypes = [ctypes.POINTER(FdsFlexRelQrArgs), ctypes.c_void_p]
        lib.fds_flexrel_qr_attn_fwd.restype = ctypes.c_int
        lib.fds_linear_fwd.argtypes = [ctypes.POINTER(FdsLinearArgs), ctypes.c_void_p]
        lib.fds_linear_fwd.restype = ctypes.c_int
        lib.fds_rope_split.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
        ]
        lib.fds_rope_split.restype = ctypes.c_int
        lib.fds_abi_version.argtypes = []
        lib.fds_abi_version.restype = ctypes.c_int
        lib.fds_last_error.argtypes = []
        lib.fds_last_error.restype = ctypes.c_char_p
        lib.fds_attn_smem_bytes.argtypes = []
        lib.fds_attn_smem_bytes.restype = ctypes.c_int
        lib.fds_attn_workspace_bytes.argtypes = [ctypes.c_int32]
        lib.fds_attn_workspace_bytes.restype = ctypes.c_int64
        lib.fds_attn_schedule.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int64, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)]
        lib.fds_attn_schedule.restype = ctypes.c_int
        if lib.fds_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{path}: ABI version {lib.fds_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def schedule(batch: int, heads: int, seq_len: int, has_kv_len: bool = False, workspace_bytes: int = 0,
             grid_ctas: int = 0) -> tuple[int, int, int]:
    """(CTAs, whole-unit CTAs, pieces of the split last wave) of a launch of this shape."""
    out = (ctypes.c_int64 * 3)()
    rc = load().fds_attn_schedule(batch, heads, seq_len, int(has_kv_len), workspace_bytes, grid_ctas, out)
    if rc != FDS_OK:
        raise RuntimeError(f"fds_attn_schedule failed ({rc}): {last_error()}")
    return int(out[0]), int(out[1]), int(out[2])


def last_error() -> str:
    return load().fds_last_error().decode(errors="replace")
